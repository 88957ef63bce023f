// breeze-synth: writes a seeded random-init Breeze-TTS-2 GGUF with the tensor names and
// `breeze.*` keys the generator reads (reference: src/config.cpp:8-99 for the keys,
// src/backbone.cpp:248-276, src/depth_decoder.cpp:40-85, src/text_encoder.cpp:8-72 for
// the tensors). Real weights are not available offline; these files stand in for them
// so the CUDA engine and the oracle read byte-identical inputs.
//
// Linear and embedding weights are N(0, 0.02) quantised to Q8_0 (same rule as gguf-py's
// Q8_0.quantize_blocks: d = amax/127, q = round-half-away(x * (1/d)), d stored as f16) or to Q4_K
// (a min/max quantiser that emits valid 144-byte blocks); norm weights are 1 + N(0, 0.02)
// in F32. Generation is deterministic for a seed and independent of the thread count.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

namespace {

enum GgufType : uint32_t { T_U8 = 0, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 };
enum GgmlType : uint32_t { G_F32 = 0, G_F16 = 1, G_Q8_0 = 8, G_Q4_K = 12 };

uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) return (uint16_t) (sign | (absx > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (absx >= 0x477ff000u) return (uint16_t) (sign | 0x7c00u);  // rounds to inf
    if (absx < 0x38800000u) {                                     // subnormal half
        if (absx < 0x33000000u) return (uint16_t) sign;
        const uint32_t m = (absx & 0x7fffffu) | 0x800000u;
        const int shift = 126 - (int) (absx >> 23) + 13;
        uint32_t h = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t) (sign | h);
    }
    uint32_t h = ((absx >> 13) - (112u << 10));
    const uint32_t rem = absx & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t) (sign | h);
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, x;
    if (e == 0) {
        if (m == 0) x = sign;
        else {
            e = 113;
            while (!(m & 0x400u)) { m <<= 1; e--; }
            x = sign | (e << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) x = sign | 0x7f800000u | (m << 13);
    else x = sign | ((e + 112u) << 23) | (m << 13);
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

uint64_t splitmix(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// element i of the standard-normal stream for (seed, tensor): Box-Muller over a hashed pair
float normal_at(uint64_t key, uint64_t i) {
    const uint64_t r = splitmix(key ^ splitmix(i >> 1));
    const double u1 = ((double) ((r >> 11) & ((1ull << 26) - 1)) + 0.5) / (double) (1ull << 26);
    const double u2 = ((double) (r >> 38) + 0.5) / (double) (1ull << 26);
    const double rad = std::sqrt(-2.0 * std::log(u1));
    return (float) ((i & 1) ? rad * std::sin(6.283185307179586 * u2) : rad * std::cos(6.283185307179586 * u2));
}

// round half away from zero without the double rounding of floor(v + 0.5f)
float round_half_away(float v) {
    const float a = std::fabs(v), f = std::floor(a);
    const float r = f + std::floor(2.0f * (a - f));
    return v < 0 ? -r : r;
}

void quant_q8_0_block(const float * x, uint8_t * out) {
    float amax = 0.0f;
    for (int j = 0; j < 32; j++) amax = std::max(amax, std::fabs(x[j]));
    const float d = amax / 127.0f;
    const float id = d == 0.0f ? 0.0f : 1.0f / d;
    const uint16_t dh = f32_to_f16(d);
    std::memcpy(out, &dh, 2);
    for (int j = 0; j < 32; j++) {
        const float q = round_half_away(x[j] * id);
        out[2 + j] = (uint8_t) (int8_t) q;
    }
}

// min/max Q4_K quantiser: 8 sub-blocks of 32, each y = d*sc*q - dmin*m with 6-bit sc, m
void quant_q4_k_block(const float * x, uint8_t * out) {
    float sub_scale[8], sub_min[8];
    for (int s = 0; s < 8; s++) {
        float lo = x[s * 32], hi = x[s * 32];
        for (int j = 1; j < 32; j++) { lo = std::min(lo, x[s * 32 + j]); hi = std::max(hi, x[s * 32 + j]); }
        lo = std::min(lo, 0.0f);
        sub_scale[s] = (hi - lo) / 15.0f;
        sub_min[s] = -lo;
    }
    float max_scale = 0, max_min = 0;
    for (int s = 0; s < 8; s++) { max_scale = std::max(max_scale, sub_scale[s]); max_min = std::max(max_min, sub_min[s]); }
    const uint16_t dh = f32_to_f16(max_scale / 63.0f), mh = f32_to_f16(max_min / 63.0f);
    const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
    uint8_t sc[8], mn[8];
    for (int s = 0; s < 8; s++) {
        sc[s] = (uint8_t) std::min(63.0f, d > 0 ? std::nearbyint(sub_scale[s] / d) : 0.0f);
        mn[s] = (uint8_t) std::min(63.0f, dmin > 0 ? std::nearbyint(sub_min[s] / dmin) : 0.0f);
    }
    std::memcpy(out, &dh, 2);
    std::memcpy(out + 2, &mh, 2);
    uint8_t * scales = out + 4;
    for (int j = 0; j < 4; j++) {
        scales[j] = (uint8_t) ((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        scales[j + 4] = (uint8_t) ((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        scales[j + 8] = (uint8_t) ((sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4));
    }
    uint8_t * qs = out + 16;
    for (int c = 0; c < 4; c++) {
        for (int half = 0; half < 2; half++) {
            const int s = c * 2 + half;
            const float ds = d * sc[s], dm = dmin * mn[s];
            for (int l = 0; l < 32; l++) {
                int q = ds > 0 ? (int) std::nearbyint((x[s * 32 + l] + dm) / ds) : 0;
                q = std::max(0, std::min(15, q));
                if (half == 0) qs[c * 32 + l] = (uint8_t) q;
                else qs[c * 32 + l] |= (uint8_t) (q << 4);
            }
        }
    }
}

struct Tensor {
    std::string name;
    std::vector<int64_t> ne;
    GgmlType type;
    int kind;  // 0 = linear N(0, 0.02), 1 = norm 1 + N(0, 0.02), 2 = N(mean, stdv)
    uint64_t offset = 0;
    uint64_t nbytes = 0;
    float mean = 0.0f, stdv = 0.0f;
};

struct Writer {
    std::vector<uint8_t> meta;
    uint64_t n_kv = 0;
    void raw(const void * p, size_t n) { const uint8_t * b = (const uint8_t *) p; meta.insert(meta.end(), b, b + n); }
    void u32(uint32_t v) { raw(&v, 4); }
    void u64(uint64_t v) { raw(&v, 8); }
    void str(const std::string & s) { u64(s.size()); raw(s.data(), s.size()); }
    void kv_u32(const std::string & k, uint32_t v) { str(k); u32(T_U32); u32(v); n_kv++; }
    void kv_f32(const std::string & k, float v) { str(k); u32(T_F32); raw(&v, 4); n_kv++; }
    void kv_str(const std::string & k, const std::string & v) { str(k); u32(T_STR); str(v); n_kv++; }
    void kv_i32_arr(const std::string & k, const std::vector<int32_t> & v) {
        str(k); u32(T_ARR); u32(T_I32); u64(v.size());
        for (int32_t x : v) raw(&x, 4);
        n_kv++;
    }
    void kv_str_arr(const std::string & k, const std::vector<std::string> & v) {
        str(k); u32(T_ARR); u32(T_STR); u64(v.size());
        for (const auto & s : v) str(s);
        n_kv++;
    }
};

struct Spec {
    int hidden = 2048, nc = 32, vs = 2051, cb_size = 2048;
    int bb_layers = 16, bb_heads = 32, bb_kv = 8, bb_hd = 64, bb_ffn = 8192;
    int dd_hidden = 1024, dd_layers = 4, dd_heads = 8, dd_kv = 2, dd_hd = 128, dd_ffn = 8192;
    int te_hidden = 1152, te_layers = 26, te_heads = 4, te_kv = 1, te_hd = 256, te_ffn = 6912, te_window = 512;
    int vocab = 128256;
    int eos_off = 0;
    int max_new_tokens = 750;
    int depth_top_k = 50;
    GgmlType qtype = G_Q8_0;
    uint64_t seed = 0;
    // vocoder (codec decoder): quantiser embedding dim, its projection, the transformer's latent
    // and hidden widths, heads, MLP, attention window, the conv stack's first width and the two
    // upsampling stages (ConvNeXt stages, then SnakeBeta blocks); 2 * 8 * 6 * 5 * 4 = 1920
    int voc_dq = 256, voc_cbdim = 512, voc_latent = 1024, voc_hidden = 512, voc_layers = 8, voc_heads = 8,
        voc_kv = 8, voc_hd = 64, voc_ffn = 1024, voc_window = 72, voc_dec = 1536;
    std::vector<int32_t> voc_ratios = { 2 }, voc_rates = { 8, 6, 5, 4 };
    // codec encoder (src/codec.cpp:80-123, src/codec_conv.cpp:60-77, src/codec_transformer.cpp:9-45):
    // SEANet filters, transformer width/layers/heads/MLP/window, codebook dim; the SEANet strides
    // run the upsampling ratios in reverse, then a stride-2 downsample: 4 * 5 * 6 * 8 * 2 = 1920
    int enc_nf = 64, enc_hidden = 512, enc_layers = 8, enc_heads = 8, enc_hd = 64, enc_ffn = 2048,
        enc_window = 250, enc_dim = 256;
    std::vector<int32_t> enc_ratios = { 8, 6, 5, 4 };
};

uint64_t tensor_bytes(const Tensor & t) {
    int64_t n = 1;
    for (int64_t d : t.ne) n *= d;
    switch (t.type) {
        case G_F32: return (uint64_t) n * 4;
        case G_F16: return (uint64_t) n * 2;
        case G_Q8_0: return (uint64_t) n / 32 * 34;
        case G_Q4_K: return (uint64_t) n / 256 * 144;
    }
    return 0;
}

void fill_tensor(const Tensor & t, uint64_t key, uint8_t * dst, int n_threads) {
    int64_t n = 1;
    for (int64_t d : t.ne) n *= d;
    const int blk = t.type == G_Q8_0 ? 32 : t.type == G_Q4_K ? 256 : 1;
    const int64_t n_blocks = n / blk;
    const int64_t per = (n_blocks + n_threads - 1) / n_threads;
    auto work = [&](int64_t b0, int64_t b1) {
        std::vector<float> buf(blk);
        for (int64_t b = b0; b < b1; b++) {
            for (int j = 0; j < blk; j++) {
                const uint64_t i = (uint64_t) (b * blk + j);
                const float z = normal_at(key, i);
                buf[j] = t.kind == 2 ? t.mean + t.stdv * z : t.kind == 1 ? 1.0f + 0.02f * z : 0.02f * z;
            }
            if (t.type == G_F32) std::memcpy(dst + b * 4, buf.data(), 4);
            else if (t.type == G_F16) { uint16_t h = f32_to_f16(buf[0]); std::memcpy(dst + b * 2, &h, 2); }
            else if (t.type == G_Q8_0) quant_q8_0_block(buf.data(), dst + b * 34);
            else quant_q4_k_block(buf.data(), dst + b * 144);
        }
    };
    std::vector<std::thread> th;
    for (int i = 0; i < n_threads; i++) {
        const int64_t b0 = i * per, b1 = std::min(n_blocks, b0 + per);
        if (b0 < b1) th.emplace_back(work, b0, b1);
    }
    for (auto & x : th) x.join();
}

int usage() {
    std::fprintf(stderr,
        "usage: breeze-synth --out PATH [--preset full|depth|tiny] [--nc N] [--quant q8_0|q4_k] [--seed S]\n"
        "                    [--eos-off] [--max-new-tokens N] [--depth-top-k K] [--threads T]\n"
        "       breeze-synth --quantize-f32 IN OUT [--quant q8_0|q4_k]   (raw f32 -> raw blocks)\n");
    return 2;
}

// quantises a raw little-endian f32 file with the writer's quantiser (used to pin it)
int quantize_file(const std::string & in, const std::string & out, GgmlType q) {
    FILE * f = std::fopen(in.c_str(), "rb");
    if (!f) return 1;
    std::vector<float> x;
    float v;
    while (std::fread(&v, 4, 1, f) == 1) x.push_back(v);
    std::fclose(f);
    const int blk = q == G_Q4_K ? 256 : 32, bb = q == G_Q4_K ? 144 : 34;
    if (x.size() % blk) return 2;
    std::vector<uint8_t> o(x.size() / blk * bb);
    for (size_t b = 0; b < x.size() / blk; b++) {
        if (q == G_Q4_K) quant_q4_k_block(x.data() + b * blk, o.data() + b * bb);
        else quant_q8_0_block(x.data() + b * blk, o.data() + b * bb);
    }
    f = std::fopen(out.c_str(), "wb");
    if (!f) return 1;
    std::fwrite(o.data(), 1, o.size(), f);
    std::fclose(f);
    return 0;
}

}  // namespace

int main(int argc, char ** argv) {
    Spec s;
    std::string out, preset = "full";
    int threads = (int) std::max(1u, std::thread::hardware_concurrency());
    int nc_override = 0;
    std::string qin, qout;
    for (int i = 1; i < argc; i++) {
        std::string a = argv[i];
        auto next = [&]() -> std::string { if (i + 1 >= argc) { std::exit(usage()); } return argv[++i]; };
        if (a == "--out") out = next();
        else if (a == "--preset") preset = next();
        else if (a == "--nc") nc_override = std::atoi(next().c_str());
        else if (a == "--quant") { std::string q = next(); s.qtype = q == "q4_k" ? G_Q4_K : G_Q8_0; }
        else if (a == "--seed") s.seed = std::strtoull(next().c_str(), nullptr, 10);
        else if (a == "--eos-off") s.eos_off = 1;
        else if (a == "--max-new-tokens") s.max_new_tokens = std::atoi(next().c_str());
        else if (a == "--depth-top-k") s.depth_top_k = std::atoi(next().c_str());
        else if (a == "--threads") threads = std::max(1, std::atoi(next().c_str()));
        else if (a == "--quantize-f32") { qin = next(); qout = next(); }
        else return usage();
    }
    if (!qin.empty()) return quantize_file(qin, qout, s.qtype);
    if (out.empty()) return usage();
    if (preset == "tiny") {
        s.hidden = 256; s.nc = 8;
        s.bb_layers = 2; s.bb_heads = 4; s.bb_kv = 2; s.bb_hd = 64; s.bb_ffn = 512;
        s.dd_hidden = 256; s.dd_layers = 2; s.dd_heads = 2; s.dd_kv = 1; s.dd_hd = 128; s.dd_ffn = 512;
        s.te_hidden = 256; s.te_layers = 2; s.te_heads = 2; s.te_kv = 1; s.te_hd = 128; s.te_ffn = 512; s.te_window = 8;
        s.voc_dq = 32; s.voc_cbdim = 64; s.voc_latent = 64; s.voc_hidden = 64; s.voc_layers = 2; s.voc_heads = 2;
        s.voc_kv = 1; s.voc_hd = 32; s.voc_ffn = 128; s.voc_window = 8; s.voc_dec = 64;
        s.enc_nf = 8; s.enc_hidden = 64; s.enc_layers = 2; s.enc_heads = 2; s.enc_hd = 32; s.enc_ffn = 128;
        s.enc_window = 8; s.enc_dim = 32;
    } else if (preset == "depth") {
        // the full-size depth decoder behind a one-layer backbone and a small text encoder: the
        // depth kernels at their real shapes in a model of a few hundred MB (profiling captures)
        s.bb_layers = 1; s.bb_ffn = 512;
        s.te_hidden = 256; s.te_layers = 1; s.te_heads = 2; s.te_kv = 1; s.te_hd = 128; s.te_ffn = 512; s.te_window = 8;
    } else if (preset != "full") return usage();
    if (nc_override > 0) s.nc = nc_override;
    // the backbone and depth linears must be whole Q4_K super-blocks; text-encoder and vocoder
    // tensors whose rows are not keep Q8_0 (lin() below)
    if (s.qtype == G_Q4_K && (s.hidden % 256 || s.dd_hidden % 256 || s.bb_ffn % 256 || s.dd_ffn % 256)) {
        std::fprintf(stderr, "Q4_K needs backbone and depth row lengths that are multiples of 256\n");
        return 2;
    }

    const GgmlType q = s.qtype;
    std::vector<Tensor> ts;
    // a Q4_K file keeps Q8_0 for tensors whose rows are not whole 256-value super-blocks (the
    // way llama.cpp's quantiser falls back), e.g. the small vocoder's 32-wide projections
    auto lin = [&](const std::string & n, int64_t in, int64_t outd, int64_t n2 = 0) {
        const GgmlType tq = (q == G_Q4_K && in % 256) ? G_Q8_0 : q;
        Tensor t{ n, n2 ? std::vector<int64_t>{ in, outd, n2 } : std::vector<int64_t>{ in, outd }, tq, 0 };
        ts.push_back(t);
    };
    auto nrm = [&](const std::string & n, int64_t d) { ts.push_back(Tensor{ n, { d }, G_F32, 1 }); };

    // text encoder (src/text_encoder.cpp:19-68)
    lin("te.token_embd.weight", s.te_hidden, s.vocab);
    for (int l = 0; l < s.te_layers; l++) {
        const std::string p = "te.blk." + std::to_string(l);
        nrm(p + ".attn_norm.weight", s.te_hidden);
        lin(p + ".attn_q.weight", s.te_hidden, (int64_t) s.te_heads * s.te_hd);
        lin(p + ".attn_k.weight", s.te_hidden, (int64_t) s.te_kv * s.te_hd);
        lin(p + ".attn_v.weight", s.te_hidden, (int64_t) s.te_kv * s.te_hd);
        nrm(p + ".attn_q_norm.weight", s.te_hd);
        nrm(p + ".attn_k_norm.weight", s.te_hd);
        lin(p + ".attn_output.weight", (int64_t) s.te_heads * s.te_hd, s.te_hidden);
        nrm(p + ".post_attn_norm.weight", s.te_hidden);
        nrm(p + ".ffn_norm.weight", s.te_hidden);
        lin(p + ".ffn_gate.weight", s.te_hidden, s.te_ffn);
        lin(p + ".ffn_up.weight", s.te_hidden, s.te_ffn);
        lin(p + ".ffn_down.weight", s.te_ffn, s.te_hidden);
        nrm(p + ".post_ffn_norm.weight", s.te_hidden);
    }
    nrm("te.output_norm.weight", s.te_hidden);
    lin("te.proj.weight", s.te_hidden, s.hidden);

    // backbone (src/backbone.cpp:223-232, 248-276, 291-295)
    lin("audio_embd.weight", s.hidden, (int64_t) s.nc * s.vs);
    for (int l = 0; l < s.bb_layers; l++) {
        const std::string p = "bb.blk." + std::to_string(l);
        nrm(p + ".attn_norm.weight", s.hidden);
        lin(p + ".attn_q.weight", s.hidden, (int64_t) s.bb_heads * s.bb_hd);
        lin(p + ".attn_k.weight", s.hidden, (int64_t) s.bb_kv * s.bb_hd);
        lin(p + ".attn_v.weight", s.hidden, (int64_t) s.bb_kv * s.bb_hd);
        nrm(p + ".attn_q_norm.weight", s.bb_hd);
        nrm(p + ".attn_k_norm.weight", s.bb_hd);
        lin(p + ".attn_output.weight", (int64_t) s.bb_heads * s.bb_hd, s.hidden);
        nrm(p + ".ffn_norm.weight", s.hidden);
        lin(p + ".ffn_gate.weight", s.hidden, s.bb_ffn);
        lin(p + ".ffn_up.weight", s.hidden, s.bb_ffn);
        lin(p + ".ffn_down.weight", s.bb_ffn, s.hidden);
    }
    nrm("bb.output_norm.weight", s.hidden);
    lin("bb.lm_head.weight", s.hidden, s.eos_off ? s.vs : s.vs + 1);

    // depth decoder (src/depth_decoder.cpp:48-50, 60-85, 119-125)
    lin("dd.in_proj.weight", s.hidden, s.dd_hidden);
    for (int l = 0; l < s.dd_layers; l++) {
        const std::string p = "dd.blk." + std::to_string(l);
        nrm(p + ".attn_norm.weight", s.dd_hidden);
        lin(p + ".attn_q.weight", s.dd_hidden, (int64_t) s.dd_heads * s.dd_hd);
        lin(p + ".attn_k.weight", s.dd_hidden, (int64_t) s.dd_kv * s.dd_hd);
        lin(p + ".attn_v.weight", s.dd_hidden, (int64_t) s.dd_kv * s.dd_hd);
        lin(p + ".attn_output.weight", (int64_t) s.dd_heads * s.dd_hd, s.dd_hidden);
        nrm(p + ".ffn_norm.weight", s.dd_hidden);
        lin(p + ".ffn_gate.weight", s.dd_hidden, s.dd_ffn);
        lin(p + ".ffn_up.weight", s.dd_hidden, s.dd_ffn);
        lin(p + ".ffn_down.weight", s.dd_ffn, s.dd_hidden);
    }
    nrm("dd.output_norm.weight", s.dd_hidden);
    lin("dd.codebooks_head.weight", s.dd_hidden, s.vs, s.nc - 1);

    // vocoder decoder (src/codec_decoder.cpp:11-98, src/codec_transformer.cpp:48-83); shapes in
    // ggml order. Appended after every generator tensor so their seeds do not move. Conv kernels
    // are F32 [K, C_in, C_out] (transposed convs [K, C_out, C_in], depthwise [C, K]) scaled by
    // 1/sqrt(fan in); SnakeBeta alpha/beta are log-space N(0, 0.1); layer scales 0.1.
    auto f32t = [&](const std::string & n, std::vector<int64_t> ne, float mean, float stdv) {
        Tensor t{ n, ne, G_F32, 2 };
        t.mean = mean;
        t.stdv = stdv;
        ts.push_back(t);
    };
    auto conv = [&](const std::string & n, int64_t K, int64_t cin, int64_t cout) {
        f32t(n + ".weight", { K, cin, cout }, 0.0f, 0.7f / std::sqrt((float) (K * cin)));
        f32t(n + ".bias", { cout }, 0.0f, 0.02f);
    };
    auto convtr = [&](const std::string & n, int64_t K, int64_t cin, int64_t cout, int64_t stride) {
        f32t(n + ".weight", { K, cout, cin }, 0.0f, 0.7f / std::sqrt((float) (cin * K / stride)));
        f32t(n + ".bias", { cout }, 0.0f, 0.02f);
    };
    f32t("codec.dq.first.0.embed", { s.voc_dq, s.vs }, 0.0f, 1.0f);
    lin("codec.dq.first.out_proj.weight", s.voc_dq, s.voc_cbdim);
    for (int cb = 1; cb < s.nc; cb++) f32t("codec.dq.rest." + std::to_string(cb - 1) + ".embed", { s.voc_dq, s.vs }, 0.0f, 1.0f);
    lin("codec.dq.rest.out_proj.weight", s.voc_dq, s.voc_cbdim);
    conv("codec.dpre.conv", 3, s.voc_cbdim, s.voc_latent);
    lin("codec.dtf.in_proj.weight", s.voc_latent, s.voc_hidden);
    f32t("codec.dtf.in_proj.bias", { s.voc_hidden }, 0.0f, 0.02f);
    for (int l = 0; l < s.voc_layers; l++) {
        const std::string p = "codec.dtf.blk." + std::to_string(l);
        nrm(p + ".attn_norm.weight", s.voc_hidden);
        lin(p + ".attn_q.weight", s.voc_hidden, (int64_t) s.voc_heads * s.voc_hd);
        lin(p + ".attn_k.weight", s.voc_hidden, (int64_t) s.voc_kv * s.voc_hd);
        lin(p + ".attn_v.weight", s.voc_hidden, (int64_t) s.voc_kv * s.voc_hd);
        lin(p + ".attn_output.weight", (int64_t) s.voc_heads * s.voc_hd, s.voc_hidden);
        f32t(p + ".attn_scale", { s.voc_hidden }, 0.1f, 0.01f);
        nrm(p + ".ffn_norm.weight", s.voc_hidden);
        lin(p + ".ffn_gate.weight", s.voc_hidden, s.voc_ffn);
        lin(p + ".ffn_up.weight", s.voc_hidden, s.voc_ffn);
        lin(p + ".ffn_down.weight", s.voc_ffn, s.voc_hidden);
        f32t(p + ".ffn_scale", { s.voc_hidden }, 0.1f, 0.01f);
    }
    nrm("codec.dtf.norm.weight", s.voc_hidden);
    lin("codec.dtf.out_proj.weight", s.voc_hidden, s.voc_latent);
    f32t("codec.dtf.out_proj.bias", { s.voc_latent }, 0.0f, 0.02f);
    for (size_t i = 0; i < s.voc_ratios.size(); i++) {
        const std::string p = "codec.dup." + std::to_string(i);
        const int r = s.voc_ratios[i];
        convtr(p + ".up.conv", 2 * r, s.voc_latent, s.voc_latent, r);
        f32t(p + ".dw.weight", { s.voc_latent, 7 }, 0.0f, 0.7f / std::sqrt(7.0f));
        f32t(p + ".dw.bias", { s.voc_latent }, 0.0f, 0.02f);
        nrm(p + ".norm.weight", s.voc_latent);
        f32t(p + ".norm.bias", { s.voc_latent }, 0.0f, 0.02f);
        lin(p + ".pw1.weight", s.voc_latent, 4 * s.voc_latent);
        f32t(p + ".pw1.bias", { 4 * s.voc_latent }, 0.0f, 0.02f);
        lin(p + ".pw2.weight", 4 * s.voc_latent, s.voc_latent);
        f32t(p + ".pw2.bias", { s.voc_latent }, 0.0f, 0.02f);
        f32t(p + ".gamma", { s.voc_latent }, 0.1f, 0.01f);
    }
    conv("codec.dhead.conv", 7, s.voc_latent, s.voc_dec);
    int64_t ch = s.voc_dec;
    for (size_t i = 0; i < s.voc_rates.size(); i++) {
        const std::string p = "codec.dblk." + std::to_string(i);
        const int r = s.voc_rates[i];
        f32t(p + ".alpha", { ch }, 0.0f, 0.1f);
        f32t(p + ".beta", { ch }, 0.0f, 0.1f);
        convtr(p + ".up.conv", 2 * r, ch, ch / 2, r);
        ch /= 2;
        for (int j = 0; j < 3; j++) {
            const std::string q = p + ".res." + std::to_string(j);
            f32t(q + ".a1", { ch }, 0.0f, 0.1f);
            f32t(q + ".b1", { ch }, 0.0f, 0.1f);
            conv(q + ".conv1.conv", 7, ch, ch);
            f32t(q + ".a2", { ch }, 0.0f, 0.1f);
            f32t(q + ".b2", { ch }, 0.0f, 0.1f);
            conv(q + ".conv2.conv", 1, ch, ch);
        }
    }
    f32t("codec.dfin.alpha", { ch }, 0.0f, 0.1f);
    f32t("codec.dfin.beta", { ch }, 0.0f, 0.1f);
    conv("codec.dfin.conv", 7, ch, 1);

    // codec encoder, appended after every decoder tensor: SEANet (conv 0; per stage a residual
    // block, ELU and a strided conv doubling the channels; ELU and conv 14), the Mimi encoder
    // transformer (LayerNorm, MHA, GELU MLP, layer scales), the stride-2 downsample and the
    // semantic / acoustic quantiser projections and codebooks (F32 [dim, codebook size])
    conv("codec.enc.0.conv", 7, 1, s.enc_nf);
    {
        const int res_idx[4] = { 1, 4, 7, 10 }, conv_idx[4] = { 3, 6, 9, 12 };
        int64_t c = s.enc_nf;
        for (int st = 0; st < 4; st++) {
            const std::string rb = "codec.enc." + std::to_string(res_idx[st]);
            conv(rb + ".block.1.conv", 3, c, c / 2);
            conv(rb + ".block.3.conv", 1, c / 2, c);
            const int r = s.enc_ratios[3 - st];
            conv("codec.enc." + std::to_string(conv_idx[st]) + ".conv", 2 * r, c, 2 * c);
            c *= 2;
        }
        conv("codec.enc.14.conv", 3, c, s.enc_hidden);
    }
    for (int l = 0; l < s.enc_layers; l++) {
        const std::string p = "codec.enct.blk." + std::to_string(l);
        nrm(p + ".attn_norm.weight", s.enc_hidden);
        f32t(p + ".attn_norm.bias", { s.enc_hidden }, 0.0f, 0.02f);
        lin(p + ".attn_q.weight", s.enc_hidden, (int64_t) s.enc_heads * s.enc_hd);
        lin(p + ".attn_k.weight", s.enc_hidden, (int64_t) s.enc_heads * s.enc_hd);
        lin(p + ".attn_v.weight", s.enc_hidden, (int64_t) s.enc_heads * s.enc_hd);
        lin(p + ".attn_output.weight", (int64_t) s.enc_heads * s.enc_hd, s.enc_hidden);
        f32t(p + ".attn_scale", { s.enc_hidden }, 0.1f, 0.01f);
        nrm(p + ".ffn_norm.weight", s.enc_hidden);
        f32t(p + ".ffn_norm.bias", { s.enc_hidden }, 0.0f, 0.02f);
        lin(p + ".ffn_up.weight", s.enc_hidden, s.enc_ffn);
        lin(p + ".ffn_down.weight", s.enc_ffn, s.enc_hidden);
        f32t(p + ".ffn_scale", { s.enc_hidden }, 0.1f, 0.01f);
    }
    f32t("codec.downsample.conv.weight", { 4, s.enc_hidden, s.enc_hidden }, 0.0f, 0.7f / std::sqrt((float) (4 * s.enc_hidden)));
    lin("codec.sq.in_proj.weight", s.enc_hidden, s.enc_dim);
    f32t("codec.sq.0.embed", { s.enc_dim, s.cb_size }, 0.0f, 0.05f);
    lin("codec.aq.in_proj.weight", s.enc_hidden, s.enc_dim);
    for (int i = 0; i < s.nc - 1; i++) f32t("codec.aq." + std::to_string(i) + ".embed", { s.enc_dim, s.cb_size }, 0.0f, 0.05f);

    Writer w;
    w.kv_str("general.architecture", "breeze");
    w.kv_str("general.name", "breeze-synthetic-" + preset);
    w.kv_u32("general.alignment", 32);
    w.kv_u32("breeze.hidden_size", s.hidden);
    w.kv_u32("breeze.num_codebooks", s.nc);
    w.kv_u32("breeze.audio_vocab_size", s.vs);
    w.kv_u32("breeze.codec_codebook_size", s.cb_size);
    w.kv_u32("breeze.backbone_eos_token_id", 2051);
    w.kv_u32("breeze.codebook_pad_token_id", 2050);
    w.kv_u32("breeze.codebook_eos_token_id", 0);
    w.kv_u32("breeze.sample_rate", 24000);
    w.kv_u32("breeze.samples_per_frame", 1920);
    w.kv_u32("breeze.max_new_tokens", s.max_new_tokens);
    w.kv_f32("breeze.temperature", 0.9f);
    w.kv_u32("breeze.top_k", 50);
    w.kv_f32("breeze.top_p", 1.0f);
    w.kv_f32("breeze.repetition_penalty", 1.1f);
    w.kv_f32("breeze.depth_temperature", 0.9f);
    w.kv_u32("breeze.depth_top_k", s.depth_top_k);
    w.kv_f32("breeze.depth_top_p", 1.0f);
    w.kv_u32("breeze.te.hidden_size", s.te_hidden);
    w.kv_u32("breeze.te.block_count", s.te_layers);
    w.kv_u32("breeze.te.head_count", s.te_heads);
    w.kv_u32("breeze.te.head_count_kv", s.te_kv);
    w.kv_u32("breeze.te.head_dim", s.te_hd);
    w.kv_u32("breeze.te.feed_forward_length", s.te_ffn);
    w.kv_f32("breeze.te.rms_eps", 1e-6f);
    w.kv_f32("breeze.te.rope_theta_full", 1000000.0f);
    w.kv_f32("breeze.te.rope_freq_scale_full", 0.125f);
    w.kv_f32("breeze.te.rope_theta_sliding", 10000.0f);
    w.kv_u32("breeze.te.sliding_window", s.te_window);
    w.kv_f32("breeze.te.query_pre_attn_scalar", (float) s.te_hd);
    w.kv_f32("breeze.te.embed_scale", 1.0f);
    {
        std::vector<int32_t> full(s.te_layers);
        for (int l = 0; l < s.te_layers; l++) full[l] = (l % 6 == 5) ? 1 : 0;
        if (preset == "tiny" && s.te_layers > 1) full[1] = 1;
        w.kv_i32_arr("breeze.te.layer_is_full", full);
    }
    w.kv_u32("breeze.bb.hidden_size", s.hidden);
    w.kv_u32("breeze.bb.block_count", s.bb_layers);
    w.kv_u32("breeze.bb.head_count", s.bb_heads);
    w.kv_u32("breeze.bb.head_count_kv", s.bb_kv);
    w.kv_u32("breeze.bb.head_dim", s.bb_hd);
    w.kv_u32("breeze.bb.feed_forward_length", s.bb_ffn);
    w.kv_f32("breeze.bb.rms_eps", 1e-5f);
    w.kv_f32("breeze.bb.rope_theta", 500000.0f);
    w.kv_u32("breeze.dd.hidden_size", s.dd_hidden);
    w.kv_u32("breeze.dd.block_count", s.dd_layers);
    w.kv_u32("breeze.dd.head_count", s.dd_heads);
    w.kv_u32("breeze.dd.head_count_kv", s.dd_kv);
    w.kv_u32("breeze.dd.head_dim", s.dd_hd);
    w.kv_u32("breeze.dd.feed_forward_length", s.dd_ffn);
    w.kv_f32("breeze.dd.rms_eps", 1e-5f);
    w.kv_f32("breeze.dd.rope_theta", 500000.0f);
    w.kv_f32("breeze.dd.rope_factor", 32.0f);
    w.kv_f32("breeze.dd.rope_high_freq_factor", 0.0078125f);
    w.kv_f32("breeze.dd.rope_low_freq_factor", 0.001953125f);
    w.kv_u32("breeze.dd.rope_orig_ctx", 16);
    w.kv_u32("breeze.codec.dec.hidden_size", s.voc_hidden);
    w.kv_u32("breeze.codec.dec.block_count", s.voc_layers);
    w.kv_u32("breeze.codec.dec.head_count", s.voc_heads);
    w.kv_u32("breeze.codec.dec.head_count_kv", s.voc_kv);
    w.kv_u32("breeze.codec.dec.head_dim", s.voc_hd);
    w.kv_u32("breeze.codec.dec.feed_forward_length", s.voc_ffn);
    w.kv_f32("breeze.codec.dec.rms_eps", 1e-5f);
    w.kv_f32("breeze.codec.dec.rope_theta", 10000.0f);
    w.kv_u32("breeze.codec.dec.sliding_window", s.voc_window);
    w.kv_u32("breeze.codec.dec.latent_dim", s.voc_latent);
    w.kv_u32("breeze.codec.dec.codebook_dim", s.voc_cbdim);
    w.kv_u32("breeze.codec.dec.decoder_dim", s.voc_dec);
    w.kv_i32_arr("breeze.codec.dec.upsample_rates", s.voc_rates);
    w.kv_i32_arr("breeze.codec.dec.upsampling_ratios", s.voc_ratios);
    w.kv_u32("breeze.codec.hidden_size", s.enc_hidden);
    w.kv_u32("breeze.codec.block_count", s.enc_layers);
    w.kv_u32("breeze.codec.head_count", s.enc_heads);
    w.kv_u32("breeze.codec.head_dim", s.enc_hd);
    w.kv_u32("breeze.codec.feed_forward_length", s.enc_ffn);
    w.kv_f32("breeze.codec.rope_theta", 10000.0f);
    w.kv_u32("breeze.codec.sliding_window", s.enc_window);
    w.kv_u32("breeze.codec.num_filters", s.enc_nf);
    w.kv_u32("breeze.codec.codebook_dim", s.enc_dim);
    w.kv_u32("breeze.codec.num_semantic", 1);
    w.kv_f32("breeze.codec.layer_norm_eps", 1e-5f);
    w.kv_i32_arr("breeze.codec.upsampling_ratios", s.enc_ratios);

    // tokenizer (src/tokenizer.cpp:19-41): every id >= 264 has a unique special spelling so an
    // id list maps to text exactly; bytes are <0xNN>; [S0]/<ins_bos>/<ins_eos> are control tokens
    {
        std::vector<std::string> toks(s.vocab);
        std::vector<int32_t> types(s.vocab, 4);
        toks[0] = "<pad>"; types[0] = 3;
        toks[1] = "<eos>"; types[1] = 3;
        toks[2] = "<bos>"; types[2] = 3;
        toks[3] = "<unk>"; types[3] = 2;
        char buf[32];
        for (int b = 0; b < 256; b++) { std::snprintf(buf, sizeof buf, "<0x%02X>", b); toks[4 + b] = buf; types[4 + b] = 6; }
        toks[260] = "[S0]"; types[260] = 3;
        toks[261] = "<ins_bos>"; types[261] = 3;
        toks[262] = "<ins_eos>"; types[262] = 3;
        toks[263] = "\xE2\x96\x81"; types[263] = 1;
        for (int i = 264; i < s.vocab; i++) { std::snprintf(buf, sizeof buf, "<|t%d|>", i); toks[i] = buf; }
        w.kv_str("tokenizer.ggml.model", "llama");
        w.kv_str_arr("tokenizer.ggml.tokens", toks);
        w.kv_i32_arr("tokenizer.ggml.token_type", types);
        w.kv_str_arr("tokenizer.ggml.merges", {});
        w.kv_u32("tokenizer.ggml.bos_token_id", 2);
        w.kv_u32("tokenizer.ggml.eos_token_id", 1);
        w.kv_u32("tokenizer.ggml.padding_token_id", 0);
        w.kv_u32("tokenizer.ggml.unknown_token_id", 3);
    }

    // tensor infos
    uint64_t off = 0;
    std::vector<uint8_t> info;
    for (auto & t : ts) {
        t.nbytes = tensor_bytes(t);
        t.offset = off;
        off += (t.nbytes + 31) / 32 * 32;
    }
    Writer ti;
    for (auto & t : ts) {
        ti.str(t.name);
        ti.u32((uint32_t) t.ne.size());
        for (int64_t d : t.ne) ti.u64((uint64_t) d);
        ti.u32(t.type);
        ti.u64(t.offset);
    }

    FILE * f = std::fopen(out.c_str(), "wb");
    if (!f) { std::perror("open"); return 1; }
    const uint32_t version = 3;
    const uint64_t n_t = ts.size();
    std::fwrite("GGUF", 1, 4, f);
    std::fwrite(&version, 4, 1, f);
    std::fwrite(&n_t, 8, 1, f);
    std::fwrite(&w.n_kv, 8, 1, f);
    std::fwrite(w.meta.data(), 1, w.meta.size(), f);
    std::fwrite(ti.meta.data(), 1, ti.meta.size(), f);
    uint64_t pos = 24 + w.meta.size() + ti.meta.size();
    const uint64_t pad = (32 - pos % 32) % 32;
    const uint8_t zeros[32] = {};
    std::fwrite(zeros, 1, pad, f);
    std::vector<uint8_t> buf;
    for (size_t i = 0; i < ts.size(); i++) {
        const Tensor & t = ts[i];
        buf.assign((t.nbytes + 31) / 32 * 32, 0);
        fill_tensor(t, splitmix(s.seed * 1000003ull + i + 1), buf.data(), threads);
        std::fwrite(buf.data(), 1, buf.size(), f);
    }
    std::fclose(f);
    return 0;
}
