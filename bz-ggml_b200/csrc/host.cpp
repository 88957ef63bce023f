#include "host.h"

#include <algorithm>
#include <climits>
#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace bzb {

uint16_t f32_to_f16_bits(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u, absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) return (uint16_t) (sign | (absx > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (absx >= 0x477ff000u) return (uint16_t) (sign | 0x7c00u);
    if (absx < 0x38800000u) {
        if (absx < 0x33000000u) return (uint16_t) sign;
        const uint32_t m = (absx & 0x7fffffu) | 0x800000u;
        const int shift = 126 - (int) (absx >> 23) + 13;
        uint32_t h = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t) (sign | h);
    }
    uint32_t h = (absx >> 13) - (112u << 10);
    const uint32_t rem = absx & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t) (sign | h);
}

float f16_bits_to_f32(uint16_t h) {
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

// ------------------------------------------------------------------------------------ GGUF
namespace {
struct Cursor {
    const uint8_t * p;
    const uint8_t * end;
    bool ok = true;
    template <class T> T get() {
        T v{};
        if ((size_t) (end - p) < sizeof(T)) { ok = false; return v; }
        std::memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || (uint64_t) (end - p) < n) { ok = false; return {}; }
        std::string s((const char *) p, (size_t) n);
        p += n;
        return s;
    }
};

uint64_t type_nbytes(uint32_t type, int64_t n, bool & ok) {
    switch (type) {
        case GT_F32: return (uint64_t) n * 4;
        case GT_F16: return (uint64_t) n * 2;
        case GT_Q8_0: if (n % 32) ok = false; return (uint64_t) n / 32 * 34;
        case GT_Q4_K: if (n % 256) ok = false; return (uint64_t) n / 256 * 144;
        default: ok = false; return 0;
    }
}
}  // namespace

GgufFile::~GgufFile() {
    if (base_) munmap(base_, size_);
}

bool GgufFile::open(const std::string & path, std::string & err) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) { err = "cannot open " + path; return false; }
    struct stat st{};
    if (fstat(fd, &st) != 0 || st.st_size < 24) { ::close(fd); err = "not a GGUF file: " + path; return false; }
    size_ = (size_t) st.st_size;
    void * m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) { err = "mmap failed for " + path; return false; }
    base_ = (uint8_t *) m;
    Cursor c{ base_, base_ + size_ };
    if (std::memcmp(base_, "GGUF", 4) != 0) { err = "bad GGUF magic in " + path; return false; }
    c.p += 4;
    const uint32_t version = c.get<uint32_t>();
    if (version < 2 || version > 3) { err = "unsupported GGUF version " + std::to_string(version); return false; }
    const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
    if (n_tensors > (1u << 20) || n_kv > (1u << 20)) { err = "implausible GGUF header counts"; return false; }
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv && c.ok; i++) {
        const std::string key = c.str();
        Kv v;
        v.type = c.get<uint32_t>();
        auto scalar = [&](uint32_t t, Kv & out) {
            switch (t) {
                case 0: out.u = c.get<uint8_t>(); out.i = (int64_t) out.u; break;
                case 1: out.i = c.get<int8_t>(); out.u = (uint64_t) out.i; break;
                case 2: out.u = c.get<uint16_t>(); out.i = (int64_t) out.u; break;
                case 3: out.i = c.get<int16_t>(); out.u = (uint64_t) out.i; break;
                case 4: out.u = c.get<uint32_t>(); out.i = (int64_t) out.u; break;
                case 5: out.i = c.get<int32_t>(); out.u = (uint64_t) out.i; break;
                case 6: out.f = c.get<float>(); break;
                case 7: out.u = c.get<uint8_t>(); out.i = (int64_t) out.u; break;
                case 8: out.s = c.str(); break;
                case 10: out.u = c.get<uint64_t>(); out.i = (int64_t) out.u; break;
                case 11: out.i = c.get<int64_t>(); out.u = (uint64_t) out.i; break;
                case 12: out.f = c.get<double>(); break;
                default: c.ok = false;
            }
        };
        if (v.type == 9) {
            v.arr_type = c.get<uint32_t>();
            const uint64_t n = c.get<uint64_t>();
            if (n > size_) { c.ok = false; break; }
            for (uint64_t j = 0; j < n && c.ok; j++) {
                Kv e;
                scalar(v.arr_type, e);
                if (v.arr_type == 8) v.arr_s.push_back(std::move(e.s));
                else v.arr_i.push_back(e.i);
            }
        } else scalar(v.type, v);
        if (key == "general.alignment" && v.u > 0) alignment = v.u;
        kv_[key] = std::move(v);
    }
    if (!c.ok) { err = "truncated GGUF metadata in " + path; return false; }
    tensors.resize(n_tensors);
    for (uint64_t i = 0; i < n_tensors && c.ok; i++) {
        GgufTensor & t = tensors[i];
        t.name = c.str();
        const uint32_t nd = c.get<uint32_t>();
        if (nd == 0 || nd > 4) { c.ok = false; break; }
        t.ne.resize(nd);
        for (uint32_t d = 0; d < nd; d++) t.ne[d] = (int64_t) c.get<uint64_t>();
        t.type = c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
    }
    if (!c.ok) { err = "truncated GGUF tensor table in " + path; return false; }
    uint64_t data_off = (uint64_t) (c.p - base_);
    data_off = (data_off + alignment - 1) / alignment * alignment;
    for (size_t i = 0; i < tensors.size(); i++) {
        GgufTensor & t = tensors[i];
        bool ok = true;
        for (int64_t d : t.ne) if (d <= 0) ok = false;
        t.nbytes = ok ? type_nbytes(t.type, t.nelem(), ok) : 0;
        if (!ok) { err = "tensor " + t.name + " has an unsupported type or shape"; return false; }
        t.offset += data_off;
        if (t.offset + t.nbytes > size_) { err = "tensor " + t.name + " runs past the end of the file"; return false; }
        index_[t.name] = i;
    }
    return true;
}

const GgufTensor * GgufFile::find(const std::string & name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors[it->second];
}

int GgufFile::kv_u32(const std::string & key, int def) const {
    auto it = kv_.find(key);
    if (it == kv_.end()) return def;
    switch (it->second.type) {
        case 4: case 5: case 10: case 11: return (int) it->second.i;
        default: return def;
    }
}

float GgufFile::kv_f32(const std::string & key, float def) const {
    auto it = kv_.find(key);
    if (it == kv_.end()) return def;
    if (it->second.type == 6 || it->second.type == 12) return (float) it->second.f;
    return def;
}

std::string GgufFile::kv_str(const std::string & key, const std::string & def) const {
    auto it = kv_.find(key);
    return (it == kv_.end() || it->second.type != 8) ? def : it->second.s;
}

std::vector<int> GgufFile::kv_i32_array(const std::string & key) const {
    auto it = kv_.find(key);
    std::vector<int> out;
    if (it == kv_.end() || it->second.type != 9) return out;
    if (it->second.arr_type != 5 && it->second.arr_type != 4) return std::vector<int>(it->second.arr_i.size(), 0);
    for (int64_t v : it->second.arr_i) out.push_back((int) v);
    return out;
}

std::vector<std::string> GgufFile::kv_str_array(const std::string & key) const {
    auto it = kv_.find(key);
    if (it == kv_.end() || it->second.type != 9) return {};
    return it->second.arr_s;
}

// ------------------------------------------------------------------------------------ config
ModelConfig parse_config(const GgufFile & g) {
    ModelConfig c{};
    c.hidden = g.kv_u32("breeze.hidden_size", 2048);
    c.nc = g.kv_u32("breeze.num_codebooks", 16);
    c.vs = g.kv_u32("breeze.audio_vocab_size", 2051);
    c.cb_size = g.kv_u32("breeze.codec_codebook_size", 2048);
    c.bb_eos = g.kv_u32("breeze.backbone_eos_token_id", 2051);
    c.cb_pad = g.kv_u32("breeze.codebook_pad_token_id", 2050);
    c.cb_eos = g.kv_u32("breeze.codebook_eos_token_id", 0);
    c.sample_rate = g.kv_u32("breeze.sample_rate", 24000);
    c.samples_per_frame = g.kv_u32("breeze.samples_per_frame", 1920);
    c.max_new_tokens = g.kv_u32("breeze.max_new_tokens", 750);
    c.temperature = g.kv_f32("breeze.temperature", 0.9f);
    c.top_k = g.kv_u32("breeze.top_k", 50);
    c.top_p = g.kv_f32("breeze.top_p", 1.0f);
    c.rep = g.kv_f32("breeze.repetition_penalty", 1.1f);
    c.depth_temperature = g.kv_f32("breeze.depth_temperature", 0.9f);
    c.depth_top_k = g.kv_u32("breeze.depth_top_k", 50);
    c.depth_top_p = g.kv_f32("breeze.depth_top_p", 1.0f);
    TeConfig & te = c.te;
    te.hidden = g.kv_u32("breeze.te.hidden_size", 1152);
    te.n_layer = g.kv_u32("breeze.te.block_count", 26);
    te.n_head = g.kv_u32("breeze.te.head_count", 4);
    te.n_kv = g.kv_u32("breeze.te.head_count_kv", 1);
    te.hd = g.kv_u32("breeze.te.head_dim", 256);
    te.ffn = g.kv_u32("breeze.te.feed_forward_length", 6912);
    te.eps = g.kv_f32("breeze.te.rms_eps", 1e-6f);
    te.theta_full = g.kv_f32("breeze.te.rope_theta_full", 1000000.0f);
    te.fscale_full = g.kv_f32("breeze.te.rope_freq_scale_full", 0.125f);
    te.theta_sliding = g.kv_f32("breeze.te.rope_theta_sliding", 10000.0f);
    te.window = g.kv_u32("breeze.te.sliding_window", 512);
    te.qpas = g.kv_f32("breeze.te.query_pre_attn_scalar", 256.0f);
    te.embed_scale = g.kv_f32("breeze.te.embed_scale", 1.0f);
    te.is_full = g.kv_i32_array("breeze.te.layer_is_full");
    BbConfig & bb = c.bb;
    bb.hidden = g.kv_u32("breeze.bb.hidden_size", 2048);
    bb.n_layer = g.kv_u32("breeze.bb.block_count", 28);
    bb.n_head = g.kv_u32("breeze.bb.head_count", 16);
    bb.n_kv = g.kv_u32("breeze.bb.head_count_kv", 8);
    bb.hd = g.kv_u32("breeze.bb.head_dim", 128);
    bb.ffn = g.kv_u32("breeze.bb.feed_forward_length", 6144);
    bb.eps = g.kv_f32("breeze.bb.rms_eps", 1e-6f);
    bb.theta = g.kv_f32("breeze.bb.rope_theta", 1000000.0f);
    DdConfig & dd = c.dd;
    dd.hidden = g.kv_u32("breeze.dd.hidden_size", 1024);
    dd.n_layer = g.kv_u32("breeze.dd.block_count", 12);
    dd.n_head = g.kv_u32("breeze.dd.head_count", 8);
    dd.n_kv = g.kv_u32("breeze.dd.head_count_kv", 2);
    dd.hd = g.kv_u32("breeze.dd.head_dim", 128);
    dd.ffn = g.kv_u32("breeze.dd.feed_forward_length", 8192);
    dd.eps = g.kv_f32("breeze.dd.rms_eps", 1e-5f);
    dd.theta = g.kv_f32("breeze.dd.rope_theta", 500000.0f);
    dd.factor = g.kv_f32("breeze.dd.rope_factor", 32.0f);
    dd.high = g.kv_f32("breeze.dd.rope_high_freq_factor", 0.0078125f);
    dd.low = g.kv_f32("breeze.dd.rope_low_freq_factor", 0.001953125f);
    dd.orig_ctx = g.kv_u32("breeze.dd.rope_orig_ctx", 16);
    c.voc.hidden = g.kv_u32("breeze.codec.dec.hidden_size", 512);
    c.voc.n_layer = g.kv_u32("breeze.codec.dec.block_count", 8);
    c.voc.n_head = g.kv_u32("breeze.codec.dec.head_count", 16);
    c.voc.n_kv = g.kv_u32("breeze.codec.dec.head_count_kv", 16);
    c.voc.hd = g.kv_u32("breeze.codec.dec.head_dim", 64);
    c.voc.ffn = g.kv_u32("breeze.codec.dec.feed_forward_length", 1024);
    c.voc.eps = g.kv_f32("breeze.codec.dec.rms_eps", 1e-5f);
    c.voc.theta = g.kv_f32("breeze.codec.dec.rope_theta", 10000.0f);
    c.voc.window = g.kv_u32("breeze.codec.dec.sliding_window", 72);
    c.voc.rates = g.kv_i32_array("breeze.codec.dec.upsample_rates");
    if (c.voc.rates.empty()) c.voc.rates = { 8, 5, 4, 3 };
    c.voc.ratios = g.kv_i32_array("breeze.codec.dec.upsampling_ratios");
    if (c.voc.ratios.empty()) c.voc.ratios = { 2, 2 };
    c.enc.hidden = g.kv_u32("breeze.codec.hidden_size", 512);
    c.enc.n_layer = g.kv_u32("breeze.codec.block_count", 8);
    c.enc.n_head = g.kv_u32("breeze.codec.head_count", 8);
    c.enc.hd = g.kv_u32("breeze.codec.head_dim", 64);
    c.enc.ffn = g.kv_u32("breeze.codec.feed_forward_length", 2048);
    c.enc.theta = g.kv_f32("breeze.codec.rope_theta", 10000.0f);
    c.enc.window = g.kv_u32("breeze.codec.sliding_window", 250);
    c.enc.nf = g.kv_u32("breeze.codec.num_filters", 64);
    c.enc.dim = g.kv_u32("breeze.codec.codebook_dim", 256);
    c.enc.n_sem = g.kv_u32("breeze.codec.num_semantic", 1);
    c.enc.eps = g.kv_f32("breeze.codec.layer_norm_eps", 1e-5f);
    c.enc.ratios = g.kv_i32_array("breeze.codec.upsampling_ratios");
    if (c.enc.ratios.empty()) c.enc.ratios = { 8, 6, 5, 4 };
    return c;
}

// ------------------------------------------------------------------------------------ tokenizer
namespace {
const char * kMeta = "\xE2\x96\x81";
int utf8_len(unsigned char c) {
    if (c < 0x80) return 1;
    if ((c >> 5) == 0x6) return 2;
    if ((c >> 4) == 0xE) return 3;
    if ((c >> 3) == 0x1E) return 4;
    return 1;
}
}  // namespace

bool Tokenizer::load(const GgufFile & g) {
    id_to_token_ = g.kv_str_array("tokenizer.ggml.tokens");
    if (id_to_token_.empty()) return false;
    const std::vector<int> types = g.kv_i32_array("tokenizer.ggml.token_type");
    std::unordered_set<size_t> lens;
    for (int i = 0; i < (int) id_to_token_.size(); i++) {
        const std::string & t = id_to_token_[i];
        token_to_id_[t] = i;
        if (t.size() == 6 && t[0] == '<' && t[1] == '0' && t[2] == 'x' && t[5] == '>')
            byte_to_id_[(int) std::strtol(t.substr(3, 2).c_str(), nullptr, 16)] = i;
        if (i < (int) types.size() && (types[i] == 3 || types[i] == 4) && !t.empty()) {
            specials_[t] = i;
            lens.insert(t.size());
        }
    }
    special_lens_.assign(lens.begin(), lens.end());
    std::sort(special_lens_.begin(), special_lens_.end(), std::greater<size_t>());
    const std::vector<std::string> merges = g.kv_str_array("tokenizer.ggml.merges");
    for (int i = 0; i < (int) merges.size(); i++) merge_rank_[merges[i]] = i;
    bos_ = g.kv_u32("tokenizer.ggml.bos_token_id", 2);
    unk_ = g.kv_u32("tokenizer.ggml.unknown_token_id", 3);
    return true;
}

void Tokenizer::bpe(const std::string & word, std::vector<int> & out) const {
    std::vector<std::string> syms;
    for (size_t i = 0; i < word.size();) {
        const int l = utf8_len((unsigned char) word[i]);
        const std::string ch = word.substr(i, l);
        i += l;
        if (token_to_id_.count(ch)) syms.push_back(ch);
        else {
            for (char b : ch) {
                auto it = byte_to_id_.find((unsigned char) b);
                syms.push_back(it != byte_to_id_.end() ? id_to_token_[it->second] : std::string(1, b));
            }
        }
    }
    while (syms.size() > 1) {
        int best = INT_MAX, best_i = -1;
        for (size_t i = 0; i + 1 < syms.size(); i++) {
            auto it = merge_rank_.find(syms[i] + " " + syms[i + 1]);
            if (it != merge_rank_.end() && it->second < best) { best = it->second; best_i = (int) i; }
        }
        if (best_i < 0) break;
        syms[best_i] += syms[best_i + 1];
        syms.erase(syms.begin() + best_i + 1);
    }
    for (const std::string & s : syms) {
        auto it = token_to_id_.find(s);
        if (it != token_to_id_.end()) out.push_back(it->second);
        else {
            for (char b : s) {
                auto bit = byte_to_id_.find((unsigned char) b);
                out.push_back(bit != byte_to_id_.end() ? bit->second : unk_);
            }
        }
    }
}

std::vector<int> Tokenizer::encode(const std::string & text, bool add_bos) const {
    std::vector<int> out;
    if (add_bos) out.push_back(bos_);
    std::string normal;
    auto flush = [&]() {
        if (normal.empty()) return;
        std::string norm;
        for (char ch : normal) {
            if (ch == ' ') norm += kMeta;
            else norm += ch;
        }
        bpe(norm, out);
        normal.clear();
    };
    for (size_t i = 0; i < text.size();) {
        bool matched = false;
        for (size_t L : special_lens_) {
            if (i + L > text.size()) continue;
            auto it = specials_.find(text.substr(i, L));
            if (it != specials_.end()) {
                flush();
                out.push_back(it->second);
                i += L;
                matched = true;
                break;
            }
        }
        if (!matched) normal += text[i++];
    }
    flush();
    return out;
}

}  // namespace bzb
