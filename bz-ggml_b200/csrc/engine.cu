// Generator engine: loading, the GPU-resident frame step and session prefill.
//
// One frame step (reference: src/c_api.cpp:764-949 with src/depth_decoder.cpp:249-365 and
// src/backbone.cpp:98-179) is captured once per batch bucket as a CUDA graph:
//   step_init -> depth sub-step 1 (2 tokens/session) -> depth sub-steps 2..nc-1 (argmax and
//   next-codebook embedding gather on the GPU) -> audio embedding sum -> backbone decode over
//   the paged KV cache -> Philox top-k sampler with repetition penalty -> frame commit.
// Session state (positions, sampler streams, penalty histories, last hidden) never leaves the
// device between steps; the host only uploads the row->slot table and seeds.
#include "engine.h"

#include <climits>
#include "rope.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>

namespace bzb {

#define CK(x)                                                                                   \
    do {                                                                                        \
        cudaError_t e_ = (x);                                                                   \
        if (e_ != cudaSuccess) throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(e_) + " (" #x ")"); \
    } while (0)

namespace {
int round_up(int x, int m) { return (x + m - 1) / m * m; }
// stored bytes of a quantised matrix: Q8_0 34 per 32 weights, Q4_K 144 per 256
size_t qmat_bytes(const QMat & q) { return q.u.q4 ? (size_t) q.M * q.K / 256 * 144 : (size_t) q.M * q.K / 32 * 34; }

std::vector<float> llama3_freq_factors(const DdConfig & c) {
    // src/depth_decoder.cpp:10-29
    const int half = c.hd / 2;
    std::vector<float> ff(half, 1.0f);
    const float pi = 3.14159265358979323846f;
    const float low_wl = (float) c.orig_ctx / c.low;
    const float high_wl = (float) c.orig_ctx / c.high;
    for (int i = 0; i < half; i++) {
        const float freq = std::pow(c.theta, -2.0f * (float) i / (float) c.hd);
        const float wavelen = 2.0f * pi / freq;
        if (wavelen > low_wl) ff[i] = c.factor;
        else if (wavelen < high_wl) ff[i] = 1.0f;
        else {
            const float smooth = ((float) c.orig_ctx / wavelen - c.low) / (c.high - c.low);
            ff[i] = 1.0f / ((1.0f - smooth) / c.factor + smooth);
        }
    }
    return ff;
}

std::string shape_str(const GgufTensor & t) {
    std::string s = "[";
    for (size_t i = 0; i < 3; i++) {
        if (i) s += ", ";
        s += i < t.ne.size() ? std::to_string(t.ne[i]) : std::string("1");
    }
    return s + "]";
}

void check_shape(const GgufTensor & t, int64_t n0, int64_t n1, int64_t n2 = -1) {
    // src/depth_decoder.cpp:31-38: a file built for another codebook or vocab count fails here
    const int64_t e0 = t.ne.size() > 0 ? t.ne[0] : 1, e1 = t.ne.size() > 1 ? t.ne[1] : 1, e2 = t.ne.size() > 2 ? t.ne[2] : 1;
    if (e0 == n0 && e1 == n1 && (n2 < 0 || e2 == n2)) return;
    throw std::runtime_error(t.name + " is " + shape_str(t) + ", expected [" + std::to_string(n0) + ", " +
                             std::to_string(n1) + ", " + (n2 < 0 ? std::string("any") : std::to_string(n2)) + "]");
}
}  // namespace

template <class T> T * Engine::dalloc(size_t n) {
    void * p = nullptr;
    CK(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
    allocs_.push_back(p);
    return (T *) p;
}

const GgufTensor * Engine::need(const std::string & name) {
    const GgufTensor * t = src().find(name);
    if (!t) throw std::runtime_error("missing tensor: " + name);
    return t;
}

QMat Engine::load_qmat(const std::vector<const GgufTensor *> & parts, bool interleave_pairs, int row0, int rows) {
    const int K = (int) parts[0]->ne[0];
    const bool q4 = parts[0]->type == GT_Q4_K;
    for (auto * t : parts) {
        if (t->type != GT_Q8_0 && t->type != GT_Q4_K)
            throw std::runtime_error(t->name + ": linear weights must be Q8_0 or Q4_K");
        if (t->type != parts[0]->type) throw std::runtime_error(t->name + ": quantisation differs from its fused partner");
        if (t->ne[0] != K) throw std::runtime_error(t->name + ": row length differs from its fused partner");
    }
    if (q4 && K % 256) throw std::runtime_error(parts[0]->name + ": Q4_K rows need a length that is a multiple of 256");
    const int KB = K / 32;
    const size_t row_bytes = q4 ? (size_t) (K / 256) * 144 : (size_t) KB * 34;
    std::vector<const uint8_t *> src_rows;
    if (interleave_pairs) {
        const int F = (int) parts[0]->rows();
        if (parts.size() != 2 || parts[1]->rows() != F || F % 8) throw std::runtime_error("gate/up pair shapes differ");
        src_rows.resize((size_t) 2 * F);
        for (int p = 0; p < 2 * F; p++) {
            const int tile = p / 16, r = p % 16;
            const GgufTensor * t = r < 8 ? parts[0] : parts[1];
            const int srow = tile * 8 + (r & 7);
            src_rows[p] = src().data(*t) + (size_t) srow * row_bytes;
        }
    } else if (rows >= 0) {
        for (int r = 0; r < rows; r++) src_rows.push_back(src().data(*parts[0]) + (size_t) (row0 + r) * row_bytes);
    } else {
        for (auto * t : parts)
            for (int64_t r = 0; r < t->rows(); r++) src_rows.push_back(src().data(*t) + (size_t) r * row_bytes);
    }
    const int M = (int) src_rows.size();
    std::vector<uint8_t> raw((size_t) M * row_bytes);
    for (int r = 0; r < M; r++) std::memcpy(raw.data() + (size_t) r * row_bytes, src_rows[r], row_bytes);
    uint8_t * raw_dev = nullptr;
    CK(cudaMalloc(&raw_dev, raw.size()));
    CK(cudaMemcpyAsync(raw_dev, raw.data(), raw.size(), cudaMemcpyHostToDevice, stream_));
    QMat q;
    q.M = M;
    q.MT = (M + 15) / 16;
    q.K = K;
    q.KB = KB;
    if (!q4) {
        // the mma.sync layout serves Q8_0 only; Q4_K matrices run on the tcgen05 path alone
        uint4 * qs = dalloc<uint4>((size_t) q.MT * KB * 32);
        half2 * ds = dalloc<half2>((size_t) q.MT * KB * 8);
        repack_q8(raw_dev, M, K, qs, ds, stream_);
        q.qs = qs;
        q.ds = ds;
    }
    if (K % 64 == 0) {
        // the tcgen05 layout pairs gate/up rows in 16-row groups instead of 8
        if (interleave_pairs) {
            const int F = M / 2;
            for (int p = 0; p < M; p++) {
                const int grp = p / 32, r = p % 32;
                const GgufTensor * t = r < 16 ? parts[0] : parts[1];
                std::memcpy(raw.data() + (size_t) p * row_bytes, src().data(*t) + (size_t) (grp * 16 + (r & 15)) * row_bytes, row_bytes);
            }
            if (F % 16) throw std::runtime_error("gate/up rows must be a multiple of 16");
            CK(cudaStreamSynchronize(stream_));
            CK(cudaMemcpyAsync(raw_dev, raw.data(), raw.size(), cudaMemcpyHostToDevice, stream_));
        }
        UMat u;
        u.M = M;
        u.MT = (M + 127) / 128;
        u.K = K;
        u.KC = K / 64;
        u.q4 = q4 ? 1 : 0;
        uint8_t * ub = dalloc<uint8_t>((size_t) u.MT * u.KC * umat_chunk_bytes(u.q4));
        if (q4) repack_umma_q4k(raw_dev, M, K, ub, stream_);
        else repack_umma(raw_dev, M, K, ub, stream_);
        u.blk = ub;
        q.u = u;
    }
    CK(cudaStreamSynchronize(stream_));
    CK(cudaFree(raw_dev));
    return q;
}

QRows Engine::load_qrows(const GgufTensor * t) {
    if (t->type != GT_Q8_0 && t->type != GT_Q4_K) throw std::runtime_error(t->name + ": embedding tables must be Q8_0 or Q4_K");
    QRows e;
    e.K = (int) t->ne[0];
    e.rows = (int) t->rows();
    uint8_t * raw_dev = nullptr;
    CK(cudaMalloc(&raw_dev, t->nbytes));
    CK(cudaMemcpyAsync(raw_dev, src().data(*t), t->nbytes, cudaMemcpyHostToDevice, stream_));
    int8_t * qs = dalloc<int8_t>((size_t) e.rows * e.K);
    half * ds = dalloc<half>((size_t) e.rows * (e.K / 32));
    if (t->type == GT_Q4_K) {
        half * ms = dalloc<half>((size_t) e.rows * (e.K / 32));
        split_q4k_rows(raw_dev, e.rows, e.K, qs, ds, ms, stream_);
        e.ms = ms;
    } else {
        split_q8_rows(raw_dev, e.rows, e.K, qs, ds, stream_);
    }
    CK(cudaStreamSynchronize(stream_));
    CK(cudaFree(raw_dev));
    e.qs = qs;
    e.ds = ds;
    return e;
}

float * Engine::load_f32(const std::string & name, int expect) {
    const GgufTensor * t = need(name);
    if (t->type != GT_F32 || t->nelem() != expect)
        throw std::runtime_error(name + ": expected an F32 vector of " + std::to_string(expect));
    float * d = dalloc<float>(expect);
    CK(cudaMemcpyAsync(d, src().data(*t), (size_t) expect * 4, cudaMemcpyHostToDevice, stream_));
    return d;
}

Engine::Engine(const std::string & path, int dev) : device(dev) {
    CK(cudaSetDevice(device));
    CK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    init_kernel_attributes();
    init_umma_attributes();
    init_depth_persist_attributes();
    {
        const char * e = std::getenv("BZB_GEMM");
        use_umma_ = !(e && std::string(e) == "mma");
        const char * d = std::getenv("BZB_DEPTH_PERSIST");
        use_dp_ = use_umma_ && !(d && d[0] == '0');
    }
    std::string err;
    if (!gg_.open(path, err)) throw std::runtime_error(err);
    cfg = parse_config(gg_);
    if (!tok_.load(gg_)) throw std::runtime_error("GGUF has no tokenizer.ggml.tokens");
    const int H = cfg.hidden, nc = cfg.nc, vs = cfg.vs;
    if (nc < 2 || nc > 64) throw std::runtime_error("num_codebooks must be in [2, 64]");
    check_shape(*need("dd.in_proj.weight"), H, cfg.dd.hidden);
    check_shape(*need("audio_embd.weight"), H, (int64_t) nc * vs);
    check_shape(*need("dd.codebooks_head.weight"), cfg.dd.hidden, vs, nc - 1);

    // backbone
    const BbConfig & bb = cfg.bb;
    for (int l = 0; l < bb.n_layer; l++) {
        const std::string p = "bb.blk." + std::to_string(l);
        LayerW w;
        w.qkv = load_qmat({ need(p + ".attn_q.weight"), need(p + ".attn_k.weight"), need(p + ".attn_v.weight") }, false);
        w.o = load_qmat({ need(p + ".attn_output.weight") }, false);
        w.gu = load_qmat({ need(p + ".ffn_gate.weight"), need(p + ".ffn_up.weight") }, true);
        w.down = load_qmat({ need(p + ".ffn_down.weight") }, false);
        w.attn_norm = load_f32(p + ".attn_norm.weight", H);
        w.ffn_norm = load_f32(p + ".ffn_norm.weight", H);
        w.q_norm = load_f32(p + ".attn_q_norm.weight", bb.hd);
        w.k_norm = load_f32(p + ".attn_k_norm.weight", bb.hd);
        if (w.qkv.M != (bb.n_head + 2 * bb.n_kv) * bb.hd || w.qkv.K != H) throw std::runtime_error(p + ": attention shapes do not match the config");
        bb_.push_back(w);
    }
    bb_out_norm_ = load_f32("bb.output_norm.weight", H);
    lm_head_ = load_qmat({ need("bb.lm_head.weight") }, false);
    vbb_ = lm_head_.M;
    if (vbb_ > 4096) throw std::runtime_error("lm_head wider than the sampler's 4096 entries");

    load_depth_weights();
    audio_embd_ = load_qrows(need("audio_embd.weight"));

    // text encoder (prefill)
    has_te_ = gg_.find("te.token_embd.weight") != nullptr;
    if (has_te_) {
        const TeConfig & te = cfg.te;
        for (int l = 0; l < te.n_layer; l++) {
            const std::string p = "te.blk." + std::to_string(l);
            LayerW w;
            w.qkv = load_qmat({ need(p + ".attn_q.weight"), need(p + ".attn_k.weight"), need(p + ".attn_v.weight") }, false);
            w.o = load_qmat({ need(p + ".attn_output.weight") }, false);
            w.gu = load_qmat({ need(p + ".ffn_gate.weight"), need(p + ".ffn_up.weight") }, true);
            w.down = load_qmat({ need(p + ".ffn_down.weight") }, false);
            w.attn_norm = load_f32(p + ".attn_norm.weight", te.hidden);
            w.ffn_norm = load_f32(p + ".ffn_norm.weight", te.hidden);
            w.q_norm = load_f32(p + ".attn_q_norm.weight", te.hd);
            w.k_norm = load_f32(p + ".attn_k_norm.weight", te.hd);
            w.post_attn = load_f32(p + ".post_attn_norm.weight", te.hidden);
            w.post_ffn = load_f32(p + ".post_ffn_norm.weight", te.hidden);
            te_.push_back(w);
        }
        te_out_norm_ = load_f32("te.output_norm.weight", te.hidden);
        te_proj_ = load_qmat({ need("te.proj.weight") }, false);
        te_embd_ = load_qrows(need("te.token_embd.weight"));
    }
    build_rope_tables();
    alloc_buffers();
    CK(cudaStreamSynchronize(stream_));
}

// the dd.* tensors of the current source file into the current depth set (the reference's
// depth decoder weights, src/depth_decoder.cpp:48-85, 119-125)
void Engine::load_depth_weights() {
    const DdConfig & dd = cfg.dd;
    const int H = cfg.hidden, nc = cfg.nc, vs = cfg.vs;
    check_shape(*need("dd.in_proj.weight"), H, dd.hidden);
    check_shape(*need("dd.codebooks_head.weight"), dd.hidden, vs, nc - 1);
    dd_.clear();
    dd_head_.clear();
    dd_in_ = load_qmat({ need("dd.in_proj.weight") }, false);
    for (int l = 0; l < dd.n_layer; l++) {
        const std::string p = "dd.blk." + std::to_string(l);
        LayerW w;
        w.qkv = load_qmat({ need(p + ".attn_q.weight"), need(p + ".attn_k.weight"), need(p + ".attn_v.weight") }, false);
        w.o = load_qmat({ need(p + ".attn_output.weight") }, false);
        w.gu = load_qmat({ need(p + ".ffn_gate.weight"), need(p + ".ffn_up.weight") }, true);
        w.down = load_qmat({ need(p + ".ffn_down.weight") }, false);
        w.attn_norm = load_f32(p + ".attn_norm.weight", dd.hidden);
        w.ffn_norm = load_f32(p + ".ffn_norm.weight", dd.hidden);
        if (w.qkv.M != (dd.n_head + 2 * dd.n_kv) * dd.hd || w.qkv.K != dd.hidden || w.gu.M != 2 * dd.ffn)
            throw std::runtime_error(p + ": depth shapes do not match the model's config");
        dd_.push_back(w);
    }
    dd_out_norm_ = load_f32("dd.output_norm.weight", dd.hidden);
    const GgufTensor * head = need("dd.codebooks_head.weight");
    for (int j = 0; j < nc - 1; j++) dd_head_.push_back(load_qmat({ head }, false, j * vs, vs));
}

void Engine::swap_depth_sets() {
    std::swap(dd_, q4_dd_);
    std::swap(dd_in_, q4_dd_in_);
    std::swap(dd_head_, q4_dd_head_);
    std::swap(dd_out_norm_, q4_dd_out_norm_);
    cur_set_ ^= 1;
}

void Engine::load_q4_depth(const std::string & path) {
    auto file = std::make_unique<GgufFile>();
    std::string err;
    if (!file->open(path, err)) throw std::runtime_error(err);
    CK(cudaStreamSynchronize(stream_));
    // the previous override, its graphs and its depth schedules go first
    for (auto it = graphs_.begin(); it != graphs_.end();) {
        if (it->first.second & kFlagQ4) {
            cudaGraphExecDestroy(it->second);
            cudaGraphDestroy(graph_defs_[it->first]);
            graph_defs_.erase(it->first);
            it = graphs_.erase(it);
        } else {
            ++it;
        }
    }
    for (auto it = dp_plans_.begin(); it != dp_plans_.end();) {
        if (it->first >> 16) {
            cudaFree(it->second.dev);
            it = dp_plans_.erase(it);
        } else {
            ++it;
        }
    }
    for (void * p : q4_allocs_) cudaFree(p);
    q4_allocs_.clear();
    has_q4_ = false;
    const size_t mark = allocs_.size();
    src_ = file.get();
    swap_depth_sets();
    try {
        load_depth_weights();
    } catch (...) {
        swap_depth_sets();
        src_ = nullptr;
        q4_allocs_.assign(allocs_.begin() + mark, allocs_.end());
        allocs_.resize(mark);
        throw;
    }
    swap_depth_sets();
    src_ = nullptr;
    CK(cudaStreamSynchronize(stream_));
    q4_allocs_.assign(allocs_.begin() + mark, allocs_.end());
    allocs_.resize(mark);
    q4_gg_ = std::move(file);
    has_q4_ = true;
}

bool Engine::session_set_q4(int sid, bool on) {
    auto it = sid_to_slot_.find(sid);
    if (it == sid_to_slot_.end()) return false;
    SlotHost & s = slots_[it->second];
    s.use_q4 = on && has_q4_;  // src/c_api.cpp:576: the flag resolves to off without a loaded override
    if (s.partner >= 0) slots_[s.partner].use_q4 = s.use_q4;
    return true;
}

Engine::~Engine() {
    cudaSetDevice(device);
    if (stream_) cudaStreamSynchronize(stream_);
    for (auto & kv : graphs_) cudaGraphExecDestroy(kv.second);
    for (auto & kv : graph_defs_) cudaGraphDestroy(kv.second);
    for (void * p : prefill_allocs_) cudaFree(p);
    for (void * p : q4_allocs_) cudaFree(p);
    for (auto & kv : dp_plans_) cudaFree(kv.second.dev);
    for (void * p : allocs_) cudaFree(p);
    if (stream_) cudaStreamDestroy(stream_);
}

void Engine::build_rope_tables() {
    const int max_ctx = 4096;
    rope_bb_max_ = max_ctx + 16;
    auto up = [&](const std::vector<float2> & v) {
        float2 * d = dalloc<float2>(v.size());
        CK(cudaMemcpyAsync(d, v.data(), v.size() * sizeof(float2), cudaMemcpyHostToDevice, stream_));
        CK(cudaStreamSynchronize(stream_));
        return d;
    };
    rope_bb_ = up(rope_table(rope_bb_max_, cfg.bb.hd, cfg.bb.theta, 1.0f, nullptr));
    const std::vector<float> ff = llama3_freq_factors(cfg.dd);
    rope_dd_ = up(rope_table(cfg.nc + 2, cfg.dd.hd, cfg.dd.theta, 1.0f, &ff));
    if (has_te_) {
        rope_te_max_ = max_ctx;
        rope_te_full_ = up(rope_table(rope_te_max_, cfg.te.hd, cfg.te.theta_full, cfg.te.fscale_full, nullptr));
        rope_te_slide_ = up(rope_table(rope_te_max_, cfg.te.hd, cfg.te.theta_sliding, 1.0f, nullptr));
    }
}

void Engine::alloc_buffers() {
    const char * env_r = std::getenv("BZB_MAX_BATCH");
    rmax_ = env_r ? std::max(8, round_up(std::atoi(env_r), 8)) : 256;
    kmax_ = 64;
    max_slots_ = 1024;
    max_pages_ = 256;  // 4096 positions per session
    const BbConfig & bb = cfg.bb;
    const DdConfig & dd = cfg.dd;
    const int H = cfg.hidden, nc = cfg.nc;
    const size_t page_elems = (size_t) bb.n_layer * 2 * bb.n_kv * 16 * bb.hd;
    size_t free_b = 0, total_b = 0;
    CK(cudaMemGetInfo(&free_b, &total_b));
    size_t pool_bytes = (size_t) 8 << 30;
    if (const char * e = std::getenv("BZB_KV_POOL_MB")) pool_bytes = (size_t) std::atoll(e) << 20;
    pool_bytes = std::min(pool_bytes, free_b / 2);
    n_pages_ = (int) std::max<size_t>(16, pool_bytes / (page_elems * sizeof(half)));
    kv_pool_ = dalloc<half>((size_t) n_pages_ * page_elems);
    free_pages_.clear();
    for (int p = n_pages_ - 1; p >= 0; p--) free_pages_.push_back(p);
    page_table_ = dalloc<int>((size_t) max_slots_ * max_pages_);
    CK(cudaMemsetAsync(page_table_, 0, (size_t) max_slots_ * max_pages_ * sizeof(int), stream_));
    st_ = dalloc<SessState>(max_slots_);
    CK(cudaMemsetAsync(st_, 0, (size_t) max_slots_ * sizeof(SessState), stream_));
    hist_ld_ = round_up(vbb_, 8);
    hist_ = dalloc<uint16_t>((size_t) max_slots_ * hist_ld_);
    hid32_ = dalloc<float>((size_t) max_slots_ * H);
    slots_.assign(max_slots_, SlotHost());
    free_slots_.clear();
    for (int s = max_slots_ - 1; s >= 0; s--) free_slots_.push_back(s);

    const int R2 = 2 * rmax_;
    const int ddq = dd.n_head * dd.hd, ddkv = dd.n_kv * dd.hd;
    row_slot_ = dalloc<int>(rmax_);
    row_active_ = dalloc<int>(rmax_);
    next_ = dalloc<int>(rmax_);
    seeds_ = dalloc<uint32_t>(rmax_);
    dseeds_ = dalloc<uint32_t>(rmax_);
    row_pair_ = dalloc<int>(rmax_);
    row_set_ = dalloc<int>(rmax_);
    force_all_ = dalloc<int>((size_t) kmax_ * rmax_ * nc);
    feed_all_ = dalloc<int>((size_t) kmax_ * rmax_ * nc);
    cur_force_ = dalloc<int>((size_t) rmax_ * nc);
    cur_feed_ = dalloc<int>((size_t) rmax_ * nc);
    create_rows_ = dalloc<int>(4);
    pslot_ = dalloc<int>(kPackSegs);
    ppair_ = dalloc<int>(kPackSegs);
    pnext_ = dalloc<int>(kPackSegs);
    plast_ = dalloc<float>((size_t) kPackSegs * H);
    plogs_ = dalloc<float>((size_t) kPackSegs * vbb_);
    cur_frames_ = dalloc<int>((size_t) rmax_ * nc);
    frames_all_ = dalloc<int>((size_t) kmax_ * rmax_ * nc);
    step_ctr_ = dalloc<int>(1);
    any_active_ = dalloc<int>(kmax_);
    slot_scalar_ = dalloc<int>(1);
    err_ = dalloc<int>(1);
    CK(cudaMemsetAsync(err_, 0, sizeof(int), stream_));
    din16_ = dalloc<half>((size_t) R2 * H);
    dx_ = dalloc<float>((size_t) R2 * dd.hidden);
    dh16_ = dalloc<half>((size_t) R2 * dd.hidden);
    dff16_ = dalloc<half>((size_t) R2 * dd.ffn);
    dqkv_ = dalloc<float>((size_t) R2 * (ddq + 2 * ddkv));
    datt16_ = dalloc<half>((size_t) R2 * ddq);
    dkv_ = dalloc<float>((size_t) dd.n_layer * rmax_ * nc * 2 * ddkv);
    dlog_ = dalloc<float>((size_t) rmax_ * cfg.vs);
    const int bbq = bb.n_head * bb.hd, bbkv = bb.n_kv * bb.hd;
    bx_ = dalloc<float>((size_t) rmax_ * H);
    bh16_ = dalloc<half>((size_t) rmax_ * H);
    bff16_ = dalloc<half>((size_t) rmax_ * bb.ffn);
    bqkv_ = dalloc<float>((size_t) rmax_ * (bbq + 2 * bbkv));
    batt16_ = dalloc<half>((size_t) rmax_ * bbq);
    battn_part_ = dalloc<float>((size_t) rmax_ * bb.n_kv * kAttnMaxSplits * 8 * (bb.hd + 2));
    battn_ctr_ = dalloc<int>((size_t) rmax_ * bb.n_kv);
    CK(cudaMemsetAsync(battn_ctr_, 0, (size_t) rmax_ * bb.n_kv * sizeof(int), stream_));
    blog_ = dalloc<float>((size_t) rmax_ * vbb_);
    scr_.ws_elems = (size_t) 16 << 20;
    scr_.ws = dalloc<float4>(scr_.ws_elems);
    scr_.n_counters = 1 << 16;
    scr_.counters = dalloc<int>(scr_.n_counters);
    CK(cudaMemsetAsync(scr_.counters, 0, (size_t) scr_.n_counters * sizeof(int), stream_));
    // persistent depth decoder: split-K partials for up to 16 splits of the widest depth
    // matrix at 2 x 64 rows (or of the head at 64 rows), row norm sums, phase counter
    dp_grid_ = depth_persist_grid();
    dp_P_floats_ = std::max((size_t) 16 * 128 * std::max(dd.hidden, ddq + 2 * ddkv), (size_t) 16 * 64 * round_up(cfg.vs, 4));
    dp_P_ = dalloc<float>(dp_P_floats_);
    dp_P2_ = dalloc<float>((size_t) rmax_ * (ddq + 2 * ddkv));
    dp_ss_ = dalloc<float>((size_t) 256 * std::max(1, dd.hidden / 64));
    CK(cudaMemsetAsync(dp_ss_, 0, (size_t) 256 * std::max(1, dd.hidden / 64) * sizeof(float), stream_));
    dp_bar_ = dalloc<unsigned>(1);
    CK(cudaMemsetAsync(din16_, 0, (size_t) R2 * H * sizeof(half), stream_));
    CK(cudaMemsetAsync(dkv_, 0, (size_t) dd.n_layer * rmax_ * nc * 2 * ddkv * sizeof(float), stream_));
}

void Engine::ensure_prefill_capacity(int T) {
    if (T <= tmax_) return;
    CK(cudaStreamSynchronize(stream_));
    for (void * p : prefill_allocs_) cudaFree(p);
    prefill_allocs_.clear();
    tmax_ = round_up(std::max(T, 256), 256);
    auto pa = [&](size_t bytes) { void * p = nullptr; CK(cudaMalloc(&p, std::max<size_t>(bytes, 16))); prefill_allocs_.push_back(p); return p; };
    const int H = cfg.hidden;
    const BbConfig & bb = cfg.bb;
    const int bbq = bb.n_head * bb.hd, bbkv = bb.n_kv * bb.hd;
    px_ = (float *) pa((size_t) tmax_ * H * 4);
    ph16_ = (half *) pa((size_t) tmax_ * H * 2);
    pff16_ = (half *) pa((size_t) tmax_ * bb.ffn * 2);
    pqkv_ = (float *) pa((size_t) tmax_ * (bbq + 2 * bbkv) * 4);
    patt16_ = (half *) pa((size_t) tmax_ * bbq * 2);
    plog_ = (float *) pa((size_t) 2 * vbb_ * 4);   // conditional and unconditional branch
    ptok_ = (int *) pa((size_t) tmax_ * 4);
    pframes_ = (int *) pa((size_t) tmax_ * cfg.nc * 4);
    pseg_ = (int *) pa((size_t) tmax_ * 4);
    pidx_ = (int *) pa((size_t) tmax_ * 4);
    psegs_ = (int4 *) pa((size_t) tmax_ * sizeof(int4));
    pqb_ = (int2 *) pa((size_t) (tmax_ + tmax_ / kPrefillQBlock + 1) * sizeof(int2));
    pstage_ = (float *) pa((size_t) tmax_ * H * 4);
    if (has_te_) {
        const TeConfig & te = cfg.te;
        const int teq = te.n_head * te.hd, tekv = te.n_kv * te.hd;
        tx_ = (float *) pa((size_t) tmax_ * te.hidden * 4);
        th16_ = (half *) pa((size_t) tmax_ * te.hidden * 2);
        tff16_ = (half *) pa((size_t) tmax_ * te.ffn * 2);
        tqkv_ = (float *) pa((size_t) tmax_ * (teq + 2 * tekv) * 4);
        tatt16_ = (half *) pa((size_t) tmax_ * teq * 2);
        ttmp_ = (float *) pa((size_t) tmax_ * te.hidden * 4);
        tk_ = (half *) pa((size_t) tmax_ * tekv * 2);
        tv_ = (half *) pa((size_t) tmax_ * tekv * 2);
    }
}

// ------------------------------------------------------------------------------------ step
void Engine::launch_gemm(const QMat & w, const half * x16, int ldx, int rows, const GemvOut & out) {
    if (w.u.blk && (use_umma_ || !w.qs) && ldx % 8 == 0) launch_umma_gemm(w.u, x16, ldx, rows, out, err_, stream_, pdl_scope());
    else if (w.qs) launch_gemv(w, x16, ldx, rows, out, scr_, stream_);
    else throw std::runtime_error("Q4_K matrices need activation rows with a stride that is a multiple of 8");
}

void Engine::gemv(const QMat & w, const half * x16, int ldx, int rows, const GemvOut & out) {
    launches_++;
    if (!prof_) {
        launch_gemm(w, x16, ldx, rows, out);
        return;
    }
    ProfRec r;
    CK(cudaEventCreate(&r.a));
    CK(cudaEventCreate(&r.b));
    const double out_bytes = (double) rows * (out.kind == EPI_STORE || out.kind == EPI_RESID ? w.M * 4.0 : w.M);
    r.bytes = (double) qmat_bytes(w) + (double) rows * w.K * 2.0 + out_bytes;
    CK(cudaEventRecord(r.a, stream_));
    launch_gemm(w, x16, ldx, rows, out);
    CK(cudaEventRecord(r.b, stream_));
    prof_->push_back(r);
}

void Engine::depth_layer(int l, int rows, int R, int n_new, int start) {
    const DdConfig & dd = cfg.dd;
    const LayerW & w = dd_[l];
    const int D = dd.hidden, q = dd.n_head * dd.hd, kv = dd.n_kv * dd.hd, qkvd = q + 2 * kv;
    launch_rmsnorm(dx_, D, w.attn_norm, D, dd.eps, dh16_, D, nullptr, 0, 0, rows, nullptr, stream_);
    gemv(w.qkv, dh16_, D, rows, GemvOut{ EPI_STORE, dqkv_, nullptr, qkvd });
    AttnDecodeArgs a;
    a.qkv = dqkv_; a.ldq = qkvd; a.n_head = dd.n_head; a.n_kv = dd.n_kv; a.hd = dd.hd;
    a.R = R; a.n_new = n_new; a.row_slot = row_slot_; a.row_active = row_active_; a.st = nullptr; a.start = start;
    a.eps = dd.eps; a.rope = rope_dd_; a.scale = 1.0f / std::sqrt((float) dd.hd);
    a.kv.flat = dkv_ + (size_t) l * rmax_ * cfg.nc * 2 * kv;
    a.kv.cap = cfg.nc;
    a.out = datt16_; a.ldo = q;
    launch_attn_decode(a, false, stream_);
    gemv(w.o, datt16_, q, rows, GemvOut{ EPI_RESID, dx_, nullptr, D });
    launch_rmsnorm(dx_, D, w.ffn_norm, D, dd.eps, dh16_, D, nullptr, 0, 0, rows, nullptr, stream_);
    gemv(w.gu, dh16_, D, rows, GemvOut{ EPI_SWIGLU, nullptr, dff16_, dd.ffn });
    gemv(w.down, dff16_, dd.ffn, rows, GemvOut{ EPI_RESID, dx_, nullptr, D });
}

void Engine::bb_decode_layer(int l, int R) {
    const BbConfig & bb = cfg.bb;
    const LayerW & w = bb_[l];
    const int H = cfg.hidden, q = bb.n_head * bb.hd, kv = bb.n_kv * bb.hd, qkvd = q + 2 * kv;
    launch_rmsnorm(bx_, H, w.attn_norm, H, bb.eps, bh16_, H, nullptr, 0, 0, R, nullptr, stream_);
    gemv(w.qkv, bh16_, H, R, GemvOut{ EPI_STORE, bqkv_, nullptr, qkvd });
    AttnDecodeArgs a;
    a.qkv = bqkv_; a.ldq = qkvd; a.n_head = bb.n_head; a.n_kv = bb.n_kv; a.hd = bb.hd;
    a.R = R; a.n_new = 1; a.row_slot = row_slot_; a.row_active = row_active_; a.st = st_;
    a.q_norm = w.q_norm; a.k_norm = w.k_norm; a.eps = bb.eps; a.rope = rope_bb_;
    a.scale = 1.0f / std::sqrt((float) bb.hd);
    a.kv.pool = kv_pool_; a.kv.page_table = page_table_; a.kv.max_pages = max_pages_; a.kv.n_layer = bb.n_layer; a.kv.layer = l;
    a.out = batt16_; a.ldo = q;
    // split the cached positions over up to 8 CTAs per (session, kv head) while the grid is
    // small (about 2048 CTAs for the whole batch); BZB_ATTN_SPLITS overrides
    int splits = std::max(1, std::min(kAttnMaxSplits, 2048 / std::max(1, R * bb.n_kv)));
    if (const char * e = std::getenv("BZB_ATTN_SPLITS")) splits = std::max(1, std::min(kAttnMaxSplits, std::atoi(e)));
    a.splits = splits; a.part = battn_part_; a.counters = battn_ctr_;
    launch_attn_decode(a, true, stream_);
    gemv(w.o, batt16_, q, R, GemvOut{ EPI_RESID, bx_, nullptr, H });
    launch_rmsnorm(bx_, H, w.ffn_norm, H, bb.eps, bh16_, H, nullptr, 0, 0, R, nullptr, stream_);
    gemv(w.gu, bh16_, H, R, GemvOut{ EPI_SWIGLU, nullptr, bff16_, bb.ffn });
    gemv(w.down, bff16_, bb.ffn, R, GemvOut{ EPI_RESID, bx_, nullptr, H });
}

bool Engine::dp_supported(int R) const {
    const DdConfig & dd = cfg.dd;
    if (!use_dp_ || dp_grid_ <= 0 || R < 1 || R > 64) return false;
    if (dd.hd != 128 || dd.n_kv <= 0 || dd.n_head % dd.n_kv || dd.n_head > 4 * dd.n_kv || dd.n_head * dd.hd != dd.hidden)
        return false;
    if (dd.hidden % 64 || cfg.hidden % 64 || dd.ffn % 64 || dd.hidden / 64 > 32) return false;
    if (cfg.nc > 32) return false;  // the attention phase holds at most 32 positions of keys and values
    if (!dd_in_.u.blk) return false;
    for (const LayerW & w : dd_)
        if (!w.qkv.u.blk || !w.o.u.blk || !w.gu.u.blk || !w.down.u.blk) return false;
    for (const QMat & h : dd_head_)
        if (!h.u.blk) return false;
    return true;
}

// The depth decoder's input from sub-step 2 on is one codebook embedding row, and in_proj is
// linear: in_proj(E_j[code]) is precomputed once per weight set for every code of codebooks
// 1..nc-2 (the same f16 embedding values and f16 weights as the in_proj phase, f32 results), so
// the arg-max phase can write the next sub-step's input directly and the plan drops one GEMM and
// one reduction phase per sub-step. [nc-2][vs][D] f32 (252 MB at nc 32).
const float * Engine::in_tab_for_set() {
    const DdConfig & dd = cfg.dd;
    const int D = dd.hidden, H = cfg.hidden, vs = cfg.vs, ncb = cfg.nc - 2;
    if (ncb <= 0 || D % 256 != 0 || audio_embd_.K != H) return nullptr;
    if (dp_in_tab_[cur_set_]) return dp_in_tab_[cur_set_];
    const long long total = (long long) ncb * vs;
    const int qkvd = dd_[0].qkv.M;
    float * tab = dalloc<float>((size_t) total * D);
    float * qtab = dalloc<float>((size_t) total * qkvd);
    const int chunk = 8192;
    half * x16 = nullptr;
    CK(cudaMalloc(&x16, (size_t) chunk * std::max(H, D) * sizeof(half)));
    try {
        for (long long r0 = 0; r0 < total; r0 += chunk) {
            const int n = (int) std::min<long long>(chunk, total - r0);
            launch_qrows_to_f16(audio_embd_, (long long) vs + r0, n, x16, stream_);  // codebook 1 starts at row vs
            launch_gemm(dd_in_, x16, H, n, GemvOut{ EPI_STORE, tab + (size_t) r0 * D, nullptr, D });
            // layer 0's q/k/v of the same rows, from the f16 norm product its GEMM phase reads
            launch_scale_rows_f16(tab + (size_t) r0 * D, dd_[0].attn_norm, n, D, x16, stream_);
            launch_gemm(dd_[0].qkv, x16, D, n, GemvOut{ EPI_STORE, qtab + (size_t) r0 * qkvd, nullptr, qkvd });
        }
        CK(cudaStreamSynchronize(stream_));
    } catch (...) {
        cudaStreamSynchronize(stream_);
        cudaFree(x16);
        throw;
    }
    CK(cudaFree(x16));
    dp_in_tab_[cur_set_] = tab;
    dp_qkv_tab_[cur_set_] = qtab;
    return tab;
}

const Engine::DpPlan * Engine::depth_plan(int R) {
    if (!dp_supported(R)) return nullptr;
    // one schedule per batch size and depth weight set (the set's weight pointers are in it)
    const int key = R | (cur_set_ << 16);
    auto it = dp_plans_.find(key);
    if (it != dp_plans_.end()) return &it->second;
    const DdConfig & dd = cfg.dd;
    const int D = dd.hidden, H = cfg.hidden, nc = cfg.nc, vs = cfg.vs, G = dp_grid_;
    const int qkvd = dd.n_head * dd.hd + 2 * dd.n_kv * dd.hd;
    const bool tab = in_tab_for_set() != nullptr;
    // activation rows go to the MMA in chunks of at most 64 (N), one unit per chunk
    const int NB1 = std::min(64, round_up(R, 16)), NB2 = std::min(64, round_up(2 * R, 16));
    std::vector<DpPhase> ph;
    // a GEMM phase: split K (up to max_splits ways) while the tiles x row chunks leave CTAs
    // idle; returns the split count its consumer sums over
    auto gemm = [&](const UMat & w, int map, int b_row0, int rows, int epi, int out_ld, int max_splits = 16) {
        DpPhase q;
        q.type = DP_GEMM;
        q.blk = w.blk; q.q4 = w.q4; q.MT = w.MT; q.KC = w.KC; q.M = w.M;
        q.row_chunks = (rows + 63) / 64;
        q.nb = std::min(64, round_up(rows, 16));
        int S = epi == DPE_PARTIAL ? std::max(1, std::min(max_splits, std::min(w.KC, G / (w.MT * q.row_chunks)))) : 1;
        q.kc_per = (w.KC + S - 1) / S;
        S = (w.KC + q.kc_per - 1) / q.kc_per;
        // partial rows are written 4 floats at a time: the pitch is a multiple of 4
        if (epi == DPE_PARTIAL && (out_ld % 4 != 0 || out_ld < w.M))
            throw std::runtime_error("persistent depth decoder: partial row pitch");
        if (epi == DPE_PARTIAL && (size_t) S * rows * out_ld > dp_P_floats_)
            throw std::runtime_error("persistent depth decoder: partial buffer too small");
        q.splits = S; q.n_units = w.MT * S * q.row_chunks;
        q.map = map; q.b_row0 = b_row0; q.rows = rows; q.epi = epi; q.out_ld = out_ld;
        ph.push_back(q);
        return S;
    };
    auto reduce = [&](int S, int rows, int resid, const float * norm_w) {
        DpPhase q;
        q.type = DP_REDUCE; q.S = S; q.rows = rows; q.resid = resid; q.norm_w = norm_w;
        ph.push_back(q);
    };
    for (int j = 1; j < nc; j++) {
        const bool first = j == 1;
        const int rows = first ? 2 * R : R, sel = first ? 0 : 1;
        int S = 1;
        if (first || !tab) {
            S = gemm(dd_in_.u, 0 + sel, 0, rows, DPE_PARTIAL, D);
            reduce(S, rows, 0, dd_[0].attn_norm);
        }
        for (int l = 0; l < dd.n_layer; l++) {
            const LayerW & w = dd_[l];
            if (w.qkv.u.M != qkvd) throw std::runtime_error("persistent depth decoder: unexpected qkv rows");
            // from the second sub-step on, layer 0's q/k/v come from the table (arg-max phase)
            const bool from_tab = l == 0 && !first && tab;
            if (!from_tab) S = gemm(w.qkv.u, 2 + sel, 0, rows, DPE_PARTIAL, qkvd);
            DpPhase a;
            a.type = DP_ATTN; a.S = from_tab ? 1 : S; a.alt = from_tab ? 1 : 0;
            a.rows = rows; a.layer = l; a.start = first ? 0 : j; a.n_new = first ? 2 : 1;
            ph.push_back(a);
            S = gemm(w.o.u, 4 + sel, 0, rows, DPE_PARTIAL, D);
            reduce(S, rows, 1, w.ffn_norm);
            gemm(w.gu.u, 2 + sel, 0, rows, DPE_SWIGLU, dd.ffn);
            S = gemm(w.down.u, 6 + sel, 0, rows, DPE_PARTIAL, D);
            reduce(S, rows, 1, l + 1 < dd.n_layer ? dd_[l + 1].attn_norm : dd_out_norm_);
        }
        // the head reads the position-1 rows in the first sub-step
        S = gemm(dd_head_[j - 1].u, 3, first ? R : 0, R, DPE_PARTIAL, round_up(vs, 4), 8);  // arg-max sums <= 8 splits
        DpPhase am;
        am.type = DP_ARGMAX; am.S = S; am.j = j; am.ss_row0 = first ? R : 0; am.out_ld = round_up(vs, 4);
        ph.push_back(am);
    }
    DpPlan plan;
    plan.n = (int) ph.size();
    CK(cudaMalloc(&plan.dev, ph.size() * sizeof(DpPhase)));
    CK(cudaMemcpyAsync(plan.dev, ph.data(), ph.size() * sizeof(DpPhase), cudaMemcpyHostToDevice, stream_));
    CK(cudaStreamSynchronize(stream_));
    plan.maps.m[0] = make_x_group_map(din16_, H, H, 2 * R, NB2, kDpGroup);
    plan.maps.m[1] = make_x_group_map(din16_, H, H, 2 * R, NB1, kDpGroup);
    plan.maps.m[2] = make_x_group_map(dh16_, D, D, 2 * R, NB2, kDpGroup);
    plan.maps.m[3] = make_x_group_map(dh16_, D, D, 2 * R, NB1, kDpGroup);
    plan.maps.m[4] = make_x_group_map(datt16_, D, D, 2 * R, NB2, kDpGroup);
    plan.maps.m[5] = make_x_group_map(datt16_, D, D, 2 * R, NB1, kDpGroup);
    plan.maps.m[6] = make_x_group_map(dff16_, dd.ffn, dd.ffn, 2 * R, NB2, kDpGroup);
    plan.maps.m[7] = make_x_group_map(dff16_, dd.ffn, dd.ffn, 2 * R, NB1, kDpGroup);
    return &(dp_plans_[key] = plan);
}

int Engine::depth_trace(double * out, int max_phases) {
    if (cur_R_ == 0) throw std::runtime_error("no batch has been stepped yet");
    const DpPlan * pl = depth_plan(cur_R_);
    if (!pl) return 0;
    const int G = dp_grid_, n = pl->n, K = kDpTraceSlots;
    const size_t count = (size_t) n * G * K;
    const size_t total = 3 + (size_t) n + count;
    if (!out) return (int) total;
    if ((size_t) max_phases < total) throw std::runtime_error("depth_trace: output needs " + std::to_string(total) + " doubles");
    unsigned long long * tr = nullptr;
    CK(cudaMalloc(&tr, count * sizeof(unsigned long long)));
    CK(cudaMemsetAsync(tr, 0, count * sizeof(unsigned long long), stream_));
    enqueue_depth(cur_R_, nullptr, nullptr, tr);
    std::vector<unsigned long long> h(count);
    CK(cudaMemcpyAsync(h.data(), tr, count * sizeof(unsigned long long), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    cudaFree(tr);
    unsigned long long t0 = ~0ull;
    for (int c = 0; c < G; c++) t0 = std::min(t0, h[(size_t) c * K]);
    std::vector<DpPhase> ph(n);
    CK(cudaMemcpy(ph.data(), pl->dev, n * sizeof(DpPhase), cudaMemcpyDeviceToHost));
    out[0] = n;
    out[1] = G;
    out[2] = K;
    for (int i = 0; i < n; i++) out[3 + i] = ph[i].type;
    // microseconds from the first CTA's start; slots never written are -1
    double * tl = out + 3 + n;
    for (size_t i = 0; i < count; i++) tl[i] = h[i] ? (double) (long long) (h[i] - t0) * 1e-3 : -1.0;
    return (int) total;
}

void Engine::raise_device_error(int code, const std::string & what) {
    // the failure is reported once: clear the word so that the next launches start clean
    CK(cudaMemsetAsync(err_, 0, sizeof(int), stream_));
    CK(cudaStreamSynchronize(stream_));
    throw std::runtime_error(what + " (device error code " + std::to_string(code) + ")");
}

void Engine::enqueue_depth(int R, const int * forced_dev, float * logits_dev, unsigned long long * trace,
                           const int * row_set, long long grid_spin) {
    const DpPlan * pl = depth_plan(R);
    if (!pl) throw std::runtime_error("persistent depth decoder: unsupported batch");
    const DdConfig & dd = cfg.dd;
    DpParams p;
    p.phases = pl->dev; p.n_phases = pl->n;
    p.R = R; p.nc = cfg.nc; p.vs = cfg.vs; p.D = dd.hidden; p.H = cfg.hidden; p.ffn = dd.ffn;
    p.n_head = dd.n_head; p.n_kv = dd.n_kv; p.hd = dd.hd;
    p.eps = dd.eps; p.attn_scale = 1.0f / std::sqrt((float) dd.hd);
    p.rope = rope_dd_;
    p.kv = dkv_; p.kv_layer = (size_t) rmax_ * cfg.nc * 2 * dd.n_kv * dd.hd;
    p.P = dp_P_; p.x = dx_; p.h16 = dh16_; p.ss = dp_ss_; p.att16 = datt16_; p.g16 = dff16_; p.din16 = din16_;
    p.embd = audio_embd_;
    p.in_tab = dp_in_tab_[cur_set_];
    p.qkv_tab = dp_qkv_tab_[cur_set_];
    p.P2 = dp_P2_;
    p.in_norm = dd_[0].attn_norm;
    p.row_active = row_active_; p.frames = cur_frames_;
    p.row_set = row_set; p.set_id = cur_set_;
    p.forced = forced_dev; p.logits_out = logits_dev;
    p.bar = dp_bar_; p.err = err_; p.trace = trace;
    p.grid_spin = grid_spin;
    if (prof_) {
        CK(cudaEventCreate(&dprof_a_));
        CK(cudaEventCreate(&dprof_b_));
        CK(cudaEventRecord(dprof_a_, stream_));
    }
    launch_depth_persist(p, pl->maps, dp_grid_, stream_);
    if (prof_) CK(cudaEventRecord(dprof_b_, stream_));
    launches_ += 2;
}

// all nc-1 depth sub-steps of the current batch with weight set `set` (0 the model's, 1 the
// Q4_K override); with kFlagQ4 only the rows of that set receive codes
void Engine::depth_pass(int R, int flags, int set, const StepArgs & sa_in) {
    const int H = cfg.hidden, nc = cfg.nc, vs = cfg.vs, D = cfg.dd.hidden;
    const bool masked = (flags & kFlagQ4) != 0;
    if (set == 1 && !has_q4_) throw std::runtime_error("no Q4_K depth override is loaded");
    if (set != cur_set_) swap_depth_sets();
    StepArgs sa = sa_in;
    sa.row_set = masked ? row_set_ : nullptr;
    sa.set_id = set;
    const bool sampled = (flags & kFlagSampled) != 0;
    try {
        // code j of every row from the depth logits; gather_cb >= 0 stages the next sub-step's input
        auto pick = [&](int j, int gather_cb) {
            if (!sampled) {
                launch_argmax_gather(sa, dlog_, vs, vs, j, gather_cb, stream_);
                return;
            }
            DepthSampleArgs da;
            da.s = sa; da.logits = dlog_; da.ld = vs; da.V = vs; da.col = j; da.gather_cb = gather_cb;
            da.row_pair = row_pair_;
            da.seeds = (flags & kFlagSeeds) ? seeds_ : nullptr;
            da.dseeds = (flags & kFlagDepthSeeds) ? dseeds_ : nullptr;
            launch_depth_sample_gather(da, stream_);
        };
        if (!sampled && dp_supported(R)) {
            // all nc-1 depth sub-steps in one persistent launch
            enqueue_depth(R, nullptr, nullptr, nullptr, sa.row_set);
        } else {
            // depth sub-step 1: position 0 = backbone hidden, position 1 = cb0 embedding
            gemv(dd_in_, din16_, H, 2 * R, GemvOut{ EPI_STORE, dx_, nullptr, D });
            for (int l = 0; l < cfg.dd.n_layer; l++) depth_layer(l, 2 * R, R, 2, 0);
            launch_rmsnorm(dx_, D, dd_out_norm_, D, cfg.dd.eps, dh16_, D, nullptr, 0, R, R, nullptr, stream_);
            gemv(dd_head_[0], dh16_, D, R, GemvOut{ EPI_STORE, dlog_, nullptr, vs });
            pick(1, nc > 2 ? 1 : -1);
            for (int j = 2; j < nc; j++) {
                gemv(dd_in_, din16_, H, R, GemvOut{ EPI_STORE, dx_, nullptr, D });
                for (int l = 0; l < cfg.dd.n_layer; l++) depth_layer(l, R, R, 1, j);
                launch_rmsnorm(dx_, D, dd_out_norm_, D, cfg.dd.eps, dh16_, D, nullptr, 0, 0, R, nullptr, stream_);
                gemv(dd_head_[j - 1], dh16_, D, R, GemvOut{ EPI_STORE, dlog_, nullptr, vs });
                pick(j, j + 1 < nc ? j : -1);
            }
        }
    } catch (...) {
        if (cur_set_ != 0) swap_depth_sets();
        throw;
    }
    if (cur_set_ != 0) swap_depth_sets();
}

void Engine::enqueue_step(int R, int flags) {
    const int H = cfg.hidden, nc = cfg.nc, vs = cfg.vs;
    StepArgs sa;
    sa.R = R; sa.nc = nc; sa.vs = vs; sa.H = H;
    sa.row_slot = row_slot_; sa.row_active = row_active_; sa.st = st_; sa.hid32 = hid32_; sa.embd = audio_embd_;
    sa.din16 = din16_; sa.frames = cur_frames_; sa.step_ctr = step_ctr_; sa.any_active = any_active_;
    if (flags & kFlagForce) {
        launch_stage_forced(force_all_, (flags & kFlagFeed) ? feed_all_ : nullptr, step_ctr_, R * nc, cur_force_, cur_feed_,
                            stream_);
        sa.force = cur_force_;
    }
    launch_step_init(sa, stream_);
    if (flags & kFlagQ4) {
        // the rows of each depth weight set take their codes from their own pass; the second
        // pass starts again from the backbone hidden and cb0 embedding rows
        depth_pass(R, flags, 0, sa);
        launch_step_init(sa, stream_);
        depth_pass(R, flags, 1, sa);
    } else {
        depth_pass(R, flags, 0, sa);
    }
    // backbone: one token per session over its own paged cache
    launch_audio_embed(audio_embd_, (flags & kFlagFeed) ? cur_feed_ : cur_frames_, nc, nc, vs, R, bx_, row_active_, stream_);
    for (int l = 0; l < cfg.bb.n_layer; l++) bb_decode_layer(l, R);
    launch_rmsnorm(bx_, H, bb_out_norm_, H, cfg.bb.eps, bh16_, H, hid32_, H, 0, R, row_slot_, stream_);
    gemv(lm_head_, bh16_, H, R, GemvOut{ EPI_STORE, blog_, nullptr, vbb_ });
    SampleArgs sm;
    sm.logits = blog_; sm.ld = vbb_; sm.V = vbb_; sm.R = R;
    sm.row_slot = row_slot_; sm.row_active = row_active_; sm.st = st_; sm.hist = hist_; sm.hist_ld = hist_ld_;
    // suppression of the non-code ids [codebook size, audio vocab) (src/c_api.cpp:348-350)
    sm.sup_lo = cfg.cb_size; sm.sup_hi = cfg.vs; sm.eos = cfg.bb_eos;
    sm.row_pair = row_pair_;
    sm.seeds = (flags & kFlagSeeds) ? seeds_ : nullptr; sm.step_ctr = step_ctr_; sm.next_out = next_;
    if (flags & kFlagForce) launch_advance(row_slot_, row_active_, row_pair_, st_, R, next_, stream_);
    else launch_sample(sm, stream_);
    launch_frames_commit(cur_frames_, frames_all_, R * nc, step_ctr_, stream_);
}

cudaGraphExec_t Engine::graph_for(int R, int flags) {
    const auto key = std::make_pair(R, flags);
    auto it = graphs_.find(key);
    if (it != graphs_.end()) return it->second;
    cudaGraph_t g = nullptr;
    if (!(flags & kFlagSampled)) {
        // the persistent schedules (one per depth weight set) are uploaded outside the capture
        depth_plan(R);
        if (flags & kFlagQ4) {
            swap_depth_sets();
            try {
                depth_plan(R);
            } catch (...) {
                swap_depth_sets();
                throw;
            }
            swap_depth_sets();
        }
    }
    CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    set_pdl_scope(true);
    try {
        enqueue_step(R, flags);
    } catch (...) {
        set_pdl_scope(false);
        cudaStreamEndCapture(stream_, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    set_pdl_scope(false);
    CK(cudaStreamEndCapture(stream_, &g));
    size_t n_nodes = 0;
    CK(cudaGraphGetNodes(g, nullptr, &n_nodes));
    graph_nodes_ = (int) n_nodes;
    cudaGraphExec_t exec = nullptr;
    CK(cudaGraphInstantiate(&exec, g, 0));
    graphs_[key] = exec;
    graph_defs_[key] = g;
    return exec;
}

int Engine::setup_step(const int * sids, int n, int K, const uint32_t * seeds, bool sampled_depth,
                       const uint32_t * depth_seeds, const StepForce * force, std::vector<int> & rs, cudaGraphExec_t * g_out) {
    const int nc = cfg.nc;
    if (n > rmax_) throw std::runtime_error("batch of " + std::to_string(n) + " sessions exceeds the engine's " + std::to_string(rmax_) + " rows (BZB_MAX_BATCH)");
    if (K > kmax_) throw std::runtime_error("burst longer than 64 steps");
    rs.assign(n, -1);
    std::vector<char> used(max_slots_, 0);
    bool any = false;
    int n_pairs = 0;
    for (int i = 0; i < n; i++) {
        auto it = sid_to_slot_.find(sids[i]);
        if (it == sid_to_slot_.end()) continue;
        const int s = it->second;
        if (!slots_[s].active || used[s]) continue;
        used[s] = 1;
        rs[i] = s;
        any = true;
        if (slots_[s].partner >= 0) n_pairs++;
    }
    if (!any) return 0;
    // rows: the listed sessions in order, then the unconditional branches of two-branch sessions
    if (n + n_pairs > rmax_) throw std::runtime_error("batch of " + std::to_string(n + n_pairs) + " branches exceeds the engine's " + std::to_string(rmax_) + " rows (BZB_MAX_BATCH)");
    const int R = std::max(8, round_up(n + n_pairs, 8));
    rs.resize(R, -1);
    std::vector<int> rp(R, -1);
    for (int i = 0, k = n; i < n; i++) {
        if (rs[i] < 0 || slots_[rs[i]].partner < 0) continue;
        rs[k] = slots_[rs[i]].partner;
        rp[i] = k;
        rp[k] = -2 - i;
        k++;
    }
    // sampled depth: any two-branch session (src/depth_decoder.cpp:252-257), or on request unless
    // every session's depth sampler is top-1 (the argmax)
    bool sampled = n_pairs > 0;
    if (!sampled && sampled_depth)
        for (int i = 0; i < n; i++)
            if (rs[i] >= 0 && slots_[rs[i]].dtop_k != 1) sampled = true;
    // rows whose sessions take their depth codes from the Q4_K override (src/c_api.cpp:622-650)
    std::vector<int> rset(R, 0);
    bool any_q4 = false;
    for (int r = 0; r < R; r++)
        if (rs[r] >= 0 && slots_[rs[r]].use_q4) rset[r] = 1, any_q4 = true;
    // teacher-forced frames run the sampled-depth kernels (forced codes bypass the draw)
    if (force) sampled = true;
    const int flags = (seeds ? kFlagSeeds : 0) | (sampled ? kFlagSampled : 0) |
                      (sampled && depth_seeds && !seeds ? kFlagDepthSeeds : 0) | (any_q4 ? kFlagQ4 : 0) |
                      (force ? kFlagForce : 0) | (force && force->feed ? kFlagFeed : 0);
    cudaGraphExec_t g = graph_for(R, flags);
    cur_R_ = R;
    cur_flags_ = flags;
    CK(cudaMemcpyAsync(row_slot_, rs.data(), R * sizeof(int), cudaMemcpyHostToDevice, stream_));
    CK(cudaMemcpyAsync(row_pair_, rp.data(), R * sizeof(int), cudaMemcpyHostToDevice, stream_));
    if (any_q4) CK(cudaMemcpyAsync(row_set_, rset.data(), R * sizeof(int), cudaMemcpyHostToDevice, stream_));
    if (force) {
        // [K][R][nc]: each listed session's frames on its row and its unconditional branch's row
        std::vector<int> fa((size_t) K * R * nc, -1), fe;
        if (force->feed) fe.assign((size_t) K * R * nc, 0);
        for (int k = 0; k < K; k++)
            for (int r = 0; r < R; r++) {
                const int lead = r < n ? r : (rp[r] <= -2 ? -2 - rp[r] : -1);
                if (lead < 0 || rs[r] < 0) continue;
                const int * src = force->codes + ((size_t) k * n + lead) * nc;
                std::copy(src, src + nc, fa.begin() + ((size_t) k * R + r) * nc);
                if (force->feed) {
                    const int * fs = force->feed + ((size_t) k * n + lead) * nc;
                    std::copy(fs, fs + nc, fe.begin() + ((size_t) k * R + r) * nc);
                }
            }
        CK(cudaMemcpyAsync(force_all_, fa.data(), fa.size() * sizeof(int), cudaMemcpyHostToDevice, stream_));
        if (force->feed) CK(cudaMemcpyAsync(feed_all_, fe.data(), fe.size() * sizeof(int), cudaMemcpyHostToDevice, stream_));
        CK(cudaStreamSynchronize(stream_));  // the host vectors go out of scope
    }
    if (seeds) {
        std::vector<uint32_t> sd(R, 0);
        for (int i = 0; i < n; i++) sd[i] = seeds[i];
        CK(cudaMemcpyAsync(seeds_, sd.data(), R * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
    }
    if (flags & kFlagDepthSeeds) {
        std::vector<uint32_t> sd(R, 0);
        for (int i = 0; i < n; i++) sd[i] = depth_seeds[i];
        CK(cudaMemcpyAsync(dseeds_, sd.data(), R * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
    }
    CK(cudaMemsetAsync(step_ctr_, 0, sizeof(int), stream_));
    CK(cudaMemsetAsync(any_active_, 0, kmax_ * sizeof(int), stream_));
    CK(cudaMemsetAsync(next_, 0xFF, R * sizeof(int), stream_));
    *g_out = g;
    return R;
}

StepResult Engine::step(const int * sids, int n, int K, const uint32_t * seeds, bool burst, int * frames_out,
                        int width, int * next_out, bool fill_inactive, bool sampled_depth,
                        const uint32_t * depth_seeds, const StepForce * force,
                        const std::function<void(int)> * after_graph) {
    StepResult res;
    const int nc = cfg.nc;
    for (int i = 0; i < n; i++) next_out[i] = -1;
    if (burst && fill_inactive) std::fill_n(frames_out, (size_t) K * n * width, -1);
    std::vector<int> rs;
    cudaGraphExec_t g = nullptr;
    const int R = setup_step(sids, n, K, seeds, sampled_depth, depth_seeds, force, rs, &g);
    if (R == 0) return res;
    for (int k = 0; k < K; k++) {
        CK(cudaGraphLaunch(g, stream_));
        if (after_graph) (*after_graph)(k);
    }
    std::vector<int> fr((size_t) K * R * nc), nx(R), aa(K);
    CK(cudaMemcpyAsync(fr.data(), frames_all_, fr.size() * sizeof(int), cudaMemcpyDeviceToHost, stream_));
    CK(cudaMemcpyAsync(nx.data(), next_, R * sizeof(int), cudaMemcpyDeviceToHost, stream_));
    CK(cudaMemcpyAsync(aa.data(), any_active_, K * sizeof(int), cudaMemcpyDeviceToHost, stream_));
    int errv = 0;
    CK(cudaMemcpyAsync(&errv, err_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    if (errv) raise_device_error(errv, "a bounded wait timed out inside the frame step");
    for (int k = 0; k < K; k++) res.steps_executed += aa[k] ? 1 : 0;
    const int wcopy = std::min(width, nc);
    for (int k = 0; k < K; k++) {
        for (int i = 0; i < n; i++) {
            if (rs[i] < 0) continue;
            const int * src = fr.data() + ((size_t) k * R + i) * nc;
            if (src[0] < 0 && !burst) continue;
            int * dst = frames_out + ((size_t) k * n + i) * width;
            for (int c = 0; c < wcopy; c++) dst[c] = src[c];
        }
    }
    for (int i = 0; i < n; i++) {
        next_out[i] = rs[i] >= 0 ? nx[i] : -1;
        if (rs[i] >= 0 && nx[i] < 0) {
            slots_[rs[i]].active = false;
            if (slots_[rs[i]].partner >= 0) slots_[slots_[rs[i]].partner].active = false;
        }
        if (next_out[i] >= 0) res.still_active++;
    }
    return res;
}

void Engine::step_device_only(int K) {
    if (cur_R_ == 0) throw std::runtime_error("no batch has been stepped yet");
    if (K > kmax_) throw std::runtime_error("burst longer than 64 steps");
    cudaGraphExec_t g = graph_for(cur_R_, cur_flags_);
    CK(cudaMemsetAsync(step_ctr_, 0, sizeof(int), stream_));
    for (int k = 0; k < K; k++) CK(cudaGraphLaunch(g, stream_));
}

void Engine::step_launch_device(const int * sids, int n, const uint32_t * seeds, int K,
                                const std::function<void(int)> & after_step) {
    for (int i = 0; i < n; i++) {
        auto it = sid_to_slot_.find(sids[i]);
        if (it == sid_to_slot_.end() || !slots_[it->second].active)
            throw std::runtime_error("device step: session " + std::to_string(sids[i]) + " is not active");
    }
    std::vector<int> rs;
    cudaGraphExec_t g = nullptr;
    if (setup_step(sids, n, K, seeds, false, nullptr, nullptr, rs, &g) == 0) return;
    for (int k = 0; k < K; k++) {
        CK(cudaGraphLaunch(g, stream_));
        if (after_step) after_step(k);
    }
}

void Engine::sync() { CK(cudaStreamSynchronize(stream_)); }

bool Engine::session_active(int sid) const {
    auto it = sid_to_slot_.find(sid);
    return it != sid_to_slot_.end() && slots_[it->second].active;
}

// ------------------------------------------------------------------------------------ sessions
int Engine::acquire_slot(int sid, int n_pages, bool register_sid) {
    if (free_slots_.empty()) throw std::runtime_error("no free session slot");
    if ((int) free_pages_.size() < n_pages) throw std::runtime_error("KV page pool exhausted");
    const int slot = free_slots_.back();
    free_slots_.pop_back();
    SlotHost & s = slots_[slot];
    s = SlotHost();
    s.sid = sid;
    for (int i = 0; i < n_pages; i++) {
        s.pages.push_back(free_pages_.back());
        free_pages_.pop_back();
    }
    std::vector<int> row(max_pages_, s.pages.empty() ? 0 : s.pages[0]);
    for (int i = 0; i < n_pages; i++) row[i] = s.pages[i];
    // a copy from pageable host memory is staged before the call returns: `row` may go
    CK(cudaMemcpyAsync(page_table_ + (size_t) slot * max_pages_, row.data(), max_pages_ * sizeof(int),
                       cudaMemcpyHostToDevice, stream_));
    if (register_sid) {
        sid_to_slot_[sid] = slot;
        sid_epoch_[sid] = ++epoch_ctr_;
    }
    else s.follower = true;
    return slot;
}

void Engine::release_slot(int slot) {
    SlotHost & s = slots_[slot];
    const int partner = s.partner;
    for (int p : s.pages) free_pages_.push_back(p);
    if (!s.follower) sid_to_slot_.erase(s.sid);
    s = SlotHost();
    free_slots_.push_back(slot);
    if (partner >= 0) release_slot(partner);  // the session's unconditional branch
}

// the slot and its pages go back to the free lists at once: whatever reuses them is enqueued on
// the same stream, after the work that still reads them
bool Engine::session_free(int sid) {
    auto it = sid_to_slot_.find(sid);
    if (it == sid_to_slot_.end()) return false;
    release_slot(it->second);
    return true;
}

void Engine::te_forward(const std::vector<int> & tokens, float * out_rows) {
    if (!has_te_) throw std::runtime_error("GGUF has no text encoder (te.*) tensors");
    const TeConfig & te = cfg.te;
    const int T = (int) tokens.size();
    if (T > rope_te_max_) throw std::runtime_error("text segment longer than 4096 tokens");
    ensure_prefill_capacity(T);
    const int D = te.hidden, q = te.n_head * te.hd, kv = te.n_kv * te.hd, qkvd = q + 2 * kv;
    CK(cudaMemcpyAsync(ptok_, tokens.data(), T * sizeof(int), cudaMemcpyHostToDevice, stream_));
    launch_embed_rows(te_embd_, ptok_, T, te.embed_scale, tx_, nullptr, D, stream_);
    for (int l = 0; l < te.n_layer; l++) {
        const LayerW & w = te_[l];
        const bool full = l < (int) te.is_full.size() && te.is_full[l] != 0;
        // layer 0's attention norm; later layers receive theirs from the previous layer's last add
        if (l == 0) launch_rmsnorm(tx_, D, w.attn_norm, D, te.eps, th16_, D, nullptr, 0, 0, T, nullptr, stream_);
        gemv(w.qkv, th16_, D, T, GemvOut{ EPI_STORE, tqkv_, nullptr, qkvd });
        PrefillArgs pa;
        pa.qkv = tqkv_; pa.ldq = qkvd; pa.T = T; pa.start = 0;
        pa.n_head = te.n_head; pa.n_kv = te.n_kv; pa.hd = te.hd;
        pa.q_norm = w.q_norm; pa.k_norm = w.k_norm; pa.eps = te.eps;
        pa.rope = full ? rope_te_full_ : rope_te_slide_;
        pa.scale = 1.0f / std::sqrt(te.qpas);
        pa.flat_k = tk_; pa.flat_v = tv_;
        pa.window = full ? 0 : te.window;
        pa.causal = false;
        pa.out = tatt16_; pa.ldo = q;
        launch_qk_prep(pa, false, stream_);
        launch_attn_prefill(pa, false, stream_);
        gemv(w.o, tatt16_, q, T, GemvOut{ EPI_STORE, ttmp_, nullptr, D });
        launch_norm_add_norm(tx_, ttmp_, D, w.post_attn, te.eps, w.ffn_norm, th16_, D, T, stream_);
        gemv(w.gu, th16_, D, T, GemvOut{ EPI_GEGLU, nullptr, tff16_, te.ffn });
        gemv(w.down, tff16_, te.ffn, T, GemvOut{ EPI_STORE, ttmp_, nullptr, D });
        // the next layer's attention norm, or the output norm after the last layer
        const float * next_norm = l + 1 < te.n_layer ? te_[l + 1].attn_norm : te_out_norm_;
        launch_norm_add_norm(tx_, ttmp_, D, w.post_ffn, te.eps, next_norm, th16_, D, T, stream_);
    }
    if (te.n_layer == 0) launch_rmsnorm(tx_, D, te_out_norm_, D, te.eps, th16_, D, nullptr, 0, 0, T, nullptr, stream_);
    gemv(te_proj_, th16_, D, T, GemvOut{ EPI_STORE, out_rows, nullptr, cfg.hidden });
}

void Engine::bb_prefill(int slot, int T, float * logits) {
    const BbConfig & bb = cfg.bb;
    const int H = cfg.hidden, q = bb.n_head * bb.hd, kv = bb.n_kv * bb.hd, qkvd = q + 2 * kv;
    for (int l = 0; l < bb.n_layer; l++) {
        const LayerW & w = bb_[l];
        launch_rmsnorm(px_, H, w.attn_norm, H, bb.eps, ph16_, H, nullptr, 0, 0, T, nullptr, stream_);
        gemv(w.qkv, ph16_, H, T, GemvOut{ EPI_STORE, pqkv_, nullptr, qkvd });
        PrefillArgs pa;
        pa.qkv = pqkv_; pa.ldq = qkvd; pa.T = T; pa.start = 0;
        pa.n_head = bb.n_head; pa.n_kv = bb.n_kv; pa.hd = bb.hd;
        pa.q_norm = w.q_norm; pa.k_norm = w.k_norm; pa.eps = bb.eps; pa.rope = rope_bb_;
        pa.scale = 1.0f / std::sqrt((float) bb.hd);
        pa.kv.pool = kv_pool_; pa.kv.n_layer = bb.n_layer; pa.kv.layer = l;
        pa.page_row = page_table_ + (size_t) slot * max_pages_;
        pa.causal = true;
        pa.out = patt16_; pa.ldo = q;
        launch_qk_prep(pa, true, stream_);
        launch_attn_prefill(pa, true, stream_);
        gemv(w.o, patt16_, q, T, GemvOut{ EPI_RESID, px_, nullptr, H });
        launch_rmsnorm(px_, H, w.ffn_norm, H, bb.eps, ph16_, H, nullptr, 0, 0, T, nullptr, stream_);
        gemv(w.gu, ph16_, H, T, GemvOut{ EPI_SWIGLU, nullptr, pff16_, bb.ffn });
        gemv(w.down, pff16_, bb.ffn, T, GemvOut{ EPI_RESID, px_, nullptr, H });
    }
    CK(cudaMemcpyAsync(slot_scalar_, &slot, sizeof(int), cudaMemcpyHostToDevice, stream_));
    launch_rmsnorm(px_, H, bb_out_norm_, H, bb.eps, ph16_, H, hid32_, H, T - 1, 1, slot_scalar_, stream_);
    gemv(lm_head_, ph16_, H, 1, GemvOut{ EPI_STORE, logits, nullptr, vbb_ });
}

SessionParams Engine::abi_params(float cfg_scale) const {
    SessionParams p;
    p.cfg = cfg_scale > 0.0f ? cfg_scale : 1.0f;
    // cb0: fixed by the generator ABI (src/c_api.cpp:343-347); depth: the GGUF's breeze.depth_*
    p.temp = 0.9f; p.top_k = 50; p.top_p = 1.0f; p.rep = 1.1f;
    p.dtemp = cfg.depth_temperature; p.dtop_k = cfg.depth_top_k; p.dtop_p = cfg.depth_top_p;
    return p;
}

void Engine::session_create(int sid, const std::string & text, const char * instruction, const char * ref_text,
                            const int * ref_codes, int ref_frames, float cfg_scale, uint32_t seed, int max_new_tokens,
                            int * out_cb0, int * out_alloc) {
    const SessionParams sp = abi_params(cfg_scale);
    // output length estimate (src/c_api.cpp:354-364)
    int est = max_new_tokens;
    if (est <= 0) {
        int words = 0;
        bool in_w = false;
        for (unsigned char ch : text) {
            if (std::isspace(ch)) in_w = false;
            else if (!in_w) { in_w = true; words++; }
        }
        est = std::min(1000, (int) std::ceil(words * 1.5f) + 30);
    }
    const std::string spk = "[S0]";
    const std::string ins = instruction ? instruction : "Speak clearly and naturally.";
    const bool has_ref = ref_codes != nullptr && ref_frames > 0 && ref_text != nullptr && std::strlen(ref_text) > 0;
    std::vector<std::vector<int>> segs, segs_u;
    if (has_ref) segs.push_back(tok_.encode(spk + ref_text, true));
    segs.push_back(tok_.encode(spk + "<ins_bos>" + ins + "<ins_eos>" + text, true));
    // the unconditional branch drops the instruction (src/c_api.cpp:411-423)
    if (sp.cfg != 1.0f) {
        if (has_ref) segs_u.push_back(segs[0]);
        segs_u.push_back(tok_.encode(spk + text, true));
    }
    session_create_tokens(sid, segs, sp.cfg != 1.0f ? &segs_u : nullptr, has_ref ? ref_codes : nullptr,
                          has_ref ? ref_frames : 0, seed, est, sp, true, out_cb0, out_alloc);
}

// Programmatic dependent launch for an eager run of kernels (a prompt's prefill): each kernel's
// CTAs start while its predecessor drains and wait (griddepcontrol.wait) before reading its
// outputs, as inside the step graphs. Host copies between the kernels keep plain stream order.
struct EagerPdl {
    EagerPdl() { set_pdl_scope(true); }
    ~EagerPdl() { set_pdl_scope(false); }
    EagerPdl(const EagerPdl &) = delete;
    EagerPdl & operator=(const EagerPdl &) = delete;
};

void Engine::prefill_prompt(int slot, const std::vector<std::vector<int>> & segs, const int * ref_codes,
                            int ref_frames, float * logits) {
    const int H = cfg.hidden, nc = cfg.nc;
    const EagerPdl pdl;
    int off = 0;
    auto add_text = [&](const std::vector<int> & toks) {
        te_forward(toks, px_ + (size_t) off * H);
        off += (int) toks.size();
    };
    auto add_frames = [&](const int * codes, int F) {
        if (F <= 0) return;  // a reference segment without frames still gets its EOS frame
        CK(cudaMemcpyAsync(pframes_, codes, (size_t) F * nc * sizeof(int), cudaMemcpyHostToDevice, stream_));
        launch_audio_embed(audio_embd_, pframes_, nc, nc, cfg.vs, F, px_ + (size_t) off * H, nullptr, stream_);
        CK(cudaStreamSynchronize(stream_));
        off += F;
    };
    if (ref_codes) {
        add_text(segs[0]);
        add_frames(ref_codes, ref_frames);
        std::vector<int> eos((size_t) nc, cfg.cb_eos);
        add_frames(eos.data(), 1);
        add_text(segs[1]);
    } else {
        add_text(segs.back());
    }
    bb_prefill(slot, off, logits);
}

void Engine::session_create_tokens(int sid, const std::vector<std::vector<int>> & segs,
                                   const std::vector<std::vector<int>> * segs_u, const int * ref_codes,
                                   int ref_frames, uint32_t seed, int est, const SessionParams & sp, bool clamp_total,
                                   int * out_cb0, int * out_alloc, bool uncond_has_ref) {
    // prompt layout (src/c_api.cpp:388-396): [ref text][ref frames][EOS frame] then the tail text
    auto prompt_len = [&](const std::vector<std::vector<int>> & sg, bool with_ref) {
        if (sg.empty() || (with_ref && sg.size() < 2)) throw std::runtime_error("prompt segments missing");
        int t = 0;
        if (with_ref) t = (int) sg[0].size() + ref_frames + 1 + (int) sg[1].size();
        else t = (int) sg.back().size();
        return t;
    };
    const bool ref_u = ref_codes && uncond_has_ref;
    const int total = prompt_len(segs, ref_codes != nullptr);
    const int total_u = segs_u ? prompt_len(*segs_u, ref_u) : 0;
    if (total <= 0 || (segs_u && total_u <= 0)) throw std::runtime_error("empty prompt");
    if (est <= 0) throw std::runtime_error("generation budget must be positive");
    if (clamp_total) {
        // src/c_api.cpp:398-403: prompt plus budget stays within 2040 positions
        const int max_available = 2040 - total;
        if (est > max_available) est = std::max(64, max_available);
    }
    const int alloc = total + est + 8;
    const int alloc_u = segs_u ? total_u + est + 8 : 0;
    const int n_pages = (alloc + 15) / 16, n_pages_u = (alloc_u + 15) / 16;
    if (n_pages > max_pages_ || n_pages_u > max_pages_)
        throw std::runtime_error("prompt plus generation budget exceeds 4096 positions");
    auto old = sid_to_slot_.find(sid);
    if (old != sid_to_slot_.end()) {
        CK(cudaStreamSynchronize(stream_));
        release_slot(old->second);
    }
    ensure_prefill_capacity(std::max(total, total_u));
    const int slot = acquire_slot(sid, n_pages);
    try {
        int slot_u = -1;
        if (segs_u) {
            slot_u = acquire_slot(sid, n_pages_u, false);
            slots_[slot].partner = slot_u;
        }
        prefill_prompt(slot, segs, ref_codes, ref_frames, plog_);
        if (segs_u) prefill_prompt(slot_u, *segs_u, ref_u ? ref_codes : nullptr, ref_frames, plog_ + vbb_);
        SessState s{};
        s.active = 1;
        s.pos = total;
        s.steps = 0;
        s.max_tokens = est;
        s.last_cb0 = -1;
        s.key = seed;
        s.draw = 0;
        s.top_k = sp.top_k; s.temp = sp.temp; s.top_p = sp.top_p; s.rep = sp.rep;
        s.cfg = segs_u ? sp.cfg : 1.0f;
        s.dtemp = sp.dtemp; s.dtop_p = sp.dtop_p; s.dtop_k = sp.dtop_k;
        CK(cudaMemcpyAsync(st_ + slot, &s, sizeof(SessState), cudaMemcpyHostToDevice, stream_));
        if (slot_u >= 0) {
            SessState su = s;
            su.pos = total_u;
            CK(cudaMemcpyAsync(st_ + slot_u, &su, sizeof(SessState), cudaMemcpyHostToDevice, stream_));
        }
        CK(cudaMemsetAsync(hist_ + (size_t) slot * hist_ld_, 0, hist_ld_ * sizeof(uint16_t), stream_));
        // the first cb0 from the prefill logits (combined with the unconditional branch's)
        const int rows[4] = { slot, slot_u, slot_u >= 0 ? 1 : -1, -2 };
        CK(cudaMemcpyAsync(create_rows_, rows, sizeof(rows), cudaMemcpyHostToDevice, stream_));
        SampleArgs sm;
        sm.logits = plog_; sm.ld = vbb_; sm.V = vbb_; sm.R = 1;
        sm.row_slot = create_rows_; sm.row_active = nullptr; sm.st = st_; sm.hist = hist_; sm.hist_ld = hist_ld_;
        sm.row_pair = create_rows_ + 2;
        sm.sup_lo = cfg.cb_size; sm.sup_hi = cfg.vs; sm.eos = cfg.bb_eos;
        sm.seeds = nullptr; sm.step_ctr = nullptr; sm.next_out = next_; sm.update_hist_first = 1;
        launch_sample(sm, stream_);
        int cb0 = -1;
        CK(cudaMemcpyAsync(&cb0, next_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
        CK(cudaStreamSynchronize(stream_));
        SlotHost & sh = slots_[slot];
        sh.active = true;
        sh.max_tokens = est;
        sh.alloc = alloc;
        sh.dtop_k = sp.dtop_k;
        if (slot_u >= 0) {
            slots_[slot_u].active = true;
            slots_[slot_u].max_tokens = est;
            slots_[slot_u].alloc = alloc_u;
        }
        *out_cb0 = cb0;
        if (out_alloc) *out_alloc = alloc + alloc_u;
    } catch (...) {
        cudaStreamSynchronize(stream_);
        release_slot(slot);
        throw;
    }
}

// ------------------------------------------------------------------------------------ packed prefill
namespace {
// per-row segment ids, the segments and the attention query blocks of packed sequences
void pack_meta(const std::vector<int4> & segs, std::vector<int> & row_seg, std::vector<int2> & qb) {
    row_seg.clear();
    qb.clear();
    for (int i = 0; i < (int) segs.size(); i++) {
        for (int r = 0; r < segs[i].y; r++) row_seg.push_back(i);
        for (int r = 0; r < segs[i].y; r += kPrefillQBlock) qb.push_back(make_int2(i, r));
    }
}
}  // namespace

void Engine::te_forward_packed(const std::vector<const std::vector<int> *> & tsegs, float * out_rows) {
    if (!has_te_) throw std::runtime_error("GGUF has no text encoder (te.*) tensors");
    const TeConfig & te = cfg.te;
    std::vector<int> toks;
    std::vector<int4> segs;
    for (const std::vector<int> * t : tsegs) {
        if (t->empty()) throw std::runtime_error("empty text segment");
        if ((int) t->size() > rope_te_max_) throw std::runtime_error("text segment longer than 4096 tokens");
        segs.push_back(make_int4((int) toks.size(), (int) t->size(), 0, 0));
        toks.insert(toks.end(), t->begin(), t->end());
    }
    const int T = (int) toks.size();
    ensure_prefill_capacity(T);
    std::vector<int> row_seg;
    std::vector<int2> qb;
    pack_meta(segs, row_seg, qb);
    CK(cudaMemcpyAsync(ptok_, toks.data(), T * sizeof(int), cudaMemcpyHostToDevice, stream_));
    CK(cudaMemcpyAsync(pseg_, row_seg.data(), T * sizeof(int), cudaMemcpyHostToDevice, stream_));
    CK(cudaMemcpyAsync(psegs_, segs.data(), segs.size() * sizeof(int4), cudaMemcpyHostToDevice, stream_));
    CK(cudaMemcpyAsync(pqb_, qb.data(), qb.size() * sizeof(int2), cudaMemcpyHostToDevice, stream_));
    const int D = te.hidden, q = te.n_head * te.hd, kv = te.n_kv * te.hd, qkvd = q + 2 * kv;
    launch_embed_rows(te_embd_, ptok_, T, te.embed_scale, tx_, nullptr, D, stream_);
    for (int l = 0; l < te.n_layer; l++) {
        const LayerW & w = te_[l];
        const bool full = l < (int) te.is_full.size() && te.is_full[l] != 0;
        // layer 0's attention norm; later layers receive theirs from the previous layer's last add
        if (l == 0) launch_rmsnorm(tx_, D, w.attn_norm, D, te.eps, th16_, D, nullptr, 0, 0, T, nullptr, stream_);
        gemv(w.qkv, th16_, D, T, GemvOut{ EPI_STORE, tqkv_, nullptr, qkvd });
        PrefillArgs pa;
        pa.qkv = tqkv_; pa.ldq = qkvd; pa.T = T; pa.start = 0;
        pa.n_head = te.n_head; pa.n_kv = te.n_kv; pa.hd = te.hd;
        pa.q_norm = w.q_norm; pa.k_norm = w.k_norm; pa.eps = te.eps;
        pa.rope = full ? rope_te_full_ : rope_te_slide_;
        pa.scale = 1.0f / std::sqrt(te.qpas);
        pa.flat_k = tk_; pa.flat_v = tv_;
        pa.window = full ? 0 : te.window;
        pa.causal = false;
        pa.out = tatt16_; pa.ldo = q;
        pa.row_seg = pseg_; pa.segs = psegs_; pa.qblocks = pqb_; pa.n_qblocks = (int) qb.size();
        launch_qk_prep(pa, false, stream_);
        launch_attn_prefill(pa, false, stream_);
        gemv(w.o, tatt16_, q, T, GemvOut{ EPI_STORE, ttmp_, nullptr, D });
        launch_norm_add_norm(tx_, ttmp_, D, w.post_attn, te.eps, w.ffn_norm, th16_, D, T, stream_);
        gemv(w.gu, th16_, D, T, GemvOut{ EPI_GEGLU, nullptr, tff16_, te.ffn });
        gemv(w.down, tff16_, te.ffn, T, GemvOut{ EPI_STORE, ttmp_, nullptr, D });
        // the next layer's attention norm, or the output norm after the last layer
        const float * next_norm = l + 1 < te.n_layer ? te_[l + 1].attn_norm : te_out_norm_;
        launch_norm_add_norm(tx_, ttmp_, D, w.post_ffn, te.eps, next_norm, th16_, D, T, stream_);
    }
    if (te.n_layer == 0) launch_rmsnorm(tx_, D, te_out_norm_, D, te.eps, th16_, D, nullptr, 0, 0, T, nullptr, stream_);
    gemv(te_proj_, th16_, D, T, GemvOut{ EPI_STORE, out_rows, nullptr, cfg.hidden });
}

void Engine::bb_prefill_packed(const std::vector<int4> & segs, float * logits) {
    const BbConfig & bb = cfg.bb;
    const int H = cfg.hidden, q = bb.n_head * bb.hd, kv = bb.n_kv * bb.hd, qkvd = q + 2 * kv;
    int T = 0;
    for (const int4 & g : segs) T = std::max(T, g.x + g.y);
    const int nb = (int) segs.size();
    std::vector<int> row_seg, last(nb), slots(nb);
    std::vector<int2> qb;
    pack_meta(segs, row_seg, qb);
    for (int b = 0; b < nb; b++) {
        last[b] = segs[b].x + segs[b].y - 1;
        slots[b] = segs[b].z;
    }
    CK(cudaMemcpyAsync(pseg_, row_seg.data(), T * sizeof(int), cudaMemcpyHostToDevice, stream_));
    CK(cudaMemcpyAsync(psegs_, segs.data(), nb * sizeof(int4), cudaMemcpyHostToDevice, stream_));
    CK(cudaMemcpyAsync(pqb_, qb.data(), qb.size() * sizeof(int2), cudaMemcpyHostToDevice, stream_));
    CK(cudaMemcpyAsync(pidx_, last.data(), nb * sizeof(int), cudaMemcpyHostToDevice, stream_));
    CK(cudaMemcpyAsync(pslot_, slots.data(), nb * sizeof(int), cudaMemcpyHostToDevice, stream_));
    for (int l = 0; l < bb.n_layer; l++) {
        const LayerW & w = bb_[l];
        launch_rmsnorm(px_, H, w.attn_norm, H, bb.eps, ph16_, H, nullptr, 0, 0, T, nullptr, stream_);
        gemv(w.qkv, ph16_, H, T, GemvOut{ EPI_STORE, pqkv_, nullptr, qkvd });
        PrefillArgs pa;
        pa.qkv = pqkv_; pa.ldq = qkvd; pa.T = T; pa.start = 0;
        pa.n_head = bb.n_head; pa.n_kv = bb.n_kv; pa.hd = bb.hd;
        pa.q_norm = w.q_norm; pa.k_norm = w.k_norm; pa.eps = bb.eps; pa.rope = rope_bb_;
        pa.scale = 1.0f / std::sqrt((float) bb.hd);
        pa.kv.pool = kv_pool_; pa.kv.n_layer = bb.n_layer; pa.kv.layer = l;
        pa.kv.page_table = page_table_; pa.kv.max_pages = max_pages_;
        pa.causal = true;
        pa.out = patt16_; pa.ldo = q;
        pa.row_seg = pseg_; pa.segs = psegs_; pa.qblocks = pqb_; pa.n_qblocks = (int) qb.size();
        launch_qk_prep(pa, true, stream_);
        launch_attn_prefill(pa, true, stream_);
        gemv(w.o, patt16_, q, T, GemvOut{ EPI_RESID, px_, nullptr, H });
        launch_rmsnorm(px_, H, w.ffn_norm, H, bb.eps, ph16_, H, nullptr, 0, 0, T, nullptr, stream_);
        gemv(w.gu, ph16_, H, T, GemvOut{ EPI_SWIGLU, nullptr, pff16_, bb.ffn });
        gemv(w.down, pff16_, bb.ffn, T, GemvOut{ EPI_RESID, px_, nullptr, H });
    }
    // each segment's last row: hidden (normed, kept per slot) and logits
    launch_copy_rows(px_, H, pidx_, plast_, H, nullptr, nb, H, stream_);
    launch_rmsnorm(plast_, H, bb_out_norm_, H, bb.eps, ph16_, H, hid32_, H, 0, nb, pslot_, stream_);
    gemv(lm_head_, ph16_, H, nb, GemvOut{ EPI_STORE, logits, nullptr, vbb_ });
}

void Engine::sessions_create_batch(const std::vector<CreateSpec> & specs, int * out_cb0, int * out_alloc) {
    const int H = cfg.hidden, nc = cfg.nc;
    const int n = (int) specs.size();
    {
        std::vector<int> ids;
        for (const CreateSpec & c : specs) ids.push_back(c.sid);
        std::sort(ids.begin(), ids.end());
        if (std::adjacent_find(ids.begin(), ids.end()) != ids.end()) throw std::runtime_error("a session id appears twice in one batch");
    }
    // the prompts, budgets and sampler of session_create for every spec
    struct Prep {
        SessionParams sp;
        std::vector<std::vector<int>> segs, segs_u;
        bool ref = false;
        int total = 0, total_u = 0, est = 0;
    };
    std::vector<Prep> prep(n);
    const std::string spk = "[S0]";
    for (int i = 0; i < n; i++) {
        const CreateSpec & c = specs[i];
        Prep & p = prep[i];
        p.sp = abi_params(c.cfg_scale);
        int est = c.max_new_tokens;
        if (est <= 0) {
            int words = 0;
            bool in_w = false;
            for (unsigned char ch : c.text) {
                if (std::isspace(ch)) in_w = false;
                else if (!in_w) { in_w = true; words++; }
            }
            est = std::min(1000, (int) std::ceil(words * 1.5f) + 30);
        }
        const std::string ins = c.instruction ? c.instruction : "Speak clearly and naturally.";
        p.ref = c.ref_codes != nullptr && c.ref_frames > 0 && c.ref_text != nullptr && std::strlen(c.ref_text) > 0;
        if (p.ref) p.segs.push_back(tok_.encode(spk + c.ref_text, true));
        p.segs.push_back(tok_.encode(spk + "<ins_bos>" + ins + "<ins_eos>" + c.text, true));
        if (p.sp.cfg != 1.0f) {
            if (p.ref) p.segs_u.push_back(p.segs[0]);
            p.segs_u.push_back(tok_.encode(spk + c.text, true));
        }
        auto len = [&](const std::vector<std::vector<int>> & sg) {
            return p.ref ? (int) sg[0].size() + c.ref_frames + 1 + (int) sg[1].size() : (int) sg.back().size();
        };
        p.total = len(p.segs);
        p.total_u = p.segs_u.empty() ? 0 : len(p.segs_u);
        const int max_available = 2040 - p.total;
        if (est > max_available) est = std::max(64, max_available);
        p.est = est;
        if ((p.total + est + 8 + 15) / 16 > max_pages_ || (p.total_u && (p.total_u + est + 8 + 15) / 16 > max_pages_))
            throw std::runtime_error("prompt plus generation budget exceeds 4096 positions");
    }
    // groups of sessions whose packed prompts stay within the row and segment budgets
    for (int g0 = 0; g0 < n;) {
        int g1 = g0, rows = 0, nseg = 0;
        while (g1 < n && (g1 == g0 || (rows + prep[g1].total + prep[g1].total_u <= kPackRows &&
                                       nseg + (prep[g1].total_u ? 2 : 1) <= kPackSegs))) {
            rows += prep[g1].total + prep[g1].total_u;
            nseg += prep[g1].total_u ? 2 : 1;
            g1++;
        }
        // slots (a reused id frees its old slot first, src/c_api.cpp:333-337); the work still
        // queued on the stream is ordered before everything enqueued here

        std::vector<int> slot_c(g1 - g0, -1), slot_u(g1 - g0, -1);
        try {
            for (int i = g0; i < g1; i++) {
                auto old = sid_to_slot_.find(specs[i].sid);
                if (old != sid_to_slot_.end()) release_slot(old->second);
                const Prep & p = prep[i];
                slot_c[i - g0] = acquire_slot(specs[i].sid, (p.total + p.est + 8 + 15) / 16);
                if (p.total_u) {
                    slot_u[i - g0] = acquire_slot(specs[i].sid, (p.total_u + p.est + 8 + 15) / 16, false);
                    slots_[slot_c[i - g0]].partner = slot_u[i - g0];
                }
            }
            ensure_prefill_capacity(rows);
            const EagerPdl pdl;
            // packed rows: branch by branch ([ref text][ref frames][EOS] tail), conditional first
            std::vector<int4> segs;                       // {first row, rows, slot, session index}
            std::vector<const std::vector<int> *> tsegs;  // text segments in encoder order
            std::vector<int> tdst, fdst, frames;          // destination rows of encoder / embedding rows
            int row = 0;
            for (int i = g0; i < g1; i++) {
                const Prep & p = prep[i];
                for (int br = 0; br < (p.total_u ? 2 : 1); br++) {
                    const std::vector<std::vector<int>> & sg = br ? p.segs_u : p.segs;
                    const int first = row;
                    auto text = [&](const std::vector<int> & t) {
                        tsegs.push_back(&t);
                        for (int r = 0; r < (int) t.size(); r++) tdst.push_back(row + r);
                        row += (int) t.size();
                    };
                    if (p.ref) {
                        text(sg[0]);
                        frames.insert(frames.end(), specs[i].ref_codes, specs[i].ref_codes + (size_t) specs[i].ref_frames * nc);
                        for (int f = 0; f < specs[i].ref_frames; f++) fdst.push_back(row + f);
                        row += specs[i].ref_frames;
                        frames.insert(frames.end(), (size_t) nc, cfg.cb_eos);
                        fdst.push_back(row++);
                        text(sg[1]);
                    } else {
                        text(sg.back());
                    }
                    segs.push_back(make_int4(first, row - first, br ? slot_u[i - g0] : slot_c[i - g0], i));
                }
            }
            // text encoder over every text segment, placed into the prompt rows
            te_forward_packed(tsegs, pstage_);
            CK(cudaMemcpyAsync(pidx_, tdst.data(), tdst.size() * sizeof(int), cudaMemcpyHostToDevice, stream_));
            launch_copy_rows(pstage_, H, nullptr, px_, H, pidx_, (int) tdst.size(), H, stream_);
            // audio-frame embeddings of the reference segments
            if (!fdst.empty()) {
                const int F = (int) fdst.size();
                CK(cudaMemcpyAsync(pframes_, frames.data(), frames.size() * sizeof(int), cudaMemcpyHostToDevice, stream_));
                launch_audio_embed(audio_embd_, pframes_, nc, nc, cfg.vs, F, pstage_, nullptr, stream_);
                CK(cudaMemcpyAsync(pidx_, fdst.data(), F * sizeof(int), cudaMemcpyHostToDevice, stream_));
                launch_copy_rows(pstage_, H, nullptr, px_, H, pidx_, F, H, stream_);
            }
            bb_prefill_packed(segs, plogs_);  // (copies from pageable host vectors are staged at the call)
            // session states, histories, and the first cb0 of every session (guidance-combined)
            const int nb = (int) segs.size();
            std::vector<int> rslot(nb), rpair(nb, -1), lead_of_spec(g1 - g0, -1);
            for (int b = 0; b < nb; b++) {
                const int i = segs[b].w;
                const Prep & p = prep[i];
                const bool is_u = segs[b].z == slot_u[i - g0];
                rslot[b] = segs[b].z;
                SessState st{};
                st.active = 1;
                st.pos = is_u ? p.total_u : p.total;
                st.max_tokens = p.est;
                st.last_cb0 = -1;
                st.key = specs[i].seed;
                st.top_k = p.sp.top_k; st.temp = p.sp.temp; st.top_p = p.sp.top_p; st.rep = p.sp.rep;
                st.cfg = p.total_u ? p.sp.cfg : 1.0f;
                st.dtemp = p.sp.dtemp; st.dtop_p = p.sp.dtop_p; st.dtop_k = p.sp.dtop_k;
                CK(cudaMemcpyAsync(st_ + segs[b].z, &st, sizeof(SessState), cudaMemcpyHostToDevice, stream_));
                if (!is_u) {
                    lead_of_spec[i - g0] = b;
                    CK(cudaMemsetAsync(hist_ + (size_t) segs[b].z * hist_ld_, 0, hist_ld_ * sizeof(uint16_t), stream_));
                } else {
                    rpair[lead_of_spec[i - g0]] = b;
                    rpair[b] = -2 - lead_of_spec[i - g0];
                }
            }
            CK(cudaMemcpyAsync(pslot_, rslot.data(), nb * sizeof(int), cudaMemcpyHostToDevice, stream_));
            CK(cudaMemcpyAsync(ppair_, rpair.data(), nb * sizeof(int), cudaMemcpyHostToDevice, stream_));
            SampleArgs sm;
            sm.logits = plogs_; sm.ld = vbb_; sm.V = vbb_; sm.R = nb;
            sm.row_slot = pslot_; sm.row_active = nullptr; sm.st = st_; sm.hist = hist_; sm.hist_ld = hist_ld_;
            sm.row_pair = ppair_;
            sm.sup_lo = cfg.cb_size; sm.sup_hi = cfg.vs; sm.eos = cfg.bb_eos;
            sm.next_out = pnext_; sm.update_hist_first = 1;
            launch_sample(sm, stream_);
            std::vector<int> nx(nb);
            CK(cudaMemcpyAsync(nx.data(), pnext_, nb * sizeof(int), cudaMemcpyDeviceToHost, stream_));
            CK(cudaStreamSynchronize(stream_));
            for (int i = g0; i < g1; i++) {
                const Prep & p = prep[i];
                SlotHost & sh = slots_[slot_c[i - g0]];
                sh.active = true;
                sh.max_tokens = p.est;
                sh.alloc = p.total + p.est + 8;
                sh.dtop_k = p.sp.dtop_k;
                if (slot_u[i - g0] >= 0) {
                    slots_[slot_u[i - g0]].active = true;
                    slots_[slot_u[i - g0]].max_tokens = p.est;
                    slots_[slot_u[i - g0]].alloc = p.total_u + p.est + 8;
                }
                out_cb0[i] = nx[lead_of_spec[i - g0]];
                if (out_alloc) out_alloc[i] = p.total + p.est + 8 + (p.total_u ? p.total_u + p.est + 8 : 0);
            }
        } catch (...) {
            cudaStreamSynchronize(stream_);
            for (int k = 0; k < g1 - g0; k++)
                if (slot_c[k] >= 0) release_slot(slot_c[k]);
            throw;
        }
        g0 = g1;
    }
}

// ------------------------------------------------------------------------------------ debug
void Engine::debug_hidden(int sid, float * out) {
    auto it = sid_to_slot_.find(sid);
    if (it == sid_to_slot_.end()) throw std::runtime_error("unknown session");
    CK(cudaMemcpyAsync(out, hid32_ + (size_t) it->second * cfg.hidden, cfg.hidden * sizeof(float),
                       cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
}

void Engine::debug_depth(int n, const float * hidden, const int * cb0, const int * forced, int * codes_out,
                         float * logits_out) {
    const int H = cfg.hidden, nc = cfg.nc, vs = cfg.vs, D = cfg.dd.hidden;
    if (n <= 0 || n > rmax_) throw std::runtime_error("debug_depth: bad row count");
    const int R = std::max(8, round_up(n, 8));
    std::vector<int> rs(R, -1), ra(R, 0);
    for (int i = 0; i < n; i++) { rs[i] = i; ra[i] = 1; }
    CK(cudaMemcpyAsync(row_slot_, rs.data(), R * sizeof(int), cudaMemcpyHostToDevice, stream_));
    CK(cudaMemcpyAsync(row_active_, ra.data(), R * sizeof(int), cudaMemcpyHostToDevice, stream_));
    std::vector<half> h16((size_t) 2 * R * H, __float2half(0.0f));
    for (int i = 0; i < n; i++)
        for (int d = 0; d < H; d++) h16[(size_t) i * H + d] = __float2half_rn(hidden[(size_t) i * H + d]);
    CK(cudaMemcpyAsync(din16_, h16.data(), h16.size() * sizeof(half), cudaMemcpyHostToDevice, stream_));
    std::vector<int> idx(R, 0);
    for (int i = 0; i < n; i++) idx[i] = cb0[i];
    ensure_prefill_capacity(R);
    CK(cudaMemcpyAsync(ptok_, idx.data(), R * sizeof(int), cudaMemcpyHostToDevice, stream_));
    launch_embed_rows(audio_embd_, ptok_, n, 1.0f, nullptr, din16_ + (size_t) R * H, H, stream_);
    StepArgs sa;
    sa.R = R; sa.nc = nc; sa.vs = vs; sa.H = H;
    sa.row_slot = row_slot_; sa.row_active = row_active_; sa.st = st_; sa.hid32 = hid32_; sa.embd = audio_embd_;
    sa.din16 = din16_; sa.frames = cur_frames_; sa.step_ctr = step_ctr_; sa.any_active = any_active_;
    std::vector<float> lg((size_t) R * vs);
    std::vector<int> fr((size_t) R * nc);
    if (dp_supported(R)) {
        // the same persistent launch the frame step uses, with teacher forcing and logits out
        int * fd = nullptr;
        float * ld = nullptr;
        CK(cudaMalloc(&ld, (size_t) R * (nc - 1) * vs * sizeof(float)));
        if (forced) {
            std::vector<int> f((size_t) R * (nc - 1), 0);
            std::memcpy(f.data(), forced, (size_t) n * (nc - 1) * sizeof(int));
            CK(cudaMalloc(&fd, f.size() * sizeof(int)));
            CK(cudaMemcpyAsync(fd, f.data(), f.size() * sizeof(int), cudaMemcpyHostToDevice, stream_));
        }
        depth_plan(R);
        enqueue_depth(R, fd, ld, nullptr, nullptr, dbg_grid_spin_);
        std::vector<float> all((size_t) R * (nc - 1) * vs);
        int errv = 0;
        CK(cudaMemcpyAsync(all.data(), ld, all.size() * sizeof(float), cudaMemcpyDeviceToHost, stream_));
        CK(cudaMemcpyAsync(fr.data(), cur_frames_, fr.size() * sizeof(int), cudaMemcpyDeviceToHost, stream_));
        CK(cudaMemcpyAsync(&errv, err_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
        CK(cudaStreamSynchronize(stream_));
        cudaFree(ld);
        if (fd) cudaFree(fd);
        if (errv) raise_device_error(errv, "persistent depth decoder: a bounded wait timed out");
        std::memcpy(logits_out, all.data(), (size_t) n * (nc - 1) * vs * sizeof(float));
        for (int i = 0; i < n; i++)
            for (int j = 1; j < nc; j++) codes_out[(size_t) i * (nc - 1) + (j - 1)] = fr[(size_t) i * nc + j];
        return;
    }
    for (int j = 1; j < nc; j++) {
        const int rows = j == 1 ? 2 * R : R;
        gemv(dd_in_, din16_, H, rows, GemvOut{ EPI_STORE, dx_, nullptr, D });
        for (int l = 0; l < cfg.dd.n_layer; l++) depth_layer(l, rows, R, j == 1 ? 2 : 1, j == 1 ? 0 : j);
        launch_rmsnorm(dx_, D, dd_out_norm_, D, cfg.dd.eps, dh16_, D, nullptr, 0, j == 1 ? R : 0, R, nullptr, stream_);
        gemv(dd_head_[j - 1], dh16_, D, R, GemvOut{ EPI_STORE, dlog_, nullptr, vs });
        launch_argmax_gather(sa, dlog_, vs, vs, j, (j + 1 < nc && !forced) ? j : -1, stream_);
        CK(cudaMemcpyAsync(lg.data(), dlog_, lg.size() * sizeof(float), cudaMemcpyDeviceToHost, stream_));
        CK(cudaStreamSynchronize(stream_));
        for (int i = 0; i < n; i++)
            std::memcpy(logits_out + ((size_t) i * (nc - 1) + (j - 1)) * vs, lg.data() + (size_t) i * vs, vs * sizeof(float));
        if (forced && j + 1 < nc) {
            for (int i = 0; i < n; i++) idx[i] = j * vs + forced[(size_t) i * (nc - 1) + (j - 1)];
            CK(cudaMemcpyAsync(ptok_, idx.data(), R * sizeof(int), cudaMemcpyHostToDevice, stream_));
            launch_embed_rows(audio_embd_, ptok_, n, 1.0f, nullptr, din16_, H, stream_);
        }
    }
    CK(cudaMemcpyAsync(fr.data(), cur_frames_, fr.size() * sizeof(int), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    for (int i = 0; i < n; i++)
        for (int j = 1; j < nc; j++) codes_out[(size_t) i * (nc - 1) + (j - 1)] = fr[(size_t) i * nc + j];
}

void Engine::debug_gemv(const char * tensor, int sub, int rows, const float * x, float * y) {
    const GgufTensor * t = need(tensor);
    QMat w = sub >= 0 ? load_qmat({ t }, false, (int) (sub * t->ne[1]), (int) t->ne[1]) : load_qmat({ t }, false);
    const int K = w.K, M = w.M;
    ensure_prefill_capacity(rows);
    std::vector<half> xh((size_t) rows * K);
    for (size_t i = 0; i < xh.size(); i++) xh[i] = __float2half_rn(x[i]);
    half * xd = nullptr;
    float * yd = nullptr;
    CK(cudaMalloc(&xd, xh.size() * sizeof(half)));
    CK(cudaMalloc(&yd, (size_t) rows * M * sizeof(float)));
    CK(cudaMemcpyAsync(xd, xh.data(), xh.size() * sizeof(half), cudaMemcpyHostToDevice, stream_));
    launch_gemm(w, xd, K, rows, GemvOut{ EPI_STORE, yd, nullptr, M });
    CK(cudaMemcpyAsync(y, yd, (size_t) rows * M * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    cudaFree(xd);
    cudaFree(yd);
}

void Engine::profile_step(double * out) {
    if (cur_R_ == 0) throw std::runtime_error("no batch has been stepped yet");
    std::vector<ProfRec> recs;
    cudaEvent_t a, b;
    CK(cudaEventCreate(&a));
    CK(cudaEventCreate(&b));
    CK(cudaMemsetAsync(step_ctr_, 0, sizeof(int), stream_));
    prof_ = &recs;
    launches_ = 0;
    CK(cudaEventRecord(a, stream_));
    try {
        enqueue_step(cur_R_, cur_flags_);
    } catch (...) {
        prof_ = nullptr;
        throw;
    }
    CK(cudaEventRecord(b, stream_));
    prof_ = nullptr;
    CK(cudaStreamSynchronize(stream_));
    float ms = 0.0f;
    CK(cudaEventElapsedTime(&ms, a, b));
    double gms = 0.0, bytes = 0.0;
    for (auto & r : recs) {
        float t = 0.0f;
        CK(cudaEventElapsedTime(&t, r.a, r.b));
        gms += t;
        bytes += r.bytes;
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    out[0] = ms;
    out[1] = gms;
    out[2] = (double) recs.size();
    out[3] = bytes;
    out[4] = (double) launches_;
    out[5] = 0.0;
    out[6] = 0.0;
    if (dprof_a_) {
        float dms = 0.0f;
        CK(cudaEventElapsedTime(&dms, dprof_a_, dprof_b_));
        cudaEventDestroy(dprof_a_);
        cudaEventDestroy(dprof_b_);
        dprof_a_ = dprof_b_ = nullptr;
        out[5] = dms;
        out[6] = (double) depth_bytes_per_step();
    }
}

size_t Engine::depth_bytes_per_step() const {
    // algorithmic bytes of the depth decode of one frame step: the Q8_0 depth weights, re-read by
    // every sub-step (the 4 layers and that sub-step's head); in_proj is read by the first
    // sub-step and, with the precomputed in_proj table, the later ones read one table row (D f32)
    // per session instead
    auto qbytes = [](const QMat & q) { return qmat_bytes(q); };
    size_t dd = qbytes(dd_head_[0]);
    for (const LayerW & w : dd_) dd += qbytes(w.qkv) + qbytes(w.o) + qbytes(w.gu) + qbytes(w.down);
    // the later sub-steps read table rows (in_proj output and layer-0 q/k/v) instead of in_proj
    // and layer 0's qkv weights
    const size_t tab_row = (size_t) (cfg.dd.hidden + dd_[0].qkv.M) * sizeof(float);
    const size_t later = dp_in_tab_[cur_set_] ? (size_t) cur_R_ * tab_row : qbytes(dd_in_) + qbytes(dd_[0].qkv);
    return (size_t) (cfg.nc - 1) * dd - (size_t) (cfg.nc - 2) * qbytes(dd_[0].qkv) + qbytes(dd_in_) +
           (size_t) (cfg.nc - 2) * later;
}

double Engine::bench_gemv(const char * tensor, int sub, int rows, int iters, int epi) {
    const GgufTensor * t = need(tensor);
    QMat w = sub >= 0 ? load_qmat({ t }, false, (int) (sub * t->ne[1]), (int) t->ne[1]) : load_qmat({ t }, false);
    half * xd = nullptr;
    float * yd = nullptr;
    CK(cudaMalloc(&xd, (size_t) rows * w.K * sizeof(half)));
    CK(cudaMalloc(&yd, (size_t) rows * w.M * sizeof(float)));
    CK(cudaMemsetAsync(xd, 0, (size_t) rows * w.K * sizeof(half), stream_));
    CK(cudaMemsetAsync(yd, 0, (size_t) rows * w.M * sizeof(float), stream_));
    GemvOut o{ epi, yd, (half *) yd, epi >= EPI_SWIGLU ? w.M / 2 : w.M };
    cudaEvent_t a, b;
    CK(cudaEventCreate(&a));
    CK(cudaEventCreate(&b));
    for (int i = 0; i < 3; i++) launch_gemm(w, xd, w.K, rows, o);
    CK(cudaEventRecord(a, stream_));
    for (int i = 0; i < iters; i++) launch_gemm(w, xd, w.K, rows, o);
    CK(cudaEventRecord(b, stream_));
    CK(cudaEventSynchronize(b));
    float ms = 0.0f;
    CK(cudaEventElapsedTime(&ms, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaFree(xd);
    cudaFree(yd);
    return ms * 1000.0 / iters;
}

const QMat * Engine::resident_any(const char * name, int * epi) const {
    *epi = EPI_STORE;
    if (const QMat * m = resident_matrix(name)) return m;
    int l = -1, n = 0;
    char part[32] = { 0 };
    if (std::sscanf(name, "dd.head.%d%n", &l, &n) == 1 && name[n] == 0)
        return l >= 0 && l < (int) dd_head_.size() ? &dd_head_[l] : nullptr;
    if (std::strcmp(name, "te.proj.weight") == 0) return has_te_ ? &te_proj_ : nullptr;
    const std::vector<LayerW> * layers = nullptr;
    int gated = EPI_SWIGLU;
    if (std::sscanf(name, "bb.blk.%d.%31[a-z_]%n", &l, part, &n) == 2 && name[n] == 0) layers = &bb_;
    else if (std::sscanf(name, "dd.blk.%d.%31[a-z_]%n", &l, part, &n) == 2 && name[n] == 0) layers = &dd_;
    else if (std::sscanf(name, "te.blk.%d.%31[a-z_]%n", &l, part, &n) == 2 && name[n] == 0) {
        layers = &te_;
        gated = EPI_GEGLU;
    }
    if (!layers || l < 0 || l >= (int) layers->size()) return nullptr;
    if (std::strcmp(part, "attn_qkv") == 0) return &(*layers)[l].qkv;
    if (std::strcmp(part, "attn_output") == 0) return &(*layers)[l].o;
    if (std::strcmp(part, "ffn_down") == 0) return &(*layers)[l].down;
    if (std::strcmp(part, "ffn_gate_up") == 0) {
        *epi = gated;
        return &(*layers)[l].gu;
    }
    return nullptr;
}

void Engine::debug_sample(const float * logits, int V, int rows, int top_k, float temp, float top_p, uint32_t seed,
                          int draws, int force_sort, int * picks) {
    if (V <= 0 || V > 4096 || rows <= 0 || draws <= 0) throw std::runtime_error("debug_sample: bad shape");
    float * lg = nullptr;
    SessState * st = nullptr;
    uint16_t * hist = nullptr;
    int * slot = nullptr, * nx = nullptr;
    auto release = [&] { cudaFree(lg); cudaFree(st); cudaFree(hist); cudaFree(slot); cudaFree(nx); };
    try {
        CK(cudaMalloc(&lg, (size_t) rows * V * sizeof(float)));
        CK(cudaMalloc(&st, (size_t) rows * sizeof(SessState)));
        CK(cudaMalloc(&hist, (size_t) rows * V * sizeof(uint16_t)));
        CK(cudaMalloc(&slot, (size_t) rows * sizeof(int)));
        CK(cudaMalloc(&nx, (size_t) rows * draws * sizeof(int)));
        std::vector<SessState> hs(rows);
        std::vector<int> hslot(rows);
        for (int r = 0; r < rows; r++) {
            SessState x{};
            x.active = 1;
            x.max_tokens = INT_MAX;
            x.last_cb0 = -1;
            x.key = seed + (uint32_t) r;
            x.top_k = top_k; x.temp = temp; x.top_p = top_p; x.rep = 1.0f; x.cfg = 1.0f;
            hs[r] = x;
            hslot[r] = r;
        }
        CK(cudaMemcpyAsync(lg, logits, (size_t) rows * V * sizeof(float), cudaMemcpyHostToDevice, stream_));
        CK(cudaMemcpyAsync(st, hs.data(), hs.size() * sizeof(SessState), cudaMemcpyHostToDevice, stream_));
        CK(cudaMemcpyAsync(slot, hslot.data(), hslot.size() * sizeof(int), cudaMemcpyHostToDevice, stream_));
        CK(cudaMemsetAsync(hist, 0, (size_t) rows * V * sizeof(uint16_t), stream_));
        SampleArgs sm;
        sm.logits = lg; sm.ld = V; sm.V = V; sm.R = rows;
        sm.row_slot = slot; sm.st = st; sm.hist = hist; sm.hist_ld = V;
        sm.sup_lo = V; sm.sup_hi = V; sm.eos = -1;
        sm.update_hist_first = 1;  // every draw returns its pick and leaves the state otherwise alone
        sm.force_sort = force_sort;
        for (int d = 0; d < draws; d++) {
            sm.next_out = nx + (size_t) d * rows;
            launch_sample(sm, stream_);
        }
        CK(cudaMemcpyAsync(picks, nx, (size_t) rows * draws * sizeof(int), cudaMemcpyDeviceToHost, stream_));
        CK(cudaStreamSynchronize(stream_));
    } catch (...) {
        cudaStreamSynchronize(stream_);
        release();
        throw;
    }
    release();
}

long long Engine::debug_gemm(const char * name, int rows, const float * x, float * y, int repeats, int flags,
                             int * where, int cap) {
    int epi = EPI_STORE;
    const QMat * wp = resident_any(name, &epi);
    if (!wp) throw std::runtime_error(std::string("debug_gemm: no resident matrix named ") + name);
    if (rows <= 0 || repeats < 0) throw std::runtime_error("debug_gemm: bad row or repeat count");
    const QMat & w = *wp;
    const bool gated = epi >= EPI_SWIGLU;
    const int K = w.K, ld = gated ? w.M / 2 : w.M;
    const size_t out_bytes = (size_t) rows * ld * (gated ? sizeof(half) : sizeof(float));
    std::vector<half> xh((size_t) rows * K);
    for (size_t i = 0; i < xh.size(); i++) xh[i] = __float2half_rn(x[i]);
    half * xd = nullptr;
    void * y0 = nullptr, * y1 = nullptr;
    int * cnt = nullptr, * wd = nullptr;
    cap = where ? std::max(cap, 0) : 0;
    CK(cudaMalloc(&xd, xh.size() * sizeof(half)));
    CK(cudaMalloc(&y0, out_bytes));
    CK(cudaMalloc(&y1, out_bytes));
    CK(cudaMalloc(&cnt, sizeof(int)));
    CK(cudaMalloc(&wd, (size_t) std::max(cap, 1) * 2 * sizeof(int)));
    long long mismatches = 0;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    auto out_of = [&](void * p) {
        return gated ? GemvOut{ epi, nullptr, static_cast<half *>(p), ld } : GemvOut{ epi, static_cast<float *>(p), nullptr, ld };
    };
    try {
        CK(cudaMemcpyAsync(xd, xh.data(), xh.size() * sizeof(half), cudaMemcpyHostToDevice, stream_));
        CK(cudaMemsetAsync(cnt, 0, sizeof(int), stream_));
        launch_gemm(w, xd, K, rows, out_of(y0));
        if (repeats > 0) {
            // the frame step's conditions: captured launches with programmatic dependent launch
            CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
            set_pdl_scope((flags & 1) == 0);
            try {
                for (int r = 0; r < repeats; r++) {
                    launch_gemm(w, xd, K, rows, out_of(y1));
                    launch_bits_diff(y0, y1, out_bytes / 4, cnt, stream_, cap ? wd : nullptr, cap, r);
                }
            } catch (...) {
                set_pdl_scope(false);
                cudaStreamEndCapture(stream_, &g);
                throw;
            }
            set_pdl_scope(false);
            CK(cudaStreamEndCapture(stream_, &g));
            CK(cudaGraphInstantiate(&ge, g, 0));
            CK(cudaGraphLaunch(ge, stream_));
        }
        std::vector<uint8_t> hb(out_bytes);
        int c = 0, errv = 0;
        CK(cudaMemcpyAsync(hb.data(), y0, out_bytes, cudaMemcpyDeviceToHost, stream_));
        CK(cudaMemcpyAsync(&c, cnt, sizeof(int), cudaMemcpyDeviceToHost, stream_));
        CK(cudaMemcpyAsync(&errv, err_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
        CK(cudaStreamSynchronize(stream_));
        if (errv) raise_device_error(errv, "debug_gemm: a bounded wait timed out in the tcgen05 GEMM");
        mismatches = c;
        if (cap > 0) CK(cudaMemcpy(where, wd, (size_t) std::min(c, cap) * 2 * sizeof(int), cudaMemcpyDeviceToHost));
        const size_t n = (size_t) rows * ld;
        if (gated)
            for (size_t i = 0; i < n; i++) y[i] = __half2float(reinterpret_cast<const half *>(hb.data())[i]);
        else
            std::memcpy(y, hb.data(), out_bytes);
    } catch (...) {
        if (ge) cudaGraphExecDestroy(ge);
        if (g) cudaGraphDestroy(g);
        cudaFree(xd); cudaFree(y0); cudaFree(y1); cudaFree(cnt); cudaFree(wd);
        throw;
    }
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
    cudaFree(xd); cudaFree(y0); cudaFree(y1); cudaFree(cnt); cudaFree(wd);
    return mismatches;
}

const QMat * Engine::resident_matrix(const char * tensor) const {
    // parsed without building strings: this lookup serves the allocation-free entry point
    int l = -1, n = 0;
    char part[32] = { 0 };
    if (std::strcmp(tensor, "bb.lm_head.weight") == 0) return &lm_head_;
    if (std::strcmp(tensor, "dd.in_proj.weight") == 0) return &dd_in_;
    const std::vector<LayerW> * layers = nullptr;
    if (std::sscanf(tensor, "bb.blk.%d.%31[a-z_].weight%n", &l, part, &n) == 2 && tensor[n] == 0) layers = &bb_;
    else if (std::sscanf(tensor, "dd.blk.%d.%31[a-z_].weight%n", &l, part, &n) == 2 && tensor[n] == 0) layers = &dd_;
    if (!layers || l < 0 || l >= (int) layers->size()) return nullptr;
    if (std::strcmp(part, "attn_output") == 0) return &(*layers)[l].o;
    if (std::strcmp(part, "ffn_down") == 0) return &(*layers)[l].down;
    return nullptr;
}

void Engine::gemm_noalloc(const char * tensor, int rows, const half * x16, int ldx, float * y, int ldy, cudaStream_t s) {
    const QMat * w = resident_matrix(tensor);
    if (!w)
        throw std::runtime_error("gemm_noalloc: not a resident unfused matrix (bb.lm_head, dd.in_proj, "
                                 "{bb,dd}.blk.N.attn_output or ffn_down): " + std::string(tensor));
    if (!x16 || !y) throw std::runtime_error("gemm_noalloc: null device buffer");
    if (!w->qs) throw std::runtime_error("gemm_noalloc: the allocation-free GEMV serves Q8_0 matrices only");
    if (ldx < w->K || (ldx & 1) || (reinterpret_cast<uintptr_t>(x16) & 3) || (reinterpret_cast<uintptr_t>(y) & 3))
        throw std::runtime_error("gemm_noalloc: x must be 4-byte aligned with an even stride >= K, y 4-byte aligned");
    // the caller's current device is restored on return
    int prev = 0;
    CK(cudaGetDevice(&prev));
    CK(cudaSetDevice(device));
    try {
        launch_gemv_static_scratch(*w, x16, ldx, rows, y, ldy, s ? s : stream_);
    } catch (...) {
        cudaSetDevice(prev);
        throw;
    }
    CK(cudaSetDevice(prev));
}

size_t Engine::weight_bytes_per_step() const {
    // algorithmic weight bytes of one frame step (Q8_0: 34 bytes per 32 weights, Q4_K: 144 per
    // 256): backbone + lm_head once, depth in_proj + layers + one head per sub-step
    auto qbytes = [](const QMat & q) { return qmat_bytes(q); };
    size_t bb = qbytes(lm_head_);
    for (const LayerW & w : bb_) bb += qbytes(w.qkv) + qbytes(w.o) + qbytes(w.gu) + qbytes(w.down);
    size_t dd = qbytes(dd_in_) + qbytes(dd_head_[0]);
    for (const LayerW & w : dd_) dd += qbytes(w.qkv) + qbytes(w.o) + qbytes(w.gu) + qbytes(w.down);
    return bb + (size_t) (cfg.nc - 1) * dd;
}

size_t Engine::kv_bytes_per_position() const {
    return (size_t) cfg.bb.n_layer * 2 * cfg.bb.n_kv * cfg.bb.hd * sizeof(half);
}

}  // namespace bzb
