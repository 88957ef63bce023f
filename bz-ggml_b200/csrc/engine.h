// The B200 generator engine: device-resident weights, a paged KV cache shared by all
// sessions, device-resident session state and one CUDA-graph frame step per batch bucket.
#pragma once

#include "depth_persist.cuh"
#include "host.h"
#include "kernels.cuh"

#include <functional>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

namespace bzb {

struct LayerW {
    QMat qkv, o, gu, down;
    float * attn_norm = nullptr, * ffn_norm = nullptr, * q_norm = nullptr, * k_norm = nullptr;
    float * post_attn = nullptr, * post_ffn = nullptr;
};

struct SlotHost {
    int sid = -1;
    bool active = false;
    int max_tokens = 0;
    int alloc = 0;
    int partner = -1;       // slot of this session's unconditional branch (two-branch sessions)
    bool follower = false;  // this slot is another session's unconditional branch
    int dtop_k = 1;         // depth sampler top-k (1: the argmax schedule serves it)
    bool use_q4 = false;    // depth codes from the Q4_K override weights (src/c_api.cpp:570-578)
    std::vector<int> pages;
};

// Sampler and guidance parameters of a new session (src/sampling.h SampleParams,
// src/c_api.cpp:340-351, src/generation.cpp:122-128).
struct SessionParams {
    float cfg = 1.0f;                               // != 1: a second, unconditional branch
    float temp = 0.9f, top_p = 1.0f, rep = 1.1f;    // cb0
    int top_k = 50;
    float dtemp = 0.9f, dtop_p = 1.0f;              // depth codes (sampled-depth mode only)
    int dtop_k = 50;
};

// teacher-forced frames for a step call (host, [K][n][nc]): `codes` holds each frame's cb0 and
// the depth codes to force (-1: the depth sampler picks); `feed`, when given, is the frame the
// backbone consumes instead of the produced one (src/generation.cpp:361-367)
struct StepForce {
    const int * codes = nullptr;
    const int * feed = nullptr;
};

// one session of a batched creation (the arguments of breeze_generator_session_create_ext)
struct CreateSpec {
    int sid = 0;
    std::string text;
    const char * instruction = nullptr, * ref_text = nullptr;
    const int * ref_codes = nullptr;
    int ref_frames = 0;
    float cfg_scale = 1.0f;
    uint32_t seed = 0;
    int max_new_tokens = 0;
};

struct StepResult {
    int steps_executed = 0;
    int still_active = 0;
};

class Engine {
public:
    Engine(const std::string & gguf_path, int device);
    ~Engine();

    ModelConfig cfg;
    int device = 0;

    // session life cycle (reference: src/c_api.cpp:325-457, 521-530, 580-582)
    void session_create(int sid, const std::string & text, const char * instruction, const char * ref_text,
                        const int * ref_codes, int ref_frames, float cfg_scale, uint32_t seed, int max_new_tokens,
                        int * out_cb0, int * out_alloc);
    // prompt = [ref text segment][ref frames][EOS frame] tail segment (the ref parts only when
    // ref_codes is non-null); `uncond` adds the unconditional branch's segments (params.cfg != 1).
    // With clamp_total the budget is clamped so prompt + budget <= 2040 (the generator ABI).
    // (uncond_has_ref false: the reference parts belong to the conditional prompt only)
    void session_create_tokens(int sid, const std::vector<std::vector<int>> & text_segments,
                               const std::vector<std::vector<int>> * uncond_segments, const int * ref_codes,
                               int ref_frames, uint32_t seed, int max_tokens, const SessionParams & params,
                               bool clamp_total, int * out_cb0, int * out_alloc, bool uncond_has_ref = true);
    // the generator ABI's sampler for a session (fixed cb0 sampler, the GGUF's depth sampler)
    SessionParams abi_params(float cfg_scale) const;
    const Tokenizer & tokenizer() const { return tok_; }
    bool session_free(int sid);
    // many session_create calls at once (the same prompts, budgets and first cb0 semantics), their
    // prompts prefilled as packed rows: one text-encoder pass and one backbone pass per group of
    // sessions instead of two per session
    void sessions_create_batch(const std::vector<CreateSpec> & specs, int * out_cb0, int * out_alloc);
    static constexpr int kPackRows = 16384;  // prompt rows of one packed prefill pass
    static constexpr int kPackSegs = 256;    // branches (prompts) of one packed prefill pass
    // the Q4_K depth override (src/c_api.cpp:532-578): dd.* of a second GGUF, used for the depth
    // codes of the sessions flagged with session_set_q4; loading again replaces it
    void load_q4_depth(const std::string & path);
    bool has_q4_depth() const { return has_q4_; }
    bool session_set_q4(int sid, bool on);
    int session_count() const { return (int) sid_to_slot_.size(); }
    bool session_active(int sid) const;
    bool session_exists(int sid) const { return sid_to_slot_.count(sid) > 0; }

    // K frame steps over a session list (reference: src/c_api.cpp:601-949). frames_out is
    // [K][n][width]; rows of sessions not stepped keep their initial contents. Depth codes are
    // the argmax unless the batch holds a two-branch session or `sampled_depth` is set (then
    // each session's depth sampler, src/depth_decoder.cpp:130-247); `depth_seeds` [n] reseeds the
    // depth draws per call (src/c_api.cpp:468).
    // after_graph (optional) is called after each step's graph launch, before the host copies
    // and the synchronisation: work it enqueues on the engine's stream reads that step's frames
    // on the device (device_frames(k)) and completes before step() returns
    StepResult step(const int * sids, int n, int K, const uint32_t * seeds, bool burst, int * frames_out,
                    int width, int * next_out, bool fill_inactive, bool sampled_depth = false,
                    const uint32_t * depth_seeds = nullptr, const StepForce * force = nullptr,
                    const std::function<void(int)> * after_graph = nullptr);

    // device-resident run of K steps for the current batch (no host copies): timing entry
    void step_device_only(int K);
    // K frame steps of the listed sessions (every one active) without host copies or a host
    // synchronisation; after each step's graph, after_step(k) may enqueue more work on the
    // engine's stream that reads that step's frames (device_frames(k), row i = session i)
    void step_launch_device(const int * sids, int n, const uint32_t * seeds, int K, const std::function<void(int)> & after_step);
    const int * device_frames(int k) const { return frames_all_ + (size_t) k * cur_R_ * cfg.nc; }
    // a counter that changes every time a session with this id is created (0: no such session)
    unsigned long long session_epoch(int sid) const {
        auto it = sid_epoch_.find(sid);
        return it == sid_epoch_.end() ? 0ull : it->second;
    }
    void sync();
    cudaStream_t stream() const { return stream_; }

    // debug accessors for parity tests
    void debug_hidden(int sid, float * out);
    void debug_depth(int n, const float * hidden, const int * cb0, const int * forced, int * codes_out,
                     float * logits_out);
    void debug_gemv(const char * tensor, int sub, int rows, const float * x, float * y);
    // one eager frame step of the current batch with CUDA events around every dequant-GEMM and
    // the persistent depth decoder: out = {step_ms, gemm_ms, gemm_launches,
    // gemm_algorithmic_bytes, launches, depth_ms, depth_algorithmic_bytes}
    void profile_step(double * out);
    size_t depth_bytes_per_step() const;
    // average microseconds of `iters` back-to-back launches of one dequant-GEMM (epilogue kind)
    double bench_gemv(const char * tensor, int sub, int rows, int iters, int epi);
    // one launch of a matrix as the frame step holds it (fused q/k/v, gate/up interleaved with
    // its SwiGLU or GeGLU epilogue, a depth head) on x [rows][K] (f32, rounded to f16); y is
    // [rows][M] for store epilogues, [rows][M/2] for the gated ones. With repeats > 0 the same
    // launch is captured `repeats` more times in one graph (programmatic dependent launch on, as
    // in the frame step), each result bit-compared on the device with the first; returns the
    // number of differing 32-bit words. flags bit 0 captures the repeats without programmatic
    // dependent launch; `where` (optional) receives the first `cap` differences as (word index,
    // repeat) pairs
    long long debug_gemm(const char * name, int rows, const float * x, float * y, int repeats, int flags = 0,
                         int * where = nullptr, int cap = 0);
    // test hook: the cb0 sampler on given logits [rows][V] (V <= 4096) with the given top-k,
    // temperature and top-p (no suppression, no penalty), `draws` draws per row from Philox key
    // seed + row; force_sort takes the full sort even where top-k <= 64 selects. picks [draws][rows]
    void debug_sample(const float * logits, int V, int rows, int top_k, float temp, float top_p, uint32_t seed, int draws,
                      int force_sort, int * picks);
    // test hook: the grid-barrier poll limit of the persistent depth launches debug_depth makes
    // (0 restores the default); frame-step graphs never use it
    void set_debug_grid_spin(long long polls) { dbg_grid_spin_ = polls > 0 ? polls : 0; }
    // the resident matrix a name refers to and the epilogue the frame step uses with it, or null
    const QMat * resident_any(const char * name, int * epi) const;
    // one eager persistent depth launch for the current batch with its timeline recorded:
    // out = {n_phases, grid, slots, type[n_phases], timeline[n_phases][grid][slots]} (microseconds
    // from the first CTA's start, -1 where a slot was not reached); returns the doubles written
    // (the size needed when out is null), 0 when the persistent decoder is not in use
    int depth_trace(double * out, int capacity);
    // y[rows][ldy] = x16[rows][ldx] . W^T for a resident, unfused Q8_0 matrix, allocating
    // nothing (static-scratch GEMV); asynchronous on `s` (the engine's stream when null)
    void gemm_noalloc(const char * tensor, int rows, const half * x16, int ldx, float * y, int ldy, cudaStream_t s);
    size_t weight_bytes_per_step() const;
    size_t kv_bytes_per_position() const;

    int max_rows() const { return rmax_; }
    const GgufFile & gguf() const { return gg_; }
    int launches_per_step() const { return graph_nodes_; }
    int nc() const { return cfg.nc; }

private:
    // loading
    QMat load_qmat(const std::vector<const GgufTensor *> & parts, bool interleave_pairs, int row0 = 0, int rows = -1);
    QRows load_qrows(const GgufTensor * t);
    float * load_f32(const std::string & name, int expect);
    const GgufTensor * need(const std::string & name);
    void alloc_buffers();
    void build_rope_tables();

    // execution
    void gemv(const QMat & w, const half * x16, int ldx, int rows, const GemvOut & out);
    void launch_gemm(const QMat & w, const half * x16, int ldx, int rows, const GemvOut & out);
    // graph flags: kFlagSeeds (per-row reseed of the samplers), kFlagSampled (sampled depth),
    // kFlagDepthSeeds (per-call depth seeds)
    // kFlagQ4 (some rows take their depth codes from the Q4_K override: two masked depth passes)
    // kFlagForce (teacher-forced frames, no cb0 draw), kFlagFeed (the backbone consumes given frames)
    static constexpr int kFlagSeeds = 1, kFlagSampled = 2, kFlagDepthSeeds = 4, kFlagQ4 = 8, kFlagForce = 16,
                         kFlagFeed = 32;
    void depth_pass(int R, int flags, int set, const StepArgs & sa);
    void load_depth_weights();
    void swap_depth_sets();
    const GgufFile & src() const { return src_ ? *src_ : gg_; }
    void enqueue_step(int R, int flags);
    // the part of step() before its graph launches: rows (the listed sessions, then the partners
    // of two-branch sessions), flags, device uploads, the graph; returns R, 0 when no listed
    // session is active (rs: row -> slot)
    int setup_step(const int * sids, int n, int K, const uint32_t * seeds, bool sampled_depth, const uint32_t * depth_seeds,
                   const StepForce * force, std::vector<int> & rs, cudaGraphExec_t * g_out);
    void prefill_prompt(int slot, const std::vector<std::vector<int>> & segs, const int * ref_codes, int ref_frames,
                        float * logits);
    void depth_layer(int l, int rows, int R, int n_new, int start);
    void bb_decode_layer(int l, int R);
    void te_forward(const std::vector<int> & tokens, float * out_rows);
    // text encoder over several token segments at once: out [sum of lengths][hidden], segment order
    void te_forward_packed(const std::vector<const std::vector<int> *> & segs, float * out_rows);
    // backbone prefill of the packed prompt rows in px_: segment b = rows [first_b, first_b + len_b)
    // of slot_b; writes each segment's last hidden to hid32[slot] and its lm_head logits to logits[b]
    void bb_prefill_packed(const std::vector<int4> & segs, float * logits);
    void bb_prefill(int slot, int T, float * logits);
    void ensure_prefill_capacity(int T);
    cudaGraphExec_t graph_for(int R, int flags);
    const QMat * resident_matrix(const char * tensor) const;

    // persistent depth decoder: one schedule (phase table + activation tensor maps) per batch
    // size R; null when R or the model shape is outside what the kernel supports
    struct DpPlan {
        DpPhase * dev = nullptr;
        int n = 0;
        DpMaps maps;
    };
    const DpPlan * depth_plan(int R);
    void enqueue_depth(int R, const int * forced_dev, float * logits_dev, unsigned long long * trace = nullptr,
                       const int * row_set = nullptr, long long grid_spin = 0);
    // clears the device error word, then throws `what` with the code
    [[noreturn]] void raise_device_error(int code, const std::string & what);
    long long dbg_grid_spin_ = 0;  // grid-barrier poll limit of debug_depth launches (0: default)
    bool dp_supported(int R) const;
    int acquire_slot(int sid, int n_pages, bool register_sid = true);
    void release_slot(int slot);

    GgufFile gg_;
    Tokenizer tok_;
    cudaStream_t stream_ = nullptr;
    std::vector<void *> allocs_;
    template <class T> T * dalloc(size_t n);

    // weights
    std::vector<LayerW> bb_, dd_, te_;
    QMat lm_head_, dd_in_, te_proj_;
    std::vector<QMat> dd_head_;
    // the other depth weight set (swapped in while a pass for the Q4_K override is enqueued)
    std::vector<LayerW> q4_dd_;
    QMat q4_dd_in_;
    std::vector<QMat> q4_dd_head_;
    float * q4_dd_out_norm_ = nullptr;
    int cur_set_ = 0;
    bool has_q4_ = false;
    std::unique_ptr<GgufFile> q4_gg_;
    const GgufFile * src_ = nullptr;   // file the loaders read (the model's own when null)
    std::vector<void *> q4_allocs_;
    QRows audio_embd_, te_embd_;
    float * bb_out_norm_ = nullptr, * dd_out_norm_ = nullptr, * te_out_norm_ = nullptr;
    float2 * rope_bb_ = nullptr, * rope_dd_ = nullptr, * rope_te_full_ = nullptr, * rope_te_slide_ = nullptr;
    int rope_bb_max_ = 0, rope_te_max_ = 0;
    int vbb_ = 0;  // lm_head rows
    bool has_te_ = false;

    // KV pool and sessions
    half * kv_pool_ = nullptr;
    int n_pages_ = 0, max_pages_ = 0, max_slots_ = 0;
    std::vector<int> free_pages_;
    int * page_table_ = nullptr;
    SessState * st_ = nullptr;
    uint16_t * hist_ = nullptr;
    int hist_ld_ = 0;
    float * hid32_ = nullptr;
    std::vector<SlotHost> slots_;
    std::vector<int> free_slots_;
    std::unordered_map<int, int> sid_to_slot_;
    std::unordered_map<int, unsigned long long> sid_epoch_;
    unsigned long long epoch_ctr_ = 0;

    // step buffers
    int rmax_ = 0, kmax_ = 0;
    int * row_slot_ = nullptr, * row_active_ = nullptr, * next_ = nullptr, * cur_frames_ = nullptr;
    int * frames_all_ = nullptr, * step_ctr_ = nullptr, * any_active_ = nullptr, * slot_scalar_ = nullptr;
    uint32_t * seeds_ = nullptr, * dseeds_ = nullptr;
    int * row_pair_ = nullptr, * create_rows_ = nullptr, * row_set_ = nullptr;
    int * force_all_ = nullptr, * feed_all_ = nullptr, * cur_force_ = nullptr, * cur_feed_ = nullptr;
    half * din16_ = nullptr, * dh16_ = nullptr, * dff16_ = nullptr, * datt16_ = nullptr;
    float * dx_ = nullptr, * dqkv_ = nullptr, * dkv_ = nullptr, * dlog_ = nullptr;
    half * bh16_ = nullptr, * bff16_ = nullptr, * batt16_ = nullptr;
    float * bx_ = nullptr, * bqkv_ = nullptr, * blog_ = nullptr;
    GemvScratch scr_;
    int cur_R_ = 0, cur_flags_ = 0;
    std::map<std::pair<int, int>, cudaGraphExec_t> graphs_;
    std::map<std::pair<int, int>, cudaGraph_t> graph_defs_;

    // prefill buffers (grown on demand)
    int tmax_ = 0;
    float * px_ = nullptr, * pqkv_ = nullptr, * plog_ = nullptr, * tx_ = nullptr, * tqkv_ = nullptr;
    float * ttmp_ = nullptr;
    half * tk_ = nullptr, * tv_ = nullptr;  // text encoder keys and values (f16, the attention's operand type)
    half * ph16_ = nullptr, * pff16_ = nullptr, * patt16_ = nullptr, * th16_ = nullptr, * tff16_ = nullptr,
         * tatt16_ = nullptr;
    int * ptok_ = nullptr, * pframes_ = nullptr;
    // packed prefill: per-row segment, segments, attention query blocks, row copy indices, the
    // text-encoder / audio-embedding output rows before they are placed, logits per segment
    int * pseg_ = nullptr, * pidx_ = nullptr, * pslot_ = nullptr, * ppair_ = nullptr, * pnext_ = nullptr;
    int4 * psegs_ = nullptr;
    int2 * pqb_ = nullptr;
    float * pstage_ = nullptr, * plast_ = nullptr, * plogs_ = nullptr;
    std::vector<void *> prefill_allocs_;

    // profiling of one eager step
    struct ProfRec { cudaEvent_t a, b; double bytes; };
    std::vector<ProfRec> * prof_ = nullptr;
    int launches_ = 0;
    int graph_nodes_ = 0;
    bool use_umma_ = true;
    bool use_dp_ = true;
    int dp_grid_ = 0;
    std::map<int, DpPlan> dp_plans_;
    // in_proj of every input code of sub-steps 2..nc-1 for each depth weight set (see DpParams::in_tab)
    float * dp_in_tab_[2] = { nullptr, nullptr };
    float * dp_qkv_tab_[2] = { nullptr, nullptr };  // layer-0 q/k/v of the same inputs (DpParams::qkv_tab)
    float * dp_P2_ = nullptr;
    float * battn_part_ = nullptr;  // split-KV partials of the backbone decode attention
    int * battn_ctr_ = nullptr;     // their per-(row, kv head) arrival counters
    static constexpr int kAttnMaxSplits = 8;
    const float * in_tab_for_set();
    float * dp_P_ = nullptr;
    size_t dp_P_floats_ = 0;
    float * dp_ss_ = nullptr;
    unsigned * dp_bar_ = nullptr;
    int * err_ = nullptr;
    cudaEvent_t dprof_a_ = nullptr, dprof_b_ = nullptr;
};

}  // namespace bzb
