// Device kernels of the B200 decode engine and their host-side launchers.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace bzb {

// Q8_0 weight matrix [M rows, K] repacked for the dequant-GEMM: for each 16-row tile and
// 32-wide K block, 32 lanes x 16 bytes laid out as the lanes' mma.m16n8k16 A fragments
// (two k16 halves), plus one half2 (scale of row g, scale of row g+8) per lane group.


// the same Q8_0 matrix in the tcgen05 kernels' layout: one contiguous block per (128-row tile,
// 64-wide K chunk), tiles major and chunks minor, so that consecutive chunks of a tile are
// consecutive blocks (one bulk copy can bring several). A block is 4 x 128 rows x 16 bytes of
// int8 (piece (block half, 16-byte half) major, row minor) followed by 2 x 128 f16 block scales
// ((block half) major, row minor). Gate/up pairs interleave in 16-row groups.
constexpr int kUChunkBytes = 128 * 64 + 2 * 128 * 2;
// The same chunk for Q4_K weights (w = d scale q - dmin min per 32-value sub-block, q in [0, 15]):
// the 4-bit quants [half][row][16 B] (each 32-bit word holds 8 consecutive values, even ones in
// nibbles 0-3 and odd ones in nibbles 4-7), then 8 bytes per row: the super-block's f16 d and
// dmin, the two sub-blocks' 6-bit scales (one byte each), then their 6-bit mins. The kernels form
// d scale and dmin min as exact f32 products, so a weight is rounded once, to f16.
constexpr int kUChunkBytesQ4 = 128 * 32 + 128 * 8;
struct UMat {
    const uint8_t * blk = nullptr;
    int M = 0, MT = 0, K = 0, KC = 0;
    int q4 = 0;                    // chunk format: 0 Q8_0, 1 Q4_K
};
__host__ __device__ inline int umat_chunk_bytes(int q4) { return q4 ? kUChunkBytesQ4 : kUChunkBytes; }

struct QMat {
    const uint4 * qs = nullptr;    // [MT][KB][32] uint4
    const half2 * ds = nullptr;    // [MT][KB][8]
    int M = 0, MT = 0, K = 0, KB = 0;
    UMat u;                        // tcgen05 layout of the same weights (when K % 64 == 0)
};

// Q8_0 rows kept for row gathers (embeddings): int8 values and f16 block scales.
// embedding rows: value = qs * ds - ms per 32-value block (ms null for Q8_0; Q4_K rows keep
// their 4-bit values in qs and the sub-block scale and min in ds and ms)
struct QRows {
    const int8_t * qs = nullptr;   // [rows][K]
    const half * ds = nullptr;     // [rows][K/32]
    const half * ms = nullptr;     // [rows][K/32] or null
    int rows = 0, K = 0;
};

// per-session state resident on the device
struct SessState {
    int active;
    int pos;          // backbone positions already in the KV cache
    int steps;        // frames generated since creation
    int max_tokens;
    int last_cb0;
    uint32_t key;     // Philox key (the session's current seed)
    uint32_t draw;    // Philox draw counter under that key
    // cb0 sampler (src/sampling.cpp:9-60 parameters; the generator ABI fixes T 0.9, top-k 50,
    // top-p 1, repetition 1.1, src/c_api.cpp:343-351)
    int top_k;
    float temp, top_p, rep;
    float cfg;        // guidance scale of a two-branch session, 1 for a single branch
    // depth sampler of the sampled-depth mode (breeze.depth_* of the GGUF, src/depth_decoder.cpp:134-140)
    float dtemp, dtop_p;
    int dtop_k;
    int pad;
};

enum Epilogue { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_GEGLU = 3 };

struct GemvOut {
    int kind = EPI_STORE;
    float * f32 = nullptr;   // STORE / RESID target [rows][ld]
    half * f16 = nullptr;    // SWIGLU / GEGLU target [rows][ld]
    int ld = 0;
};

struct GemvScratch {
    float4 * ws = nullptr;   // split-K partials
    size_t ws_elems = 0;     // capacity in float4
    int * counters = nullptr;
    int n_counters = 0;
};

// sets the kernels' shared-memory limits; once per device before the first launch or capture
void init_kernel_attributes();
// launches of this thread use programmatic dependent launch while `on` (graph capture only)
void set_pdl_scope(bool on);

// y[rows, M] = x16[rows, K] . W^T with the chosen epilogue; rows may exceed 64 (column chunks)
// fit_scratch: choose at most the split-K plan `scr` holds (the allocation-free entry point's
// fixed scratch) and ignore the BZB_GEMV_SPLITS override
void launch_gemv(const QMat & w, const half * x16, int ldx, int rows, const GemvOut & out,
                 const GemvScratch & scr, cudaStream_t s, bool fit_scratch = false);

void repack_q8(const uint8_t * raw_dev, int M, int K, uint4 * qs, half2 * ds, cudaStream_t s);

// The same GEMV with its split-K partials and tile counters in fixed-size static device arrays
// instead of caller-provided scratch, for callers that must not allocate (see
// bzb_generator_gemm_noalloc). Limits: rows <= kStaticGemvMaxRows, and the split plan must fit
// kStaticGemvWsElems partials and kStaticGemvCounters counters (checked: std::runtime_error).
// The first call on a device looks up the arrays' addresses (once per device, with that device
// current); make it before any stream capture. Concurrent calls on one device share the
// arrays and race.
constexpr int kStaticGemvMaxRows = 256;
constexpr size_t kStaticGemvWsElems = (size_t) 640 << 10;   // float4: 10 MiB of partials
constexpr int kStaticGemvCounters = 4096;
void launch_gemv_static_scratch(const QMat & w, const half * x16, int ldx, int rows, float * y, int ldy,
                                cudaStream_t s);

// tcgen05 dequant-GEMM (umma_gemm.cu): same contract as launch_gemv; `err` receives 1 if a
// bounded pipeline wait gave up
void init_umma_attributes();
void repack_umma(const uint8_t * raw_dev, int M, int K, uint8_t * blk, cudaStream_t s);
// Q4_K rows (144-byte super-blocks of 256 values, K % 256 == 0) into kUChunkBytesQ4 chunks
void repack_umma_q4k(const uint8_t * raw_dev, int M, int K, uint8_t * blk, cudaStream_t s);
void launch_umma_gemm(const UMat & w, const half * x16, int ldx, int rows, const GemvOut & out, int * err,
                      cudaStream_t s, bool pdl);
bool pdl_scope();
// runs the tcgen05 pipelines' bounded mbarrier wait (limit polls) on a barrier nothing arrives on,
// in a one-thread kernel on the current device; returns the error code the wait recorded
int probe_mbar_timeout(long long limit);
void split_q8_rows(const uint8_t * raw_dev, int rows, int K, int8_t * qs, half * ds, cudaStream_t s);
// Q4_K rows into 4-bit values (one per byte), sub-block scales and mins
void split_q4k_rows(const uint8_t * raw_dev, int rows, int K, int8_t * qs, half * ds, half * ms, cudaStream_t s);

// out16[r] = f16(rmsnorm(x[r]) * w) (and out32 when non-null) for rows [r0, r0 + n)
void launch_rmsnorm(const float * x, int ldx, const float * w, int D, float eps, half * out16, int ld16,
                    float * out32, int ld32, int r0, int n, const int * row_map, cudaStream_t s);
// dst[dst_idx ? dst_idx[i] : i][:cols] = src[src_idx ? src_idx[i] : i][:cols] for i < n (f32 rows)
// rows [row0, row0 + n) of a quantised table as f16 rows [n][K]: f16(q * d - m), the embedding
// value the depth decoder's input gather writes
void launch_qrows_to_f16(const QRows & e, long long row0, int n, half * out, cudaStream_t s);
// out[r][c] = f16(x[r][c] * w[c]) for n rows of D columns (the norm product a GEMM phase reads)
void launch_scale_rows_f16(const float * x, const float * w, int n, int D, half * out, cudaStream_t s);
void launch_copy_rows(const float * src, int lds, const int * src_idx, float * dst, int ldd, const int * dst_idx, int n,
                      int cols, cudaStream_t s);
// x[r] += rmsnorm(t[r]) * w  (Gemma post-norms)
void launch_norm_add(float * x, const float * t, int D, const float * w, float eps, int rows, cudaStream_t s);
// x += RMSNorm(t) w, then y16 = RMSNorm(x) w2 (row stride ld16)
void launch_norm_add_norm(float * x, const float * t, int D, const float * w, float eps, const float * w2, half * y16,
                          int ld16, int rows, cudaStream_t s);

// dst[r] = f16/f32 dequantised row idx[r] of an embedding table, scaled
void launch_embed_rows(const QRows & e, const int * idx, int n, float scale, float * out32, half * out16,
                       int ld, cudaStream_t s);
// x[r] = sum over codebooks of audio_embd[frames[r][cb] + cb*vs]
void launch_audio_embed(const QRows & e, const int * frames, int ld_frames, int nc, int vs, int n,
                        float * out32, const int * row_active, cudaStream_t s);

struct AttnKV {
    // paged f16 backbone cache
    half * pool = nullptr;
    const int * page_table = nullptr;   // [slot][max_pages]
    int max_pages = 0, n_layer = 0, layer = 0;
    // flat f32 cache (depth decoder) [rows][cap][2][n_kv][hd] for this layer
    float * flat = nullptr;
    int cap = 0;
};

struct AttnDecodeArgs {
    const float * qkv = nullptr;
    int ldq = 0;
    int n_head = 0, n_kv = 0, hd = 0;
    int R = 0;              // sessions (rows per token)
    int n_new = 1;          // new tokens per session (1 or 2); token i of row b is at b + i*R
    const int * row_slot = nullptr;   // session slot of each row (paged mode)
    const int * row_active = nullptr; // 1 when the row is stepped this frame
    const SessState * st = nullptr;   // start position = st[slot].pos when non-null
    int start = 0;                    // otherwise this start position
    const float * q_norm = nullptr, * k_norm = nullptr;
    float eps = 0;
    const float2 * rope = nullptr;    // [pos][hd/2] (cos, sin)
    float scale = 0;
    AttnKV kv;
    half * out = nullptr;
    int ldo = 0;
    // split-KV: each (session, kv head) runs `splits` CTAs over equal 32-aligned position ranges,
    // each writing its (max, sum, weighted values) per query head to `part`; the last CTA to
    // arrive (per-(session, kv head) counter, left at zero) combines them. 1: no split.
    int splits = 1;
    float * part = nullptr;   // [R][n_kv][splits][4 heads][2 tokens][hd + 2]
    int * counters = nullptr; // [R][n_kv], zero between launches
};
void launch_attn_decode(const AttnDecodeArgs & a, bool paged, cudaStream_t s);

struct PrefillArgs {
    float * qkv = nullptr;  // [T][ldq], q normed/roped in place by launch_qk_prep
    int ldq = 0, T = 0, start = 0;
    int n_head = 0, n_kv = 0, hd = 0;
    const float * q_norm = nullptr, * k_norm = nullptr;
    float eps = 0;
    const float2 * rope = nullptr;
    float scale = 0;
    // paged destination (slot's page row) or flat f16 k/v [T][n_kv][hd]
    AttnKV kv;
    const int * page_row = nullptr;
    half * flat_k = nullptr, * flat_v = nullptr;
    int window = 0;         // bidirectional window (0 = full) for the text encoder
    bool causal = true;
    half * out = nullptr;
    int ldo = 0;
    // packed prefill of several sequences in one launch (null: one sequence from `start`): each
    // row's segment, each segment's {first row, length, KV slot (paged), 0}, and the attention's
    // query blocks {segment, first query row within it}; positions start at 0 in every segment
    const int * row_seg = nullptr;
    const int4 * segs = nullptr;
    const int2 * qblocks = nullptr;
    int n_qblocks = 0;
};
void launch_qk_prep(const PrefillArgs & a, bool paged, cudaStream_t s);
constexpr int kPrefillQBlock = 64;  // query rows per attention-prefill CTA
void launch_attn_prefill(const PrefillArgs & a, bool paged, cudaStream_t s);

struct StepArgs {
    int R = 0, nc = 0, vs = 0, H = 0;
    const int * row_slot = nullptr;
    int * row_active = nullptr;
    SessState * st = nullptr;
    const float * hid32 = nullptr;  // [slot][H] last normed backbone hidden
    QRows embd;
    half * din16 = nullptr;         // [2R][H]
    int * frames = nullptr;         // current frame [R][nc]
    int * step_ctr = nullptr;       // burst step index
    int * any_active = nullptr;     // [Kmax]
    // depth passes of one weight set: rows whose row_set differs from set_id are left alone
    const int * row_set = nullptr;
    int set_id = 0;
    // teacher-forced steps: codes [R][nc] of this step (cb0 always, depth codes where >= 0)
    const int * force = nullptr;
};
void launch_step_init(const StepArgs & a, cudaStream_t s);
// codes[r] = first argmax of logits[r]; frames[..][r][col] = code; when gather_cb >= 0 the
// next sub-step's input row din16[r] = embedding row (gather_cb*vs + code)
void launch_argmax_gather(const StepArgs & a, const float * logits, int ld, int V, int col, int gather_cb,
                          cudaStream_t s);

// Row pairing of two-branch (classifier-free guidance) sessions: row_pair[r] = the row of r's
// unconditional branch (r leads), -2 - leader for that branch's own row (r follows), -1 for a
// single-branch row. A leader's logits are combined as lu + cfg (lc - lu) (src/c_api.cpp:148-155,
// src/depth_decoder.cpp:149-152) and its pick is written to both rows.
//
// Sampled depth sub-step (src/depth_decoder.cpp:130-161, 163-247): codes[r] = the depth sampler's
// pick from logits[r] (the session's dtemp / dtop_k / dtop_p; dtop_k 1 is the first argmax), with
// the Philox uniform for (key, draw, codebook col): key/draw are the session's, or (seeds[r] +
// step, 0) / (dseeds[r], 0) when those per-row reseeds are given; frames and the next input row
// as launch_argmax_gather.
struct DepthSampleArgs {
    StepArgs s;
    const float * logits = nullptr;
    int ld = 0, V = 0, col = 1, gather_cb = -1;
    const int * row_pair = nullptr;
    const uint32_t * seeds = nullptr;    // batched reseed: key = seeds[r] + step
    const uint32_t * dseeds = nullptr;   // per-call depth seed: key = dseeds[r]
};
void launch_depth_sample_gather(const DepthSampleArgs & a, cudaStream_t s);

struct SampleArgs {
    const float * logits = nullptr;
    int ld = 0, V = 0, R = 0;
    const int * row_slot = nullptr;
    const int * row_active = nullptr;
    SessState * st = nullptr;
    uint16_t * hist = nullptr;      // [slot][hist_ld]
    int hist_ld = 0;
    int sup_lo = 0, sup_hi = 0, eos = 0;
    // temperature, top-k, top-p, repetition penalty and guidance scale are the session's (SessState)
    const int * row_pair = nullptr;     // two-branch pairing (see DepthSampleArgs), or null
    const uint32_t * seeds = nullptr;   // per-row reseed (key = seeds[r] + step) when non-null
    const int * step_ctr = nullptr;
    int * next_out = nullptr;           // [R]
    int clamp_on_finish = 0;            // burst: last_cb0 = -1 on finish
    int advance_pos = 1;
    int update_hist_first = 0;          // prefill: first cb0 is always recorded
    int force_sort = 0;                 // test hook: the full sort even for top-k <= 64
};
void launch_sample(const SampleArgs & a, cudaStream_t s);
// teacher-forced steps: copies step *step_ctr's rows of force_all / feed_all ([K][n] ints) into
// cur_force / cur_feed (feed may be null)
void launch_stage_forced(const int * force_all, const int * feed_all, const int * step_ctr, int n, int * cur_force,
                         int * cur_feed, cudaStream_t s);
// teacher-forced steps draw no cb0: every active leading row advances its (and its pair's)
// position and step count, next_out[r] = 0 (still active)
void launch_advance(const int * row_slot, const int * row_active, const int * row_pair, SessState * st, int R,
                    int * next_out, cudaStream_t s);
// copies the current frame into frames_all[step] and advances the burst step counter
void launch_frames_commit(const int * cur, int * frames_all, int n, int * step_ctr, cudaStream_t s);
// adds to *count the number of 32-bit words of b that differ bitwise from a (n_words each); with
// `where` the first `cap` differences overall are recorded as (word index, tag) int pairs
void launch_bits_diff(const void * a, const void * b, size_t n_words, int * count, cudaStream_t s,
                      int * where = nullptr, int cap = 0, int tag = 0);

// Philox4x32-10 uniform in [0, 1): top 24 bits of the first output word for (key, draw)
__host__ __device__ inline uint32_t philox_word0(uint32_t key, uint32_t draw_lo, uint32_t draw_hi) {
    uint32_t c0 = draw_lo, c1 = draw_hi, c2 = 0, c3 = 0, k0 = key, k1 = 0x42524545u;
    for (int r = 0; r < 10; r++) {
        const uint64_t p0 = (uint64_t) 0xD2511F53u * c0, p1 = (uint64_t) 0xCD9E8D57u * c2;
        const uint32_t hi0 = (uint32_t) (p0 >> 32), lo0 = (uint32_t) p0;
        const uint32_t hi1 = (uint32_t) (p1 >> 32), lo1 = (uint32_t) p1;
        const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c0;
}

}  // namespace bzb
