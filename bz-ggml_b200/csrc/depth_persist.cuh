// Persistent depth decoder: every sub-step of one frame step's depth decode (codebooks 1..nc-1,
// reference src/depth_decoder.cpp:249-365) in one launch of one CTA per SM, with grid-wide
// phase barriers instead of kernel boundaries.
#pragma once

#include "kernels.cuh"

#include <cuda.h>

namespace bzb {

enum DpType { DP_GEMM = 0, DP_REDUCE = 1, DP_ATTN = 2, DP_ARGMAX = 3 };
enum DpEpi { DPE_PARTIAL = 0, DPE_SWIGLU = 1 };
constexpr int kDpTraceSlots = 57;  // 9 phase events + 3 x 16 per-chunk events

// One phase of the schedule. GEMM phases split a Q8_0 matrix (tcgen05 layout) into units of one
// 128-row weight tile, one K range and up to 64 activation rows; CTA c runs units c', c' + grid,
// ... where c' is c rotated by the phase index.
struct alignas(16) DpPhase {
    int type = DP_GEMM;
    int q4 = 0;                     // GEMM weight chunk format (UMat::q4)
    // GEMM
    const uint8_t * blk = nullptr;  // tcgen05 layout (UMat::blk)
    int MT = 0, KC = 0, M = 0, splits = 1, kc_per = 0, n_units = 0;
    int row_chunks = 1; // activation rows are taken in chunks of 64 (one unit each)
    int map = 0;        // activation tensor map (DpMaps index)
    int b_row0 = 0;     // first activation row read
    int nb = 0;         // MMA N: activation rows per unit, a multiple of 16, at most 64
    int rows = 0;       // activation rows whose results are kept
    int epi = DPE_PARTIAL;
    int out_ld = 0;     // partial (and arg-max): row pitch of the partials, M rounded up to 4; SwiGLU: the FFN width
    int ss_row0 = 0;    // rows whose RMS scale applies (SwiGLU, arg-max) start here in `ss`
    // consumers of partials
    int S = 1;          // splits of the GEMM that produced the partials
    int resid = 0;      // REDUCE: add the sum into the residual stream
    const float * norm_w = nullptr;  // REDUCE: weight of the norm that the next GEMM applies
    int layer = 0, start = 0, n_new = 1;  // ATTN
    int j = 0;          // ARGMAX: codebook
    int alt = 0;        // ATTN: the q/k/v come from P2 (written by the arg-max phase), not from partials
};

// activation buffers as 3-D tensors {64 columns, rows, K / 64 chunks}: one TMA box brings up to
// 4 consecutive 64-wide chunks of up to 64 rows, each chunk landing as its own 128-byte-swizzled
// tile
constexpr int kDpGroup = 4;
struct DpMaps {
    CUtensorMap m[8];   // {in, h, att, ff} x {box of 2R rows, box of R rows}
};

struct DpParams {
    const DpPhase * phases = nullptr;
    int n_phases = 0;
    int R = 0, nc = 0, vs = 0, D = 0, H = 0, ffn = 0, n_head = 0, n_kv = 0, hd = 0;
    float eps = 0.0f, attn_scale = 0.0f;
    const float2 * rope = nullptr;      // [positions][hd/2] (cos, sin)
    float * kv = nullptr;               // depth cache, layer stride kv_layer
    size_t kv_layer = 0;
    float * P = nullptr;                // split-K partials [S][rows][M]
    float * P2 = nullptr;               // layer 0's q/k/v rows from qkv_tab [R][q + 2 kv]
    float * x = nullptr;                // residual stream [2R][D] f32
    half * h16 = nullptr;               // x * norm weight [2R][D] (the next GEMM's input)
    float * ss = nullptr;               // per-row sums of squares in 64-column chunks [2R][D/64]
    half * att16 = nullptr;             // attention output [2R][D]
    half * g16 = nullptr;               // SwiGLU output [2R][ffn]
    half * din16 = nullptr;             // in_proj input [2R][H]
    QRows embd;                         // audio embedding table
    // in_proj of every code of codebooks 1..nc-2, [nc-2][vs][D] f32, or null: the arg-max phase
    // then writes sub-step j+1's input (x, x * in_norm, chunk sums of squares) from row
    // (j-1, code) instead of the embedding gather, and the plan has no in_proj phases after the
    // first sub-step
    const float * in_tab = nullptr;
    const float * in_norm = nullptr;    // layer 0's attention norm weight
    // layer 0's q/k/v projection of the same inputs, [nc-2][vs][q + 2 kv] f32, or null: with it
    // the arg-max phase also writes P2 and the plan has no layer-0 qkv phase after the first
    // sub-step (the RMS scale is applied by the attention phase, as for partials)
    const float * qkv_tab = nullptr;
    const int * row_active = nullptr;   // [R]
    const int * row_set = nullptr;      // [R] depth weight set of each row, or null (all rows)
    int set_id = 0;                     // the set this launch's weights are; other rows are left alone
    int * frames = nullptr;             // [R][nc]
    const int * forced = nullptr;       // [R][nc-1] teacher-forced codes, or null
    float * logits_out = nullptr;       // [R][nc-1][vs] or null
    unsigned * bar = nullptr;           // phase-arrival counter, zero at launch
    int * err = nullptr;
    // polls of a grid phase barrier before the CTA gives up (error code 3); 0 keeps the default
    // (about a second). A shorter limit lets a test make the barrier run out on purpose.
    long long grid_spin = 0;
    // optional timeline [n_phases][grid][kDpTraceSlots] of %globaltimer (ns) per CTA and phase:
    // 0 epilogue start, 1 epilogue end, 2 activation loads start, 3 first activation chunk
    // landed, 4 first weight tile dequantised, 5 last MMA issued, 6 accumulator ready,
    // 7 first weight copy issued, 8 first weight chunk landed; for chunks c < 16 of the unit:
    // 9 + c activation chunk ready, 25 + c weight tile ready (as the MMA issuer sees them),
    // 41 + c MMAs issued;
    // null in production launches
    unsigned long long * trace = nullptr;
};

// activation rows [rows][K] f16 with row stride ldx, read as 64 x box_rows tiles in the
// 128-byte swizzle; rows past `rows` read as zero (umma_gemm.cu)
CUtensorMap make_x_map(const half * x, int K, int ldx, int rows, int box_rows);
// the same rows viewed as {64, rows, K / 64}: boxes of `group` consecutive 64-wide chunks
CUtensorMap make_x_group_map(const half * x, int K, int ldx, int rows, int box_rows, int group);

// grid size (CTAs) of the persistent kernel on the current device; 0 when it cannot run
int depth_persist_grid();
void init_depth_persist_attributes();
// the counter at p.bar must be zero (the launcher clears it on `s` first)
void launch_depth_persist(const DpParams & p, const DpMaps & maps, int grid, cudaStream_t s);

}  // namespace bzb
