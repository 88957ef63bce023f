// tcgen05 (5th-generation tensor core) dequant-GEMM for Q8_0 and Q4_K weights, sm_100a.
//
// y[rows, M] = x[rows, K] . W^T with W stored as Q8_0. Each CTA owns one 128-row weight tile
// (the MMA's M), up to 64 activation rows (the MMA's N) and a K range, processed in 64-wide
// chunks, two chunks per pipeline stage, by a warp-specialised pipeline:
//   * a loader warp streams each stage's int8 weights and block scales (2 x 8.5 KB, contiguous
//     in the repacked layout) with one 1-D bulk async copy into a 4-stage raw ring;
//   * a second loader warp brings the activation rows with 2-D TMA tensor loads that write the
//     128-byte-swizzled K-major layout the MMA reads;
//   * 8 producer warps dequantise the raw ring (one Q8_0 block of one weight row per thread)
//     into the swizzled f16 A stage;
//   * one MMA warp issues four tcgen05.mma.cta_group::1.kind::f16 (128 x N x 16) per chunk into
//     a TMEM accumulator and commits each stage's MMAs to its "empty" barriers.
// Every hand-over is an mbarrier; no thread holds global loads in flight across a fence. The raw
// weight ring is read by the producers with generic shared-memory loads and refilled by bulk
// copies, which write through the async proxy: the loader issues fence.proxy.async after it has
// acquired an empty slot, or a copy can land before the last reads of the slot are performed
// (measured: without the fence 5-20 % of back-to-back launches of a 256-CTA grid returned a few
// wrong weight rows in one CTA; with it none in thousands).

// Split-K partials of one tile are reduced on chip: the splits form a thread-block cluster, each
// CTA pushes the rows another split owns into that split's receive buffer (distributed shared
// memory stores) and sums the slices of its own rows in rank order.
#include "kernels.cuh"
#include "q4k.cuh"
#include "tc_ptx.cuh"

#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <stdexcept>
#include <string>

namespace cg = cooperative_groups;

namespace bzb {

namespace {

using namespace tc;

constexpr int kTileM = 128;     // weight rows per CTA (MMA M)
constexpr int kChunkK = 64;     // K per stage: one 128-byte swizzle atom of f16
constexpr int kThreads = 256;
constexpr int kABytes = kTileM * kChunkK * 2;

#define UCHECK(x)                                                                             \
    do {                                                                                      \
        cudaError_t e_ = (x);                                                                 \
        if (e_ != cudaSuccess) throw std::runtime_error(std::string("CUDA: ") + cudaGetErrorString(e_) + " at " #x); \
    } while (0)

struct UParams {
    const uint8_t * blk;
    int q4;          // chunk format (UMat::q4)
    int M, MT, KC, kc_per_split, splits;
    const half * x;
    int ldx, rows;
    GemvOut out;
    int * err;
};

// epilogue of one output element pair source: value v for (row n, weight row m)
template <int EPI>
__device__ __forceinline__ void store_out(const UParams & p, int n, int m, float v) {
    float * dst = p.out.f32 + (size_t) n * p.out.ld + m;
    if (EPI == EPI_RESID) *dst += v;
    else *dst = v;
}

// roles: warps 0-7 dequantise, warp 8 issues MMAs, warp 9 loads weights, warp 10 loads activations.
// Every ring moves stages of kSC chunks: each mbarrier wait costs the waiting thread ~220 cycles
// even on a completed phase (measured), so a hand-over per two chunks halves that cost per chunk.
// Rings are sized so that no load waits on a recent MMA: activations run up to kBStages stages
// ahead and weights kRawStages stages ahead; the dequantised A tile only needs double buffering.
constexpr int kSC = 2;
constexpr int kRawStages = 8 / kSC;
constexpr int kAStages = 2;
constexpr int kBStages = 6 / kSC;
constexpr int kRawBytes = kTileM * kChunkK + 2 * kTileM * 2;   // 8 KB int8 + 512 B scales
constexpr int kAllThreads = kThreads + 96;

// one producer thread's share of a chunk (weight row r, half hb: two Q8_0 blocks' halves or one
// Q4_K sub-block), read from the raw ring into registers so the ring slot can be released before
// the thread waits for its A stage
struct RawPiece {
    uint4 q0, q1;
    uint2 meta;  // Q8_0: the block scale bits in x; Q4_K: the row's d, dmin, scales and mins
};

__device__ __forceinline__ RawPiece read_piece(const uint8_t * raw, int q4, int r, int hb) {
    RawPiece pc;
    if (q4) {
        pc.q0 = *reinterpret_cast<const uint4 *>(raw + (hb * kTileM + r) * 16);
        pc.q1 = pc.q0;
        pc.meta = *reinterpret_cast<const uint2 *>(raw + kTileM * 32 + r * 8);
    } else {
        pc.q0 = *reinterpret_cast<const uint4 *>(raw + ((hb * 2 + 0) * kTileM + r) * 16);
        pc.q1 = *reinterpret_cast<const uint4 *>(raw + ((hb * 2 + 1) * kTileM + r) * 16);
        pc.meta = make_uint2(*reinterpret_cast<const unsigned short *>(raw + kTileM * kChunkK + (hb * kTileM + r) * 2), 0u);
    }
    return pc;
}

// the piece dequantised to f16 into row r of a swizzled A stage (arow = the row's 128 bytes)
__device__ __forceinline__ void write_piece(const RawPiece & pc, int q4, int r, int hb, uint8_t * arow) {
    if (q4) {
        float a, b;
        q4k_chunk_scale_min(pc.meta, hb, a, b);
        const uint32_t w4[4] = { pc.q0.x, pc.q0.y, pc.q0.z, pc.q0.w };
#pragma unroll
        for (int q = 0; q < 4; q++) {
            uint32_t o[4];
            dq8_nib_f32(w4[q], a, b, o);
            const int j = hb * 4 + q;
            *reinterpret_cast<uint4 *>(arow + ((j ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        return;
    }
    const half sc = __ushort_as_half((unsigned short) pc.meta.x);
    const half2 s2 = __halves2half2(sc, sc);
    const uint32_t w8[8] = { pc.q0.x, pc.q0.y, pc.q0.z, pc.q0.w, pc.q1.x, pc.q1.y, pc.q1.z, pc.q1.w };
#pragma unroll
    for (int q = 0; q < 4; q++) {
        uint4 o;
        dq4(w8[2 * q], s2, o.x, o.y);
        dq4(w8[2 * q + 1], s2, o.z, o.w);
        const int j = hb * 4 + q;
        *reinterpret_cast<uint4 *>(arow + ((j ^ (r & 7)) << 4)) = o;
    }
}

template <int NT16>
constexpr int umma_smem_bytes() {
    return 1024 + kSC * (kAStages * kABytes + kBStages * (16 * NT16 * kChunkK * 2) + kRawStages * kRawBytes) +
           kTileM * (16 * NT16 + 4) * 4;  // split-K receive buffer
}

__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
static_assert(umma_smem_bytes<4>() <= 227 * 1024, "decode GEMM shared memory");

template <int NT16, int EPI>
__global__ void __launch_bounds__(kAllThreads, 1) umma_gemm_kernel(const UParams p, const __grid_constant__ CUtensorMap xmap) {
    constexpr int N = 16 * NT16;
    constexpr int kBBytes = N * kChunkK * 2;
    constexpr uint32_t kCols = N <= 32 ? 32 : 64;
    constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t) (N >> 3) << 17) | ((uint32_t) (kTileM >> 4) << 24);
    constexpr int kPartLd = N + 4;  // padded partial rows: consecutive weight rows land in different banks
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t a_full[kAStages], a_empty[kAStages], b_full[kBStages], b_empty[kBStages];
    __shared__ uint64_t raw_full[kRawStages], raw_empty[kRawStages], done_bar;
    __shared__ uint32_t tmem_slot;
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t) 1023);
    uint8_t * sA = smem;
    uint8_t * sB = sA + kSC * kAStages * kABytes;
    uint8_t * sR = sB + kSC * kBStages * kBBytes;
    float * recv = reinterpret_cast<float *>(sR + kSC * kRawStages * kRawBytes);  // [splits][128 / splits][N + 4]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.x, split = blockIdx.y, chunk = blockIdx.z;
    const int c_beg = split * p.kc_per_split;
    const int nch = max(0, min(p.KC, c_beg + p.kc_per_split) - c_beg);
    const int nst = (nch + kSC - 1) / kSC;  // stages; the last one may hold fewer than kSC chunks
    const int row0 = chunk * 64;
    const int rows_here = min(64, p.rows - row0);

    if (warp == 8) tmem_alloc(&tmem_slot, kCols);
    if (tid == 0) {
        for (int i = 0; i < kAStages; i++) {
            mbar_init(&a_full[i], kThreads);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < kBStages; i++) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < kRawStages; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kThreads);
        }
        mbar_init(&done_bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    // the next kernel may start only once this CTA holds its TMEM columns, so a waiting
    // successor can never take columns this grid still needs
    pdl_trigger();
    // split-K: the first cluster phase only tells each CTA that its peers have started (their
    // shared memory may be written); it completes long before the partial sums are pushed
    if (p.splits > 1) cluster_arrive_relaxed();
    bool ok = true;

    // A role stops at its first failed (bounded) wait; then the loaders wait for the copies they
    // issued and the MMA thread for its MMAs, so that no copy lands in shared memory and no MMA
    // touches tensor memory after the CTA has released them.
    const int cb = umat_chunk_bytes(p.q4);
    if (warp < 8) {
        // producer: weight row r, Q8_0 block hb of every chunk
        const int r = tid & (kTileM - 1), hb = tid >> 7;
        for (int s = 0; s < nst && ok; s++) {
            const int rs = s % kRawStages, ab = s % kAStages, nsub = min(kSC, nch - s * kSC);
            ok = mbar_wait(&raw_full[rs], (uint32_t) (s / kRawStages) & 1u, p.err);
            if (!ok) break;
            RawPiece pc[kSC];
#pragma unroll
            for (int j = 0; j < kSC; j++)
                if (j < nsub) pc[j] = read_piece(sR + rs * kSC * kRawBytes + j * cb, p.q4, r, hb);
            mbar_arrive(&raw_empty[rs]);
            if (s >= kAStages) ok = mbar_wait(&a_empty[ab], (uint32_t) ((s / kAStages) - 1) & 1u, p.err);
            if (!ok) break;
#pragma unroll
            for (int j = 0; j < kSC; j++)
                if (j < nsub) write_piece(pc[j], p.q4, r, hb, sA + (ab * kSC + j) * kABytes + (r >> 3) * 1024 + (r & 7) * 128);
            fence_proxy_async();
            mbar_arrive(&a_full[ab]);
        }
    } else if (warp == 8) {
        if (lane == 0) {
            for (int s = 0; s < nst && ok; s++) {
                const int ab = s % kAStages, bb = s % kBStages, nsub = min(kSC, nch - s * kSC);
                ok = mbar_wait(&b_full[bb], (uint32_t) (s / kBStages) & 1u, p.err);
                if (ok) ok = mbar_wait(&a_full[ab], (uint32_t) (s / kAStages) & 1u, p.err);
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (int j = 0; j < kSC; j++) {
                    if (j < nsub) {
                        const uint32_t a0 = smem_u32(sA + (ab * kSC + j) * kABytes), b0 = smem_u32(sB + (bb * kSC + j) * kBBytes);
#pragma unroll
                        for (int kk = 0; kk < kChunkK / 16; kk++)
                            umma_f16(tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), kIdesc, (s > 0 || j > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                umma_commit(&a_empty[ab]);
                umma_commit(&b_empty[bb]);
            }
            umma_commit(&done_bar);  // arrives once every MMA above has completed
            // tensor memory is released after the block barrier below: the MMAs must be done first
            if (!mbar_drain(&done_bar, 0u, p.err)) ok = false;
        }
    } else if (warp == 9) {
        if (lane == 0) {
            // weights and scales are constant: stream them before the predecessor finishes;
            // one bulk copy per stage: a tile's chunks are contiguous in the repacked layout
            const uint8_t * base = p.blk + (size_t) (mt * p.KC + c_beg) * cb;
            int issued = 0;
            for (int s = 0; s < nst; s++) {
                const int rs = s % kRawStages, nsub = min(kSC, nch - s * kSC);
                if (s >= kRawStages) ok = mbar_wait(&raw_empty[rs], (uint32_t) ((s / kRawStages) - 1) & 1u, p.err);
                if (!ok) break;
                // the producers read this slot with generic loads; without a proxy fence the bulk
                // copy (async proxy) may overwrite it before those reads are performed
                fence_proxy_async();
                mbar_expect_tx(&raw_full[rs], (uint32_t) (nsub * cb));
                bulk_g2s(sR + rs * kSC * kRawBytes, base + (size_t) s * kSC * cb, (uint32_t) (nsub * cb), &raw_full[rs]);
                issued = s + 1;
            }
            // the copies still in flight land before the CTA can exit
            for (int s = max(0, issued - kRawStages); s < issued; s++)
                mbar_drain(&raw_full[s % kRawStages], (uint32_t) (s / kRawStages) & 1u, p.err);
        }
    } else {
        if (lane == 0) {
            pdl_wait();  // activations come from the previous kernel
            int issued = 0;
            for (int s = 0; s < nst; s++) {
                const int bb = s % kBStages, nsub = min(kSC, nch - s * kSC);
                if (s >= kBStages) ok = mbar_wait(&b_empty[bb], (uint32_t) ((s / kBStages) - 1) & 1u, p.err);
                if (!ok) break;
                // one 3-D box per stage (kSC chunk tiles; every copy costs the SM about the same
                // time whatever its size): chunks past K read as zeros and are never multiplied
                (void) nsub;
                mbar_expect_tx(&b_full[bb], (uint32_t) (kSC * kBBytes));
                tma_3d(sB + bb * kSC * kBBytes, &xmap, 0, row0, c_beg + s * kSC, &b_full[bb]);
                issued = s + 1;
            }
            for (int s = max(0, issued - kBStages); s < issued; s++)
                mbar_drain(&b_full[s % kBStages], (uint32_t) (s / kBStages) & 1u, p.err);
        }
    }
    pdl_wait();  // every thread: outputs are read/written below only after the predecessor completed

    // accumulator rows 32w..32w+31 (warps 0-3), all N columns
    float v[N];
    if (warp < 4) {
        if (!mbar_wait(&done_bar, 0u, p.err)) ok = false;
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t) (32 * warp) << 16);
#pragma unroll
        for (int j = 0; j < N / 16; j++) tmem_ld16(taddr + 16 * j, v + 16 * j);
        tmem_wait_ld();
        // the loaded registers are only valid after the wait: tie every use to it
#pragma unroll
        for (int j = 0; j < N; j++) asm volatile("" : "+f"(v[j]));
        if (nch == 0 || !ok)
#pragma unroll
            for (int j = 0; j < N; j++) v[j] = 0.0f;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) tmem_dealloc(tmem, kCols);

    const int m_loc = 32 * warp + lane;
    if (p.splits == 1) {
        if (warp >= 4) return;
        const int m = mt * kTileM + m_loc;
        if (EPI == EPI_STORE || EPI == EPI_RESID) {
            if (m < p.M) {
#pragma unroll
                for (int n0 = 0; n0 < N; n0 += 16) {
                    if (EPI == EPI_RESID) {
                        // gather 16 residual values at a time so their loads overlap
                        float old[16];
#pragma unroll
                        for (int e = 0; e < 16; e++)
                            old[e] = n0 + e < rows_here ? p.out.f32[(size_t) (row0 + n0 + e) * p.out.ld + m] : 0.0f;
#pragma unroll
                        for (int e = 0; e < 16; e++) v[n0 + e] += old[e];
                    }
#pragma unroll
                    for (int e = 0; e < 16; e++)
                        if (n0 + e < rows_here) p.out.f32[(size_t) (row0 + n0 + e) * p.out.ld + m] = v[n0 + e];
                }
            }
        } else {
            // 16-row interleave: lanes 0-15 hold gate rows, lanes 16-31 the matching up rows
            const int j = mt * (kTileM / 2) + 16 * warp + lane;
#pragma unroll
            for (int n = 0; n < N; n++) {
                const float up = __shfl_sync(0xffffffffu, v[n], lane + 16);
                if (lane < 16 && n < rows_here && j < (p.M >> 1)) {
                    const float g = v[n];
                    const float act = EPI == EPI_SWIGLU ? silu_f(g) : gelu_tanh_f(g);
                    p.out.f16[(size_t) (row0 + n) * p.out.ld + j] = __float2half_rn(act * up);
                }
            }
        }
        return;
    }

    // split-K: each CTA pushes the rows of its partial tile that another split owns into that
    // split's receive buffer (distributed shared memory stores, no remote loads), then sums the
    // splits' slices of its own rows in rank order (deterministic)
    cg::cluster_group cluster = cg::this_cluster();
    const int S = p.splits;
    const int rank = (int) cluster.block_rank();
    const int rows_per = kTileM / S;
    const int mbeg = rank * rows_per;
    cluster_wait();
    if (warp < 4) {
        float * dst = cluster.map_shared_rank(recv, m_loc / rows_per) + (size_t) (rank * rows_per + m_loc % rows_per) * kPartLd;
#pragma unroll
        for (int n = 0; n < N; n += 4)
            *reinterpret_cast<float4 *>(dst + n) = make_float4(v[n], v[n + 1], v[n + 2], v[n + 3]);
    }
    cluster_arrive();
    cluster_wait();
    // peers[q] + ml * kPartLd addresses split q's partial of tile row ml (mbeg <= ml < mbeg + rows_per)
    const float * peers[8];
#pragma unroll
    for (int q = 0; q < 8; q++) peers[q] = recv + (ptrdiff_t) (q * rows_per - mbeg) * kPartLd;
    const int nq = (rows_here + 3) / 4;
    if (EPI == EPI_STORE || EPI == EPI_RESID) {
        // lane -> weight row (coalesced stores per activation row), 4 activation rows per item
        for (int idx = tid; idx < rows_per * nq; idx += kAllThreads) {
            const int ml = mbeg + idx % rows_per, n4 = (idx / rows_per) * 4;
            float4 pv[8];
#pragma unroll
            for (int q = 0; q < 8; q++)
                if (q < S) pv[q] = *reinterpret_cast<const float4 *>(peers[q] + (size_t) ml * kPartLd + n4);
            float4 acc = pv[0];
#pragma unroll
            for (int q = 1; q < 8; q++)
                if (q < S) { acc.x += pv[q].x; acc.y += pv[q].y; acc.z += pv[q].z; acc.w += pv[q].w; }
            const int m = mt * kTileM + ml;
            if (m < p.M) {
                const float av[4] = { acc.x, acc.y, acc.z, acc.w };
#pragma unroll
                for (int e = 0; e < 4; e++)
                    if (n4 + e < rows_here) store_out<EPI>(p, row0 + n4 + e, m, av[e]);
            }
        }
    } else {
        // whole 32-row gate/up groups per slice (at most 4 splits for these epilogues)
        const int pairs = rows_per / 2;
        for (int idx = tid; idx < pairs * nq; idx += kAllThreads) {
            const int pi = idx % pairs, n4 = (idx / pairs) * 4;
            const int grp = mbeg + (pi / 16) * 32, i = pi % 16;
            float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
#pragma unroll
            for (int q = 0; q < 4; q++) {
                if (q < S) {
                    const float4 gq = *reinterpret_cast<const float4 *>(peers[q] + (size_t) (grp + i) * kPartLd + n4);
                    const float4 uq = *reinterpret_cast<const float4 *>(peers[q] + (size_t) (grp + 16 + i) * kPartLd + n4);
                    g.x += gq.x; g.y += gq.y; g.z += gq.z; g.w += gq.w;
                    u.x += uq.x; u.y += uq.y; u.z += uq.z; u.w += uq.w;
                }
            }
            const int j = mt * (kTileM / 2) + grp / 2 + i;
            if (j < (p.M >> 1)) {
                const float gv[4] = { g.x, g.y, g.z, g.w }, uv[4] = { u.x, u.y, u.z, u.w };
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    if (n4 + e < rows_here) {
                        const float act = EPI == EPI_SWIGLU ? silu_f(gv[e]) : gelu_tanh_f(gv[e]);
                        p.out.f16[(size_t) (row0 + n4 + e) * p.out.ld + j] = __float2half_rn(act * uv[e]);
                    }
                }
            }
        }
    }
}

// Prefill shape: 256 activation rows per CTA (MMA N = 256), so each dequantised weight chunk feeds
// four times the rows of the decode shape and the MMA issues 4x the work per instruction. One CTA
// per (128-row weight tile, 256-row activation tile) over the whole K, no split; the same roles
// as the decode kernel, and the 8 dequantising warps drain the 128 x 256 f32 accumulator (warp w
// reads TMEM lanes 32 (w % 4) .. + 31, activation rows 128 (w / 4) .. + 127).
constexpr int kPN = 256;
constexpr int kPRawStages = 4;
constexpr int kPStages = 3;   // stages of the dequantised weight tile and the activation tile together
constexpr int kPBBytes = kPN * kChunkK * 2;
constexpr int kPrefillSmem = 1024 + kPStages * (kABytes + kPBBytes) + kPRawStages * kRawBytes;
static_assert(kPrefillSmem <= 227 * 1024, "prefill GEMM shared memory");

template <int EPI>
__global__ void __launch_bounds__(kAllThreads, 1) umma_prefill_kernel(const UParams p, const __grid_constant__ CUtensorMap xmap) {
    constexpr uint32_t kCols = kPN;
    constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t) (kPN >> 3) << 17) | ((uint32_t) (kTileM >> 4) << 24);
    extern __shared__ uint8_t smem_raw[];
    // one ring for both MMA operands: stage s is full once the 8 producer warps have written its
    // weight tile and its activation tile has landed, and empty once the MMAs reading it are done,
    // so the MMA thread waits and commits once per chunk
    __shared__ uint64_t st_full[kPStages], st_empty[kPStages];
    __shared__ uint64_t raw_full[kPRawStages], raw_empty[kPRawStages], done_bar;
    __shared__ uint32_t tmem_slot;
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t) 1023);
    uint8_t * sA = smem;
    uint8_t * sB = sA + kPStages * kABytes;
    uint8_t * sR = sB + kPStages * kPBBytes;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.x, row0 = blockIdx.y * kPN;
    const int rows_here = min(kPN, p.rows - row0);
    const int nch = p.KC;

    if (warp == 8) tmem_alloc(&tmem_slot, kCols);
    if (tid == 0) {
        for (int i = 0; i < kPStages; i++) {
            mbar_init(&st_full[i], 8 + 1);  // producer warps + the activation copy's expect_tx
            mbar_init(&st_empty[i], 1);
        }
        for (int i = 0; i < kPRawStages; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], 8);    // one arrival per producer warp
        }
        mbar_init(&done_bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    pdl_trigger();
    bool ok = true;

    // failure handling as in the decode kernel: stop at the first failed wait, then let the
    // issued copies and MMAs land before shared and tensor memory are released
    if (warp < 8) {
        const int r = tid & (kTileM - 1), hb = tid >> 7;
        for (int c = 0; c < nch; c++) {
            const int rs = c % kPRawStages, st = c % kPStages;
            ok = mbar_wait(&raw_full[rs], (uint32_t) (c / kPRawStages) & 1u, p.err);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            const RawPiece pc = read_piece(sR + rs * kRawBytes, p.q4, r, hb);
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[rs]);
            if (c >= kPStages) ok = mbar_wait(&st_empty[st], (uint32_t) ((c / kPStages) - 1) & 1u, p.err, kSpinLimit, 32);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            write_piece(pc, p.q4, r, hb, sA + st * kABytes + (r >> 3) * 1024 + (r & 7) * 128);
            fence_proxy_async();  // each thread's stores before the warp's arrival
            __syncwarp();
            if (lane == 0) mbar_arrive(&st_full[st]);
        }
    } else if (warp == 8) {
        if (lane == 0) {
            for (int c = 0; c < nch; c++) {
                const int st = c % kPStages;
                ok = mbar_wait(&st_full[st], (uint32_t) (c / kPStages) & 1u, p.err);
                if (!ok) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(sA + st * kABytes), b0 = smem_u32(sB + st * kPBBytes);
#pragma unroll
                for (int kk = 0; kk < kChunkK / 16; kk++)
                    umma_f16(tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), kIdesc, (c > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&st_empty[st]);
            }
            umma_commit(&done_bar);
            if (!mbar_drain(&done_bar, 0u, p.err)) ok = false;
        }
    } else if (warp == 9) {
        if (lane == 0) {
            const int cb = umat_chunk_bytes(p.q4);
            const uint8_t * base = p.blk + (size_t) mt * p.KC * cb;
            int issued = 0;
            for (int c = 0; c < nch; c++) {
                const int rs = c % kPRawStages;
                if (c >= kPRawStages) ok = mbar_wait(&raw_empty[rs], (uint32_t) ((c / kPRawStages) - 1) & 1u, p.err, kSpinLimit, 32);
                if (!ok) break;
                fence_proxy_async();  // generic reads of the slot before the async-proxy overwrite
                mbar_expect_tx(&raw_full[rs], (uint32_t) cb);
                bulk_g2s(sR + rs * kRawBytes, base + (size_t) c * cb, (uint32_t) cb, &raw_full[rs]);
                issued = c + 1;
            }
            for (int c = max(0, issued - kPRawStages); c < issued; c++)
                mbar_drain(&raw_full[c % kPRawStages], (uint32_t) (c / kPRawStages) & 1u, p.err);
        }
    } else {
        if (lane == 0) {
            pdl_wait();  // activations come from the previous kernel
            int issued = 0;
            for (int c = 0; c < nch; c++) {
                const int st = c % kPStages;
                if (c >= kPStages) ok = mbar_wait(&st_empty[st], (uint32_t) ((c / kPStages) - 1) & 1u, p.err, kSpinLimit, 32);
                if (!ok) break;
                mbar_expect_tx(&st_full[st], kPBBytes);
                tma_2d(sB + st * kPBBytes, &xmap, c * kChunkK, row0, &st_full[st]);
                issued = c + 1;
            }
            // the copies still in flight land before the CTA can exit. A stage's full phase also
            // needs the producers' arrivals, which a failed run may never make: the wait is bounded
            // (some 65,000 polls, far longer than any copy takes to land) and then gives up
            for (int c = max(0, issued - kPStages); c < issued; c++)
                mbar_drain(&st_full[c % kPStages], (uint32_t) (c / kPStages) & 1u, p.err, kSpinLimit / 64);
        }
    }
    pdl_wait();  // every thread: outputs are read/written below only after the predecessor completed

    if (warp < 8) {
        if (!mbar_wait(&done_bar, 0u, p.err)) ok = false;
        tc_fence_after();
        const int q = warp & 3, h = warp >> 2;
        const uint32_t taddr = tmem + ((uint32_t) (32 * q) << 16) + (uint32_t) (128 * h);
        const int m = mt * kTileM + 32 * q + lane;
        for (int sl = 0; sl < 8; sl++) {
            const int n0 = 128 * h + 16 * sl;  // warp-uniform
            if (n0 >= rows_here) break;
            float v[16];
            tmem_ld16(taddr + 16 * sl, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; e++) asm volatile("" : "+f"(v[e]));
            if (!ok)
#pragma unroll
                for (int e = 0; e < 16; e++) v[e] = 0.0f;
            if (EPI == EPI_STORE || EPI == EPI_RESID) {
                if (m < p.M) {
                    if (EPI == EPI_RESID) {
                        float old[16];
#pragma unroll
                        for (int e = 0; e < 16; e++)
                            old[e] = n0 + e < rows_here ? p.out.f32[(size_t) (row0 + n0 + e) * p.out.ld + m] : 0.0f;
#pragma unroll
                        for (int e = 0; e < 16; e++) v[e] += old[e];
                    }
#pragma unroll
                    for (int e = 0; e < 16; e++)
                        if (n0 + e < rows_here) p.out.f32[(size_t) (row0 + n0 + e) * p.out.ld + m] = v[e];
                }
            } else {
                // 16-row interleave: lanes 0-15 hold gate rows, lanes 16-31 the matching up rows
                const int j = mt * (kTileM / 2) + 16 * q + lane;
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    const float up = __shfl_sync(0xffffffffu, v[e], lane + 16);
                    if (lane < 16 && n0 + e < rows_here && j < (p.M >> 1)) {
                        const float g = v[e];
                        const float act = EPI == EPI_SWIGLU ? silu_f(g) : gelu_tanh_f(g);
                        p.out.f16[(size_t) (row0 + n0 + e) * p.out.ld + j] = __float2half_rn(act * up);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) tmem_dealloc(tmem, kCols);
}

// one thread per (tile, chunk, sub-block half, row): the Q4_K sub-block's values repacked into
// words of 8 (even values in nibbles 0-3, odd in 4-7), with the row's d and dmin (half 0 writes
// them) and the sub-block's 6-bit scale and min bytes
__global__ void repack_umma_q4k_kernel(const uint8_t * raw, int M, int K, int KC, uint8_t * blk) {
    const long long idx = (long long) blockIdx.x * blockDim.x + threadIdx.x;
    const int MT = (M + kTileM - 1) / kTileM;
    if (idx >= (long long) MT * KC * 2 * kTileM) return;
    const int r = (int) (idx % kTileM), hb = (int) ((idx / kTileM) % 2);
    const long long tc = idx / (2 * kTileM);
    const int c = (int) (tc % KC), mt = (int) (tc / KC);
    const int row = mt * kTileM + r;
    uint32_t w[4] = { 0u, 0u, 0u, 0u };
    uint16_t d = 0, dmin = 0;  // padded rows: zero scales give zero weights
    int sc = 0, mn = 0;
    if (row < M) {
        const int v0 = c * kChunkK + hb * 32;  // first value of the sub-block within the row
        const uint8_t * sblk = raw + ((size_t) row * (K / kQ4KBlockValues) + (size_t) (v0 / kQ4KBlockValues)) * kQ4KBlockBytes;
        uint8_t q[32];
        q4k_sub_block_raw(sblk, (v0 % kQ4KBlockValues) / 32, d, dmin, sc, mn, q);
#pragma unroll
        for (int wi = 0; wi < 4; wi++)
#pragma unroll
            for (int k = 0; k < 4; k++)
                w[wi] |= ((uint32_t) q[8 * wi + 2 * k] << (4 * k)) | ((uint32_t) q[8 * wi + 2 * k + 1] << (16 + 4 * k));
    }
    uint8_t * bp = blk + (size_t) tc * kUChunkBytesQ4;
    *reinterpret_cast<uint4 *>(bp + ((size_t) hb * kTileM + r) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    uint8_t * meta = bp + kTileM * 32 + (size_t) r * 8;
    if (hb == 0) *reinterpret_cast<uint32_t *>(meta) = (uint32_t) d | ((uint32_t) dmin << 16);
    meta[4 + hb] = (uint8_t) sc;
    meta[6 + hb] = (uint8_t) mn;
}

__global__ void repack_umma_kernel(const uint8_t * raw, int M, int KB, int KC, uint8_t * blk) {
    const long long idx = (long long) blockIdx.x * blockDim.x + threadIdx.x;
    const int MT = (M + kTileM - 1) / kTileM;
    if (idx >= (long long) MT * KC * 4 * kTileM) return;
    const int r = (int) (idx % kTileM);
    const long long rest = idx / kTileM;
    const int pc = (int) (rest % 2), hb = (int) ((rest / 2) % 2);
    const long long tc = rest / 4;
    const int c = (int) (tc % KC), mt = (int) (tc / KC);
    const int row = mt * kTileM + r, qb = 2 * c + hb;
    uint32_t w[4] = { 0u, 0u, 0u, 0u };
    unsigned short d = 0;
    if (row < M) {
        const uint8_t * src = raw + ((size_t) row * KB + qb) * 34;
        d = (unsigned short) (src[0] | (src[1] << 8));
        const uint8_t * q = src + 2 + pc * 16;
        for (int i = 0; i < 4; i++) w[i] = q[4 * i] | (q[4 * i + 1] << 8) | (q[4 * i + 2] << 16) | ((uint32_t) q[4 * i + 3] << 24);
    }
    uint8_t * b = blk + (size_t) tc * kUChunkBytes;
    *reinterpret_cast<uint4 *>(b + ((size_t) (hb * 2 + pc) * kTileM + r) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    if (pc == 0) *reinterpret_cast<unsigned short *>(b + kTileM * kChunkK + ((size_t) hb * kTileM + r) * 2) = d;
}

template <int NT16, int EPI>
void set_attr_one() {
    cudaFuncSetAttribute(umma_gemm_kernel<NT16, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, umma_smem_bytes<NT16>());
    cudaFuncSetAttribute(umma_gemm_kernel<NT16, EPI>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
}

template <int NT16>
void set_attr_nt() {
    set_attr_one<NT16, EPI_STORE>();
    set_attr_one<NT16, EPI_RESID>();
    set_attr_one<NT16, EPI_SWIGLU>();
    set_attr_one<NT16, EPI_GEGLU>();
}

template <int NT16, int EPI>
void launch_one(const UParams & p, const CUtensorMap & map, dim3 grid, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kAllThreads);
    cfg.dynamicSmemBytes = umma_smem_bytes<NT16>();
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (p.splits > 1) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = 1;
        at[na].val.clusterDim.y = p.splits;
        at[na].val.clusterDim.z = 1;
        na++;
    }
    if (pdl) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    UCHECK(cudaLaunchKernelEx(&cfg, umma_gemm_kernel<NT16, EPI>, p, map));
}

template <int EPI>
void launch_prefill_one(const UParams & p, const CUtensorMap & map, dim3 grid, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kAllThreads);
    cfg.dynamicSmemBytes = kPrefillSmem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    int na = 0;
    if (pdl) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    UCHECK(cudaLaunchKernelEx(&cfg, umma_prefill_kernel<EPI>, p, map));
}

template <int NT16>
void launch_nt(const UParams & p, const CUtensorMap & map, dim3 grid, cudaStream_t s, bool pdl) {
    switch (p.out.kind) {
        case EPI_STORE: launch_one<NT16, EPI_STORE>(p, map, grid, s, pdl); break;
        case EPI_RESID: launch_one<NT16, EPI_RESID>(p, map, grid, s, pdl); break;
        case EPI_SWIGLU: launch_one<NT16, EPI_SWIGLU>(p, map, grid, s, pdl); break;
        default: launch_one<NT16, EPI_GEGLU>(p, map, grid, s, pdl); break;
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void * f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !f)
            throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}


}  // namespace

// activation rows [rows][K] f16 with row stride ldx, read as 64 x box_rows tiles in the
// 128-byte swizzle; rows past `rows` read as zero
CUtensorMap make_x_map(const half * x, int K, int ldx, int rows, int box_rows) {
    CUtensorMap m;
    const cuuint64_t dims[2] = { (cuuint64_t) K, (cuuint64_t) rows };
    const cuuint64_t strides[1] = { (cuuint64_t) ldx * sizeof(half) };
    const cuuint32_t box[2] = { (cuuint32_t) kChunkK, (cuuint32_t) box_rows };
    const cuuint32_t estr[2] = { 1, 1 };
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<half *>(x), dims, strides, box, estr,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed (" + std::to_string((int) r) + ")");
    return m;
}

CUtensorMap make_x_group_map(const half * x, int K, int ldx, int rows, int box_rows, int group) {
    CUtensorMap m;
    const cuuint64_t dims[3] = { (cuuint64_t) kChunkK, (cuuint64_t) rows, (cuuint64_t) (K / kChunkK) };
    const cuuint64_t strides[2] = { (cuuint64_t) ldx * sizeof(half), (cuuint64_t) kChunkK * sizeof(half) };
    const cuuint32_t box[3] = { (cuuint32_t) kChunkK, (cuuint32_t) box_rows, (cuuint32_t) group };
    const cuuint32_t estr[3] = { 1, 1, 1 };
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<half *>(x), dims, strides, box, estr,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (3-D chunk groups) failed (" + std::to_string((int) r) + ")");
    return m;
}


namespace {
// one thread waits, with the GEMM pipelines' bounded wait, on a barrier that nothing arrives on
__global__ void mbar_timeout_probe_kernel(int * err, long long limit) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0 && mbar_wait(&bar, 0u, err, limit)) atomicExch(err, -1);  // must not complete
}
}  // namespace

int probe_mbar_timeout(long long limit) {
    int * err = nullptr;
    UCHECK(cudaMalloc(&err, sizeof(int)));
    int code = 0;
    try {
        UCHECK(cudaMemset(err, 0, sizeof(int)));
        mbar_timeout_probe_kernel<<<1, 32>>>(err, limit);
        UCHECK(cudaGetLastError());
        UCHECK(cudaMemcpy(&code, err, sizeof(int), cudaMemcpyDeviceToHost));
    } catch (...) {
        cudaFree(err);
        throw;
    }
    cudaFree(err);
    return code;
}

void init_umma_attributes() {
    for (const void * f : { (const void *) umma_prefill_kernel<EPI_STORE>, (const void *) umma_prefill_kernel<EPI_RESID>,
                            (const void *) umma_prefill_kernel<EPI_SWIGLU>, (const void *) umma_prefill_kernel<EPI_GEGLU> }) {
        cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kPrefillSmem);
        cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    }
    set_attr_nt<1>();
    set_attr_nt<2>();
    set_attr_nt<3>();
    set_attr_nt<4>();
    UCHECK(cudaGetLastError());
}

void repack_umma(const uint8_t * raw_dev, int M, int K, uint8_t * blk, cudaStream_t s) {
    if (K % kChunkK) throw std::runtime_error("tcgen05 layout needs K % 64 == 0");
    const int MT = (M + kTileM - 1) / kTileM, KC = K / kChunkK;
    const long long n = (long long) MT * KC * 4 * kTileM;
    repack_umma_kernel<<<(unsigned) ((n + 255) / 256), 256, 0, s>>>(raw_dev, M, K / 32, KC, blk);
    UCHECK(cudaGetLastError());
}

void repack_umma_q4k(const uint8_t * raw_dev, int M, int K, uint8_t * blk, cudaStream_t s) {
    if (K % kQ4KBlockValues) throw std::runtime_error("Q4_K rows need a length that is a multiple of 256");
    const int MT = (M + kTileM - 1) / kTileM, KC = K / kChunkK;
    const long long n = (long long) MT * KC * 2 * kTileM;
    repack_umma_q4k_kernel<<<(unsigned) ((n + 255) / 256), 256, 0, s>>>(raw_dev, M, K, KC, blk);
    UCHECK(cudaGetLastError());
}

void launch_umma_gemm(const UMat & w, const half * x16, int ldx, int rows, const GemvOut & out, int * err,
                      cudaStream_t s, bool pdl) {
    if (rows <= 0) return;
    if (ldx % 8 != 0 || w.K % kChunkK != 0 || (reinterpret_cast<uintptr_t>(x16) & 15))
        throw std::runtime_error("umma gemm: activations must be 16-byte aligned with a stride multiple of 8");
    const int chunks = (rows + 63) / 64;
    const int n_rows = std::min(rows, 64);
    const int NT16 = (n_rows + 15) / 16;
    const int tiles_chunks = w.MT * chunks;
    // one wave of one CTA per SM: split K while the tiles leave SMs idle; the cluster reduction
    // costs more than it saves beyond 4 splits unless the matrix has at most 8 tiles
    const int max_splits = (tiles_chunks <= 8 && out.kind < EPI_SWIGLU) ? 8 : 4;
    int splits = 1;
    while (splits * 2 * tiles_chunks <= 148 && splits * 2 <= max_splits && w.KC / (splits * 2) >= 2) splits *= 2;
    if (const char * e = std::getenv("BZB_UMMA_SPLITS")) {
        const int f = std::atoi(e);
        if (f == 1 || f == 2 || f == 4 || f == 8) splits = std::min(f, (out.kind >= EPI_SWIGLU) ? 4 : 8);
    }
    // Over 64 rows, the 256-row shape runs when it takes fewer chunk steps per SM: a chunk costs
    // both shapes about the same time (measured), so compare waves of CTAs x chunks per CTA.
    // BZB_PREFILL_GEMM=0 / 1 forces the decode / prefill shape.
    if (rows > 64) {
        const int row_tiles = (rows + kPN - 1) / kPN;
        const long long t_decode = (long long) ((tiles_chunks * splits + 147) / 148) * ((w.KC + splits - 1) / splits);
        const long long t_prefill = (long long) ((w.MT * row_tiles + 147) / 148) * w.KC;
        const char * pm = std::getenv("BZB_PREFILL_GEMM");
        const int mode = pm ? std::atoi(pm) : -1;
        if (mode == 1 || (mode != 0 && t_prefill < t_decode)) {
            UParams p;
            p.blk = w.blk; p.q4 = w.q4; p.M = w.M; p.MT = w.MT; p.KC = w.KC;
            p.kc_per_split = w.KC; p.splits = 1;
            p.x = x16; p.ldx = ldx; p.rows = rows; p.out = out; p.err = err;
            const CUtensorMap map = make_x_map(x16, w.K, ldx, rows, kPN);
            const dim3 grid(w.MT, row_tiles);
            switch (out.kind) {
                case EPI_STORE: launch_prefill_one<EPI_STORE>(p, map, grid, s, pdl); break;
                case EPI_RESID: launch_prefill_one<EPI_RESID>(p, map, grid, s, pdl); break;
                case EPI_SWIGLU: launch_prefill_one<EPI_SWIGLU>(p, map, grid, s, pdl); break;
                default: launch_prefill_one<EPI_GEGLU>(p, map, grid, s, pdl); break;
            }
            return;
        }
    }
    UParams p;
    p.blk = w.blk; p.q4 = w.q4; p.M = w.M; p.MT = w.MT; p.KC = w.KC;
    p.kc_per_split = (w.KC + splits - 1) / splits;
    p.splits = splits;
    p.x = x16; p.ldx = ldx; p.rows = rows; p.out = out; p.err = err;
    const CUtensorMap map = make_x_group_map(x16, w.K, ldx, rows, 16 * NT16, kSC);
    dim3 grid(w.MT, splits, chunks);
    switch (NT16) {
        case 1: launch_nt<1>(p, map, grid, s, pdl); break;
        case 2: launch_nt<2>(p, map, grid, s, pdl); break;
        case 3: launch_nt<3>(p, map, grid, s, pdl); break;
        default: launch_nt<4>(p, map, grid, s, pdl); break;
    }
}

}  // namespace bzb
