// Persistent depth decoder for sm_100a.
//
// The nc-1 sub-steps of a frame step's depth decode (reference src/depth_decoder.cpp:249-365:
// in_proj, 4 pre-norm GQA layers, output norm, head j, argmax feeding the next embedding) run in
// ONE launch of one CTA per SM. The work is a fixed schedule of phases (DpPhase) separated by
// grid-wide barriers: a monotonically increasing arrival counter that every CTA bumps once per
// phase (release) and polls (acquire) before it consumes another CTA's output.
//
// Roles inside a CTA (480 threads):
//   warps 0-3   epilogue group: drains the TMEM accumulators of GEMM units, and runs the
//               element-wise phases (split-K reduction + residual + norm preparation, attention,
//               arg-max + next embedding);
//   warps 4-11  dequantise raw Q8_0 chunks into the f16 A tile, written straight to tensor
//               memory (tcgen05.st): the MMA reads A from TMEM, so the weight tile never passes
//               through shared memory as f16 (half of the shared-memory traffic per chunk);
//   warp 12     issues tcgen05.mma (128 x N x 16, A from TMEM, B from shared memory) and owns
//               the TMEM columns;
//   warp 13     streams weight chunks with bulk async copies;
//   warp 14     loads activation chunks with 2-D TMA after the phase's input is complete.
// Weights never depend on activations, so warps 4-13 run ahead across phase boundaries and
// keep the next phases' weights streaming while the grid waits at a barrier; only warp 14 and
// the epilogue group wait for other CTAs.
//
// RMSNorm is split around the GEMM it feeds: the reduction phase writes x * w (f16) and each
// row's sum of squares in 64-column chunks; the consumer applies 1/sqrt(mean + eps) per row
// after the matrix product (the norm is linear in the row scale), so no phase needs a whole
// row before the GEMM starts.
//
// Every wait is bounded; on a timeout the CTA records an error code in p.err, every other wait
// notices it and returns, copies and MMAs in flight are drained, TMEM is freed, and the host
// reports the failure.
#include "depth_persist.cuh"
#include "q4k.cuh"
#include "tc_ptx.cuh"

#include <climits>
#include <stdexcept>
#include <string>

namespace bzb {

namespace {

using namespace tc;

constexpr int kTileM = 128;
constexpr int kChunkK = 64;
// Every bulk or tensor copy costs the SM a roughly fixed ~0.4 us of issue time whatever its size
// up to 32 KB, so weights and activations move in groups of kDpGroup chunks per copy.
constexpr int kRawGroups = 2;                            // weight ring: groups of 4 chunks
constexpr int kRawGroupBytes = kDpGroup * kUChunkBytes;
// dequantised A ring in TMEM: stages of kASC chunks (32 columns each), handed to the MMA thread
// with one arrival and released with one commit per stage (a unit's last stage may hold one chunk)
constexpr int kASC = 2;
constexpr int kAStages = 2;
constexpr int kACols = kChunkK / 2;                      // a 128 x 64 f16 chunk: 32 columns
constexpr int kBGroups = 2;                              // activation ring: groups of 4 chunks
constexpr int kBChunkMax = 64 * kChunkK * 2;             // one chunk of up to 64 activation rows
constexpr int kBGroupBytes = kDpGroup * kBChunkMax;
constexpr int kEpiThreads = 128;
constexpr int kDqThreads = 256;
constexpr int kMmaWarp = 12, kWeightWarp = 13, kActWarp = 14;
constexpr int kThreads = 480;
constexpr int kAccCols = 128;                            // two 64-column accumulators
constexpr int kTmemCols = 256;                           // accumulators, then the A ring
static_assert(kAccCols + kAStages * kASC * kACols <= kTmemCols, "TMEM columns");
constexpr int kQFloats = 4 * 2 * 128;                    // query heads of one attention task
constexpr long long kGridSpin = 1ll << 23;
constexpr int kMaxSplitsK = 16;                          // the split-K partials a reduction sums at most

constexpr int kStageFloats = 32 * kTileM;                // epilogue stage: 32 activation rows x 128 f32
constexpr int kRedFloats = 4 * kMaxSplitsK * 32 * 4;     // reduction landing areas: 4 warps x 16 splits x 32 float4
static_assert(kRedFloats >= 32 * 2 * 128, "attention reuses the reduction landing area for 32 positions of keys and values");
constexpr int kSmemBytes = 1024 + kBGroups * kBGroupBytes + kRawGroups * kRawGroupBytes +
                           (kQFloats + 256 + 16 + kStageFloats + kRedFloats) * 4;

#define DCHECK(x)                                                                             \
    do {                                                                                      \
        cudaError_t e_ = (x);                                                                 \
        if (e_ != cudaSuccess) throw std::runtime_error(std::string("CUDA: ") + cudaGetErrorString(e_) + " at " #x); \
    } while (0)

__device__ __forceinline__ int ld_volatile(const int * p) {
    int v;
    asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// bounded mbarrier wait that also gives up as soon as any CTA has recorded an error. It polls
// with the non-suspending test_wait: on this critical path a suspended waiter is woken later
// than a spinning one sees the phase flip.
// `backoff_ns` > 0 sleeps between polls after the first few: the waiting warps then leave the
// shared-memory pipe to the tensor core's operand reads and the copies (only the MMA issuer,
// whose latency paces everything, polls without pause).
__device__ __forceinline__ bool dwait(uint64_t * bar, uint32_t parity, int * err, unsigned backoff_ns = 0) {
    const uint32_t a = smem_u32(bar);
    for (long long i = 0; i < kSpinLimit * 16; i++) {
        uint32_t done;
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(done) : "r"(a), "r"(parity) : "memory");
        if (done) return true;
        if ((i & 4095) == 4095 && ld_volatile(err)) return false;
        if (backoff_ns && i >= 4) __nanosleep(backoff_ns);
    }
    atomicExch(err, 2);
    return false;
}
constexpr unsigned kBackoff = 64;

// the wait for copies and MMAs a role has issued, after a failure: unlike dwait it does not
// return early because an error is recorded, so the CTA releases its shared and tensor memory
// only after they have landed (error code 5 if even they time out)
__device__ __forceinline__ bool ddrain(uint64_t * bar, uint32_t parity, int * err) {
    const uint32_t a = smem_u32(bar);
    for (long long i = 0; i < kSpinLimit * 16; i++) {
        uint32_t done;
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(done) : "r"(a), "r"(parity) : "memory");
        if (done) return true;
    }
    atomicCAS(err, 0, 5);
    return false;
}

// wait until `target` phase arrivals have been counted (every phase before the current one
// complete on every CTA)
__device__ __forceinline__ bool grid_wait(const unsigned * bar, unsigned target, int * err, long long limit) {
    for (long long i = 0; i < limit; i++) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
        if (v >= target) return true;
        if ((i & 63) == 63 && ld_volatile(err)) return false;
        if (i >= 8) __nanosleep(32);
    }
    atomicExch(err, 3);
    return false;
}

__device__ __forceinline__ void grid_arrive(unsigned * bar) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// true on every thread of the epilogue group when `v` is true on all of them
__device__ __forceinline__ bool epi_all(bool v) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
                 : "=r"(r) : "r"((uint32_t) v) : "memory");
    return r != 0;
}

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float wmax(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// the phase table is constant for the whole launch: read it through the non-coherent path into
// registers once per phase, so that stores to the output buffers (which the compiler cannot
// prove do not alias the table) never force the fields to be reloaded
__device__ __forceinline__ DpPhase load_phase(const DpPhase * src) {
    static_assert(sizeof(DpPhase) % 16 == 0, "phase descriptor must be a whole number of 16-byte words");
    DpPhase out;
    const uint4 * s = reinterpret_cast<const uint4 *>(src);
    uint4 * d = reinterpret_cast<uint4 *>(&out);
#pragma unroll
    for (int k = 0; k < (int) (sizeof(DpPhase) / 16); k++) d[k] = __ldg(s + k);
    return out;
}

// which unit of GEMM phase `i` this CTA runs (valid when below n_units); rotating the
// assignment spreads the idle CTAs, and with them the early weight streaming, over the grid
__device__ __forceinline__ int unit_of(int i, int cta, int G) { return (int) (((long long) cta + 17ll * i) % G); }

struct UnitRange {
    int tile, split, c0, nch, row0;
};
__device__ __forceinline__ UnitRange unit_range(const DpPhase ph, int u) {
    UnitRange r;
    const int per_rows = ph.MT * ph.splits;
    const int rem = u % per_rows;
    r.row0 = (u / per_rows) * 64;
    r.tile = rem % ph.MT;
    r.split = rem / ph.MT;
    r.c0 = r.split * ph.kc_per;
    r.nch = min(ph.KC - r.c0, ph.kc_per);
    return r;
}

constexpr int kMaxSplits = kMaxSplitsK;
constexpr int kArgSplits = 8;   // the head's split-K is capped at this

// x[e] = sum over s < S of P[s * split_stride + off + 32 e], e < 4, with all loads in flight
// before the first add (a loop that adds as it loads waits one L2 round trip per split)
__device__ __forceinline__ void sum_partials(const float * P, int S, size_t split_stride, size_t off, float (&x)[4]) {
#pragma unroll
    for (int e = 0; e < 4; e++) {
        float v[kMaxSplits];
#pragma unroll
        for (int s = 0; s < kMaxSplits; s++) v[s] = s < S ? __ldcg(P + s * split_stride + off + 32 * e) : 0.0f;
        float a = 0.0f;
#pragma unroll
        for (int s = 0; s < kMaxSplits; s++) a += v[s];
        x[e] = a;
    }
}

// NEOX rotation of one 128-wide head held as x[e] = head[lane + 32 e]
__device__ __forceinline__ void rope128(float (&x)[4], const float2 * cs, int lane) {
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const float2 c = cs[lane + 32 * j];
        const float x0 = x[j], x1 = x[j + 2];
        x[j] = x0 * c.x - x1 * c.y;
        x[j + 2] = x0 * c.y + x1 * c.x;
    }
}

// 1 / sqrt(mean square + eps) of a row from its 64-column partial sums (lanes < nch hold one)
__device__ __forceinline__ float row_scale(const DpParams & p, int row, int lane) {
    const int nch = p.D / kChunkK;
    const float s = lane < nch ? __ldcg(p.ss + (size_t) row * nch + lane) : 0.0f;
    return 1.0f / sqrtf(wsum(s) / (float) p.D + p.eps);
}

// the same for `rows` rows at once, one thread per row (D / 64 <= 32 partial loads in flight)
__device__ __forceinline__ void row_scales(const DpParams & p, int row0, int rows, int tid, float * out) {
    const int nch = p.D / kChunkK;
    for (int n = tid; n < rows; n += kEpiThreads) {
        const float * src = p.ss + (size_t) (row0 + n) * nch;
        float v[32];
#pragma unroll
        for (int c = 0; c < 32; c++) v[c] = c < nch ? __ldcg(src + c) : 0.0f;
        float a = 0.0f;
#pragma unroll
        for (int c = 0; c < 32; c++) a += v[c];
        out[n] = 1.0f / sqrtf(a / (float) p.D + p.eps);
    }
}

// ---- element-wise phases (epilogue group: 128 threads, warps 0-3) -------------------------
__device__ __forceinline__ void cp_async16(void * dst_smem, const void * src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// sRed: this warp's [kMaxSplits][32] float4 landing area
__device__ void phase_reduce(const DpParams & p, const DpPhase ph, int cta, int G, int warp, int lane, float4 * sRed) {
    const int D = p.D, nch = D / kChunkK, rows = ph.rows;
    const int W = G * 4, nt2 = (nch + 1) / 2;
    // A warp task is 128 columns, two 64-column chunks, 4 per lane (lanes 0-15 the first chunk):
    // 64 rows of 1,024 columns are 512 tasks, one round on 592 warps, so no warp waits for two L2
    // round trips in a row. The S partials of a lane land in shared memory by cp.async, all in
    // flight at once without holding registers.
    for (int t = cta * 4 + warp; t < rows * nt2; t += W) {
        const int n = t / nt2, c = (t % nt2) * 2 + (lane >> 4);
        const bool valid = c < nch;
        const int col = c * kChunkK + 4 * (lane & 15);
        if (valid)
            for (int s = 0; s < ph.S; s++) cp_async16(sRed + s * 32 + lane, p.P + ((size_t) s * rows + n) * D + col);
        const float4 xo = ph.resid && valid ? __ldcg(reinterpret_cast<const float4 *>(p.x + (size_t) n * D + col))
                                            : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        cp_async_wait_all();
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (valid)
            for (int s = 0; s < ph.S; s++) {
                const float4 v = sRed[s * 32 + lane];
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
        const float4 xn = ph.resid ? make_float4(xo.x + acc.x, xo.y + acc.y, xo.z + acc.z, xo.w + acc.w) : acc;
        float sq = 0.0f;
        if (valid) {
            __stcg(reinterpret_cast<float4 *>(p.x + (size_t) n * D + col), xn);
            const float4 w = *reinterpret_cast<const float4 *>(ph.norm_w + col);
            half2 h[2] = { __floats2half2_rn(xn.x * w.x, xn.y * w.y), __floats2half2_rn(xn.z * w.z, xn.w * w.w) };
            __stcg(reinterpret_cast<uint2 *>(p.h16 + (size_t) n * D + col), *reinterpret_cast<uint2 *>(h));
            sq = xn.x * xn.x + xn.y * xn.y + xn.z * xn.z + xn.w * xn.w;
        }
        // the chunk's sum of squares over its 16 lanes
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if ((lane & 15) == 0 && valid) __stcg(p.ss + (size_t) n * nch + c, sq);
        __syncwarp();  // every lane has read its landing slots before the next task refills them
    }
}

// sKV: [32 positions][2][128] f32 landing area (the reductions' area, unused during attention)
__device__ void phase_attn(const DpParams & p, const DpPhase ph, int cta, int G, int warp, int lane, float * sQ,
                           float * sKV) {
    const int R = p.R, hd = 128, nkv = p.n_kv, nh = p.n_head, D = p.D;
    const int M = nh * hd + 2 * nkv * hd;
    const int rows = ph.rows, S = ph.alt ? 1 : ph.S, n_new = ph.n_new;
    const float * part = ph.alt ? p.P2 : p.P;
    const int Gq = nh / nkv;  // query heads per kv head (1..4): warps >= Gq only append k/v
    const bool qwarp = warp < Gq;
    float * kvl = p.kv + (size_t) ph.layer * p.kv_layer;
    for (int t = cta; t < R * nkv; t += G) {
        const int b = t / nkv, g = t % nkv;
        const int qh = g * Gq + warp;
        if (!p.row_active[b]) {
            if (qwarp)
                for (int i = 0; i < n_new; i++)
#pragma unroll
                    for (int e = 0; e < 4; e++) p.att16[(size_t) (b + i * R) * D + qh * hd + lane + 32 * e] = __float2half_rn(0.0f);
            continue;
        }
        float scale[2] = { 1.0f, 1.0f };
        for (int i = 0; i < n_new; i++) scale[i] = row_scale(p, b + i * R, lane);
        // this task's new keys and values: warp w < 2 n_new handles position w / 2, k or v
        if (warp < 2 * n_new) {
            const int i = warp >> 1, isv = warp & 1;
            const int row = b + i * R, pos = ph.start + i;
            const int col0 = nh * hd + isv * nkv * hd + g * hd;
            float x[4];
            sum_partials(part, S, (size_t) rows * M, (size_t) row * M + col0 + lane, x);
#pragma unroll
            for (int e = 0; e < 4; e++) x[e] *= scale[i];
            if (!isv) rope128(x, p.rope + (size_t) pos * (hd / 2), lane);
            float * dst = kvl + (((size_t) b * p.nc + pos) * 2 + isv) * nkv * hd + (size_t) g * hd;
#pragma unroll
            for (int e = 0; e < 4; e++) __stcg(dst + lane + 32 * e, x[e]);
        }
        // this warp's query head at each new position
        for (int i = 0; i < n_new && qwarp; i++) {
            const int row = b + i * R, pos = ph.start + i;
            float x[4];
            sum_partials(part, S, (size_t) rows * M, (size_t) row * M + qh * hd + lane, x);
#pragma unroll
            for (int e = 0; e < 4; e++) x[e] *= scale[i];
            rope128(x, p.rope + (size_t) pos * (hd / 2), lane);
#pragma unroll
            for (int e = 0; e < 4; e++) sQ[(warp * 2 + i) * hd + lane + 32 * e] = x[e];
        }
        epi_sync();  // appended keys/values and the queries visible to the group
        const float * kb = kvl + (size_t) b * p.nc * 2 * nkv * hd + (size_t) g * hd;
        const size_t pstride = (size_t) 2 * nkv * hd;  // floats between consecutive positions
        // The task's key and value rows (positions 0 .. start + n_new - 1, at most 32) land in
        // shared memory once for the query warps by cp.async, all in flight together: sKV
        // [position][key, value][hd] f32. Reading them row block by row block from L2 cost each
        // warp one round trip per 8 positions.
        {
            const int lim_all = ph.start + n_new;
            const int tid = warp * 32 + lane;
            for (int q = tid; q < lim_all * 2 * (hd / 4); q += kEpiThreads) {
                const int pp = q / (2 * (hd / 4)), rem = q % (2 * (hd / 4));
                const int isv = rem / (hd / 4), c4 = rem % (hd / 4);
                cp_async16(sKV + (pp * 2 + isv) * hd + 4 * c4, kb + (size_t) pp * pstride + isv * nkv * hd + 4 * c4);
            }
            cp_async_wait_all();
        }
        epi_sync();
        for (int i = 0; i < n_new && qwarp; i++) {
            const int lim = ph.start + i + 1;
            // scores: the warp reads one key row per position (lane = 4 dims), 8 rows in flight;
            // lane pp % 32 keeps the score of position pp
            const float4 q4 = *reinterpret_cast<const float4 *>(sQ + (warp * 2 + i) * hd + 4 * lane);
            float sc[2] = { -INFINITY, -INFINITY };
            for (int pp0 = 0; pp0 < lim; pp0 += 8) {
                float4 k4[8];
#pragma unroll
                for (int k = 0; k < 8; k++)
                    k4[k] = pp0 + k < lim ? *(reinterpret_cast<const float4 *>(sKV + (pp0 + k) * 2 * hd) + lane)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const int pp = pp0 + k;
                    const float d = wsum(q4.x * k4[k].x + q4.y * k4[k].y + q4.z * k4[k].z + q4.w * k4[k].w);
                    if (pp < lim && lane == (pp & 31)) sc[pp >> 5] = d * p.attn_scale;
                }
            }
            const float mx = wmax(fmaxf(sc[0], sc[1]));
            const float pr0 = lane < lim ? expf(sc[0] - mx) : 0.0f;
            const float pr1 = lane + 32 < lim ? expf(sc[1] - mx) : 0.0f;
            const float l = wsum(pr0 + pr1);
            // values: 8 rows in flight, lane = dims lane + 32 e
            float o[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
            for (int pp0 = 0; pp0 < lim; pp0 += 8) {
                float vv[8][4];
#pragma unroll
                for (int k = 0; k < 8; k++)
#pragma unroll
                    for (int e = 0; e < 4; e++)
                        vv[k][e] = pp0 + k < lim ? sKV[((pp0 + k) * 2 + 1) * hd + lane + 32 * e] : 0.0f;
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const int pp = pp0 + k;
                    const float pj = __shfl_sync(0xffffffffu, pp < 32 ? pr0 : pr1, pp & 31);
                    if (pp < lim)
#pragma unroll
                        for (int e = 0; e < 4; e++) o[e] += pj * vv[k][e];
                }
            }
            const float inv = 1.0f / l;
#pragma unroll
            for (int e = 0; e < 4; e++)
                p.att16[(size_t) (b + i * R) * D + qh * hd + lane + 32 * e] = __float2half_rn(o[e] * inv);
        }
        epi_sync();  // sQ is reused by the next task
    }
}

__device__ void phase_argmax(const DpParams & p, const DpPhase ph, int cta, int G, int tid, int warp, int lane,
                             float * sMisc) {
    const int R = p.R, V = p.vs, nc = p.nc, j = ph.j;
    float * sv = sMisc;
    int * si = reinterpret_cast<int *>(sMisc + 4);
    int * scode = reinterpret_cast<int *>(sMisc + 8);
    float * sscale = sMisc + 9;
    for (int b = cta; b < R; b += G) {
        if (p.row_set && p.row_set[b] != p.set_id) continue;  // a row of the other weight set's pass
        if (!p.row_active[b]) {
            if (tid == 0) p.frames[(size_t) b * nc + j] = -1;
            continue;
        }
        if (warp == 0) {
            const float s = row_scale(p, ph.ss_row0 + b, lane);
            if (lane == 0) *sscale = s;
        }
        epi_sync();
        const float scale = *sscale;
        float best = -INFINITY;
        int bi = INT_MAX;
        // 8 columns per pass, all S partial loads of the pass issued before the adds
        for (int v0 = tid; v0 < V; v0 += 8 * kEpiThreads) {
            float part[kArgSplits][8];
#pragma unroll
            for (int s = 0; s < kArgSplits; s++)
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const int v = v0 + k * kEpiThreads;
                    part[s][k] = (s < ph.S && v < V) ? __ldcg(p.P + ((size_t) s * R + b) * ph.out_ld + v) : 0.0f;
                }
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const int v = v0 + k * kEpiThreads;
                if (v >= V) break;
                float a = 0.0f;
#pragma unroll
                for (int s = 0; s < kArgSplits; s++)
                    if (s < ph.S) a += part[s][k];
                const float logit = a * scale;
                if (p.logits_out) p.logits_out[((size_t) b * (nc - 1) + (j - 1)) * V + v] = logit;
                if (logit > best || (bi == INT_MAX && !(logit < best))) {
                    best = logit;
                    bi = v;
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > best || (ov == best && oi < bi)) {
                best = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            sv[warp] = best;
            si[warp] = bi;
        }
        epi_sync();
        if (tid == 0) {
            float bv = sv[0];
            int i0 = si[0];
            for (int w = 1; w < 4; w++)
                if (sv[w] > bv || (sv[w] == bv && si[w] < i0)) {
                    bv = sv[w];
                    i0 = si[w];
                }
            if (i0 == INT_MAX) i0 = 0;
            p.frames[(size_t) b * nc + j] = i0;
            *scode = i0;
        }
        epi_sync();
        if (j + 1 < nc && p.in_tab) {
            int next = p.forced ? p.forced[(size_t) b * (nc - 1) + (j - 1)] : *scode;
            if (next < 0 || next >= V) next = 0;
            // the next sub-step's layer-0 input, as its in_proj + reduce phases would leave it:
            // x (f32), x * norm weight (f16) and the sum of squares of each 64-column chunk
            const int D = p.D;
            const float * src = p.in_tab + ((size_t) (j - 1) * V + next) * D;
            for (int c0 = tid * 8; c0 < D; c0 += kEpiThreads * 8) {
                const float4 a = __ldcg(reinterpret_cast<const float4 *>(src + c0));
                const float4 b2 = __ldcg(reinterpret_cast<const float4 *>(src + c0 + 4));
                const float4 wa = *reinterpret_cast<const float4 *>(p.in_norm + c0);
                const float4 wb = *reinterpret_cast<const float4 *>(p.in_norm + c0 + 4);
                __stcg(reinterpret_cast<float4 *>(p.x + (size_t) b * D + c0), a);
                __stcg(reinterpret_cast<float4 *>(p.x + (size_t) b * D + c0 + 4), b2);
                half2 h[4] = { __floats2half2_rn(a.x * wa.x, a.y * wa.y), __floats2half2_rn(a.z * wa.z, a.w * wa.w),
                               __floats2half2_rn(b2.x * wb.x, b2.y * wb.y), __floats2half2_rn(b2.z * wb.z, b2.w * wb.w) };
                __stcg(reinterpret_cast<uint4 *>(p.h16 + (size_t) b * D + c0), *reinterpret_cast<uint4 *>(h));
                // 8 consecutive threads cover one 64-column chunk
                float sq = a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b2.x * b2.x + b2.y * b2.y + b2.z * b2.z + b2.w * b2.w;
                sq += __shfl_xor_sync(0xffffffffu, sq, 1);
                sq += __shfl_xor_sync(0xffffffffu, sq, 2);
                sq += __shfl_xor_sync(0xffffffffu, sq, 4);
                if ((lane & 7) == 0) __stcg(p.ss + (size_t) b * (D / kChunkK) + c0 / kChunkK, sq);
            }
            if (p.qkv_tab) {
                const int M = p.n_head * p.hd + 2 * p.n_kv * p.hd;
                const float * qs = p.qkv_tab + ((size_t) (j - 1) * V + next) * M;
                for (int c0 = tid * 4; c0 < M; c0 += kEpiThreads * 4)
                    __stcg(reinterpret_cast<float4 *>(p.P2 + (size_t) b * M + c0), __ldcg(reinterpret_cast<const float4 *>(qs + c0)));
            }
        } else if (j + 1 < nc) {
            int next = p.forced ? p.forced[(size_t) b * (nc - 1) + (j - 1)] : *scode;
            if (next < 0 || next >= V) next = 0;
            const size_t row = (size_t) j * V + next;
            const int8_t * q = p.embd.qs + row * p.embd.K;
            const half * d = p.embd.ds + row * (p.embd.K / 32);
            const half * mn = p.embd.ms ? p.embd.ms + row * (p.embd.K / 32) : nullptr;
            for (int c = tid; c < p.embd.K / 8; c += kEpiThreads) {
                const uint2 u = *reinterpret_cast<const uint2 *>(q + c * 8);
                const float sc = __half2float(d[c >> 2]), m = mn ? __half2float(mn[c >> 2]) : 0.0f;
                const int8_t * bq = reinterpret_cast<const int8_t *>(&u);
                half2 o[4];
#pragma unroll
                for (int k = 0; k < 4; k++) o[k] = __floats2half2_rn((float) bq[2 * k] * sc - m, (float) bq[2 * k + 1] * sc - m);
                __stcg(reinterpret_cast<uint4 *>(p.din16 + (size_t) b * p.H + c * 8), *reinterpret_cast<uint4 *>(o));
            }
        }
        epi_sync();  // sMisc is reused by the next row
    }
}

__global__ void __launch_bounds__(kThreads, 1) depth_persist_kernel(const DpParams p, const __grid_constant__ DpMaps maps) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t raw_full[kRawGroups], raw_empty[kRawGroups];
    __shared__ uint64_t a_full[kAStages], a_empty[kAStages], b_full[kBGroups], b_empty[kBGroups];
    __shared__ uint64_t acc_full[2], acc_empty[2], drain_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ int s_abort;
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t) 1023);
    uint8_t * sB = smem;
    uint8_t * sR = sB + kBGroups * kBGroupBytes;
    float * sQ = reinterpret_cast<float *>(sR + kRawGroups * kRawGroupBytes);
    float * sScale = sQ + kQFloats;
    float * sMisc = sScale + 256;
    float * sStage = sMisc + 16;  // 16-byte aligned: every region before it is a multiple of 16 bytes
    float4 * sRed = reinterpret_cast<float4 *>(sStage + kStageFloats);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    int * err = p.err;
    const long long grid_spin = p.grid_spin > 0 ? p.grid_spin : kGridSpin;

    if (warp == kMmaWarp) tmem_alloc(&tmem_slot, kTmemCols);
    if (tid == 0) {
        // producer and epilogue barriers count warps: each warp syncs, then its lane 0 arrives
        for (int i = 0; i < kRawGroups; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kDqThreads / 32);
        }
        for (int i = 0; i < kAStages; i++) {
            mbar_init(&a_full[i], kDqThreads / 32);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < kBGroups; i++) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kEpiThreads / 32);
        }
        mbar_init(&drain_bar, 1);
        s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp < 4) {
        // ---------------------------------------------------------------- epilogue group
        // s_stop is written by thread 0 only between two group barriers, so the whole group
        // reads one value and leaves the loop together (a partial group would stall bar.sync)
        __shared__ int s_stop;
        uint32_t uc = 0;
        for (int i = 0; i < p.n_phases; i++) {
            const DpPhase ph = load_phase(p.phases + i);
            if (tid == 0) {
                s_stop = (s_abort || !grid_wait(p.bar, (unsigned) i * G, err, grid_spin)) ? 1 : 0;
                if (p.trace) p.trace[((size_t) i * G + cta) * kDpTraceSlots] = gtimer();
            }
            epi_sync();
            if (s_stop) break;
            if (ph.type == DP_GEMM) {
                const int v0 = unit_of(i, cta, G);
                if (ph.epi == DPE_SWIGLU && v0 < ph.n_units) {
                    // per-row RMS scale of this phase's activation rows
                    row_scales(p, ph.ss_row0, ph.rows, tid, sScale);
                    epi_sync();
                }
                for (int u = v0; u < ph.n_units; u += G) {
                    const UnitRange ur = unit_range(ph, u);
                    const int acc = uc & 1;
                    bool ok = dwait(&acc_full[acc], (uc >> 1) & 1, err, kBackoff);
                    // one outcome for the whole group: the body below has group barriers
                    ok = epi_all(ok);
                    if (p.trace && tid == 0) p.trace[((size_t) i * G + cta) * kDpTraceSlots + 6] = gtimer();
                    tc_fence_after();
                    const uint32_t taddr = tmem + (uint32_t) (acc * 64) + ((uint32_t) (32 * warp) << 16);
                    const int m_loc = 32 * warp + lane;
                    if (!ok) {
                        if (tid == 0) s_abort = 1;
                    } else if (ph.epi == DPE_PARTIAL) {
                        // The accumulator goes to global memory through shared memory, 32 activation
                        // rows at a time: TMEM -> stage [32][128] f32, then 16-byte stores of 4
                        // consecutive matrix rows (a warp instruction writes 512 contiguous bytes;
                        // scalar stores of one matrix row per lane take four times the instructions
                        // and are what limits this epilogue).
                        const int ld = ph.out_ld;  // partial row pitch, a multiple of 4
                        float * dst0 = p.P + (size_t) ur.split * ph.rows * ld;
                        for (int h = 0; h < ph.nb; h += 32) {
                            for (int n0 = h; n0 < h + 32 && n0 < ph.nb; n0 += 16) {
                                float v[16];
                                tmem_ld16(taddr + n0, v);
                                tmem_wait_ld();
#pragma unroll
                                for (int e = 0; e < 16; e++) asm volatile("" : "+f"(v[e]));
#pragma unroll
                                for (int e = 0; e < 16; e++) sStage[(n0 - h + e) * kTileM + m_loc] = v[e];
                            }
                            if (h + 32 >= ph.nb) {
                                // every TMEM read of the unit is done: the MMA may reuse the accumulator
                                tc_fence_before();
                                __syncwarp();
                                if (lane == 0) mbar_arrive(&acc_empty[acc]);
                            }
                            epi_sync();
                            const int nr = min(32, ph.nb - h);
                            for (int idx = tid; idx < nr * (kTileM / 4); idx += kEpiThreads) {
                                const int r = idx / (kTileM / 4), c4 = idx % (kTileM / 4);
                                const int n = ur.row0 + h + r, m = ur.tile * kTileM + 4 * c4;
                                if (n < ph.rows && m < ph.M)
                                    __stcg(reinterpret_cast<float4 *>(dst0 + (size_t) n * ld + m),
                                           *reinterpret_cast<const float4 *>(sStage + r * kTileM + 4 * c4));
                            }
                            epi_sync();  // the stage is refilled next
                        }
                    } else {
                        // 16-row gate/up interleave: lanes 0-15 hold gate rows, lanes 16-31 the
                        // matching up rows. Partners swap values so that every lane finishes half of
                        // the columns: lane l < 16 the even ones, lane l + 16 the odd. The row scales
                        // are read into registers first (a shared-memory read between global stores
                        // would wait for each of them and chain the rows), and the products go to a
                        // shared stage [rows][64 + 16] f16 (the pad puts the even and odd rows of one
                        // store in different banks), written out with 16-byte stores.
                        const int pr = lane & 15;
                        const bool gate_lane = lane < 16;
                        half * stage = reinterpret_cast<half *>(sStage);
                        constexpr int kGp = kTileM / 2 + 16;
                        for (int n0 = 0; n0 < ph.nb; n0 += 16) {
                            float v[16];
                            tmem_ld16(taddr + n0, v);
                            tmem_wait_ld();
#pragma unroll
                            for (int e = 0; e < 16; e++) asm volatile("" : "+f"(v[e]));
                            const int nbase = ur.row0 + n0;  // activation row of v[0]
                            float scv[8];
#pragma unroll
                            for (int e2 = 0; e2 < 8; e2++) scv[e2] = sScale[min(nbase + 2 * e2 + (gate_lane ? 0 : 1), 255)];
#pragma unroll
                            for (int e2 = 0; e2 < 8; e2++) {
                                // lanes < 16 finish row n0 + 2 e2, lanes >= 16 row n0 + 2 e2 + 1
                                const float oe = __shfl_xor_sync(0xffffffffu, v[2 * e2], 16);
                                const float oo = __shfl_xor_sync(0xffffffffu, v[2 * e2 + 1], 16);
                                const float gt = (gate_lane ? v[2 * e2] : oo) * scv[e2];
                                const float up = (gate_lane ? oe : v[2 * e2 + 1]) * scv[e2];
                                const float act = __fdividef(gt, 1.0f + __expf(-gt));
                                stage[(n0 + 2 * e2 + (gate_lane ? 0 : 1)) * kGp + 16 * warp + pr] = __float2half_rn(act * up);
                            }
                        }
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[acc]);
                        epi_sync();
                        for (int idx = tid; idx < ph.nb * 8; idx += kEpiThreads) {
                            const int r = idx >> 3, c8 = idx & 7;
                            const int n = ur.row0 + r, jc = ur.tile * (kTileM / 2) + 8 * c8;
                            if (n < ph.rows && jc < ph.out_ld)
                                *reinterpret_cast<uint4 *>(p.g16 + (size_t) n * p.ffn + jc) =
                                    *reinterpret_cast<const uint4 *>(stage + r * kGp + 8 * c8);
                        }
                        epi_sync();  // the stage is refilled by the next unit
                    }
                    if (!ok) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[acc]);
                    }
                    uc++;
                }
            } else if (ph.type == DP_REDUCE) {
                phase_reduce(p, ph, cta, G, warp, lane, sRed + warp * (kMaxSplits * 32));
            } else if (ph.type == DP_ATTN) {
                phase_attn(p, ph, cta, G, warp, lane, sQ, reinterpret_cast<float *>(sRed));
            } else {
                phase_argmax(p, ph, cta, G, tid, warp, lane, sMisc);
            }
            epi_sync();
            if (tid == 0) {
                if (p.trace) p.trace[((size_t) i * G + cta) * kDpTraceSlots + 1] = gtimer();
                // the group barrier orders the group's writes before this thread's release, which
                // publishes them at GPU scope; the proxy fence lets TMA loads in other CTAs see them
                fence_proxy_async_global();
                grid_arrive(p.bar);
            }
        }
        if (tid == 0 && (s_abort || s_stop)) atomicCAS(err, 0, 4);
    } else if (warp < 4 + kDqThreads / 32) {
        // ---------------------------------------------------------------- dequantising producers
        const int t = tid - kEpiThreads;
        const int r = t & (kTileM - 1), hb = t >> 7;
        uint32_t rg = 0, as = 0;
        bool ok = true;
        for (int i = 0; i < p.n_phases && ok; i++) {
            const DpPhase ph = load_phase(p.phases + i);
            if (ph.type != DP_GEMM) continue;
            for (int u = unit_of(i, cta, G); u < ph.n_units && ok; u += G) {
                const UnitRange ur = unit_range(ph, u);
                for (int c = 0; c < ur.nch && ok; c++) {
                    const int within = c % kDpGroup, gs = min(kDpGroup, ur.nch - (c - within));
                    const int rs = rg % kRawGroups, ab = as % kAStages, sub = c % kASC;
                    const bool stage_end = sub == kASC - 1 || c == ur.nch - 1;
                    // every wait's outcome is made warp-uniform: the TMEM stores below are warp-collective
                    if (within == 0) ok = __all_sync(0xffffffffu, dwait(&raw_full[rs], (rg / kRawGroups) & 1u, err, kBackoff));
                    if (!ok) break;
                    if (p.trace && t == 0 && c == 0) p.trace[((size_t) i * G + cta) * kDpTraceSlots + 8] = gtimer();
                    const uint8_t * raw = sR + rs * kRawGroupBytes + within * umat_chunk_bytes(ph.q4);
                    uint4 q0, q1;
                    half sc = __float2half_rn(0.0f);
                    uint2 meta = make_uint2(0u, 0u);
                    if (ph.q4) {
                        // one 32-value Q4_K sub-block: 16 bytes of nibbles, the row's scale data
                        q0 = *reinterpret_cast<const uint4 *>(raw + (hb * kTileM + r) * 16);
                        q1 = q0;
                        meta = *reinterpret_cast<const uint2 *>(raw + kTileM * 32 + r * 8);
                    } else {
                        q0 = *reinterpret_cast<const uint4 *>(raw + ((hb * 2 + 0) * kTileM + r) * 16);
                        q1 = *reinterpret_cast<const uint4 *>(raw + ((hb * 2 + 1) * kTileM + r) * 16);
                        sc = *reinterpret_cast<const half *>(raw + kTileM * kChunkK + (hb * kTileM + r) * 2);
                    }
                    if (within == gs - 1) {
                        __syncwarp();  // the whole warp has read the group
                        if (lane == 0) mbar_arrive(&raw_empty[rs]);
                        rg++;
                    }
                    if (sub == 0 && as >= kAStages)
                        ok = __all_sync(0xffffffffu, dwait(&a_empty[ab], ((as / kAStages) - 1) & 1u, err, kBackoff));
                    if (!ok) break;
                    const half2 s2 = __halves2half2(sc, sc);
                    // this thread's 32 K values (half hb of the chunk) of A row r, as 16 columns of
                    // its TMEM lane; the stage's MMAs were complete (a_empty) before the first write
                    if (sub == 0) tc_fence_after();
                    uint32_t o16[16];
                    if (ph.q4) {
                        float qa, qb;
                        q4k_chunk_scale_min(meta, hb, qa, qb);
                        const uint32_t w4[4] = { q0.x, q0.y, q0.z, q0.w };
#pragma unroll
                        for (int q = 0; q < 4; q++) {
                            uint32_t o[4];
                            dq8_nib_f32(w4[q], qa, qb, o);
#pragma unroll
                            for (int k = 0; k < 4; k++) o16[4 * q + k] = o[k];
                        }
                    } else {
                        const uint32_t w8[8] = { q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w };
#pragma unroll
                        for (int q = 0; q < 4; q++) {
                            dq4(w8[2 * q], s2, o16[4 * q], o16[4 * q + 1]);
                            dq4(w8[2 * q + 1], s2, o16[4 * q + 2], o16[4 * q + 3]);
                        }
                    }
                    tmem_st16(tmem + ((uint32_t) (32 * (warp & 3)) << 16) + (uint32_t) (kAccCols + (ab * kASC + sub) * kACols + hb * 16),
                              o16);
                    if (stage_end) {
                        tmem_wait_st();  // this thread's TMEM stores of the stage complete
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&a_full[ab]);
                        as++;
                    }

                }
            }
        }
        tmem_wait_st();
        if (!ok) s_abort = 1;
    } else if (warp == kMmaWarp) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            uint32_t as = 0, bg = 0, uc = 0;
            bool ok = true;
            for (int i = 0; i < p.n_phases && ok; i++) {
                const DpPhase ph = load_phase(p.phases + i);
                if (ph.type != DP_GEMM) continue;
                for (int u = unit_of(i, cta, G); u < ph.n_units && ok; u += G) {
                    const UnitRange ur = unit_range(ph, u);
                    const int acc = uc & 1;
                    if (uc >= 2) ok = dwait(&acc_empty[acc], ((uc >> 1) - 1) & 1u, err);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t idesc = (1u << 4) | ((uint32_t) (ph.nb >> 3) << 17) | ((uint32_t) (kTileM >> 4) << 24);
                    const uint32_t d = tmem + (uint32_t) (acc * 64);
                    for (int c = 0; c < ur.nch; c++) {
                        const int within = c % kDpGroup, gs = min(kDpGroup, ur.nch - (c - within));
                        const int ab = as % kAStages, bs = bg % kBGroups, sub = c % kASC;
                        const bool stage_end = sub == kASC - 1 || c == ur.nch - 1;
                        if (within == 0) ok = dwait(&b_full[bs], (bg / kBGroups) & 1u, err);
                        if (p.trace && c == 0) p.trace[((size_t) i * G + cta) * kDpTraceSlots + 3] = gtimer();
                        if (p.trace && c < 16) p.trace[((size_t) i * G + cta) * kDpTraceSlots + 9 + c] = gtimer();
                        if (sub == 0) ok = ok && dwait(&a_full[ab], (as / kAStages) & 1u, err);
                        if (p.trace && c == 0) p.trace[((size_t) i * G + cta) * kDpTraceSlots + 4] = gtimer();
                        if (p.trace && c < 16) p.trace[((size_t) i * G + cta) * kDpTraceSlots + 25 + c] = gtimer();
                        if (!ok) break;
                        // the A stage was written to TMEM by the dequantisers (tcgen05.st, wait,
                        // fence before their arrival): order this thread's MMAs after that wait
                        if (sub == 0) tc_fence_after();
                        const uint32_t a0 = tmem + (uint32_t) (kAccCols + (ab * kASC + sub) * kACols);
                        const uint32_t b0 = smem_u32(sB + bs * kBGroupBytes + within * ph.nb * kChunkK * 2);
#pragma unroll
                        for (int kk = 0; kk < kChunkK / 16; kk++)
                            umma_f16_tmem_a(d, a0 + kk * 8, sw128_desc(b0 + kk * 32), idesc, (c > 0 || kk > 0) ? 1u : 0u);
                        if (stage_end) {
                            umma_commit(&a_empty[ab]);  // the stage's MMAs release its A tiles
                            as++;
                        }
                        if (within == gs - 1) {
                            umma_commit(&b_empty[bs]);  // the group's last chunk releases its stage
                            bg++;
                        }
                        if (p.trace && c < 16) p.trace[((size_t) i * G + cta) * kDpTraceSlots + 41 + c] = gtimer();
                    }
                    if (!ok) break;
                    if (p.trace) p.trace[((size_t) i * G + cta) * kDpTraceSlots + 5] = gtimer();
                    umma_commit(&acc_full[acc]);
                    uc++;
                }
            }
            // every MMA issued above has completed before TMEM is released
            umma_commit(&drain_bar);
            ddrain(&drain_bar, 0, err);
            if (!ok) s_abort = 1;
        }
    } else if (warp == kWeightWarp) {
        // ---------------------------------------------------------------- weight stream
        if (lane == 0) {
            uint32_t rg = 0;
            bool ok = true;
            for (int i = 0; i < p.n_phases && ok; i++) {
                const DpPhase ph = load_phase(p.phases + i);
                if (ph.type != DP_GEMM) continue;
                for (int u = unit_of(i, cta, G); u < ph.n_units && ok; u += G) {
                    const UnitRange ur = unit_range(ph, u);
                    const int cb = umat_chunk_bytes(ph.q4);
                    const uint8_t * base = ph.blk + (size_t) (ur.tile * ph.KC + ur.c0) * cb;
                    for (int g0 = 0; g0 < ur.nch; g0 += kDpGroup, rg++) {
                        const int gs = min(kDpGroup, ur.nch - g0);
                        const int rs = rg % kRawGroups;
                        if (rg >= kRawGroups) ok = dwait(&raw_empty[rs], ((rg / kRawGroups) - 1) & 1u, err, kBackoff);
                        if (!ok) break;
                        // the producers read this slot with generic loads: order those reads before
                        // the bulk copy's async-proxy writes into it
                        fence_proxy_async();
                        if (p.trace && g0 == 0) p.trace[((size_t) i * G + cta) * kDpTraceSlots + 7] = gtimer();
                        mbar_expect_tx(&raw_full[rs], (uint32_t) (gs * cb));
                        bulk_g2s(sR + rs * kRawGroupBytes, base + (size_t) g0 * cb, (uint32_t) (gs * cb), &raw_full[rs]);
                    }
                }
            }
            // copies still in flight land before the CTA exits
            for (uint32_t k = rg > (uint32_t) kRawGroups ? rg - kRawGroups : 0; k < rg; k++)
                ddrain(&raw_full[k % kRawGroups], (k / kRawGroups) & 1u, err);
            if (!ok) s_abort = 1;
        }
    } else {
        // ---------------------------------------------------------------- activation loads
        if (lane == 0) {
            uint32_t bg = 0;
            bool ok = true;
            for (int i = 0; i < p.n_phases && ok; i++) {
                const DpPhase ph = load_phase(p.phases + i);
                if (ph.type != DP_GEMM) continue;
                const int v0 = unit_of(i, cta, G);
                if (v0 >= ph.n_units) continue;
                ok = grid_wait(p.bar, (unsigned) i * G, err, grid_spin);
                if (!ok) break;
                fence_proxy_async_global();
                if (p.trace) p.trace[((size_t) i * G + cta) * kDpTraceSlots + 2] = gtimer();
                // a box always spans kDpGroup chunks (those past the unit are loaded and unused)
                const uint32_t bytes = (uint32_t) kDpGroup * ph.nb * kChunkK * 2;
                for (int u = v0; u < ph.n_units && ok; u += G) {
                    const UnitRange ur = unit_range(ph, u);
                    for (int g0 = 0; g0 < ur.nch; g0 += kDpGroup, bg++) {
                        const int bs = bg % kBGroups;
                        if (bg >= kBGroups) ok = dwait(&b_empty[bs], ((bg / kBGroups) - 1) & 1u, err, kBackoff);
                        if (!ok) break;
                        mbar_expect_tx(&b_full[bs], bytes);
                        tma_3d(sB + bs * kBGroupBytes, &maps.m[ph.map], 0, ph.b_row0 + ur.row0, ur.c0 + g0, &b_full[bs]);
                    }
                }
            }
            for (uint32_t k = bg > (uint32_t) kBGroups ? bg - kBGroups : 0; k < bg; k++)
                ddrain(&b_full[k % kBGroups], (k / kBGroups) & 1u, err);
            if (!ok) s_abort = 1;
        }
    }
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

int depth_persist_grid() {
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, depth_persist_kernel, kThreads, kSmemBytes) != cudaSuccess)
        return 0;
    return per_sm >= 1 ? sms : 0;
}

void init_depth_persist_attributes() {
    DCHECK(cudaFuncSetAttribute(depth_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    DCHECK(cudaFuncSetAttribute(depth_persist_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
}

void launch_depth_persist(const DpParams & p, const DpMaps & maps, int grid, cudaStream_t s) {
    if (grid <= 0) throw std::runtime_error("persistent depth decoder: no grid");
    DCHECK(cudaMemsetAsync(p.bar, 0, sizeof(unsigned), s));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    // all CTAs must be resident at once: the phase barriers wait for every one of them
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    DCHECK(cudaLaunchKernelEx(&cfg, depth_persist_kernel, p, maps));
}

}  // namespace bzb
