// CUDA kernels of the B200 decode engine (sm_100a).
//
// Weight contractions are dequant-GEMMs over Q8_0 weights repacked once at load into the
// mma.m16n8k16 A-fragment order, so each lane streams its weights with one 128-bit load per
// 16x32 tile and dequantises them in registers; the (few) activation rows are staged once
// per CTA in shared memory in B-fragment order. Split-K partials are reduced in a fixed order
// by the last CTA of each output tile, so results do not depend on scheduling.
#include "kernels.cuh"
#include "q4k.cuh"

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <utility>
#include <cfloat>
#include <cmath>
#include <stdexcept>
#include <string>

namespace bzb {

#define BZB_CUDA_CHECK(x)                                                                     \
    do {                                                                                      \
        cudaError_t e_ = (x);                                                                 \
        if (e_ != cudaSuccess) throw std::runtime_error(std::string("CUDA: ") + cudaGetErrorString(e_) + " at " #x); \
    } while (0)

namespace {

// PDL is switched on only while a step graph is being captured, whose nodes are all kernels;
// eager sequences interleave host copies, which keep plain stream ordering
thread_local bool g_pdl_scope = false;

bool pdl_enabled() {
    static const bool allowed = [] { const char * e = std::getenv("BZB_PDL"); return !(e && e[0] == '0'); }();
    return allowed && g_pdl_scope;
}

template <typename... KArgs, typename... Args>
void launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args &&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    BZB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// programmatic dependent launch: every kernel of a step lets the next one start its
// independent prologue early (trigger) and waits for its predecessor's results (wait)
// before touching them; the wait is a no-op for launches without the PDL attribute
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint4 ld_stream(const uint4 * p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

__device__ __forceinline__ void mma16816(float * c, const uint32_t * a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// four int8 (rows g, g, g+8, g+8) -> two half2 scaled by their rows' Q8_0 scales. 0x64XX as
// f16 is 1024 + XX, so flipping the sign bit and subtracting 1152 recovers the int8 exactly.
__device__ __forceinline__ void dq_word(uint32_t w, half2 s_g, half2 s_g8, uint32_t & lo, uint32_t & hi) {
    const uint32_t u = w ^ 0x80808080u;
    uint32_t l = __byte_perm(u, 0x64646464u, 0x5140u);
    uint32_t h = __byte_perm(u, 0x64646464u, 0x7362u);
    const half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    half2 hl = __hmul2(__hsub2(*reinterpret_cast<half2 *>(&l), bias), s_g);
    half2 hh = __hmul2(__hsub2(*reinterpret_cast<half2 *>(&h), bias), s_g8);
    lo = *reinterpret_cast<uint32_t *>(&hl);
    hi = *reinterpret_cast<uint32_t *>(&hh);
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float gelu_tanh_f(float x) {
    const float c = 0.7978845608028654f;
    return 0.5f * x * (1.0f + tanhf(c * x * (1.0f + 0.044715f * x * x)));
}

// ------------------------------------------------------------------------------------ GEMM
struct GemvParams {
    const uint4 * qs;
    const half2 * ds;
    int MT, M, KB, kper, splits, MG;
    const half * x;
    int ldx, rows;
    GemvOut out;
    float4 * ws;
    int * counters;
};

constexpr int kGemvThreads = 256;
constexpr int kSub = 8;        // k32 blocks per staged activation sub-chunk (= weight prefetch depth)
constexpr int kMaxSplits = 8;

// activations are written by the previous kernel while this one may already be running
// (programmatic dependent launch), so they are read with coherent loads, never ld.global.nc
__device__ __forceinline__ uint32_t ldg32(const half * p) { return *reinterpret_cast<const unsigned int *>(p); }

// Each CTA owns 8 m16 row tiles (one per warp), one 64-row activation chunk and a K range.
// Activations for kSub k32 blocks are staged in shared memory in mma B-fragment order, double
// buffered through registers; weights stream through an 8-deep per-lane register ring that
// runs across sub-chunk boundaries. Split-K partials (at most kMaxSplits) are reduced in split
// order by the last CTA of each row group.
template <int NT, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(const GemvParams p) {
    extern __shared__ uint4 smem_b[];  // [2][kSub][NT][32]
    __shared__ int s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mg = blockIdx.x, split = blockIdx.y, chunk = blockIdx.z;
    const int kb_beg = split * p.kper;
    const int nkb = min(p.KB, kb_beg + p.kper) - kb_beg;
    const int mt = mg * 8 + warp;
    const bool mt_ok = mt < p.MT;
    const int row0 = chunk * 64;
    const uint4 * wq = p.qs + ((size_t) mt * p.KB + kb_beg) * 32 + lane;
    const half2 * wd = p.ds + ((size_t) mt * p.KB + kb_beg) * 8 + (lane >> 2);

    pdl_trigger();
    uint4 a[kSub];
    half2 sc[kSub];
#pragma unroll
    for (int i = 0; i < kSub; i++) {
        if (mt_ok && i < nkb) {
            a[i] = ld_stream(wq + (size_t) i * 32);
            sc[i] = wd[(size_t) i * 8];
        }
    }
    pdl_wait();  // weights are constant; activations and outputs belong to the previous kernels

    // this thread's NT staged fragments per sub-chunk: fragment f = tid + 256*r covers
    // (k block f / (NT*32), row tile (f / 32) % NT, lane f % 32)
    uint4 st[NT];
    auto load_stage = [&](int s) {
        const int kbs = s * kSub;
#pragma unroll
        for (int r = 0; r < NT; r++) {
            const int f = tid + r * kGemvThreads;
            const int kbl = f / (NT * 32), nt = (f / 32) % NT, L = f & 31;
            const int n = row0 + nt * 8 + (L >> 2);
            const int kb = kbs + kbl;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (kb < nkb && n < p.rows) {
                const half * src = p.x + (size_t) n * p.ldx + (size_t) (kb_beg + kb) * 32 + 2 * (L & 3);
                v.x = ldg32(src);
                v.y = ldg32(src + 8);
                v.z = ldg32(src + 16);
                v.w = ldg32(src + 24);
            }
            st[r] = v;
        }
    };
    auto store_stage = [&](int buf) {
        uint4 * dst = smem_b + (size_t) buf * kSub * NT * 32;
#pragma unroll
        for (int r = 0; r < NT; r++) dst[tid + r * kGemvThreads] = st[r];
    };

    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;

    const int nsubs = (nkb + kSub - 1) / kSub;
    load_stage(0);
    store_stage(0);
    __syncthreads();
    for (int s = 0; s < nsubs; s++) {
        if (s + 1 < nsubs) load_stage(s + 1);
        if (mt_ok) {
            const uint4 * sbuf = smem_b + (size_t) (s & 1) * kSub * NT * 32 + lane;
#pragma unroll
            for (int i = 0; i < kSub; i++) {
                const int kb = s * kSub + i;
                if (kb < nkb) {
                    uint32_t A[8];
                    const half2 sg = __low2half2(sc[i]), sg8 = __high2half2(sc[i]);
                    dq_word(a[i].x, sg, sg8, A[0], A[1]);
                    dq_word(a[i].y, sg, sg8, A[2], A[3]);
                    dq_word(a[i].z, sg, sg8, A[4], A[5]);
                    dq_word(a[i].w, sg, sg8, A[6], A[7]);
                    if (kb + kSub < nkb) {
                        a[i] = ld_stream(wq + (size_t) (kb + kSub) * 32);
                        sc[i] = wd[(size_t) (kb + kSub) * 8];
                    }
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) {
                        const uint4 b = sbuf[(i * NT + nt) * 32];
                        mma16816(acc[nt], A, b.x, b.y);
                        mma16816(acc[nt], A + 4, b.z, b.w);
                    }
                }
            }
        }
        if (s + 1 < nsubs) store_stage((s + 1) & 1);
        __syncthreads();
    }

    if (p.splits > 1) {
        if (mt_ok) {
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
                __stcg(&p.ws[(((size_t) (chunk * p.splits + split) * p.MT + mt) * NT + nt) * 32 + lane],
                       make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]));
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = atomicAdd(&p.counters[chunk * p.MG + mg], 1) == p.splits - 1;
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        if (mt_ok) {
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                float4 v[kMaxSplits];
#pragma unroll
                for (int sp = 0; sp < kMaxSplits; sp++)
                    if (sp < p.splits)
                        v[sp] = __ldcg(&p.ws[(((size_t) (chunk * p.splits + sp) * p.MT + mt) * NT + nt) * 32 + lane]);
                float4 t = v[0];
#pragma unroll
                for (int sp = 1; sp < kMaxSplits; sp++)
                    if (sp < p.splits) { t.x += v[sp].x; t.y += v[sp].y; t.z += v[sp].z; t.w += v[sp].w; }
                acc[nt][0] = t.x; acc[nt][1] = t.y; acc[nt][2] = t.z; acc[nt][3] = t.w;
            }
        }
        if (tid == 0) p.counters[chunk * p.MG + mg] = 0;
    }
    if (!mt_ok) return;

    const int g = lane >> 2, t = lane & 3;
    if (EPI == EPI_RESID) {
        // gather every residual value first so the loads overlap instead of alternating with
        // stores the compiler cannot prove disjoint
        float old[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int m = mt * 16 + g + (e >= 2 ? 8 : 0), n = row0 + nt * 8 + 2 * t + (e & 1);
                old[nt][e] = (m < p.M && n < p.rows) ? p.out.f32[(size_t) n * p.out.ld + m] : 0.0f;
            }
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[nt][e] += old[nt][e];
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const int n0 = row0 + nt * 8 + 2 * t;
        if (EPI == EPI_STORE || EPI == EPI_RESID) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int m = mt * 16 + g + (e >= 2 ? 8 : 0);
                const int n = n0 + (e & 1);
                if (m < p.M && n < p.rows) p.out.f32[(size_t) n * p.out.ld + m] = acc[nt][e];
            }
        } else {
            const int j = mt * 8 + g;
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int n = n0 + e;
                if (n < p.rows && j < (p.M >> 1)) {
                    const float gate = acc[nt][e], up = acc[nt][2 + e];
                    const float act = EPI == EPI_SWIGLU ? silu_f(gate) : gelu_tanh_f(gate);
                    p.out.f16[(size_t) n * p.out.ld + j] = __float2half_rn(act * up);
                }
            }
        }
    }
}

template <int NT>
void launch_gemv_nt(const GemvParams & p, dim3 grid, size_t smem, cudaStream_t s) {
    switch (p.out.kind) {
        case EPI_STORE: launch_k(gemv_kernel<NT, EPI_STORE>, grid, kGemvThreads, smem, s, p); break;
        case EPI_RESID: launch_k(gemv_kernel<NT, EPI_RESID>, grid, kGemvThreads, smem, s, p); break;
        case EPI_SWIGLU: launch_k(gemv_kernel<NT, EPI_SWIGLU>, grid, kGemvThreads, smem, s, p); break;
        default: launch_k(gemv_kernel<NT, EPI_GEGLU>, grid, kGemvThreads, smem, s, p); break;
    }
}

template <int NT>
void set_gemv_attr() {
    const int mx = 2 * kSub * NT * 32 * (int) sizeof(uint4);
    cudaFuncSetAttribute(gemv_kernel<NT, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    cudaFuncSetAttribute(gemv_kernel<NT, EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    cudaFuncSetAttribute(gemv_kernel<NT, EPI_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    cudaFuncSetAttribute(gemv_kernel<NT, EPI_GEGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
}

// ------------------------------------------------------------------------------------ repack
__global__ void repack_q8_kernel(const uint8_t * raw, int M, int KB, uint4 * qs, half2 * ds) {
    pdl_trigger();
    pdl_wait();
    const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int MT = (M + 15) / 16;
    if (warp_global >= MT * KB) return;
    const int mt = warp_global / KB, kb = warp_global % KB;
    const int g = lane >> 2, t = lane & 3;
    const int r0 = mt * 16 + g, r1 = r0 + 8;
    auto q_at = [&](int r, int k) -> uint32_t {
        if (r >= M) return 0u;
        return raw[((size_t) r * KB + kb) * 34 + 2 + k];
    };
    uint32_t w[4];
    for (int hlf = 0; hlf < 2; hlf++) {
        const int k0 = hlf * 16 + 2 * t;
        w[hlf * 2 + 0] = q_at(r0, k0) | (q_at(r0, k0 + 1) << 8) | (q_at(r1, k0) << 16) | (q_at(r1, k0 + 1) << 24);
        w[hlf * 2 + 1] = q_at(r0, k0 + 8) | (q_at(r0, k0 + 9) << 8) | (q_at(r1, k0 + 8) << 16) | (q_at(r1, k0 + 9) << 24);
    }
    qs[((size_t) mt * KB + kb) * 32 + lane] = make_uint4(w[0], w[1], w[2], w[3]);
    if (lane < 8) {
        auto d_at = [&](int r) -> unsigned short {
            if (r >= M) return 0;
            const uint8_t * b = raw + ((size_t) r * KB + kb) * 34;
            return (unsigned short) (b[0] | (b[1] << 8));
        };
        ds[((size_t) mt * KB + kb) * 8 + lane] = __halves2half2(__ushort_as_half(d_at(mt * 16 + lane)),
                                                               __ushort_as_half(d_at(mt * 16 + lane + 8)));
    }
}

__global__ void split_q8_rows_kernel(const uint8_t * raw, long long n_blocks, int8_t * qs, half * ds) {
    pdl_trigger();
    pdl_wait();
    const long long b = (long long) blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_blocks) return;
    const uint8_t * src = raw + b * 34;
    ds[b] = __ushort_as_half((unsigned short) (src[0] | (src[1] << 8)));
    for (int j = 0; j < 32; j++) qs[b * 32 + j] = (int8_t) src[2 + j];
}

// one thread per (row, 32-value sub-block) of Q4_K rows
__global__ void split_q4k_rows_kernel(const uint8_t * raw, long long n_sub, int8_t * qs, half * ds, half * ms) {
    pdl_trigger();
    pdl_wait();
    const long long b = (long long) blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_sub) return;
    const uint8_t * blk = raw + (b / 8) * kQ4KBlockBytes;
    half a, mn;
    uint8_t q[32];
    q4k_sub_block(blk, (int) (b % 8), a, mn, q);
    ds[b] = a;
    ms[b] = mn;
    for (int j = 0; j < 32; j++) qs[b * 32 + j] = (int8_t) q[j];
}

// ------------------------------------------------------------------------------------ norms
__device__ float block_sum(float v, float * red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
    for (int i = 0; i < nw; i++) s += red[i];
    return s;
}

__global__ void rmsnorm_kernel(const float * x, int ldx, const float * w, int D, float eps, half * o16, int ld16,
                               float * o32, int ld32, int r0, const int * row_map) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    const int i = blockIdx.x;
    const float4 * xr = reinterpret_cast<const float4 *>(x + (size_t) (r0 + i) * ldx);
    const float4 * w4 = reinterpret_cast<const float4 *>(w);
    const int D4 = D >> 2;
    float4 v[4];
    float ss = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int c = threadIdx.x + q * blockDim.x;
        v[q] = c < D4 ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        ss += v[q].x * v[q].x + v[q].y * v[q].y + v[q].z * v[q].z + v[q].w * v[q].w;
    }
    for (int c = threadIdx.x + 4 * blockDim.x; c < D4; c += blockDim.x) {
        const float4 t = xr[c];
        ss += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
    }
    ss = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(ss / (float) D + eps);
    const int orow = row_map ? row_map[i] : i;
    for (int c = threadIdx.x; c < D4; c += blockDim.x) {
        const float4 t = xr[c], ww = w4[c];
        const float4 y = make_float4((t.x * scale) * ww.x, (t.y * scale) * ww.y, (t.z * scale) * ww.z, (t.w * scale) * ww.w);
        if (o16) {
            half2 h0 = __floats2half2_rn(y.x, y.y), h1 = __floats2half2_rn(y.z, y.w);
            uint2 u;
            u.x = *reinterpret_cast<uint32_t *>(&h0);
            u.y = *reinterpret_cast<uint32_t *>(&h1);
            *reinterpret_cast<uint2 *>(o16 + (size_t) i * ld16 + 4 * c) = u;
        }
        if (o32 && orow >= 0) *reinterpret_cast<float4 *>(o32 + (size_t) orow * ld32 + 4 * c) = y;
    }
}

__global__ void norm_add_kernel(float * x, const float * t, int D, const float * w, float eps) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    const int r = blockIdx.x;
    const float * tr = t + (size_t) r * D;
    float ss = 0.0f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) ss += tr[d] * tr[d];
    ss = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(ss / (float) D + eps);
    for (int d = threadIdx.x; d < D; d += blockDim.x) x[(size_t) r * D + d] += (tr[d] * scale) * w[d];
}

// x += RMSNorm(t) * w (a sub-block's post-norm and residual add), then y16 = RMSNorm(x) * w2, the
// norm that feeds the next sub-block (each thread re-reads only the elements it wrote)
__global__ void norm_add_norm_kernel(float * x, const float * t, int D, const float * w, float eps, const float * w2,
                                     half * y16, int ld16) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    const int r = blockIdx.x;
    const float * tr = t + (size_t) r * D;
    float * xr = x + (size_t) r * D;
    float ss = 0.0f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) ss += tr[d] * tr[d];
    ss = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(ss / (float) D + eps);
    float ss2 = 0.0f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        const float v = xr[d] + (tr[d] * scale) * w[d];
        xr[d] = v;
        ss2 += v * v;
    }
    ss2 = block_sum(ss2, red);
    const float scale2 = 1.0f / sqrtf(ss2 / (float) D + eps);
    for (int d = threadIdx.x; d < D; d += blockDim.x) y16[(size_t) r * ld16 + d] = __float2half_rn((xr[d] * scale2) * w2[d]);
}

// ------------------------------------------------------------------------------------ embeddings
__global__ void embed_rows_kernel(QRows e, const int * idx, float scale, float * o32, half * o16, int ld) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x;
    int row = idx[r];
    row = (row < 0 || row >= e.rows) ? 0 : row;
    const int8_t * q = e.qs + (size_t) row * e.K;
    const half * d = e.ds + (size_t) row * (e.K / 32);
    const half * mn = e.ms ? e.ms + (size_t) row * (e.K / 32) : nullptr;
    for (int k = threadIdx.x; k < e.K; k += blockDim.x) {
        const float v = ((float) q[k] * __half2float(d[k >> 5]) - (mn ? __half2float(mn[k >> 5]) : 0.0f)) * scale;
        if (o32) o32[(size_t) r * ld + k] = v;
        if (o16) o16[(size_t) r * ld + k] = __float2half_rn(v);
    }
}

__global__ void audio_embed_kernel(QRows e, const int * frames, int ldf, int nc, int vs, float * out,
                                   const int * row_active) {
    pdl_trigger();
    pdl_wait();
    // one CTA per frame; a thread owns 8 consecutive columns (one 8-byte load of int8 quants per
    // codebook) and sums the codebooks in order, eight rows of loads in flight at a time
    __shared__ int codes[128];
    const int r = blockIdx.x;
    const bool act = row_active ? row_active[r] != 0 : true;
    for (int cb = threadIdx.x; cb < nc && cb < 128; cb += blockDim.x) {
        const int c = frames[(size_t) r * ldf + cb];
        codes[cb] = (c < 0 || c >= vs) ? 0 : c;
    }
    __syncthreads();
    const int kb = e.K / 32;
    for (int c8 = threadIdx.x; c8 < e.K / 8; c8 += blockDim.x) {
        float acc[8];
#pragma unroll
        for (int q = 0; q < 8; q++) acc[q] = 0.0f;
        if (act) {
            for (int cb0 = 0; cb0 < nc; cb0 += 8) {
                uint2 u[8];
                float d[8], m[8];
#pragma unroll
                for (int t = 0; t < 8; t++) {
                    const int cb = cb0 + t;
                    u[t] = make_uint2(0u, 0u);
                    d[t] = m[t] = 0.0f;
                    if (cb < nc) {
                        const size_t row = (size_t) cb * vs + (cb < 128 ? codes[cb] : 0);
                        u[t] = *reinterpret_cast<const uint2 *>(e.qs + row * e.K + c8 * 8);
                        d[t] = __half2float(e.ds[row * kb + (c8 >> 2)]);
                        m[t] = e.ms ? __half2float(e.ms[row * kb + (c8 >> 2)]) : 0.0f;
                    }
                }
#pragma unroll
                for (int t = 0; t < 8; t++) {
                    if (cb0 + t >= nc) break;
                    const int8_t * q8 = reinterpret_cast<const int8_t *>(&u[t]);
#pragma unroll
                    for (int q = 0; q < 8; q++) acc[q] += (float) q8[q] * d[t] - m[t];
                }
            }
        }
        float4 * o = reinterpret_cast<float4 *>(out + (size_t) r * e.K + c8 * 8);
        o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
}

// ------------------------------------------------------------------------------------ attention
template <int HD>
__device__ __forceinline__ void rope_apply(float (&x)[HD / 32], const float2 * cs, int lane) {
    constexpr int E = HD / 32;
#pragma unroll
    for (int j = 0; j < E / 2; j++) {
        const float2 c = cs[lane + 32 * j];
        const float x0 = x[j], x1 = x[j + E / 2];
        x[j] = x0 * c.x - x1 * c.y;
        x[j + E / 2] = x0 * c.y + x1 * c.x;
    }
}

template <int HD>
__device__ __forceinline__ void head_rmsnorm(float (&x)[HD / 32], const float * w, float eps, int lane) {
    constexpr int E = HD / 32;
    float ss = 0.0f;
#pragma unroll
    for (int e = 0; e < E; e++) ss += x[e] * x[e];
    ss = warp_sum(ss);
    const float scale = 1.0f / sqrtf(ss / (float) HD + eps);
#pragma unroll
    for (int e = 0; e < E; e++) x[e] = (x[e] * scale) * w[lane + 32 * e];
}

__device__ __forceinline__ size_t paged_off(const AttnKV & kv, const int * page_row, int p, int kvsel, int h,
                                            int n_kv, int HD) {
    const int page = page_row[p >> 4];
    return ((((size_t) page * kv.n_layer + kv.layer) * 2 + kvsel) * n_kv + h) * 16 * HD + (size_t) (p & 15) * HD;
}

// K/V tile of 32 positions of one kv head, fetched by the 128 threads of a decode CTA into
// registers (so the next tile's loads overlap this tile's math) and stored as f32 in shared
// memory; positions past `lim` read as zero
template <int HD, bool PAGED>
struct KvTileRegs {
    static constexpr int VEC = PAGED ? 8 : 4;
    static constexpr int PER_ROW = HD / VEC;
    static constexpr int NV = 32 * PER_ROW;
    static constexpr int PT = NV / 128;
    uint4 k[PT], v[PT];

    __device__ __forceinline__ void load(const AttnKV & kv, const int * page_row, int b, int h, int n_kv, int t0, int lim) {
        int pg0 = 0, pg1 = 0;
        if (PAGED) {
            pg0 = page_row[t0 >> 4];
            pg1 = ((t0 >> 4) + 1 < kv.max_pages) ? page_row[(t0 >> 4) + 1] : pg0;
        }
#pragma unroll
        for (int i = 0; i < PT; i++) {
            const int vi = threadIdx.x + i * 128;
            const int j = vi / PER_ROW, c = vi % PER_ROW;
            const int p = t0 + j;
            k[i] = v[i] = make_uint4(0u, 0u, 0u, 0u);
            if (p < lim) {
                if (PAGED) {
                    const int page = (j < 16) ? pg0 : pg1;
                    const size_t base = ((((size_t) page * kv.n_layer + kv.layer) * 2) * n_kv + h) * 16 * HD +
                                        (size_t) (p & 15) * HD + c * 8;
                    const size_t vstride = (size_t) n_kv * 16 * HD;
                    k[i] = *reinterpret_cast<const uint4 *>(kv.pool + base);
                    v[i] = *reinterpret_cast<const uint4 *>(kv.pool + base + vstride);
                } else {
                    const size_t base = (((size_t) b * kv.cap + p) * 2) * n_kv * HD + (size_t) h * HD + c * 4;
                    k[i] = *reinterpret_cast<const uint4 *>(kv.flat + base);
                    v[i] = *reinterpret_cast<const uint4 *>(kv.flat + base + (size_t) n_kv * HD);
                }
            }
        }
    }

    __device__ __forceinline__ void store(float (*sk)[HD + 1], float (*sv)[HD + 1]) const {
#pragma unroll
        for (int i = 0; i < PT; i++) {
            const int vi = threadIdx.x + i * 128;
            const int j = vi / PER_ROW, c = vi % PER_ROW;
            if (PAGED) {
                const half2 * hk = reinterpret_cast<const half2 *>(&k[i]);
                const half2 * hv = reinterpret_cast<const half2 *>(&v[i]);
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float2 fk = __half22float2(hk[q]), fv = __half22float2(hv[q]);
                    sk[j][c * 8 + 2 * q] = fk.x;
                    sk[j][c * 8 + 2 * q + 1] = fk.y;
                    sv[j][c * 8 + 2 * q] = fv.x;
                    sv[j][c * 8 + 2 * q + 1] = fv.y;
                }
            } else {
                const float * fk = reinterpret_cast<const float *>(&k[i]);
                const float * fv = reinterpret_cast<const float *>(&v[i]);
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    sk[j][c * 4 + q] = fk[q];
                    sv[j][c * 4 + q] = fv[q];
                }
            }
        }
    }
};

template <int HD>
struct DecodeSmem {
    float k[32][HD + 1];
    float v[32][HD + 1];
    float q[4][2][HD];
};

// decode attention for one session and one kv head: 128 threads; warp w < G (the GQA group,
// at most 4) owns query head h*G + w. The CTA first normalises, rotates and appends the new
// tokens' keys and values (1 token, or 2 for the depth decoder's first sub-step), then runs an
// online softmax over 32-position tiles of the session's cache.
template <int HD, bool PAGED>
__global__ void __launch_bounds__(128) attn_decode_kernel(const AttnDecodeArgs a) {
    pdl_trigger();
    pdl_wait();
    constexpr int E = HD / 32;
    __shared__ DecodeSmem<HD> sm;
    const int b = blockIdx.x, h = blockIdx.y, z = blockIdx.z, S = a.splits;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.n_head / a.n_kv;
    const bool qwarp = warp < G;
    const int slot = a.row_slot ? a.row_slot[b] : b;
    const bool act = (a.row_active ? a.row_active[b] != 0 : true) && slot >= 0;
    const int n_new = a.n_new;
    const int qh = h * G + warp;
    if (!act) {
        if (qwarp && z == 0)
            for (int i = 0; i < n_new; i++)
                for (int e = 0; e < E; e++)
                    a.out[(size_t) (b + i * a.R) * a.ldo + qh * HD + lane + 32 * e] = __float2half_rn(0.0f);
        return;
    }
    const int start = a.st ? a.st[slot].pos : a.start;
    const int L = start + n_new;
    const int * page_row = PAGED ? a.kv.page_table + (size_t) slot * a.kv.max_pages : nullptr;
    // this CTA's positions [p0, p1): equal 32-aligned shares of the cache
    const int share = ((L + S - 1) / S + 31) & ~31;
    const int p0 = min(L, z * share), p1 = min(L, p0 + share);

    // 1. normalise, rotate and append the new tokens' keys and values (each split appends the
    //    new positions in its own range, the only ones it reads)
    for (int task = warp; task < 2 * n_new; task += 4) {
        const int i = task >> 1;
        const int isv = task & 1;
        if (start + i < p0 || start + i >= p1) continue;
        const int row = b + i * a.R;
        const float * src = a.qkv + (size_t) row * a.ldq + a.n_head * HD + isv * a.n_kv * HD + h * HD;
        float x[E];
#pragma unroll
        for (int e = 0; e < E; e++) x[e] = src[lane + 32 * e];
        if (!isv) {
            if (a.k_norm) head_rmsnorm<HD>(x, a.k_norm, a.eps, lane);
            rope_apply<HD>(x, a.rope + (size_t) (start + i) * (HD / 2), lane);
        }
        const int p = start + i;
        if (PAGED) {
            half * dst = a.kv.pool + paged_off(a.kv, page_row, p, isv, h, a.n_kv, HD);
#pragma unroll
            for (int e = 0; e < E; e++) dst[lane + 32 * e] = __float2half_rn(x[e]);
        } else {
            float * dst = a.kv.flat + (((size_t) b * a.kv.cap + p) * 2 + isv) * a.n_kv * HD + (size_t) h * HD;
#pragma unroll
            for (int e = 0; e < E; e++) dst[lane + 32 * e] = x[e];
        }
    }
    // 2. this warp's query head for each new token
    if (qwarp) {
        for (int i = 0; i < n_new; i++) {
            const float * src = a.qkv + (size_t) (b + i * a.R) * a.ldq + qh * HD;
            float x[E];
#pragma unroll
            for (int e = 0; e < E; e++) x[e] = src[lane + 32 * e];
            if (a.q_norm) head_rmsnorm<HD>(x, a.q_norm, a.eps, lane);
            rope_apply<HD>(x, a.rope + (size_t) (start + i) * (HD / 2), lane);
#pragma unroll
            for (int e = 0; e < E; e++) sm.q[warp][i][lane + 32 * e] = x[e];
        }
    }
    __syncthreads();  // appended keys/values visible to the whole CTA before the first tile load

    float m[2] = { -INFINITY, -INFINITY }, l[2] = { 0.0f, 0.0f };
    float acc[2][E];
#pragma unroll
    for (int i = 0; i < 2; i++)
#pragma unroll
        for (int e = 0; e < E; e++) acc[i][e] = 0.0f;

    KvTileRegs<HD, PAGED> regs;
    if (p0 < p1) regs.load(a.kv, page_row, b, h, a.n_kv, p0, p1);
    for (int t0 = p0; t0 < p1; t0 += 32) {
        __syncthreads();
        regs.store(sm.k, sm.v);
        __syncthreads();
        if (t0 + 32 < p1) regs.load(a.kv, page_row, b, h, a.n_kv, t0 + 32, p1);
        if (!qwarp) continue;
#pragma unroll
        for (int i = 0; i < 2; i++) {
            if (i >= n_new) break;
            const int lim = min(start + i + 1, p1);
            const int p = t0 + lane;
            float sc = -INFINITY;
            if (p < lim) {
                float dot = 0.0f;
#pragma unroll 16
                for (int d = 0; d < HD; d++) dot += sm.q[warp][i][d] * sm.k[lane][d];
                sc = dot * a.scale;
            }
            const float tmax = warp_max(sc);
            if (tmax == -INFINITY) continue;
            const float mn = fmaxf(m[i], tmax);
            const float corr = expf(m[i] - mn);
            const float pr = p < lim ? expf(sc - mn) : 0.0f;
            l[i] = l[i] * corr + warp_sum(pr);
#pragma unroll
            for (int e = 0; e < E; e++) acc[i][e] *= corr;
            const int jmax = min(32, lim - t0);
            for (int j = 0; j < jmax; j++) {
                const float pj = __shfl_sync(0xffffffffu, pr, j);
#pragma unroll
                for (int e = 0; e < E; e++) acc[i][e] += pj * sm.v[j][lane + 32 * e];
            }
            m[i] = mn;
        }
    }
    if (S == 1) {
        if (!qwarp) return;
#pragma unroll
        for (int i = 0; i < 2; i++) {
            if (i >= n_new) break;
            const float inv = 1.0f / l[i];
#pragma unroll
            for (int e = 0; e < E; e++)
                a.out[(size_t) (b + i * a.R) * a.ldo + qh * HD + lane + 32 * e] = __float2half_rn(acc[i][e] * inv);
        }
        return;
    }
    // split-KV: publish this range's state, then the last CTA of (b, h) combines every range
    constexpr int PL = HD + 2;
    float * base = a.part + ((size_t) (b * a.n_kv + h) * S) * (4 * 2 * PL);
    if (qwarp) {
        for (int i = 0; i < n_new; i++) {
            float * pp = base + ((size_t) z * 8 + warp * 2 + i) * PL;
#pragma unroll
            for (int e = 0; e < E; e++) pp[lane + 32 * e] = acc[i][e];
            if (lane == 0) {
                pp[HD] = m[i];
                pp[HD + 1] = l[i];
            }
        }
    }
    __threadfence();
    __syncthreads();
    __shared__ int s_last;
    if (threadIdx.x == 0) {
        int * ctr = a.counters + (size_t) b * a.n_kv + h;
        const int prev = atomicAdd(ctr, 1);
        s_last = prev == S - 1;
        if (s_last) *ctr = 0;  // ready for the next launch
    }
    __syncthreads();
    if (!s_last || !qwarp) return;
    __threadfence();
    for (int i = 0; i < n_new; i++) {
        float mx = -INFINITY;
        for (int zz = 0; zz < S; zz++) mx = fmaxf(mx, __ldcg(base + ((size_t) zz * 8 + warp * 2 + i) * PL + HD));
        float lsum = 0.0f, o[E];
#pragma unroll
        for (int e = 0; e < E; e++) o[e] = 0.0f;
        for (int zz = 0; zz < S; zz++) {
            const float * pp = base + ((size_t) zz * 8 + warp * 2 + i) * PL;
            const float mz = __ldcg(pp + HD), lz = __ldcg(pp + HD + 1);
            if (lz == 0.0f || mz == -INFINITY) continue;  // an empty range
            const float w = expf(mz - mx);
            lsum += lz * w;
#pragma unroll
            for (int e = 0; e < E; e++) o[e] += w * __ldcg(pp + lane + 32 * e);
        }
        const float inv = lsum > 0.0f ? 1.0f / lsum : 0.0f;
#pragma unroll
        for (int e = 0; e < E; e++)
            a.out[(size_t) (b + i * a.R) * a.ldo + qh * HD + lane + 32 * e] = __float2half_rn(o[e] * inv);
    }
}

// prefill: normalise/rotate q in place, k likewise, and write k,v to the cache or flat buffers
template <int HD, bool PAGED>
__global__ void qk_prep_kernel(const PrefillArgs a) {
    pdl_trigger();
    pdl_wait();
    constexpr int E = HD / 32;
    const int r = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    int p = a.start + r;
    const int * page_row = a.page_row;
    if (a.segs) {
        const int4 sg = a.segs[a.row_seg[r]];
        p = r - sg.x;
        if (PAGED) page_row = a.kv.page_table + (size_t) sg.z * a.kv.max_pages;
    }
    float * row = a.qkv + (size_t) r * a.ldq;
    const int tasks = a.n_head + 2 * a.n_kv;
    for (int task = warp; task < tasks; task += nw) {
        float x[E];
        float * src;
        int kind, h;
        if (task < a.n_head) { kind = 0; h = task; src = row + h * HD; }
        else if (task < a.n_head + a.n_kv) { kind = 1; h = task - a.n_head; src = row + (a.n_head + h) * HD; }
        else { kind = 2; h = task - a.n_head - a.n_kv; src = row + (a.n_head + a.n_kv + h) * HD; }
#pragma unroll
        for (int e = 0; e < E; e++) x[e] = src[lane + 32 * e];
        if (kind == 0 && a.q_norm) head_rmsnorm<HD>(x, a.q_norm, a.eps, lane);
        if (kind == 1 && a.k_norm) head_rmsnorm<HD>(x, a.k_norm, a.eps, lane);
        if (kind < 2) rope_apply<HD>(x, a.rope + (size_t) p * (HD / 2), lane);
        if (kind == 0) {
#pragma unroll
            for (int e = 0; e < E; e++) src[lane + 32 * e] = x[e];
        } else if (PAGED) {
            half * dst = a.kv.pool + paged_off(a.kv, page_row, p, kind - 1, h, a.n_kv, HD);
#pragma unroll
            for (int e = 0; e < E; e++) dst[lane + 32 * e] = __float2half_rn(x[e]);
        } else {
            half * dst = (kind == 1 ? a.flat_k : a.flat_v) + ((size_t) r * a.n_kv + h) * HD;
#pragma unroll
            for (int e = 0; e < E; e++) dst[lane + 32 * e] = __float2half_rn(x[e]);
        }
    }
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t & r0, uint32_t & r1, uint32_t & r2, uint32_t & r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t & r0, uint32_t & r1, uint32_t & r2, uint32_t & r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void * src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Backbone decode attention on the tensor cores (mma.sync m16n8k16, f16 operands, f32
// accumulation): one CTA per (session, kv head, position range) as in attn_decode_kernel, for one
// new token and head_dim HD in the paged cache. The G query heads of the kv head are the first G
// rows of a 16-row A tile (the rest zero); the range is read in chunks of 64 positions (four
// 16-position pages, one per warp) that asynchronous copies bring from the f16 cache to shared
// memory unchanged, one chunk ahead of the MMAs, so
// S = Q K^T and O += P V are two MMAs per 8 positions or 8 values instead of one FMA per
// (position, value). Each warp keeps an online softmax over its pages; the four warps' states
// are merged in shared memory, and split ranges are published and combined exactly as in
// attn_decode_kernel.
template <int HD>
__global__ void __launch_bounds__(128) attn_decode_mma_kernel(const AttnDecodeArgs a) {
    pdl_trigger();
    pdl_wait();
    constexpr int E = HD / 32, LD = HD + 8, CH = 64, PL = HD + 2;
    constexpr int V4 = CH * HD / 8 / 128;  // 16-byte pieces of K (and of V) per thread per chunk
    __shared__ __align__(16) half sq[16 * LD];
    __shared__ __align__(16) half sk2[2][CH * LD];
    __shared__ __align__(16) half sv2[2][CH * LD];
    __shared__ float sst[4][4][PL];  // per warp, per query head: weighted values, max (log2 units), sum
    __shared__ int s_last;
    const int b = blockIdx.x, h = blockIdx.y, z = blockIdx.z, S = a.splits;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tg = lane & 3;
    const int G = a.n_head / a.n_kv;
    const int slot = a.row_slot ? a.row_slot[b] : b;
    const bool act = (a.row_active ? a.row_active[b] != 0 : true) && slot >= 0;
    if (!act) {
        if (warp < G && z == 0)
            for (int e = 0; e < E; e++) a.out[(size_t) b * a.ldo + (h * G + warp) * HD + lane + 32 * e] = __float2half_rn(0.0f);
        return;
    }
    const int start = a.st ? a.st[slot].pos : a.start;
    const int L = start + 1;
    const int * page_row = a.kv.page_table + (size_t) slot * a.kv.max_pages;
    const int share = ((L + S - 1) / S + 31) & ~31;
    const int p0 = min(L, z * share), p1 = min(L, p0 + share);

    // 1. the new token's key and value (if in this range) and the query heads, as f16 rows
    if (warp < 2 && start >= p0 && start < p1) {
        const int isv = warp;
        const float * src = a.qkv + (size_t) b * a.ldq + a.n_head * HD + isv * a.n_kv * HD + h * HD;
        float x[E];
#pragma unroll
        for (int e = 0; e < E; e++) x[e] = src[lane + 32 * e];
        if (!isv) {
            if (a.k_norm) head_rmsnorm<HD>(x, a.k_norm, a.eps, lane);
            rope_apply<HD>(x, a.rope + (size_t) start * (HD / 2), lane);
        }
        half * dst = a.kv.pool + paged_off(a.kv, page_row, start, isv, h, a.n_kv, HD);
#pragma unroll
        for (int e = 0; e < E; e++) dst[lane + 32 * e] = __float2half_rn(x[e]);
    }
    if (warp < G) {
        const float * src = a.qkv + (size_t) b * a.ldq + (h * G + warp) * HD;
        float x[E];
#pragma unroll
        for (int e = 0; e < E; e++) x[e] = src[lane + 32 * e];
        if (a.q_norm) head_rmsnorm<HD>(x, a.q_norm, a.eps, lane);
        rope_apply<HD>(x, a.rope + (size_t) start * (HD / 2), lane);
#pragma unroll
        for (int e = 0; e < E; e++) sq[warp * LD + lane + 32 * e] = __float2half_rn(x[e]);
    }
    for (int i = tid; i < (16 - G) * HD; i += 128) sq[(G + i / HD) * LD + i % HD] = __float2half_rn(0.0f);

    // 2. chunks of 64 positions, double-buffered: positions past the range are zero-filled
    auto load_chunk = [&](int t0, int buf) {
        const uint32_t ku = (uint32_t) __cvta_generic_to_shared(sk2[buf]), vu = (uint32_t) __cvta_generic_to_shared(sv2[buf]);
#pragma unroll
        for (int i = 0; i < V4; i++) {
            const int vi = tid + 128 * i, j = vi / (HD / 8), c8 = vi % (HD / 8), pos = t0 + j;
            const bool valid = pos < p1;
            const size_t off = valid ? paged_off(a.kv, page_row, pos, 0, h, a.n_kv, HD) + 8 * c8 : 0;
            const size_t vstride = valid ? (size_t) a.n_kv * 16 * HD : 0;
            const uint32_t so = (uint32_t) (j * LD + 8 * c8) * 2;
            cp_async16(ku + so, a.kv.pool + off, valid);
            cp_async16(vu + so, a.kv.pool + off + vstride, valid);
        }
    };
    __syncthreads();  // the appended key/value (global) and the query rows (shared) are visible
    const float sl2 = a.scale * 1.4426950408889634f;
    float o[HD / 8][4];
#pragma unroll
    for (int n = 0; n < HD / 8; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;
    const uint32_t sq_u = (uint32_t) __cvta_generic_to_shared(sq);
    if (p0 < p1) load_chunk(p0, 0);
    cp_async_commit();
    for (int t0 = p0, it = 0; t0 < p1; t0 += CH, it++) {
        if (t0 + CH < p1) load_chunk(t0 + CH, (it + 1) & 1);
        cp_async_commit();  // possibly empty: the wait below always leaves exactly the newest group
        cp_async_wait1();
        __syncthreads();    // every thread's copies of this chunk have landed
        const uint32_t sk_u = (uint32_t) __cvta_generic_to_shared(sk2[it & 1]), sv_u = (uint32_t) __cvta_generic_to_shared(sv2[it & 1]);
        const int w0 = t0 + 16 * warp;  // this warp's page
        if (w0 < p1) {
            float sc[2][4];
#pragma unroll
            for (int n = 0; n < 2; n++) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < HD / 16; kk++) {
                uint32_t af[4], b0, b1, b2, b3;
                const int qr = (lane & 7) + ((lane >> 3) & 1) * 8, qc = 16 * kk + (lane >> 4) * 8;
                ldsm_x4(sq_u + (uint32_t) (qr * LD + qc) * 2, af[0], af[1], af[2], af[3]);
                const int kr_ = 16 * warp + (lane & 7) + (lane >> 4) * 8, kc = 16 * kk + ((lane >> 3) & 1) * 8;
                ldsm_x4(sk_u + (uint32_t) (kr_ * LD + kc) * 2, b0, b1, b2, b3);
                mma16816(sc[0], af, b0, b1);
                mma16816(sc[1], af, b2, b3);
            }
            float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
            for (int n = 0; n < 2; n++) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const bool ok = w0 + 8 * n + 2 * tg + e < p1;
                    sc[n][e] = ok ? sc[n][e] * sl2 : -INFINITY;
                    sc[n][2 + e] = ok ? sc[n][2 + e] * sl2 : -INFINITY;
                    mx_a = fmaxf(mx_a, sc[n][e]);
                    mx_b = fmaxf(mx_b, sc[n][2 + e]);
                }
            }
#pragma unroll
            for (int off = 1; off <= 2; off <<= 1) {
                mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
                mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
            }
            // every page holds at least one valid position, so the new maxima are finite
            const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
            const float c_a = exp2f(m_a - mn_a), c_b = exp2f(m_b - mn_b);
            m_a = mn_a;
            m_b = mn_b;
            float sum_a = 0.0f, sum_b = 0.0f;
#pragma unroll
            for (int n = 0; n < 2; n++) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    sc[n][e] = sc[n][e] == -INFINITY ? 0.0f : exp2f(sc[n][e] - mn_a);
                    sc[n][2 + e] = sc[n][2 + e] == -INFINITY ? 0.0f : exp2f(sc[n][2 + e] - mn_b);
                    sum_a += sc[n][e];
                    sum_b += sc[n][2 + e];
                }
            }
            l_a = l_a * c_a + sum_a;
            l_b = l_b * c_b + sum_b;
            uint32_t pf[4];
            pf[0] = pack_h2(sc[0][0], sc[0][1]);
            pf[1] = pack_h2(sc[0][2], sc[0][3]);
            pf[2] = pack_h2(sc[1][0], sc[1][1]);
            pf[3] = pack_h2(sc[1][2], sc[1][3]);
#pragma unroll
            for (int n2 = 0; n2 < HD / 16; n2++) {
                o[2 * n2][0] *= c_a; o[2 * n2][1] *= c_a; o[2 * n2][2] *= c_b; o[2 * n2][3] *= c_b;
                o[2 * n2 + 1][0] *= c_a; o[2 * n2 + 1][1] *= c_a; o[2 * n2 + 1][2] *= c_b; o[2 * n2 + 1][3] *= c_b;
                uint32_t b0, b1, b2, b3;
                const int vr_ = 16 * warp + (lane & 7) + ((lane >> 3) & 1) * 8, vc = 16 * n2 + (lane >> 4) * 8;
                ldsm_x4_t(sv_u + (uint32_t) (vr_ * LD + vc) * 2, b0, b1, b2, b3);
                mma16816(o[2 * n2], pf, b0, b1);
                mma16816(o[2 * n2 + 1], pf, b2, b3);
            }
        }
        __syncthreads();  // every warp is done with this buffer before the copies after next refill it
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) l_a += __shfl_xor_sync(0xffffffffu, l_a, off);

    // 3. merge the four warps' states of each query head (rows g < G live in lanes 0..4G-1)
    if (g < G) {
#pragma unroll
        for (int n = 0; n < HD / 8; n++) {
            sst[warp][g][8 * n + 2 * tg] = o[n][0];
            sst[warp][g][8 * n + 2 * tg + 1] = o[n][1];
        }
        if (tg == 0) {
            sst[warp][g][HD] = m_a;
            sst[warp][g][HD + 1] = l_a;
        }
    }
    __syncthreads();
    float * base = a.part + ((size_t) (b * a.n_kv + h) * S) * (4 * 2 * PL);
    for (int i = tid; i < G * HD; i += 128) {
        const int r = i / HD, d = i % HD;
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; w++) mx = fmaxf(mx, sst[w][r][HD]);
        float ov = 0.0f, lv = 0.0f;
        if (mx != -INFINITY) {
#pragma unroll
            for (int w = 0; w < 4; w++) {
                const float mw = sst[w][r][HD];
                if (mw == -INFINITY) continue;
                const float f = exp2f(mw - mx);
                ov += f * sst[w][r][d];
                lv += f * sst[w][r][HD + 1];
            }
        }
        if (S == 1) {
            a.out[(size_t) b * a.ldo + (h * G + r) * HD + d] = __float2half_rn(lv > 0.0f ? ov / lv : 0.0f);
        } else {
            // the published state in natural-log units, as attn_decode_kernel writes it
            float * pp = base + ((size_t) z * 8 + r * 2) * PL;
            pp[d] = ov;
            if (d == 0) {
                pp[HD] = mx == -INFINITY ? -INFINITY : mx * 0.6931471805599453f;
                pp[HD + 1] = lv;
            }
        }
    }
    if (S == 1) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        int * ctr = a.counters + (size_t) b * a.n_kv + h;
        const int prev = atomicAdd(ctr, 1);
        s_last = prev == S - 1;
        if (s_last) *ctr = 0;  // ready for the next launch
    }
    __syncthreads();
    if (!s_last || warp >= G) return;
    __threadfence();
    float mx = -INFINITY;
    for (int zz = 0; zz < S; zz++) mx = fmaxf(mx, __ldcg(base + ((size_t) zz * 8 + warp * 2) * PL + HD));
    float lsum = 0.0f, ov[E];
#pragma unroll
    for (int e = 0; e < E; e++) ov[e] = 0.0f;
    for (int zz = 0; zz < S; zz++) {
        const float * pp = base + ((size_t) zz * 8 + warp * 2) * PL;
        const float mz = __ldcg(pp + HD), lz = __ldcg(pp + HD + 1);
        if (lz == 0.0f || mz == -INFINITY) continue;  // an empty range
        const float w = expf(mz - mx);
        lsum += lz * w;
#pragma unroll
        for (int e = 0; e < E; e++) ov[e] += w * __ldcg(pp + lane + 32 * e);
    }
    const float inv = lsum > 0.0f ? 1.0f / lsum : 0.0f;
#pragma unroll
    for (int e = 0; e < E; e++) a.out[(size_t) b * a.ldo + (h * G + warp) * HD + lane + 32 * e] = __float2half_rn(ov[e] * inv);
}

template <int HD>
__host__ __device__ constexpr int prefill_kb() { return HD >= 256 ? 32 : 64; }
template <int HD>
constexpr size_t prefill_smem() { return (size_t) (kPrefillQBlock + 4 * prefill_kb<HD>()) * (HD + 8) * sizeof(half); }

// Prefill attention on the tensor cores (mma.sync m16n8k16, f16 operands, f32 accumulation and
// online softmax): one CTA per (query block of 64 rows of one sequence, query head), 4 warps of
// 16 query rows. Q is staged once as f16; K and V tiles of KB f16 positions come by cp.async into
// two shared-memory buffers, the next tile's copies in flight while the current one is used
// (rows padded by 8 halves so ldmatrix rows fall in distinct banks). S = Q K^T
// comes from ldmatrix fragments of Q and K, P = exp(S - max) is repacked from the accumulator
// registers into A fragments, and V is read with the transposing ldmatrix. Causal, windowed
// (text encoder) and full spans are per query row, as in the f32 restatement.
template <int HD, bool PAGED>
__global__ void __launch_bounds__(128) attn_prefill_kernel(const PrefillArgs a) {
    pdl_trigger();
    pdl_wait();
    constexpr int QB = kPrefillQBlock, KB = prefill_kb<HD>(), LD = HD + 8;
    extern __shared__ __align__(16) unsigned char psm_raw[];
    half * sq = reinterpret_cast<half *>(psm_raw);  // [QB][LD]
    half * sk = sq + QB * LD;                        // [2][KB][LD]
    half * sv = sk + 2 * KB * LD;                    // [2][KB][LD]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tg = lane & 3;
    // this CTA's sequence: rows [base, base + T) of the packed rows (one sequence: all of them)
    int base = 0, T = a.T, r0 = blockIdx.x * QB;
    const int * page_row = a.page_row;
    if (a.qblocks) {
        const int2 qb = a.qblocks[blockIdx.x];
        const int4 sg = a.segs[qb.x];
        base = sg.x; T = sg.y; r0 = qb.y;
        if (PAGED) page_row = a.kv.page_table + (size_t) sg.z * a.kv.max_pages;
    }
    const int qh = blockIdx.y, h = qh / (a.n_head / a.n_kv);
    const int nq = min(QB, T - r0);
    const int left = (a.window + 1) / 2, right = a.window / 2 + 1;
    auto span = [&](int r, int & lo, int & hi) {
        if (a.causal) { lo = 0; hi = a.start + r + 1; }
        else if (a.window > 0) { lo = max(0, r - left + 1); hi = min(T, r + right); }
        else { lo = 0; hi = T; }
    };
    int lo_min, hi_max, tmp;
    span(r0, lo_min, tmp);
    span(r0 + nq - 1, tmp, hi_max);
    // Q block as f16 (rows past the sequence are zero)
    for (int i = threadIdx.x; i < QB * (HD / 4); i += blockDim.x) {
        const int row = i / (HD / 4), c4 = i - row * (HD / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row < nq) v = *reinterpret_cast<const float4 *>(a.qkv + (size_t) (base + r0 + row) * a.ldq + qh * HD + 4 * c4);
        half2 * d = reinterpret_cast<half2 *>(sq + row * LD + 4 * c4);
        d[0] = __floats2half2_rn(v.x, v.y);
        d[1] = __floats2half2_rn(v.z, v.w);
    }
    // this thread's two query rows and their spans
    const int ra = r0 + 16 * warp + g, rb = ra + 8;
    int lo_a = 0, hi_a = 0, lo_b = 0, hi_b = 0;
    if (ra < r0 + nq) span(ra, lo_a, hi_a);
    if (rb < r0 + nq) span(rb, lo_b, hi_b);
    const float sl2 = a.scale * 1.4426950408889634f;  // scores in log2 units
    float o[HD / 8][4];
#pragma unroll
    for (int n = 0; n < HD / 8; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;
    const uint32_t sq_u = (uint32_t) __cvta_generic_to_shared(sq), sk_u = (uint32_t) __cvta_generic_to_shared(sk),
                   sv_u = (uint32_t) __cvta_generic_to_shared(sv);
    // K and V of positions [t0, t0 + KB) into buffer b (positions past hi_max read as zeros; their
    // copy addresses stay on a position the CTA reads anyway)
    auto load_tile = [&](int t0, int b) {
        const uint32_t dk = sk_u + (uint32_t) (b * KB * LD) * 2, dv = sv_u + (uint32_t) (b * KB * LD) * 2;
        for (int i = threadIdx.x; i < KB * (HD / 8); i += blockDim.x) {
            const int j = i / (HD / 8), c8 = i - j * (HD / 8);
            const int pos = t0 + j;
            const bool valid = pos < hi_max;
            const int pc = valid ? pos : lo_min;
            const half * ks, * vs;
            if (PAGED) {
                ks = a.kv.pool + paged_off(a.kv, page_row, pc, 0, h, a.n_kv, HD) + 8 * c8;
                vs = a.kv.pool + paged_off(a.kv, page_row, pc, 1, h, a.n_kv, HD) + 8 * c8;
            } else {
                const size_t off = ((size_t) (base + pc) * a.n_kv + h) * HD + 8 * c8;
                ks = a.flat_k + off;
                vs = a.flat_v + off;
            }
            const uint32_t so = (uint32_t) (j * LD + 8 * c8) * 2;
            cp_async16(dk + so, ks, valid);
            cp_async16(dv + so, vs, valid);
        }
    };
    const int t_first = (lo_min / KB) * KB;
    if (t_first < hi_max) load_tile(t_first, 0);
    cp_async_commit();
    int buf = 0;
    for (int t0 = t_first; t0 < hi_max; t0 += KB, buf ^= 1) {
        if (t0 + KB < hi_max) load_tile(t0 + KB, buf ^ 1);
        cp_async_commit();  // possibly empty: the wait leaves only the newest group in flight
        cp_async_wait1();
        __syncthreads();
        const uint32_t skb = sk_u + (uint32_t) (buf * KB * LD) * 2, svb = sv_u + (uint32_t) (buf * KB * LD) * 2;
        // S = Q K^T for rows 16w..16w+15 and the tile's KB positions
        float sc[KB / 8][4];
#pragma unroll
        for (int n = 0; n < KB / 8; n++) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
            uint32_t af[4];
            const int qr = 16 * warp + (lane & 7) + ((lane >> 3) & 1) * 8, qc = 16 * kk + (lane >> 4) * 8;
            ldsm_x4(sq_u + (uint32_t) (qr * LD + qc) * 2, af[0], af[1], af[2], af[3]);
#pragma unroll
            for (int n2 = 0; n2 < KB / 16; n2++) {
                uint32_t b0, b1, b2, b3;
                const int kr = 16 * n2 + (lane & 7) + (lane >> 4) * 8, kc = 16 * kk + ((lane >> 3) & 1) * 8;
                ldsm_x4(skb + (uint32_t) (kr * LD + kc) * 2, b0, b1, b2, b3);
                mma16816(sc[2 * n2], af, b0, b1);
                mma16816(sc[2 * n2 + 1], af, b2, b3);
            }
        }
        // masks, running maxima and probabilities (rows ra: elements 0-1, rb: elements 2-3)
        float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
        for (int n = 0; n < KB / 8; n++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int pos = t0 + 8 * n + 2 * tg + e;
                sc[n][e] = (pos >= lo_a && pos < hi_a) ? sc[n][e] * sl2 : -INFINITY;
                sc[n][2 + e] = (pos >= lo_b && pos < hi_b) ? sc[n][2 + e] * sl2 : -INFINITY;
                mx_a = fmaxf(mx_a, sc[n][e]);
                mx_b = fmaxf(mx_b, sc[n][2 + e]);
            }
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
            mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
            mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
        }
        const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
        // a row with no position yet keeps its (zero) state: its scores are all -inf
        const float c_a = mn_a == -INFINITY ? 1.0f : exp2f(m_a - mn_a);
        const float c_b = mn_b == -INFINITY ? 1.0f : exp2f(m_b - mn_b);
        m_a = mn_a;
        m_b = mn_b;
        float sum_a = 0.0f, sum_b = 0.0f;
#pragma unroll
        for (int n = 0; n < KB / 8; n++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                sc[n][e] = sc[n][e] == -INFINITY ? 0.0f : exp2f(sc[n][e] - mn_a);
                sc[n][2 + e] = sc[n][2 + e] == -INFINITY ? 0.0f : exp2f(sc[n][2 + e] - mn_b);
                sum_a += sc[n][e];
                sum_b += sc[n][2 + e];
            }
        }
        l_a = l_a * c_a + sum_a;
        l_b = l_b * c_b + sum_b;
#pragma unroll
        for (int n = 0; n < HD / 8; n++) {
            o[n][0] *= c_a; o[n][1] *= c_a;
            o[n][2] *= c_b; o[n][3] *= c_b;
        }
        // O += P V: P's accumulator layout is the A fragment layout of two adjacent position tiles
#pragma unroll
        for (int k2 = 0; k2 < KB / 16; k2++) {
            uint32_t pf[4];
            pf[0] = pack_h2(sc[2 * k2][0], sc[2 * k2][1]);
            pf[1] = pack_h2(sc[2 * k2][2], sc[2 * k2][3]);
            pf[2] = pack_h2(sc[2 * k2 + 1][0], sc[2 * k2 + 1][1]);
            pf[3] = pack_h2(sc[2 * k2 + 1][2], sc[2 * k2 + 1][3]);
#pragma unroll
            for (int n2 = 0; n2 < HD / 16; n2++) {
                uint32_t b0, b1, b2, b3;
                const int vr = 16 * k2 + (lane & 7) + ((lane >> 3) & 1) * 8, vc = 16 * n2 + (lane >> 4) * 8;
                ldsm_x4_t(svb + (uint32_t) (vr * LD + vc) * 2, b0, b1, b2, b3);
                mma16816(o[2 * n2], pf, b0, b1);
                mma16816(o[2 * n2 + 1], pf, b2, b3);
            }
        }
        __syncthreads();  // every warp is done with buffer buf before the next tile's copies reuse it
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
        l_a += __shfl_xor_sync(0xffffffffu, l_a, off);
        l_b += __shfl_xor_sync(0xffffffffu, l_b, off);
    }
    const float inv_a = l_a > 0.0f ? 1.0f / l_a : 0.0f, inv_b = l_b > 0.0f ? 1.0f / l_b : 0.0f;
#pragma unroll
    for (int n = 0; n < HD / 8; n++) {
        const int col = qh * HD + 8 * n + 2 * tg;
        if (ra < r0 + nq)
            *reinterpret_cast<half2 *>(a.out + (size_t) (base + ra) * a.ldo + col) = __floats2half2_rn(o[n][0] * inv_a, o[n][1] * inv_a);
        if (rb < r0 + nq)
            *reinterpret_cast<half2 *>(a.out + (size_t) (base + rb) * a.ldo + col) = __floats2half2_rn(o[n][2] * inv_b, o[n][3] * inv_b);
    }
}

// ------------------------------------------------------------------------------------ step glue
__global__ void step_init_kernel(const StepArgs a) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x;
    const int slot = a.row_slot[r];
    const bool act = slot >= 0 && a.st[slot].active != 0;
    const int k = *a.step_ctr;
    if (threadIdx.x == 0) {
        a.row_active[r] = act ? 1 : 0;
        a.frames[(size_t) r * a.nc] = act ? (a.force ? a.force[(size_t) r * a.nc] : a.st[slot].last_cb0) : -1;
        if (act) atomicOr(&a.any_active[k], 1);
    }
    const int cb0 = act ? (a.force ? a.force[(size_t) r * a.nc] : a.st[slot].last_cb0) : 0;
    const int row = (cb0 < 0 || cb0 >= a.embd.rows) ? 0 : cb0;
    for (int d = threadIdx.x; d < a.H; d += blockDim.x) {
        half h0 = __float2half_rn(0.0f), h1 = __float2half_rn(0.0f);
        if (act) {
            h0 = __float2half_rn(a.hid32[(size_t) slot * a.H + d]);
            const size_t sb = (size_t) row * (a.embd.K / 32) + (d >> 5);
            const float e = (float) a.embd.qs[(size_t) row * a.embd.K + d] * __half2float(a.embd.ds[sb]) -
                            (a.embd.ms ? __half2float(a.embd.ms[sb]) : 0.0f);
            h1 = __float2half_rn(e);
        }
        a.din16[(size_t) r * a.H + d] = h0;
        a.din16[(size_t) (a.R + r) * a.H + d] = h1;
    }
}

// dst[0..K) = f16(q * d) of one Q8_0 embedding row, 8 values per 8-byte load
__device__ __forceinline__ void embed_row_f16(const QRows & e, size_t row, half * dst) {
    const int8_t * q = e.qs + row * e.K;
    const half * d = e.ds + row * (e.K / 32);
    const half * mn = e.ms ? e.ms + row * (e.K / 32) : nullptr;
    for (int c = threadIdx.x; c < e.K / 8; c += blockDim.x) {
        const uint2 u = *reinterpret_cast<const uint2 *>(q + c * 8);
        const float sc = __half2float(d[c >> 2]), m = mn ? __half2float(mn[c >> 2]) : 0.0f;
        const int8_t * b = reinterpret_cast<const int8_t *>(&u);
        half2 o[4];
#pragma unroll
        for (int j = 0; j < 4; j++) o[j] = __floats2half2_rn((float) b[2 * j] * sc - m, (float) b[2 * j + 1] * sc - m);
        *reinterpret_cast<uint4 *>(dst + c * 8) = *reinterpret_cast<uint4 *>(o);
    }
}

__global__ void argmax_gather_kernel(const StepArgs a, const float * logits, int ld, int V, int col, int gather_cb) {
    pdl_trigger();
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ int s_code;
    const int r = blockIdx.x;
    if (a.row_set && a.row_set[r] != a.set_id) return;
    if (!a.row_active[r]) {
        if (threadIdx.x == 0) a.frames[(size_t) r * a.nc + col] = -1;
        return;
    }
    const float * lr = logits + (size_t) r * ld;
    float best = -INFINITY;
    int bi = INT_MAX;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = lr[i];
        if (v > best || (bi == INT_MAX && !(v < best))) { best = v; bi = i; }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sv[warp] = best; si[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = sv[0];
        int i0 = si[0];
        for (int w = 1; w < (int) (blockDim.x >> 5); w++)
            if (sv[w] > b || (sv[w] == b && si[w] < i0)) { b = sv[w]; i0 = si[w]; }
        if (i0 == INT_MAX) i0 = 0;
        s_code = i0;
        a.frames[(size_t) r * a.nc + col] = i0;
    }
    __syncthreads();
    if (gather_cb < 0) return;
    embed_row_f16(a.embd, (size_t) gather_cb * a.vs + s_code, a.din16 + (size_t) r * a.H);
}

__device__ __forceinline__ unsigned int f2ord(float f) {
    const unsigned int b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

constexpr int kSortN = 4096;

// sort key: logit descending, then index ascending (the order of std::partial_sort's survivors
// when logits tie is unspecified; this picks the lowest index first)
__device__ __forceinline__ unsigned long long sort_key(float l, int i) {
    return ((unsigned long long) f2ord(l) << 32) | (unsigned long long) (0xFFFFFFFFu - (unsigned) i);
}
__device__ __forceinline__ int key_index(unsigned long long k) {
    return (int) (0xFFFFFFFFu - (unsigned) (k & 0xFFFFFFFFull));
}
// the logit back from its key (f2ord is a bijection on the bit patterns)
__device__ __forceinline__ float key_logit(unsigned long long k) {
    const unsigned int o = (unsigned int) (k >> 32);
    return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}

// descending bitonic sort of kSortN keys by the whole block
__device__ void sort_keys_desc(unsigned long long * keys) {
    for (int kk = 2; kk <= kSortN; kk <<= 1) {
        for (int j = kk >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < kSortN; i += blockDim.x) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long x = keys[i], y = keys[ixj];
                    const bool desc = (i & kk) == 0;
                    if (desc ? (x < y) : (x > y)) { keys[i] = y; keys[ixj] = x; }
                }
            }
            __syncthreads();
        }
    }
}

// One thread: src/sampling.cpp:25-59 over the sorted keys of the modified logits: keep the top k,
// softmax at the temperature, optional top-p cut with renormalisation, then the inverse CDF at the
// uniform u in place of std::discrete_distribution.
__device__ int pick_from_sorted(const unsigned long long * keys, int V, float temp_in, int top_k, float top_p,
                                float u) {
    const int keep = (top_k > 0 && top_k < V) ? top_k : V;
    const float temp = temp_in > 0.0f ? temp_in : 1.0f;
    const float maxl = key_logit(keys[0]);
    float sum = 0.0f;
    for (int i = 0; i < keep; i++) sum += expf((key_logit(keys[i]) - maxl) / temp);
    int cut = keep;
    float total = 1.0f;
    if (top_p < 1.0f) {
        float cum = 0.0f;
        for (int i = 0; i < keep; i++) {
            cum += expf((key_logit(keys[i]) - maxl) / temp) / sum;
            if (cum >= top_p) { cut = i + 1; break; }
        }
        total = 0.0f;
        for (int i = 0; i < cut; i++) total += expf((key_logit(keys[i]) - maxl) / temp) / sum;
    }
    // cdf over the kept probabilities (renormalised by `total` when top-p cut them)
    float cdf_last = 0.0f;
    for (int i = 0; i < cut; i++) {
        float pi = expf((key_logit(keys[i]) - maxl) / temp) / sum;
        if (top_p < 1.0f) pi = pi / total;
        cdf_last += pi;
    }
    const float target = u * cdf_last;
    int pick = key_index(keys[cut - 1]);
    float cdf = 0.0f;
    for (int i = 0; i < cut; i++) {
        float pi = expf((key_logit(keys[i]) - maxl) / temp) / sum;
        if (top_p < 1.0f) pi = pi / total;
        cdf += pi;
        if (target < cdf) { pick = key_index(keys[i]); break; }
    }
    return pick;
}

// The `keep` largest of the block's keys (each thread holds kv[0..3], unique keys, padding 0),
// sorted descending into sel[0..64) (the rest 0): a radix select finds the keep-th largest key
// one byte at a time from the top (8 histogram passes over the candidates still matching the
// bytes found), the keys at or above it are gathered, and one warp sorts those <= 64 keys.
// The result equals the first `keep` entries of sort_keys_desc over the same keys.
__device__ void select_top_keys(const unsigned long long (&kv)[4], int keep, unsigned long long * sel, int * hist,
                                unsigned long long * s_prefix, int * s_rem) {
    const int tid = threadIdx.x, lane = tid & 31;
    unsigned long long prefix = 0ull;
    int rem = keep;
    for (int d = 7; d >= 0; d--) {
        if (tid < 256) hist[tid] = 0;
        __syncthreads();
        const unsigned long long hi = d == 7 ? 0ull : (~0ull << (8 * (d + 1)));
#pragma unroll
        for (int q = 0; q < 4; q++)
            if ((kv[q] & hi) == (prefix & hi)) atomicAdd(&hist[(kv[q] >> (8 * d)) & 255], 1);
        __syncthreads();
        if (tid < 32) {
            // lane l scans bins 255 - 8 l down to 248 - 8 l: lanes in order visit the bins from the top
            int c = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) c += hist[255 - 8 * lane - j];
            int incl = c;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += t;
            }
            const unsigned m = __ballot_sync(0xffffffffu, incl >= rem);
            const int L = __ffs(m) - 1;
            if (lane == L) {
                int acc = incl - c;
                int b = 255 - 8 * lane - 7;
                for (int j = 0; j < 8; j++) {
                    const int h = hist[255 - 8 * lane - j];
                    if (acc + h >= rem) { b = 255 - 8 * lane - j; break; }
                    acc += h;
                }
                *s_prefix = prefix | ((unsigned long long) b << (8 * d));
                *s_rem = rem - acc;
            }
        }
        __syncthreads();
        prefix = *s_prefix;
        rem = *s_rem;
    }
    // prefix is now the keep-th largest key: exactly `keep` keys are >= it
    __syncthreads();  // every thread has read the last pass's shared results
    if (tid < 64) sel[tid] = 0ull;
    if (tid == 0) *s_rem = 0;
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 4; q++)
        if (kv[q] >= prefix) sel[atomicAdd(s_rem, 1)] = kv[q];
    __syncthreads();
    if (tid < 32) {
        for (int kk = 2; kk <= 64; kk <<= 1) {
            for (int j = kk >> 1; j > 0; j >>= 1) {
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int i = lane + 32 * h, ixj = i ^ j;
                    if (ixj > i) {
                        const unsigned long long x = sel[i], y = sel[ixj];
                        const bool desc = (i & kk) == 0;
                        if (desc ? (x < y) : (x > y)) { sel[i] = y; sel[ixj] = x; }
                    }
                }
                __syncwarp();
            }
        }
    }
    __syncthreads();
}

__device__ __forceinline__ float philox_unit(uint32_t key, uint32_t draw, uint32_t hi) {
    return (float) (philox_word0(key, draw, hi) >> 8) * (1.0f / 16777216.0f);
}

__global__ void __launch_bounds__(1024) sample_kernel(const SampleArgs a) {
    pdl_trigger();
    pdl_wait();
    __shared__ unsigned long long keys[kSortN];
    const int r = blockIdx.x;
    const int slot = a.row_slot[r];
    if (slot < 0) return;
    if (a.row_active && !a.row_active[r]) return;
    const int pr = a.row_pair ? a.row_pair[r] : -1;
    if (pr <= -2) return;  // the unconditional branch of a pair: its leader samples for both
    SessState & s = a.st[slot];
    if (!s.active) return;
    const float * lr = a.logits + (size_t) r * a.ld;
    const float * lu = pr >= 0 ? a.logits + (size_t) pr * a.ld : nullptr;
    const float cfg = s.cfg, rep = s.rep;
    const uint16_t * hr = a.hist + (size_t) slot * a.hist_ld;
    unsigned long long kv[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int i = threadIdx.x + q * blockDim.x;
        unsigned long long key = 0ull;
        if (i < a.V) {
            float l = lr[i];
            if (lu) l = lu[i] + cfg * (l - lu[i]);
            if (i >= a.sup_lo && i < a.sup_hi) l = -INFINITY;
            if (rep != 1.0f && i < a.hist_ld) {
                const int c = hr[i];
                for (int q2 = 0; q2 < c; q2++) l = l > 0.0f ? l / rep : l * rep;
            }
            key = sort_key(l, i);
        }
        kv[q] = key;
    }
    // top-k of at most 64 (the reference's 50): select instead of sorting every key
    const int keep = (s.top_k > 0 && s.top_k < a.V) ? s.top_k : a.V;
    __shared__ int s_hist[256];
    __shared__ unsigned long long s_sel[64], s_prefix;
    __shared__ int s_rem;
    const unsigned long long * sorted = keys;
    if (keep <= 64 && !a.force_sort) {
        select_top_keys(kv, keep, s_sel, s_hist, &s_prefix, &s_rem);
        sorted = s_sel;
    } else {
#pragma unroll
        for (int q = 0; q < 4; q++) keys[threadIdx.x + q * blockDim.x] = kv[q];
        __syncthreads();
        sort_keys_desc(keys);
    }
    if (threadIdx.x != 0) return;
    uint32_t key = s.key, draw = s.draw;
    if (a.seeds) { key = a.seeds[r] + (uint32_t) (a.step_ctr ? *a.step_ctr : 0); draw = 0; }
    const int pick = pick_from_sorted(sorted, a.V, s.temp, s.top_k, s.top_p, philox_unit(key, draw, 0u));
    s.key = key;
    s.draw = draw + 1;
    SessState * u = pr >= 0 ? &a.st[a.row_slot[pr]] : nullptr;  // the unconditional branch's state
    uint16_t * hw = a.hist + (size_t) slot * a.hist_ld;
    if (a.update_hist_first) {
        if (pick < a.hist_ld) hw[pick] = (uint16_t) min(65535, hw[pick] + 1);
        s.last_cb0 = pick;
        if (u) u->last_cb0 = pick;
        a.next_out[r] = pick;
        return;
    }
    s.steps += 1;
    if (a.advance_pos) s.pos += 1;
    if (u) {
        u->steps = s.steps;
        if (a.advance_pos) u->pos += 1;
    }
    if (pick == a.eos || s.steps >= s.max_tokens) {
        s.active = 0;
        if (u) u->active = 0;
        if (a.clamp_on_finish) {
            // src/c_api.cpp:924-930: both branches' positions clamp to max_tokens - 1
            s.last_cb0 = -1;
            s.pos = min(s.pos, s.max_tokens - 1);
            if (u) {
                u->last_cb0 = -1;
                u->pos = min(u->pos, s.max_tokens - 1);
            }
        }
        a.next_out[r] = -1;
    } else {
        if (pick < a.hist_ld) hw[pick] = (uint16_t) min(65535, hw[pick] + 1);
        s.last_cb0 = pick;
        if (u) u->last_cb0 = pick;
        a.next_out[r] = pick;
    }
}

__global__ void __launch_bounds__(1024) depth_sample_kernel(const DepthSampleArgs a) {
    pdl_trigger();
    pdl_wait();
    __shared__ unsigned long long keys[kSortN];
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ int s_code;
    const StepArgs & sa = a.s;
    const int r = blockIdx.x;
    if (sa.row_set && sa.row_set[r] != sa.set_id) return;
    if (!sa.row_active[r]) {
        if (threadIdx.x == 0) sa.frames[(size_t) r * sa.nc + a.col] = -1;
        return;
    }
    const int pr = a.row_pair ? a.row_pair[r] : -1;
    if (pr <= -2) return;  // written by its leader
    const SessState & s = sa.st[sa.row_slot[r]];
    const float * lc = a.logits + (size_t) r * a.ld;
    const float * lu = pr >= 0 ? a.logits + (size_t) pr * a.ld : nullptr;
    const float cfg = s.cfg;
    const int V = a.V;
    const int forced = sa.force ? sa.force[(size_t) r * sa.nc + a.col] : -1;
    if (forced >= 0) {
        // a teacher-forced code (src/depth_decoder.cpp:158-159): no draw
        if (threadIdx.x == 0) s_code = forced;
    } else if (s.dtop_k == 1) {
        // top-1 is the first argmax (no draw)
        float best = -INFINITY;
        int bi = INT_MAX;
        for (int i = threadIdx.x; i < V; i += blockDim.x) {
            float v = lc[i];
            if (lu) v = lu[i] + cfg * (v - lu[i]);
            if (v > best || (bi == INT_MAX && !(v < best))) { best = v; bi = i; }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
        }
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        if (lane == 0) { sv[warp] = best; si[warp] = bi; }
        __syncthreads();
        if (threadIdx.x == 0) {
            float b = sv[0];
            int i0 = si[0];
            for (int w = 1; w < (int) (blockDim.x >> 5); w++)
                if (sv[w] > b || (sv[w] == b && si[w] < i0)) { b = sv[w]; i0 = si[w]; }
            s_code = i0 == INT_MAX ? 0 : i0;
        }
    } else {
        for (int i = threadIdx.x; i < kSortN; i += blockDim.x) {
            unsigned long long key = 0ull;
            if (i < V) {
                float l = lc[i];
                if (lu) l = lu[i] + cfg * (l - lu[i]);
                key = sort_key(l, i);
            }
            keys[i] = key;
        }
        __syncthreads();
        sort_keys_desc(keys);
        if (threadIdx.x == 0) {
            uint32_t key = s.key, draw = s.draw;
            if (a.seeds) { key = a.seeds[r] + (uint32_t) *sa.step_ctr; draw = 0; }
            else if (a.dseeds) { key = a.dseeds[r]; draw = 0; }
            s_code = pick_from_sorted(keys, V, s.dtemp, s.dtop_k, s.dtop_p, philox_unit(key, draw, (uint32_t) a.col));
        }
    }
    __syncthreads();
    const int code = s_code;
    if (threadIdx.x == 0) {
        sa.frames[(size_t) r * sa.nc + a.col] = code;
        if (pr >= 0) sa.frames[(size_t) pr * sa.nc + a.col] = code;
    }
    if (a.gather_cb < 0) return;
    embed_row_f16(sa.embd, (size_t) a.gather_cb * sa.vs + code, sa.din16 + (size_t) r * sa.H);
    if (pr >= 0) embed_row_f16(sa.embd, (size_t) a.gather_cb * sa.vs + code, sa.din16 + (size_t) pr * sa.H);
}

__global__ void copy_rows_kernel(const float * src, int lds, const int * src_idx, float * dst, int ldd, const int * dst_idx,
                                 int cols) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x;
    const float * sr = src + (size_t) (src_idx ? src_idx[i] : i) * lds;
    float * dr = dst + (size_t) (dst_idx ? dst_idx[i] : i) * ldd;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) dr[c] = sr[c];
}

__global__ void stage_forced_kernel(const int * force_all, const int * feed_all, const int * ctr, int n, int * cur_force,
                                    int * cur_feed) {
    pdl_trigger();
    pdl_wait();
    const size_t base = (size_t) (*ctr) * n;
    for (int i = threadIdx.x + blockIdx.x * blockDim.x; i < n; i += blockDim.x * gridDim.x) {
        cur_force[i] = force_all[base + i];
        if (feed_all) cur_feed[i] = feed_all[base + i];
    }
}

__global__ void advance_kernel(const int * row_slot, const int * row_active, const int * row_pair, SessState * st, int R,
                               int * next_out) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= R) return;
    const int slot = row_slot[r];
    if (slot < 0 || !row_active[r]) return;
    const int pr = row_pair ? row_pair[r] : -1;
    if (pr <= -2) return;  // the unconditional branch: its leader advances it
    SessState & s = st[slot];
    s.steps += 1;
    s.pos += 1;
    if (pr >= 0) {
        SessState & u = st[row_slot[pr]];
        u.steps = s.steps;
        u.pos += 1;
    }
    next_out[r] = 0;
}

__global__ void frames_commit_kernel(const int * cur, int * all, int n, int * ctr) {
    pdl_trigger();
    pdl_wait();
    const int k = *ctr;
    for (int i = threadIdx.x; i < n; i += blockDim.x) all[(size_t) k * n + i] = cur[i];
    __syncthreads();
    if (threadIdx.x == 0) *ctr = k + 1;
}

// counts the 32-bit words of b that differ bitwise from a (repeat-launch determinism probe);
// with `where` non-null the first `cap` differences are recorded as (word index, tag) pairs
__global__ void bits_diff_kernel(const uint32_t * a, const uint32_t * b, size_t n, int * count, int * where, int cap,
                                 int tag) {
    pdl_trigger();
    pdl_wait();
    for (size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t) gridDim.x * blockDim.x) {
        if (a[i] != b[i]) {
            const int k = atomicAdd(count, 1);
            if (where && k < cap) {
                where[2 * k] = (int) i;
                where[2 * k + 1] = tag;
            }
        }
    }
}

}  // namespace

// ------------------------------------------------------------------------------------ launchers

void set_pdl_scope(bool on) { g_pdl_scope = on; }
bool pdl_scope() { return pdl_enabled(); }

void init_kernel_attributes() {
    set_gemv_attr<1>(); set_gemv_attr<2>(); set_gemv_attr<3>(); set_gemv_attr<4>();
    set_gemv_attr<5>(); set_gemv_attr<6>(); set_gemv_attr<7>(); set_gemv_attr<8>();
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_gemv(const QMat & w, const half * x16, int ldx, int rows, const GemvOut & out,
                 const GemvScratch & scr, cudaStream_t s, bool fit_scratch) {
    if (rows <= 0) return;
    if (ldx % 2 != 0 || w.K % 32 != 0) throw std::runtime_error("gemv: activation stride or K not aligned");
    const int chunks = (rows + 63) / 64;
    const int NT = rows >= 64 ? 8 : (rows + 7) / 8;
    const int MG = (w.MT + 7) / 8;
    // split K only as far as needed to fill one wave (2 CTAs on each of the 148 SMs), at most
    // kMaxSplits, each split at least one sub-chunk
    const int wave = 2 * 148;
    int splits = std::max(1, wave / (MG * chunks));
    splits = std::min(splits, std::min(kMaxSplits, std::max(1, w.KB / kSub)));
    const char * e = fit_scratch ? nullptr : std::getenv("BZB_GEMV_SPLITS");
    if (e) splits = std::max(1, std::min(kMaxSplits, std::atoi(e)));
    int kper = (w.KB + splits - 1) / splits;
    splits = (w.KB + kper - 1) / kper;
    // a fixed scratch: fewer splits until the partials and the tile counters fit
    while (fit_scratch && splits > 1 && ((size_t) chunks * splits * w.MT * NT * 32 > scr.ws_elems ||
                                         (size_t) chunks * MG > (size_t) scr.n_counters)) {
        kper = (w.KB + splits - 2) / (splits - 1);
        splits = (w.KB + kper - 1) / kper;
    }
    if (splits > 1 && (size_t) chunks * splits * w.MT * NT * 32 > scr.ws_elems) throw std::runtime_error("gemv: split-K scratch too small");
    if (splits > 1 && (size_t) chunks * MG > (size_t) scr.n_counters) throw std::runtime_error("gemv: counter scratch too small");
    GemvParams p;
    p.qs = w.qs; p.ds = w.ds; p.MT = w.MT; p.M = w.M; p.KB = w.KB; p.kper = kper; p.splits = splits; p.MG = MG;
    p.x = x16; p.ldx = ldx; p.rows = rows; p.out = out; p.ws = scr.ws; p.counters = scr.counters;
    const size_t smem = (size_t) 2 * kSub * NT * 32 * sizeof(uint4);
    dim3 grid(MG, splits, chunks);
    switch (NT) {
        case 1: launch_gemv_nt<1>(p, grid, smem, s); break;
        case 2: launch_gemv_nt<2>(p, grid, smem, s); break;
        case 3: launch_gemv_nt<3>(p, grid, smem, s); break;
        case 4: launch_gemv_nt<4>(p, grid, smem, s); break;
        case 5: launch_gemv_nt<5>(p, grid, smem, s); break;
        case 6: launch_gemv_nt<6>(p, grid, smem, s); break;
        case 7: launch_gemv_nt<7>(p, grid, smem, s); break;
        default: launch_gemv_nt<8>(p, grid, smem, s); break;
    }
    BZB_CUDA_CHECK(cudaGetLastError());
}

// Scratch of launch_gemv_static_scratch: file-scope device arrays, so the allocation-free
// entry point needs no cudaMalloc. Zero-initialised at module load; the counters are cleared
// again on the stream before every launch.
static __device__ __align__(256) float4 g_static_gemv_ws[kStaticGemvWsElems];
static __device__ __align__(256) int g_static_gemv_counters[kStaticGemvCounters];

namespace {
constexpr int kMaxStaticDevices = 64;
std::mutex g_static_mu;
GemvScratch g_static_scr[kMaxStaticDevices];
bool g_static_ready[kMaxStaticDevices] = {};

// addresses of the static scratch on the current device, looked up once per device (the
// lookup may load the module on first use, which is why the first call precedes any capture)
GemvScratch static_scratch() {
    int dev = 0;
    BZB_CUDA_CHECK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxStaticDevices) throw std::runtime_error("gemv (static scratch): device index out of range");
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_ready[dev]) {
        GemvScratch s;
        cudaError_t e = cudaGetSymbolAddress((void **) &s.ws, g_static_gemv_ws);
        if (e != cudaSuccess)
            throw std::runtime_error(std::string("gemv (static scratch): cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
        e = cudaGetSymbolAddress((void **) &s.counters, g_static_gemv_counters);
        if (e != cudaSuccess)
            throw std::runtime_error(std::string("gemv (static scratch): cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
        s.ws_elems = kStaticGemvWsElems;
        s.n_counters = kStaticGemvCounters;
        g_static_scr[dev] = s;
        g_static_ready[dev] = true;
    }
    return g_static_scr[dev];
}
}  // namespace

void launch_gemv_static_scratch(const QMat & w, const half * x16, int ldx, int rows, float * y, int ldy,
                                cudaStream_t s) {
    if (rows <= 0 || rows > kStaticGemvMaxRows)
        throw std::runtime_error("gemv (static scratch): rows must be in [1, " + std::to_string(kStaticGemvMaxRows) + "]");
    if (ldy < w.M) throw std::runtime_error("gemv (static scratch): output stride is below the matrix rows");
    const GemvScratch scr = static_scratch();
    // tile counters must start at zero; a launch that did not finish could have left them set
    const size_t n_ctr = std::min((size_t) kStaticGemvCounters, (size_t) ((rows + 63) / 64) * ((w.MT + 7) / 8));
    BZB_CUDA_CHECK(cudaMemsetAsync(scr.counters, 0, n_ctr * sizeof(int), s));
    // the split plan is reduced to what the fixed scratch holds (BZB_GEMV_SPLITS does not apply);
    // a plan that still cannot fit is rejected before anything is launched
    launch_gemv(w, x16, ldx, rows, GemvOut{ EPI_STORE, y, nullptr, ldy }, scr, s, true);
}

void repack_q8(const uint8_t * raw_dev, int M, int K, uint4 * qs, half2 * ds, cudaStream_t s) {
    const int KB = K / 32, MT = (M + 15) / 16;
    const long long warps = (long long) MT * KB;
    const int threads = 256;
    const long long blocks = (warps * 32 + threads - 1) / threads;
    launch_k(repack_q8_kernel, (unsigned) blocks, threads, 0, s, raw_dev, M, KB, qs, ds);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void split_q8_rows(const uint8_t * raw_dev, int rows, int K, int8_t * qs, half * ds, cudaStream_t s) {
    const long long nb = (long long) rows * (K / 32);
    launch_k(split_q8_rows_kernel, (unsigned) ((nb + 255) / 256), 256, 0, s, raw_dev, nb, qs, ds);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void split_q4k_rows(const uint8_t * raw_dev, int rows, int K, int8_t * qs, half * ds, half * ms, cudaStream_t s) {
    if (K % kQ4KBlockValues) throw std::runtime_error("Q4_K rows need a length that is a multiple of 256");
    const long long nb = (long long) rows * (K / 32);
    launch_k(split_q4k_rows_kernel, (unsigned) ((nb + 255) / 256), 256, 0, s, raw_dev, nb, qs, ds, ms);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_rmsnorm(const float * x, int ldx, const float * w, int D, float eps, half * out16, int ld16,
                    float * out32, int ld32, int r0, int n, const int * row_map, cudaStream_t s) {
    if (n <= 0) return;
    launch_k(rmsnorm_kernel, n, 256, 0, s, x, ldx, w, D, eps, out16, ld16, out32, ld32, r0, row_map);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_norm_add(float * x, const float * t, int D, const float * w, float eps, int rows, cudaStream_t s) {
    if (rows <= 0) return;
    launch_k(norm_add_kernel, rows, 256, 0, s, x, t, D, w, eps);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_norm_add_norm(float * x, const float * t, int D, const float * w, float eps, const float * w2, half * y16,
                          int ld16, int rows, cudaStream_t s) {
    if (rows <= 0) return;
    launch_k(norm_add_norm_kernel, rows, 256, 0, s, x, t, D, w, eps, w2, y16, ld16);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_embed_rows(const QRows & e, const int * idx, int n, float scale, float * out32, half * out16, int ld,
                       cudaStream_t s) {
    if (n <= 0) return;
    launch_k(embed_rows_kernel, n, 256, 0, s, e, idx, scale, out32, out16, ld);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_audio_embed(const QRows & e, const int * frames, int ld_frames, int nc, int vs, int n, float * out32,
                        const int * row_active, cudaStream_t s) {
    if (n <= 0) return;
    if (nc > 128 || e.K % 32) throw std::runtime_error("audio embedding: at most 128 codebooks, rows a multiple of 32");
    launch_k(audio_embed_kernel, n, 256, 0, s, e, frames, ld_frames, nc, vs, out32, row_active);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_attn_decode(const AttnDecodeArgs & a, bool paged, cudaStream_t s) {
    const int G = a.n_head / a.n_kv;
    if (G < 1 || G > 4 || a.n_head % a.n_kv) throw std::runtime_error("decode attention: query heads per kv head must be 1..4");
    if (a.n_new < 1 || a.n_new > 2) throw std::runtime_error("attention: 1 or 2 new tokens per session");
    if (a.splits < 1 || a.splits > 16 || (a.splits > 1 && (!a.part || !a.counters)))
        throw std::runtime_error("decode attention: split-KV needs 1..16 splits, scratch and counters");
    dim3 grid(a.R, a.n_kv, a.splits);
    const int threads = 128;
    // one new token over the paged cache at head_dim 64 (the backbone): the tensor-core kernel;
    // BZB_ATTN_MMA=0 selects the scalar one
    static const bool mma_off = [] { const char * e = std::getenv("BZB_ATTN_MMA"); return e && std::atoi(e) == 0; }();
    if (paged && a.hd == 64 && a.n_new == 1 && !mma_off) {
        launch_k(attn_decode_mma_kernel<64>, grid, threads, 0, s, a);
        BZB_CUDA_CHECK(cudaGetLastError());
        return;
    }
    if (a.hd == 64) {
        if (paged) launch_k(attn_decode_kernel<64, true>, grid, threads, 0, s, a);
        else launch_k(attn_decode_kernel<64, false>, grid, threads, 0, s, a);
    } else if (a.hd == 128) {
        if (paged) launch_k(attn_decode_kernel<128, true>, grid, threads, 0, s, a);
        else launch_k(attn_decode_kernel<128, false>, grid, threads, 0, s, a);
    } else throw std::runtime_error("attention: head_dim must be 64 or 128 for decode");
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_qk_prep(const PrefillArgs & a, bool paged, cudaStream_t s) {
    if (a.T <= 0) return;
    switch (a.hd) {
        case 64: if (paged) launch_k(qk_prep_kernel<64, true>, a.T, 128, 0, s, a); else launch_k(qk_prep_kernel<64, false>, a.T, 128, 0, s, a); break;
        case 128: if (paged) launch_k(qk_prep_kernel<128, true>, a.T, 128, 0, s, a); else launch_k(qk_prep_kernel<128, false>, a.T, 128, 0, s, a); break;
        case 256: if (paged) launch_k(qk_prep_kernel<256, true>, a.T, 128, 0, s, a); else launch_k(qk_prep_kernel<256, false>, a.T, 128, 0, s, a); break;
        default: throw std::runtime_error("prefill: head_dim must be 64, 128 or 256");
    }
    BZB_CUDA_CHECK(cudaGetLastError());
}

template <int HD, bool PAGED>
static void launch_prefill_t(const PrefillArgs & a, cudaStream_t s) {
    const size_t smem = prefill_smem<HD>();
    cudaFuncSetAttribute(attn_prefill_kernel<HD, PAGED>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    dim3 grid(a.qblocks ? a.n_qblocks : (a.T + kPrefillQBlock - 1) / kPrefillQBlock, a.n_head);
    launch_k(attn_prefill_kernel<HD, PAGED>, grid, 128, smem, s, a);
}

void launch_attn_prefill(const PrefillArgs & a, bool paged, cudaStream_t s) {
    if (a.T <= 0) return;
    if (a.n_kv < 1 || a.n_head % a.n_kv) throw std::runtime_error("prefill attention: unsupported head grouping");
    switch (a.hd) {
        case 64: if (paged) launch_prefill_t<64, true>(a, s); else launch_prefill_t<64, false>(a, s); break;
        case 128: if (paged) launch_prefill_t<128, true>(a, s); else launch_prefill_t<128, false>(a, s); break;
        case 256: if (paged) launch_prefill_t<256, true>(a, s); else launch_prefill_t<256, false>(a, s); break;
        default: throw std::runtime_error("prefill attention: head_dim must be 64, 128 or 256");
    }
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_step_init(const StepArgs & a, cudaStream_t s) {
    launch_k(step_init_kernel, a.R, 256, 0, s, a);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_argmax_gather(const StepArgs & a, const float * logits, int ld, int V, int col, int gather_cb,
                          cudaStream_t s) {
    launch_k(argmax_gather_kernel, a.R, 256, 0, s, a, logits, ld, V, col, gather_cb);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_sample(const SampleArgs & a, cudaStream_t s) {
    if (a.V > kSortN) throw std::runtime_error("sampler: vocabulary larger than 4096");
    static_assert(kSortN == 4 * 1024, "the sampler's threads hold four keys each");
    launch_k(sample_kernel, a.R, 1024, 0, s, a);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_depth_sample_gather(const DepthSampleArgs & a, cudaStream_t s) {
    if (a.V > kSortN) throw std::runtime_error("depth sampler: vocabulary larger than 4096");
    if (a.col < 1 || a.col >= a.s.nc) throw std::runtime_error("depth sampler: codebook out of range");
    launch_k(depth_sample_kernel, a.s.R, 1024, 0, s, a);
    BZB_CUDA_CHECK(cudaGetLastError());
}

__global__ void qrows_to_f16_kernel(const QRows e, long long row0, int n, half * out) {
    const long long i = (long long) blockIdx.x * blockDim.x + threadIdx.x;  // one 8-value group
    const int g = e.K / 8;
    if (i >= (long long) n * g) return;
    const long long row = row0 + i / g;
    const int c = (int) (i % g);
    const uint2 u = *reinterpret_cast<const uint2 *>(e.qs + row * e.K + c * 8);
    const float sc = __half2float(e.ds[row * (e.K / 32) + (c >> 2)]);
    const float m = e.ms ? __half2float(e.ms[row * (e.K / 32) + (c >> 2)]) : 0.0f;
    const int8_t * bq = reinterpret_cast<const int8_t *>(&u);
    half2 o[4];
#pragma unroll
    for (int k = 0; k < 4; k++) o[k] = __floats2half2_rn((float) bq[2 * k] * sc - m, (float) bq[2 * k + 1] * sc - m);
    *reinterpret_cast<uint4 *>(out + (i / g) * e.K + c * 8) = *reinterpret_cast<uint4 *>(o);
}

__global__ void scale_rows_f16_kernel(const float * x, const float * w, long long total, int D, half * out) {
    const long long i = (long long) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    out[i] = __float2half_rn(x[i] * w[i % D]);
}

void launch_scale_rows_f16(const float * x, const float * w, int n, int D, half * out, cudaStream_t s) {
    const long long total = (long long) n * D;
    if (total <= 0) return;
    scale_rows_f16_kernel<<<(unsigned) ((total + 255) / 256), 256, 0, s>>>(x, w, total, D, out);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_qrows_to_f16(const QRows & e, long long row0, int n, half * out, cudaStream_t s) {
    if (n <= 0) return;
    if (e.K % 32 || row0 < 0 || row0 + n > e.rows) throw std::runtime_error("qrows_to_f16: rows out of the table");
    const long long groups = (long long) n * (e.K / 8);
    qrows_to_f16_kernel<<<(unsigned) ((groups + 255) / 256), 256, 0, s>>>(e, row0, n, out);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_copy_rows(const float * src, int lds, const int * src_idx, float * dst, int ldd, const int * dst_idx, int n,
                      int cols, cudaStream_t s) {
    if (n <= 0) return;
    launch_k(copy_rows_kernel, (unsigned) n, 256, 0, s, src, lds, src_idx, dst, ldd, dst_idx, cols);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_stage_forced(const int * force_all, const int * feed_all, const int * step_ctr, int n, int * cur_force,
                         int * cur_feed, cudaStream_t s) {
    launch_k(stage_forced_kernel, (unsigned) std::max(1, std::min(64, (n + 255) / 256)), 256, 0, s, force_all, feed_all,
             step_ctr, n, cur_force, cur_feed);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_advance(const int * row_slot, const int * row_active, const int * row_pair, SessState * st, int R,
                    int * next_out, cudaStream_t s) {
    launch_k(advance_kernel, (unsigned) ((R + 127) / 128), 128, 0, s, row_slot, row_active, row_pair, st, R, next_out);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_frames_commit(const int * cur, int * frames_all, int n, int * step_ctr, cudaStream_t s) {
    launch_k(frames_commit_kernel, 1, 256, 0, s, cur, frames_all, n, step_ctr);
    BZB_CUDA_CHECK(cudaGetLastError());
}

void launch_bits_diff(const void * a, const void * b, size_t n_words, int * count, cudaStream_t s, int * where, int cap,
                      int tag) {
    const unsigned grid = (unsigned) std::max<size_t>(1, std::min<size_t>((n_words + 255) / 256, 148 * 4));
    launch_k(bits_diff_kernel, grid, 256, 0, s, static_cast<const uint32_t *>(a), static_cast<const uint32_t *>(b),
             n_words, count, where, cap, tag);
    BZB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace bzb
