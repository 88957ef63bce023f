// Codec decoder on the GPU (reference: src/codec_decoder.cpp:11-98, src/codec_conv.cpp:9-59,
// src/codec_transformer.cpp:48-83, src/codec.cpp:15-59, src/c_api.cpp:952-1229).
//
// Activations of the convolution stack are [channels][time] f32 (the reference's ggml [L, C]
// tensors, time contiguous); the transformer and the ConvNeXt MLPs work on [time][channels] rows
// so that their Q8_0 linears run through the dequant-GEMV. Convolutions are direct f32 kernels
// tiled 64 output channels x 64 time steps with the input window and kernel slice staged in
// shared memory.
#include "vocoder.h"
#include "rope.h"
#include "tc_ptx.cuh"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>

namespace bzb {

#define VCHECK(x)                                                                             \
    do {                                                                                      \
        cudaError_t e_ = (x);                                                                 \
        if (e_ != cudaSuccess) throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(e_) + " (" #x ")"); \
    } while (0)

namespace {


// sum over codebooks of the quantiser embeddings (src/codec_decoder.cpp:41-62): out_first[t] =
// E_first[code0], out_rest[t] = sum_{cb>=1} E_rest[cb-1][code_cb], both f16 for the projections
__global__ void voc_embed_kernel(const float * first, const float * rest, const int * codes, int nc, int n_cb, int dq,
                                 int vs, half * out_first, half * out_rest) {
    const int t = blockIdx.x;
    for (int d = threadIdx.x; d < dq; d += blockDim.x) {
        int c0 = codes[(size_t) t * nc];
        c0 = min(max(c0, 0), vs - 1);
        out_first[(size_t) t * dq + d] = __float2half_rn(first[(size_t) c0 * dq + d]);
        float acc = 0.0f;
        for (int cb = 1; cb < n_cb; cb++) {
            int c = codes[(size_t) t * nc + cb];
            c = min(max(c, 0), vs - 1);
            acc += rest[((size_t) (cb - 1) * vs + c) * dq + d];
        }
        out_rest[(size_t) t * dq + d] = __float2half_rn(acc);
    }
}

// dst[j][c] = src[rows[j]][c] for m rows of nc codes (src row stride ld)
__global__ void voc_gather_rows_kernel(const int * src, int ld, const int * rows, int m, int nc, int * dst) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < m * nc; i += gridDim.x * blockDim.x) {
        const int j = i / nc, c = i - j * nc;
        dst[i] = src[(size_t) rows[j] * ld + c];
    }
}

// out[c][r] = in[r][c] (+ add[c][r] when non-null)
__global__ void voc_transpose_kernel(const float * in, int R, int C, float * out, const float * add) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        tile[i][threadIdx.x] = (r < R && c < C) ? in[(size_t) r * C + c] : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int c = c0 + i, r = r0 + threadIdx.x;
        if (c < C && r < R) {
            float v = tile[threadIdx.x][i];
            if (add) v += add[(size_t) c * R + r];
            out[(size_t) c * R + r] = v;
        }
    }
}

// Causal convolutions as TF32 tensor-core implicit GEMMs (mma.sync m16n8k8):
//   y[o][t] = b[o] + sum_{k,i} W[o][k][i] * x[i][t - (taps-1-k) dil]
// M = output channels, N = time, reduction = taps x input channels, ordered as 32-channel
// chunks outer and taps inner. Each chunk's input window x[i][t0 - halo .. t0 + 63] is staged in
// shared memory once and every tap reads its shifted view of it, so the im2col is free. The
// weights are laid out tap-major at load, so a (tap, chunk) weight tile is 64 rows of 32
// contiguous floats. A stride-s transposed conv (src/codec_conv.cpp:25-32) is s such convs with
// 2 taps, one per output phase p: y[o][s t + p] = b[o] + sum_{i,m} w[i][o][p + m s] x[i][t - m].
// When the grid is small (a few frames) the channel chunks are split across CTAs, which write
// partial sums that a second kernel adds. The epilogue (bias, optional residual, SnakeBeta of
// the stored value and/or of a second copy for the next consumer, PCM clamp) runs in whichever
// kernel finishes the sum.
constexpr int kCBM = 64, kCBN = 64, kCCI = 32, kCThreads = 128;

struct ConvArgs {
    const float * x = nullptr;          // input [cin][L] (with istride > 1: see below)
    int cin = 0, L = 0;                 // reduction channels, output length
    // a stride-s conv runs as a causal conv over s phase channels per input channel: channel
    // i*s + r at step t reads x[i][t*s + r] of the [cin/s][Lin] input (istride 1: Lin = L)
    int istride = 1, Lin = 0;
    const float * w = nullptr;          // [phases][cout][taps][cin]
    int taps = 1, dil = 1;
    const float * bias = nullptr;
    int cout = 0;
    float * y = nullptr;                // y[o * ldy + t * ostride + phase]
    int ldy = 0, ostride = 1;
    const float * res = nullptr;        // residual added before the activations (same indexing), or null
    const float * sa = nullptr, * sb = nullptr;     // SnakeBeta (alpha, 1 / beta) of the stored value, or null
    float * y2 = nullptr;               // second output: SnakeBeta(value) with (s2a, 1 / s2b), or ELU(value), or null
    const float * s2a = nullptr, * s2b = nullptr;
    int elu1 = 0, elu2 = 0;             // ELU instead of SnakeBeta for the stored value / the second output
    int clamp = 0;
    // split of the input channels over blockIdx.z / phases (1: no split); partial sums go to
    // part[conv_part_index(split, o, t, phase)]
    int splits = 1, ci_per_split = 0;
    float * part = nullptr;
    int lxp = 0;                        // staged window row stride (floats)
    // Segments: the L steps are S = L / seg_len independent sequences of seg_len steps each (one
    // per decoded stream; seg_len 0: one sequence of L steps). Each segment's first
    // P = (taps - 1) dil inputs come from its state -- the last P inputs of the stream's previous
    // call -- instead of zeros, so consecutive calls continue one causal sequence. A stream slot
    // keeps two copies of this layer's state, [2][cin][P] floats at st + slot * st_stride; segment
    // b reads copy seg_par[b] (-1: a new stream, zero state) of slot seg_slot[b], and the tile that
    // holds a segment's last step writes its new state (the last P inputs of [state | data]) to
    // copy voc_state_next(seg_par[b]). st null: zero state, nothing written.
    int seg_len = 0;
    float * st = nullptr;
    size_t st_stride = 0;
    const int * seg_slot = nullptr, * seg_par = nullptr;
};

// the state copy a segment writes: the other one, or copy 0 after a zero (new-stream) state
__host__ __device__ inline int voc_state_next(int par) { return par < 0 ? 0 : 1 - par; }

__device__ __forceinline__ uint32_t to_tf32(float f) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(f));
    return r;
}

__device__ __forceinline__ void mma_tf32(float c[4], const uint32_t a[4], const uint32_t b[2]) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// SnakeBeta x + sin(alpha x)^2 / beta with the reciprocal of beta stored at load: one fused
// multiply-add after the hardware sine (absolute error ~2^-21 |alpha x|, far below the PCM bar)
__device__ __forceinline__ float snake_beta(float v, float alpha, float inv_beta) {
    const float s = __sinf(v * alpha);
    return fmaf(s * s, inv_beta, v);
}

// ELU as ggml_elu: x for x > 0, exp(x) - 1 otherwise
__device__ __forceinline__ float elu_f(float v) { return v > 0.0f ? v : expm1f(v); }

// stores v = conv + bias (+ residual) of output channel o at idx, with its activations
__device__ __forceinline__ void conv_store(const ConvArgs & a, int o, size_t idx, float v) {
    float out = a.elu1 ? elu_f(v) : a.sa ? snake_beta(v, __ldg(a.sa + o), __ldg(a.sb + o)) : v;
    if (a.clamp) out = fminf(1.0f, fmaxf(-1.0f, out));
    a.y[idx] = out;
    if (a.y2) a.y2[idx] = a.elu2 ? elu_f(v) : snake_beta(v, __ldg(a.s2a + o), __ldg(a.s2b + o));
}

__device__ __forceinline__ void conv_epilogue(const ConvArgs & a, int o, size_t idx, float v) {
    v += a.bias ? __ldg(a.bias + o) : 0.0f;
    if (a.res) v += a.res[idx];
    conv_store(a, o, idx, v);
}

// the partial sum of input-channel split sp for output (o, step t, phase ph): phase-major planes
// [split][phase][cout][L], so that a warp's consecutive steps store to consecutive addresses
__device__ __forceinline__ size_t conv_part_index(const ConvArgs & a, int sp, int o, int t, int ph) {
    return (((size_t) sp * a.ostride + ph) * a.cout + o) * (size_t) a.L + t;
}

__global__ void __launch_bounds__(kCThreads) voc_conv_mma_kernel(const ConvArgs a) {
    extern __shared__ float csm[];
    constexpr int kAld = kCCI + 4;
    float * As = csm;                                   // [2][kCBM][kAld]: weight tile of one tap
    float * xs = csm + 2 * kCBM * kAld;                 // [kCCI][lxp]: input window of one chunk
    int * wseg = reinterpret_cast<int *>(xs + kCCI * a.lxp);  // [lxp]: segment of each window entry
    int * wtau = wseg + a.lxp;                          // [lxp]: its step in the segment (< 0: state)
    const int phases = a.ostride;
    const int phase = blockIdx.z % phases, split = blockIdx.z / phases;
    const int ci_beg = split * a.ci_per_split, ci_end = min(a.cin, ci_beg + a.ci_per_split);
    const float * W = a.w + (size_t) phase * a.cout * a.taps * a.cin;
    const int t0 = blockIdx.x * kCBN, o0 = blockIdx.y * kCBM;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = (warp >> 1) * 32, wn = (warp & 1) * 32;
    const int g = lane >> 2, t4 = lane & 3;
    const int halo = (a.taps - 1) * a.dil;
    // The window holds the tile's steps in the padded sequence where every segment is preceded
    // by its P = halo state inputs: step n (segment n / seg) sits at padded index
    // n + P (n / seg) + P, and the window starts P entries before the tile's first step.
    const int seg = a.seg_len > 0 ? a.seg_len : a.L;
    const int n_last = min(t0 + kCBN, a.L) - 1;
    const int b_first = t0 / seg;
    const int wbeg = t0 + halo * b_first;
    const int lx = n_last + halo * (n_last / seg) + halo - wbeg + 1;
    for (int u = tid; u < lx; u += kCThreads) {
        const int v = wbeg + u, b = v / (halo + seg);
        wseg[u] = b;
        wtau[u] = v - b * (halo + seg) - halo;
    }
    // window column of this thread's output steps for tap taps-1 (the unshifted one)
    int cbase[4];
#pragma unroll
    for (int ni = 0; ni < 4; ni++) {
        const int n = min(t0 + wn + ni * 8 + g, a.L - 1);
        cbase[ni] = n + halo * (n / seg) - wbeg;
    }
    float acc[2][4][4];
#pragma unroll
    for (int mi = 0; mi < 2; mi++)
#pragma unroll
        for (int ni = 0; ni < 4; ni++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[mi][ni][e] = 0.0f;
    const int n_chunks = max(0, (ci_end - ci_beg + kCCI - 1) / kCCI);
    const int n_iter = n_chunks * a.taps;  // (chunk, tap) steps
    float4 ra[4];
    // weight tile of step it: rows o0.., tap k, channels c0..c0+31 (8 float4 per row)
    auto load_a = [&](int it) {
        const int c0 = ci_beg + (it / a.taps) * kCCI, k = it % a.taps;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int e = tid + kCThreads * j;          // 512 float4 of the 64 x 32 tile
            const int r = e >> 3, c = (e & 7) * 4;
            const int o = o0 + r, ci = c0 + c;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (o < a.cout) {
                const float * src = W + ((size_t) o * a.taps + k) * a.cin + ci;
                if (ci + 3 < ci_end && ((reinterpret_cast<uintptr_t>(src) & 15) == 0)) {
                    v = __ldg(reinterpret_cast<const float4 *>(src));
                } else {
                    if (ci < ci_end) v.x = __ldg(src);
                    if (ci + 1 < ci_end) v.y = __ldg(src + 1);
                    if (ci + 2 < ci_end) v.z = __ldg(src + 2);
                    if (ci + 3 < ci_end) v.w = __ldg(src + 3);
                }
            }
            ra[j] = v;
        }
    };
    auto store_a = [&](int buf) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int e = tid + kCThreads * j;
            *reinterpret_cast<float4 *>(As + ((size_t) buf * kCBM + (e >> 3)) * kAld + (e & 7) * 4) = ra[j];
        }
    };
    if (n_iter > 0) {
        load_a(0);
        store_a(0);
    }
    for (int it = 0; it < n_iter; it++) {
        const int k = it % a.taps, cur = it & 1;
        if (k == 0) {
            // a new channel chunk: stage its input window (a segment's state before its first
            // step: zero without a state; zero past the chunk and past the last step)
            __syncthreads();  // every warp is done with the previous window
            const int c0 = ci_beg + (it / a.taps) * kCCI;
            for (int e = tid; e < kCCI * lx; e += kCThreads) {
                const int i = e / lx, u = e - i * lx;
                const int ci = c0 + i, b = wseg[u], tau = wtau[u];
                float v = 0.0f;
                if (ci < ci_end) {
                    if (tau < 0) {
                        const int par = a.st && b * seg < a.L ? a.seg_par[b] : -1;
                        if (par >= 0)
                            v = a.st[(size_t) a.seg_slot[b] * a.st_stride + ((size_t) par * a.cin + ci) * halo + (tau + halo)];
                    } else {
                        const int t = b * seg + tau;
                        if (t < a.L) {
                            const int src = ci / a.istride, ph = ci - src * a.istride;
                            v = a.x[(size_t) src * a.Lin + (size_t) t * a.istride + ph];
                        }
                    }
                }
                xs[i * a.lxp + u] = v;
            }
        }
        __syncthreads();  // weight tile `cur` and the window are in place
        if (k == 0 && a.st && halo > 0 && blockIdx.y == 0 && phase == 0) {
            // segments whose last step is in this tile: their new state is the last `halo`
            // entries of [state | data], at padded indices b (halo + seg) + seg + r
            const int c0 = ci_beg + (it / a.taps) * kCCI;
            for (int b = b_first; b * seg + seg - 1 <= n_last; b++) {
                if ((b + 1) * seg - 1 < t0) continue;
                float * dst = a.st + (size_t) a.seg_slot[b] * a.st_stride + (size_t) voc_state_next(a.seg_par[b]) * a.cin * halo;
                const int u0 = b * (halo + seg) + seg - wbeg;
                for (int e = tid; e < kCCI * halo; e += kCThreads) {
                    const int i = e / halo, r = e - i * halo;
                    if (c0 + i < ci_end) dst[(size_t) (c0 + i) * halo + r] = xs[i * a.lxp + u0 + r];
                }
            }
        }
        if (it + 1 < n_iter) load_a(it + 1);  // next tile's global loads overlap these MMAs
        const float * At = As + (size_t) cur * kCBM * kAld;
        const int shift = halo - (a.taps - 1 - k) * a.dil;  // tap k reads (taps-1-k) dil steps back
#pragma unroll
        for (int kk = 0; kk < kCCI; kk += 8) {
            uint32_t af[2][4], bf[4][2];
#pragma unroll
            for (int mi = 0; mi < 2; mi++) {
                const int r = wm + mi * 16 + g;
                af[mi][0] = to_tf32(At[r * kAld + kk + t4]);
                af[mi][1] = to_tf32(At[(r + 8) * kAld + kk + t4]);
                af[mi][2] = to_tf32(At[r * kAld + kk + t4 + 4]);
                af[mi][3] = to_tf32(At[(r + 8) * kAld + kk + t4 + 4]);
            }
#pragma unroll
            for (int ni = 0; ni < 4; ni++) {
                const int col = cbase[ni] + shift;
                bf[ni][0] = to_tf32(xs[(kk + t4) * a.lxp + col]);
                bf[ni][1] = to_tf32(xs[(kk + t4 + 4) * a.lxp + col]);
            }
#pragma unroll
            for (int mi = 0; mi < 2; mi++)
#pragma unroll
                for (int ni = 0; ni < 4; ni++) mma_tf32(acc[mi][ni], af[mi], bf[ni]);
        }
        if (it + 1 < n_iter) store_a(cur ^ 1);  // the other buffer was last read before this step's barrier
    }
#pragma unroll
    for (int mi = 0; mi < 2; mi++) {
#pragma unroll
        for (int ni = 0; ni < 4; ni++) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int o = o0 + wm + mi * 16 + g + (e >= 2 ? 8 : 0);
                const int t = t0 + wn + ni * 8 + 2 * t4 + (e & 1);
                if (o >= a.cout || t >= a.L) continue;
                const size_t idx = (size_t) o * a.ldy + (size_t) t * a.ostride + phase;
                if (a.splits > 1) a.part[conv_part_index(a, split, o, t, phase)] = acc[mi][ni][e];
                else conv_epilogue(a, o, idx, acc[mi][ni][e]);
            }
        }
    }
}

// The decoder's convolutions on the 5th-generation tensor cores (tcgen05): an implicit GEMM with
// the time steps as M (128 per CTA), the output channels as N (a tile of nt <= 256) and
// (64-channel chunk, tap) pairs as K steps of 64. Per chunk, the 8 producer warps stage the
// chunk's input window time-major as f16 (128-byte rows of 64 channels, the 16-byte pieces of
// row u XOR-swizzled by u mod 8), with each segment's state in front of its steps exactly as the
// TF32 kernel stages it; for every tap they then copy the 128 rows that tap reads -- a row shift
// of (taps-1-k) dil -- into a 128-byte-swizzled K-major A stage. One thread streams the f16 weight
// tiles (pre-tiled at load, one bulk copy of nt x 128 bytes per K step) into the B ring, one
// issues four tcgen05.mma kind::f16 (128 x nt x 16) per K step into a TMEM accumulator, and the
// producers finally read the accumulator back and apply the same epilogue (bias, residual,
// SnakeBeta of the stored value and of a second copy, PCM clamp). Every wait is bounded; after a
// failed wait a role stops, the loader lets its copies land and the MMA thread its MMAs before
// shared and tensor memory are released.
constexpr int kTM = 128;             // time steps per CTA (MMA M)
constexpr int kTThreads = 320;       // warps 0-7 producers and epilogue, 8 MMA, 9 weight loader
constexpr int kTAB = kTM * 128;      // one A stage: 128 rows x 64 f16
constexpr int kTSmemMax = 226 * 1024;  // the 227 KB opt-in limit covers static shared memory too

struct TcConv {
    ConvArgs a;                      // geometry, epilogue, segments and states (istride 1)
    const half * w16 = nullptr;      // [phases][otiles][kchunks][taps] tiles of nt x 64 f16
    int nt = 0, otiles = 0, kchunks = 0;
    int win_rows = 0;                // window capacity (rows of 64 f16)
    int a_stages = 3, b_stages = 3;  // at most 4 each
    // input-channel split across CTAs (blockIdx.z / phases): chunks [split cps, (split + 1) cps);
    // with splits > 1 the raw sums go to a.part[split][...] and voc_conv_reduce_kernel finishes
    int splits = 1, cps = 0;
    int * err = nullptr;
};

// The fused epilogue of one output step t (the calling thread's TMEM lane) over accumulator
// columns [c_lo, c_hi): column g = ot nt + c is output channel g / P, phase g % P (P = ostride).
// With input-channel splits the raw sums go to the phase-major partials; otherwise bias, the
// residual, the activations and the stores. The residual of a 16-column group is loaded one
// group ahead of its use (the first one by the caller before its wait for the accumulator), so
// that its latency hides behind the MMAs and the previous group's stores; the loads of one group
// never touch another group's outputs, so reading ahead of in-place stores is safe.
struct TcEpi {
    const ConvArgs & a;
    int nt, ot, P, split, splits;
    bool have_sum, want_res;
    int t;
    size_t tcol;
    __device__ __forceinline__ TcEpi(const ConvArgs & a_, int nt_, int ot_, int split_, int splits_, bool have_sum_, int t_,
                                     bool row_ok)
        : a(a_), nt(nt_), ot(ot_), P(a_.ostride), split(split_), splits(splits_), have_sum(have_sum_),
          want_res(a_.res && splits_ == 1 && row_ok), t(t_), tcol((size_t) t_ * a_.ostride) {}

    __device__ __forceinline__ void load_res(int c0, float * r) const {
        const int ob = ot * nt + c0, ne = min(16, a.cout * P - ob);
        int o = ob / P, ph = ob - (ob / P) * P;
#pragma unroll
        for (int e = 0; e < 16; e++) {
            r[e] = (want_res && e < ne) ? a.res[(size_t) o * a.ldy + tcol + ph] : 0.0f;
            if (++ph == P) {
                ph = 0;
                o++;
            }
        }
    }

    // warp-uniform loop: every lane takes part in each tensor-memory load
    __device__ __forceinline__ void run(uint32_t taddr, int c_lo, int c_hi, bool live, float * rn) const {
        for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
            float r[16];
#pragma unroll
            for (int e = 0; e < 16; e++) r[e] = rn[e];
            if (c0 + 16 < c_hi) load_res(c0 + 16, rn);
            float v[16];
            tc::tmem_ld16(taddr + (uint32_t) c0, v);
            tc::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; e++) asm volatile("" : "+f"(v[e]));
            const int ob = ot * nt + c0, ne = min(16, a.cout * P - ob);
            const int o0 = ob / P, ph0 = ob - o0 * P;
            if (live && splits > 1) {
                int o = o0, ph = ph0;
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    if (e < ne) a.part[conv_part_index(a, split, o, t, ph)] = have_sum ? v[e] : 0.0f;
                    if (++ph == P) {
                        ph = 0;
                        o++;
                    }
                }
            } else if (live) {
                int o = o0, ph = ph0;
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    if (e < ne) conv_store(a, o, (size_t) o * a.ldy + tcol + ph, v[e] + r[e] + (a.bias ? __ldg(a.bias + o) : 0.0f));
                    if (++ph == P) {
                        ph = 0;
                        o++;
                    }
                }
            }
        }
    }
};

__device__ __forceinline__ void bar_producers() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__global__ void __launch_bounds__(kTThreads, 2) voc_conv_tc_kernel(const __grid_constant__ TcConv p) {
    using namespace tc;
    const ConvArgs & a = p.a;
    extern __shared__ uint8_t tsm_raw[];
    __shared__ uint64_t a_full[4], a_empty[4], b_full[4], b_empty[4], done_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ int s_abort;
    uint8_t * sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tsm_raw) + 1023) & ~(uintptr_t) 1023);
    uint8_t * sA = sm;
    uint8_t * sB = sA + p.a_stages * kTAB;
    const uint32_t tb = (uint32_t) p.nt * 128;
    uint8_t * sW = sB + p.b_stages * tb;
    int * wseg = reinterpret_cast<int *>(sW + (size_t) p.win_rows * 128);
    int * wtau = wseg + p.win_rows;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.z, ot = blockIdx.y;
    const int c_beg = split * p.cps, c_end = min(p.kchunks, c_beg + p.cps);
    const int t0 = blockIdx.x * kTM;
    const int halo = (a.taps - 1) * a.dil;
    const int seg = a.seg_len > 0 ? a.seg_len : a.L;
    const int n_last = min(t0 + kTM, a.L) - 1;
    const int b_first = t0 / seg;
    const int wbeg = t0 + halo * b_first;
    const int lx = n_last + halo * (n_last / seg) + halo - wbeg + 1;
    const int AS = p.a_stages, BS = p.b_stages;
    const int n_it = max(0, c_end - c_beg) * a.taps;
    const uint32_t cols = p.nt <= 32 ? 32u : p.nt <= 64 ? 64u : p.nt <= 128 ? 128u : 256u;
    const uint32_t idesc = (1u << 4) | ((uint32_t) (p.nt >> 3) << 17) | ((uint32_t) (kTM >> 4) << 24);

    if (warp == 8) tmem_alloc(&tmem_slot, cols);
    if (tid == 0) {
        for (int i = 0; i < AS; i++) {
            mbar_init(&a_full[i], 8);   // one arrival per producer warp
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < BS; i++) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        mbar_init(&done_bar, 1);
        fence_mbar_init();
        s_abort = 0;
    }
    for (int u = tid; u < lx; u += kTThreads) {
        const int v = wbeg + u, b = v / (halo + seg);
        wseg[u] = b;
        wtau[u] = v - b * (halo + seg) - halo;
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    bool ok = true;

    if (warp < 8) {
        // copies per tap: rows r = tid / 8 + 32 m (m < 4), 16-byte piece j = tid mod 8
        const int j = tid & 7;
        int cb[4];
#pragma unroll
        for (int m = 0; m < 4; m++) {
            const int n = min(t0 + (tid >> 3) + 32 * m, a.L - 1);
            cb[m] = n + halo * (n / seg) - wbeg;
        }
        int it = 0;
        for (int c = c_beg; c < c_end; c++) {
            bar_producers();  // every producer is done with the previous window
            if (*reinterpret_cast<volatile int *>(&s_abort)) break;
            // the chunk's window: warp w stages piece w (channels c 64 + 8 w ...) of every row,
            // its lanes taking consecutive rows (coalesced loads of consecutive steps); each lane
            // loads 4 rows before converting any, so that 32 loads are in flight
            {
                const int ci0 = c * 64 + warp * 8, nq = min(8, a.cin - ci0);
                for (int ub = 0; ub < lx; ub += 128) {
                    float f[4][8];
#pragma unroll
                    for (int m = 0; m < 4; m++) {
#pragma unroll
                        for (int q = 0; q < 8; q++) f[m][q] = 0.0f;
                        const int u = ub + 32 * m + lane;
                        if (u >= lx || nq <= 0) continue;
                        const int b = wseg[u], tau = wtau[u];
                        if (tau < 0) {
                            const int par = a.st && b * seg < a.L ? a.seg_par[b] : -1;
                            if (par >= 0) {
                                const float * stp = a.st + (size_t) a.seg_slot[b] * a.st_stride +
                                                    ((size_t) par * a.cin + ci0) * halo + tau + halo;
#pragma unroll
                                for (int q = 0; q < 8; q++)
                                    if (q < nq) f[m][q] = stp[(size_t) q * halo];
                            }
                        } else {
                            const int t = b * seg + tau;
                            if (t < a.L) {
                                const float * xp = a.x + (size_t) ci0 * a.L + t;
#pragma unroll
                                for (int q = 0; q < 8; q++)
                                    if (q < nq) f[m][q] = xp[(size_t) q * a.L];
                            }
                        }
                    }
#pragma unroll
                    for (int m = 0; m < 4; m++) {
                        const int u = ub + 32 * m + lane;
                        if (u >= lx) continue;
                        uint32_t w[4];
#pragma unroll
                        for (int q = 0; q < 4; q++) {
                            const half2 h2 = __floats2half2_rn(f[m][2 * q], f[m][2 * q + 1]);
                            w[q] = *reinterpret_cast<const uint32_t *>(&h2);
                        }
                        *reinterpret_cast<uint4 *>(sW + (size_t) u * 128 + ((warp ^ (u & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
            bar_producers();  // the window is complete
            if (a.st && halo > 0 && ot == 0) {
                // segments whose last step is in this tile: the new state of this chunk's channels
                for (int b = b_first; b * seg + seg - 1 <= n_last; b++) {
                    float * dst = a.st + (size_t) a.seg_slot[b] * a.st_stride + (size_t) voc_state_next(a.seg_par[b]) * a.cin * halo;
                    const int u0 = b * (halo + seg) + seg - wbeg;
                    for (int e = tid; e < 64 * halo; e += 256) {
                        const int i = e / halo, r = e - i * halo, ci = c * 64 + i, u = u0 + r;
                        if (ci < a.cin) {
                            const half hv = *reinterpret_cast<const half *>(sW + (size_t) u * 128 + (((i >> 3) ^ (u & 7)) << 4) + (i & 7) * 2);
                            dst[(size_t) ci * halo + r] = __half2float(hv);
                        }
                    }
                }
            }
            for (int k = 0; k < a.taps; k++, it++) {
                const int st = it % AS;
                if (ok && it >= AS) ok = mbar_wait(&a_empty[st], (uint32_t) ((it / AS) - 1) & 1u, p.err, kSpinLimit, 32);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) {
                    s_abort = 1;
                    continue;
                }
                const int shift = halo - (a.taps - 1 - k) * a.dil;
                uint8_t * A = sA + st * kTAB;
#pragma unroll
                for (int m = 0; m < 4; m++) {
                    const int r = (tid >> 3) + 32 * m, u = cb[m] + shift;
                    const uint4 v = *reinterpret_cast<const uint4 *>(sW + (size_t) u * 128 + ((j ^ (u & 7)) << 4));
                    *reinterpret_cast<uint4 *>(A + (r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4)) = v;
                }
                fence_proxy_async();  // each thread's stores before the warp's arrival
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_full[st]);
            }
        }
    } else if (warp == 8) {
        if (lane == 0) {
            for (int it = 0; it < n_it; it++) {
                const int st = it % AS, sb = it % BS;
                ok = mbar_wait(&b_full[sb], (uint32_t) (it / BS) & 1u, p.err);
                if (ok) ok = mbar_wait(&a_full[st], (uint32_t) (it / AS) & 1u, p.err);
                if (!ok) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(sA + st * kTAB), b0 = smem_u32(sB + sb * tb);
#pragma unroll
                for (int kk = 0; kk < 4; kk++)
                    umma_f16(tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), idesc, (it > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&a_empty[st]);
                umma_commit(&b_empty[sb]);
            }
            umma_commit(&done_bar);
            if (!mbar_drain(&done_bar, 0u, p.err)) ok = false;
        }
    } else {
        if (lane == 0) {
            const uint8_t * base = reinterpret_cast<const uint8_t *>(p.w16) + ((size_t) ot * p.kchunks + c_beg) * a.taps * (size_t) tb;
            int issued = 0;
            for (int it = 0; it < n_it; it++) {
                const int sb = it % BS;
                if (it >= BS) ok = mbar_wait(&b_empty[sb], (uint32_t) ((it / BS) - 1) & 1u, p.err, kSpinLimit, 64);
                if (!ok) break;
                mbar_expect_tx(&b_full[sb], tb);
                bulk_g2s(sB + sb * tb, base + (size_t) it * tb, tb, &b_full[sb]);
                issued = it + 1;
            }
            for (int it = max(0, issued - BS); it < issued; it++)
                mbar_drain(&b_full[it % BS], (uint32_t) (it / BS) & 1u, p.err);
        }
    }

    if (warp < 8) {
        const int q = warp & 3, hh = warp >> 2, half_cols = p.nt / 2;
        const int t = t0 + 32 * q + lane;
        const TcEpi ep(a, p.nt, ot, split, p.splits, n_it > 0, t, t < a.L);
        float rn[16];
        ep.load_res(hh * half_cols, rn);
        if (!mbar_wait(&done_bar, 0u, p.err, kSpinLimit, 128)) ok = false;
        tc_fence_after();
        ep.run(tmem + ((uint32_t) (32 * q) << 16), hh * half_cols, (hh + 1) * half_cols, ok && t < a.L, rn);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) tmem_dealloc(tmem, cols);
}

// The same convolution with the staged window itself as the A operand, for segments of 96 steps
// and more: a CTA's 128 steps lie in one segment (tiles are laid out per segment, the
// last one of a segment partly empty), so output step r of tap k reads window row r + k dil and
// the tap's A operand is the window from row k dil on: a shared-memory descriptor that starts
// k dil rows into the 1024-byte-aligned window, whose 16-byte pieces are stored at the XOR of the
// row's own address bits like every 128-byte-swizzled tile (the swizzle follows the absolute
// address, so the descriptor's matrix base offset stays 0: setting it to the start row's phase
// fails the parity tests). The producers stage one window per
// 64-channel chunk (two buffers) and hand each over once for all its taps; there are no per-tap
// copies. Rows past the window's data are never stored (their outputs belong to steps past the
// segment).
struct TcConvW {
    ConvArgs a;
    const half * w16 = nullptr;
    int nt = 0, otiles = 0, kchunks = 0;
    int tps = 0;         // tiles per segment
    int win_rows = 0;    // window rows per buffer (a multiple of 8: 128 + halo rounded up)
    int b_stages = 3;    // at most 4
    int splits = 1, cps = 0;
    int * err = nullptr;
};

__global__ void __launch_bounds__(kTThreads, 2) voc_conv_tcw_kernel(const __grid_constant__ TcConvW p) {
    using namespace tc;
    const ConvArgs & a = p.a;
    extern __shared__ uint8_t tsm_raw[];
    __shared__ uint64_t w_full[2], w_empty[2], b_full[4], b_empty[4], done_bar;
    __shared__ uint32_t tmem_slot;
    uint8_t * sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tsm_raw) + 1023) & ~(uintptr_t) 1023);
    const uint32_t wbytes = (uint32_t) p.win_rows * 128;
    uint8_t * sWin = sm;                 // [2][win_rows][128 B]
    uint8_t * sB = sm + 2 * wbytes;      // [b_stages][nt][128 B]
    const uint32_t tb = (uint32_t) p.nt * 128;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.z, ot = blockIdx.y;
    const int c_beg = split * p.cps, c_end = min(p.kchunks, c_beg + p.cps);
    const int seg = a.seg_len > 0 ? a.seg_len : a.L;
    const int b = blockIdx.x / p.tps, tau0 = (blockIdx.x % p.tps) * kTM;
    const int rows = min(kTM, seg - tau0);
    const int halo = (a.taps - 1) * a.dil;
    const int lx = rows + halo;
    const int n_ch = max(0, c_end - c_beg), n_it = n_ch * a.taps;
    const int BS = p.b_stages;
    const uint32_t cols = p.nt <= 32 ? 32u : p.nt <= 64 ? 64u : p.nt <= 128 ? 128u : 256u;
    const uint32_t idesc = (1u << 4) | ((uint32_t) (p.nt >> 3) << 17) | ((uint32_t) (kTM >> 4) << 24);

    if (warp == 8) tmem_alloc(&tmem_slot, cols);
    if (tid == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(&w_full[i], 8);   // one arrival per producer warp
            mbar_init(&w_empty[i], 1);
        }
        for (int i = 0; i < BS; i++) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        mbar_init(&done_bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    bool ok = true;

    if (warp < 8) {
        // warp w stages piece w (channels c 64 + 8 w ...) of every window row, lanes on consecutive
        // rows (coalesced loads of consecutive steps), 4 rows per lane in flight
        const int par = (a.st && halo > 0) ? a.seg_par[b] : -1;
        const float * stb = par >= 0 ? a.st + (size_t) a.seg_slot[b] * a.st_stride + (size_t) par * a.cin * halo : nullptr;
        const float * xb = a.x + (size_t) b * seg;
        for (int ci = 0; ci < n_ch; ci++) {
            const int c = c_beg + ci, wb = ci & 1;
            if (ok && ci >= 2) ok = mbar_wait(&w_empty[wb], (uint32_t) ((ci / 2) - 1) & 1u, p.err, kSpinLimit, 32);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            uint8_t * W = sWin + wb * wbytes;
            const int ci0 = c * 64 + warp * 8, nq = min(8, a.cin - ci0);
            for (int ub = 0; ub < lx; ub += 128) {
                float f[4][8];
#pragma unroll
                for (int m = 0; m < 4; m++) {
#pragma unroll
                    for (int q = 0; q < 8; q++) f[m][q] = 0.0f;
                    const int u = ub + 32 * m + lane;
                    if (u >= lx || nq <= 0) continue;
                    const int tau = tau0 + u - halo;
                    if (tau < 0) {
                        if (stb) {
#pragma unroll
                            for (int q = 0; q < 8; q++)
                                if (q < nq) f[m][q] = stb[(size_t) (ci0 + q) * halo + tau + halo];
                        }
                    } else {
                        const float * xp = xb + (size_t) ci0 * a.L + tau;
#pragma unroll
                        for (int q = 0; q < 8; q++)
                            if (q < nq) f[m][q] = xp[(size_t) q * a.L];
                    }
                }
#pragma unroll
                for (int m = 0; m < 4; m++) {
                    const int u = ub + 32 * m + lane;
                    if (u >= lx) continue;
                    uint32_t w[4];
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const half2 h2 = __floats2half2_rn(f[m][2 * q], f[m][2 * q + 1]);
                        w[q] = *reinterpret_cast<const uint32_t *>(&h2);
                    }
                    *reinterpret_cast<uint4 *>(W + (size_t) u * 128 + ((warp ^ (u & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
            __syncwarp();
            // the tile holding the segment's last step writes the segment's new state for this
            // warp's channels: the last halo rows of [state | data] (from the f16 window, as read)
            if (a.st && halo > 0 && ot == 0 && tau0 + rows == seg && nq > 0) {
                float * dst = a.st + (size_t) a.seg_slot[b] * a.st_stride + (size_t) voc_state_next(a.seg_par[b]) * a.cin * halo;
                for (int e = lane; e < 8 * halo; e += 32) {
                    const int i = e / halo, r = e - i * halo, u = lx - halo + r;
                    if (i < nq) {
                        const half hv = *reinterpret_cast<const half *>(W + (size_t) u * 128 + ((warp ^ (u & 7)) << 4) + i * 2);
                        dst[(size_t) (ci0 + i) * halo + r] = __half2float(hv);
                    }
                }
            }
            fence_proxy_async();  // each thread's window stores before the warp's arrival
            __syncwarp();
            if (lane == 0) mbar_arrive(&w_full[wb]);
        }
    } else if (warp == 8) {
        if (lane == 0) {
            int it = 0;
            for (int ci = 0; ci < n_ch && ok; ci++) {
                const int wb = ci & 1;
                ok = mbar_wait(&w_full[wb], (uint32_t) (ci / 2) & 1u, p.err);
                if (!ok) break;
                tc_fence_after();
                const uint32_t wa = smem_u32(sWin + wb * wbytes);
                for (int k = 0; k < a.taps; k++, it++) {
                    const int sb = it % BS;
                    ok = mbar_wait(&b_full[sb], (uint32_t) (it / BS) & 1u, p.err);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t a0 = wa + (uint32_t) (k * a.dil) * 128, b0 = smem_u32(sB + sb * tb);
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        umma_f16(tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), idesc, (it > 0 || kk > 0) ? 1u : 0u);
                    umma_commit(&b_empty[sb]);
                }
                if (!ok) break;
                umma_commit(&w_empty[wb]);
            }
            umma_commit(&done_bar);
            if (!mbar_drain(&done_bar, 0u, p.err)) ok = false;
        }
    } else {
        if (lane == 0) {
            const uint8_t * base = reinterpret_cast<const uint8_t *>(p.w16) + ((size_t) ot * p.kchunks + c_beg) * a.taps * (size_t) tb;
            int issued = 0;
            for (int it = 0; it < n_it; it++) {
                const int sb = it % BS;
                if (it >= BS) ok = mbar_wait(&b_empty[sb], (uint32_t) ((it / BS) - 1) & 1u, p.err, kSpinLimit, 64);
                if (!ok) break;
                mbar_expect_tx(&b_full[sb], tb);
                bulk_g2s(sB + sb * tb, base + (size_t) it * tb, tb, &b_full[sb]);
                issued = it + 1;
            }
            for (int it = max(0, issued - BS); it < issued; it++)
                mbar_drain(&b_full[it % BS], (uint32_t) (it / BS) & 1u, p.err);
        }
    }

    if (warp < 8) {
        const int q = warp & 3, hh = warp >> 2, half_cols = p.nt / 2;
        const int r = 32 * q + lane;
        const int t = b * seg + tau0 + r;
        const TcEpi ep(a, p.nt, ot, split, p.splits, n_it > 0, t, r < rows);
        float rn[16];
        ep.load_res(hh * half_cols, rn);
        if (!mbar_wait(&done_bar, 0u, p.err, kSpinLimit, 128)) ok = false;
        tc_fence_after();
        ep.run(tmem + ((uint32_t) (32 * q) << 16), hh * half_cols, (hh + 1) * half_cols, ok && r < rows, rn);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) tmem_dealloc(tmem, cols);
}

// sums the channel-split partials in split order and applies the epilogue: blockIdx.y is the
// output channel, threads take consecutive outputs i = t ostride + phase of its row
__global__ void voc_conv_reduce_kernel(const ConvArgs a) {
    const int P = a.ostride, n_row = a.L * P;
    for (int o = blockIdx.y; o < a.cout; o += gridDim.y)
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_row; i += gridDim.x * blockDim.x) {
            const int t = i / P, ph = i - t * P;
            float v = 0.0f;
            for (int sp = 0; sp < a.splits; sp++) v += a.part[conv_part_index(a, sp, o, t, ph)];
            conv_epilogue(a, o, (size_t) o * a.ldy + i, v);
        }
}

void launch_conv_reduce(const ConvArgs & a, cudaStream_t s) {
    const dim3 grid((unsigned) std::min((a.L * a.ostride + 255) / 256, 65535), (unsigned) std::min(a.cout, 65535));
    voc_conv_reduce_kernel<<<grid, 256, 0, s>>>(a);
}

// causal depthwise conv (src/codec_conv.cpp:42-59), w [K][C], y[c][t] = b[c] + sum_k w[k][c]
// x[c][t - (K-1) + k], over S segments of seg steps each (x [C][S seg]); a segment's first
// K-1 inputs come from copy seg_par of its slot's state ([2][C][K-1] at st + slot st_stride;
// -1 or st null: zero). Threads past the outputs write each segment's new state (the last K-1
// inputs of [state | data]) to copy voc_state_next(seg_par).
__global__ void voc_depthwise_seg_kernel(const float * x, int C, int S, int seg, const float * w, const float * b, int K,
                                         float * y, float * st, size_t st_stride, const int * seg_slot, const int * seg_par) {
    const int P = K - 1, L = S * seg;
    const size_t n_out = (size_t) C * L, n_st = st ? (size_t) S * C * P : 0;
    for (size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x; idx < n_out + n_st; idx += (size_t) gridDim.x * blockDim.x) {
        if (idx < n_out) {
            const int c = (int) (idx / L), n = (int) (idx % L), sg = n / seg, tau = n - sg * seg;
            const int par = st ? seg_par[sg] : -1;
            const float * sin_ = par >= 0 ? st + (size_t) seg_slot[sg] * st_stride + ((size_t) par * C + c) * P : nullptr;
            float acc = 0.0f;
            for (int k = 0; k < K; k++) {
                const int tt = tau - P + k;
                const float v = tt >= 0 ? x[(size_t) c * L + (size_t) sg * seg + tt] : (sin_ ? sin_[P + tt] : 0.0f);
                acc += w[(size_t) k * C + c] * v;
            }
            y[idx] = acc + (b ? b[c] : 0.0f);
        } else {
            const size_t j = idx - n_out;
            const int r = (int) (j % P), c = (int) ((j / P) % C), sg = (int) (j / ((size_t) P * C));
            const int par = seg_par[sg];
            float * slot = st + (size_t) seg_slot[sg] * st_stride;
            const int q = r + seg;  // index into [state (P) | data (seg)]
            const float v = q < P ? (par >= 0 ? slot[((size_t) par * C + c) * P + q] : 0.0f)
                                  : x[(size_t) c * L + (size_t) sg * seg + (q - P)];
            slot[((size_t) voc_state_next(par) * C + c) * P + r] = v;
        }
    }
}

// K and V of T new frames of S streams into their rings: row s T + t is position pos0[s] + t of
// ring slot[s] (k rotated by NEOX RoPE at that position). Ring layout per slot:
// [R positions][2 (k, v)][nkv hd] floats, position p at p mod R.
__global__ void voc_kv_ring_append_kernel(const float * k, const float * v, int ld, int S, int T, int nkv, int hd,
                                          const float2 * rope, float * ring, size_t slot_stride, int R,
                                          const int * slots, const int * pos0) {
    const int kvd = nkv * hd, half_d = hd / 2;
    const size_t n = (size_t) S * T * kvd;
    for (size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += (size_t) gridDim.x * blockDim.x) {
        const int e = (int) (idx % kvd), row = (int) (idx / kvd), sgm = row / T, t = row - sgm * T;
        const int d = e % hd;
        const int pos = pos0[sgm] + t;
        const int dp = d < half_d ? d + half_d : d - half_d;
        const float x0 = k[(size_t) row * ld + e], x1 = k[(size_t) row * ld + e - d + dp];
        const float2 cs = rope[(size_t) pos * half_d + (d < half_d ? d : d - half_d)];
        const float kr = d < half_d ? x0 * cs.x - x1 * cs.y : x1 * cs.y + x0 * cs.x;
        float * dst = ring + (size_t) slots[sgm] * slot_stride + (size_t) (pos % R) * 2 * kvd;
        dst[e] = kr;
        dst[kvd + e] = v[(size_t) row * ld + e];
    }
}

// causal sliding-window attention of T new frames per stream over its ring (keys already
// rotated): one warp per (row s T + t, head h), query at position pos0[s] + t, keys
// pos - window < j <= pos; hd <= 128, a multiple of 4. The positions go in blocks of 32, one per
// lane: each lane forms its position's score from the whole key row (the rotated query sits in
// shared memory), so the key loads of a block are independent of one another; the block's
// softmax weights are then broadcast lane by lane into the value sums of the lane's dims (online
// rescaling between blocks).
__global__ void __launch_bounds__(128) voc_attn_ring_kernel(const float * q, int ldq, int S, int T, int nh, int nkv, int hd, int window,
                                     const float2 * rope, float scale, const float * ring, size_t slot_stride, int R,
                                     const int * slots, const int * pos0, half * out) {
    __shared__ float qs[4][128];
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    if (warp >= S * T * nh) return;
    const int row = warp / nh, h = warp % nh, sgm = row / T, t = row - sgm * T, g = h / (nh / nkv);
    const int E = hd / 32, half_d = hd / 2, kvd = nkv * hd;
    const int pos = pos0[sgm] + t;
    const float * base = ring + (size_t) slots[sgm] * slot_stride + (size_t) g * hd;
    for (int d = lane; d < hd; d += 32) {
        const int dp = d < half_d ? d + half_d : d - half_d;
        const float x0 = q[(size_t) row * ldq + (size_t) h * hd + d], x1 = q[(size_t) row * ldq + (size_t) h * hd + dp];
        const float2 cs = rope[(size_t) pos * half_d + (d < half_d ? d : d - half_d)];
        qs[wib][d] = d < half_d ? x0 * cs.x - x1 * cs.y : x1 * cs.y + x0 * cs.x;
    }
    __syncwarp();
    const int j0 = max(0, window > 0 ? pos - window + 1 : 0);
    float m = -INFINITY, l = 0.0f, acc[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
    for (int jb = j0; jb <= pos; jb += 32) {
        const int j = jb + lane;
        float sc = -INFINITY;
        if (j <= pos) {
            const float4 * kr = reinterpret_cast<const float4 *>(base + (size_t) (j % R) * 2 * kvd);
            float dot = 0.0f;
            for (int i = 0; i < hd / 4; i++) {
                const float4 kk = kr[i];
                dot += qs[wib][4 * i] * kk.x + qs[wib][4 * i + 1] * kk.y + qs[wib][4 * i + 2] * kk.z + qs[wib][4 * i + 3] * kk.w;
            }
            sc = dot * scale;
        }
        float mb = sc;
        for (int o = 16; o > 0; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
        const float mn = fmaxf(m, mb);
        const float corr = expf(m - mn);
        const float p = j <= pos ? expf(sc - mn) : 0.0f;
        float ps = p;
        for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
        l = l * corr + ps;
#pragma unroll
        for (int e = 0; e < 4; e++) acc[e] *= corr;
        // value rows eight at a time, every load of a group issued before its sums (the loads of
        // consecutive positions do not wait on one another)
        const int nb = min(32, pos - jb + 1);
        for (int j8 = 0; j8 < nb; j8 += 8) {
            float vv[8][4];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float * vr = base + (size_t) ((jb + j8 + u) % R) * 2 * kvd + kvd;
#pragma unroll
                for (int e = 0; e < 4; e++) vv[u][e] = (j8 + u < nb && e < E) ? vr[lane + 32 * e] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float pj = __shfl_sync(0xffffffffu, p, (j8 + u) & 31);  // zero past the last position
#pragma unroll
                for (int e = 0; e < 4; e++) acc[e] += pj * vv[u][e];
            }
        }
        m = mn;
    }
#pragma unroll
    for (int e = 0; e < 4; e++)
        if (e < E) out[((size_t) row * nh + h) * hd + lane + 32 * e] = __float2half_rn(acc[e] / l);
}

// layer norm over each row of [R][C] (mean and variance in double, src/common.cpp:131-134) -> f16
__global__ void voc_layernorm_kernel(const float * x, int C, const float * w, const float * b, float eps, half * y) {
    __shared__ double red[2][32];
    const int r = blockIdx.x;
    const float * xr = x + (size_t) r * C;
    double s = 0.0;
    for (int c = threadIdx.x; c < C; c += blockDim.x) s += xr[c];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (lane == 0) red[0][warp] = s;
    __syncthreads();
    double mean = 0.0;
    for (int i = 0; i < nw; i++) mean += red[0][i];
    mean /= C;
    const float mf = (float) mean;
    double v = 0.0;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float d = xr[c] - mf;
        v += (double) d * d;
    }
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[1][warp] = v;
    __syncthreads();
    double var = 0.0;
    for (int i = 0; i < nw; i++) var += red[1][i];
    var /= C;
    const float scale = 1.0f / sqrtf((float) var + eps);
    for (int c = threadIdx.x; c < C; c += blockDim.x)
        y[(size_t) r * C + c] = __float2half_rn(((xr[c] - mf) * scale) * w[c] + b[c]);
}

// rows [R][C] += bias, then GELU (erf) to f16 when `gelu`, else plain f32 in place
__global__ void voc_bias_gelu_kernel(float * x, size_t n, int C, const float * b, half * y16) {
    for (size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t) gridDim.x * blockDim.x) {
        const float v = x[i] + (b ? b[i % C] : 0.0f);
        y16[i] = __float2half_rn(0.5f * v * (1.0f + erff(v * 0.70710678118654752f)));
    }
}

// h[r][c] = (h[r][c] + b[c]) * scale[c] (bias and layer scale of a branch), or with b null just
// the scale
__global__ void voc_bias_scale_kernel(float * x, size_t n, int C, const float * b, const float * scale) {
    for (size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t) gridDim.x * blockDim.x) {
        const int c = (int) (i % C);
        x[i] = (x[i] + (b ? b[c] : 0.0f)) * (scale ? scale[c] : 1.0f);
    }
}

// h[i] += o[i] * scale[i % C]
__global__ void voc_scaled_add_kernel(float * h, const float * o, size_t n, int C, const float * scale) {
    for (size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t) gridDim.x * blockDim.x)
        h[i] += o[i] * scale[i % C];
}

// row r of h += o * scale (a branch's output and its layer scale), then y16 = RMSNorm(h) * w:
// the residual add of one block and the norm that feeds the next (one CTA per row)
__global__ void voc_add_rmsnorm_kernel(float * h, const float * o, const float * scale, int C, const float * w, float eps,
                                       half * y16) {
    __shared__ float red[32];
    const int r = blockIdx.x;
    float * hr = h + (size_t) r * C;
    const float * orow = o + (size_t) r * C;
    float ss = 0.0f;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float v = hr[c] + orow[c] * scale[c];
        hr[c] = v;
        ss += v * v;
    }
    for (int k = 16; k > 0; k >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, k);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < nw; i++) tot += red[i];
    const float inv = 1.0f / sqrtf(tot / (float) C + eps);
    for (int c = threadIdx.x; c < C; c += blockDim.x) y16[(size_t) r * C + c] = __float2half_rn((hr[c] * inv) * w[c]);
}


// x16 = f16(x) for [R][C] rows
__global__ void voc_to_f16_kernel(const float * x, size_t n, half * y) {
    for (size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t) gridDim.x * blockDim.x)
        y[i] = __float2half_rn(x[i]);
}

// causal sliding-window GQA attention with NEOX RoPE on q and k (src/codec_transformer.cpp:60-70,
// src/common.cpp:147-173): one warp per (query t, head h); keys t - window < k <= t; hd <= 128
__global__ void voc_attn_kernel(const float * q, const float * k, const float * v, int T, int nh, int nkv, int hd,
                                int window, const float2 * rope, float scale, half * out) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T * nh) return;
    const int t = warp / nh, h = warp % nh, g = h / (nh / nkv);
    const int E = hd / 32, half_d = hd / 2;
    float qv[4];
    // rotated query: element d pairs with d +- hd/2
    for (int e = 0; e < E; e++) {
        const int d = lane + 32 * e;
        const int dp = d < half_d ? d + half_d : d - half_d;
        const float x0 = q[((size_t) t * nh + h) * hd + d], x1 = q[((size_t) t * nh + h) * hd + dp];
        const float2 cs = rope[(size_t) t * half_d + (d < half_d ? d : d - half_d)];
        qv[e] = d < half_d ? x0 * cs.x - x1 * cs.y : x1 * cs.y + x0 * cs.x;
    }
    const int k0 = max(0, window > 0 ? t - window + 1 : 0);
    float m = -INFINITY, l = 0.0f, acc[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
    for (int kk = k0; kk <= t; kk++) {
        float dot = 0.0f;
        for (int e = 0; e < E; e++) {
            const int d = lane + 32 * e;
            const int dp = d < half_d ? d + half_d : d - half_d;
            const float x0 = k[((size_t) kk * nkv + g) * hd + d], x1 = k[((size_t) kk * nkv + g) * hd + dp];
            const float2 cs = rope[(size_t) kk * half_d + (d < half_d ? d : d - half_d)];
            const float kr = d < half_d ? x0 * cs.x - x1 * cs.y : x1 * cs.y + x0 * cs.x;
            dot += qv[e] * kr;
        }
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const float sc = dot * scale;
        const float mn = fmaxf(m, sc);
        const float corr = expf(m - mn), p = expf(sc - mn);
        l = l * corr + p;
        for (int e = 0; e < E; e++) acc[e] = acc[e] * corr + p * v[((size_t) kk * nkv + g) * hd + lane + 32 * e];
        m = mn;
    }
    for (int e = 0; e < E; e++) out[((size_t) t * nh + h) * hd + lane + 32 * e] = __float2half_rn(acc[e] / l);
}

unsigned grid_for(size_t n) { return (unsigned) std::min<size_t>((n + 255) / 256, 148 * 16); }

size_t conv_smem_bytes(int lxp) {
    return ((size_t) 2 * kCBM * (kCCI + 4) + (size_t) kCCI * lxp) * sizeof(float) + (size_t) 2 * lxp * sizeof(int);
}
// window row stride: at least the widest window a tile stages -- 64 steps plus `halo` state
// entries for every segment the tile touches (a 64-step tile touches at most
// ceil(63 / seg_len) + 1 segments) -- and 8 mod 32 so that the 4 x 8 B-fragment reads of a warp
// fall in distinct banks. seg_len 0: one segment.
int conv_lxp(int taps, int dil, int seg_len = 0, int n_seg = 1) {
    const int halo = (taps - 1) * dil;
    const int touched = seg_len > 0 ? std::min(n_seg, (kCBN - 1 + seg_len - 1) / seg_len + 1) : 1;
    const int lx = kCBN + halo * touched;
    return (lx + 23) / 32 * 32 + 8;
}

// the conv kernel's dynamic shared-memory limit is a per-device function attribute shared by every
// vocoder and encoder in the process: it only ever grows
void raise_conv_smem_limit(size_t bytes) {
    static std::mutex mu;
    static std::map<int, size_t> set_on;
    int dev = 0;
    VCHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    if (bytes <= set_on[dev]) return;
    if (bytes > 227 * 1024) throw std::runtime_error("vocoder: convolution window too wide");
    VCHECK(cudaFuncSetAttribute(voc_conv_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) bytes));
    set_on[dev] = bytes;
}

// `a` with x, w, y, ... set; fills the launch shape (and the channel split when the grid would
// leave SMs idle and the scratch can hold the partials)
void launch_conv(ConvArgs a, int phases, float * scratch, size_t scratch_floats, cudaStream_t s) {
    if (a.L <= 0) return;
    if (a.Lin == 0) a.Lin = a.L;
    const int tiles = ((a.L + kCBN - 1) / kCBN) * ((a.cout + kCBM - 1) / kCBM) * phases;
    const int chunks = (a.cin + kCCI - 1) / kCCI;
    int splits = 1;
    while (tiles * splits * 2 <= 2 * 148 && splits * 2 <= chunks && splits < 16 &&
           (size_t) splits * 2 * a.cout * a.ldy <= scratch_floats)
        splits *= 2;
    a.splits = splits;
    a.ci_per_split = ((chunks + splits - 1) / splits) * kCCI;
    a.part = scratch;
    a.lxp = conv_lxp(a.taps, a.dil, a.seg_len, a.seg_len > 0 ? a.L / a.seg_len : 1);
    raise_conv_smem_limit(conv_smem_bytes(a.lxp));
    const dim3 grid((unsigned) ((a.L + kCBN - 1) / kCBN), (unsigned) ((a.cout + kCBM - 1) / kCBM), (unsigned) (phases * splits));
    voc_conv_mma_kernel<<<grid, kCThreads, conv_smem_bytes(a.lxp), s>>>(a);
    if (splits > 1) launch_conv_reduce(a, s);
}

// the tcgen05 convolution of `a` (istride 1) with weights tiled as `c` describes
void launch_conv_tc(ConvArgs a, const half * w16, int nt, int otiles, int kchunks, int * err,
                    float * scratch, size_t scratch_floats, cudaStream_t s) {
    if (a.L <= 0) return;
    if (a.istride != 1) throw std::runtime_error("tcgen05 conv: strided input is not supported");
    a.Lin = a.L;
    static std::mutex mu;
    static std::map<int, bool> attr_set;
    int dev = 0;
    VCHECK(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_set[dev]) {
            VCHECK(cudaFuncSetAttribute(voc_conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTSmemMax));
            VCHECK(cudaFuncSetAttribute(voc_conv_tcw_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTSmemMax));
            attr_set[dev] = true;
        }
    }
    const int halo = (a.taps - 1) * a.dil;
    const int seg = a.seg_len > 0 ? a.seg_len : a.L;
    const int n_seg = a.L / seg;
    const size_t two_per_sm = (size_t) 113 * 1024;
    // segments of at least 96 steps: tiles per segment (at most a quarter of a tile's rows unused)
    // and the window itself as the A operand of every tap (measured, 64 streams x 1 frame: 96
    // steps and up 2.87 ms per decode, 112 and up 3.02 ms, every stage 3.02 ms)
    if (seg >= 96) {
        TcConvW q;
        q.w16 = w16;
        q.nt = nt;
        q.otiles = otiles;
        q.kchunks = kchunks;
        q.err = err;
        q.tps = (seg + kTM - 1) / kTM;
        q.win_rows = (kTM + halo + 7) / 8 * 8;
        const int tiles = n_seg * q.tps * otiles;
        int splits = 1;
        while (tiles * splits * 2 <= 2 * 148 && splits * 2 <= kchunks && splits < 16 &&
               (size_t) splits * 2 * a.cout * a.ldy <= scratch_floats)
            splits *= 2;
        a.splits = splits;
        a.part = scratch;
        q.a = a;
        q.splits = splits;
        q.cps = (kchunks + splits - 1) / splits;
        auto smem = [&](int bs) { return (size_t) 1024 + (size_t) 2 * q.win_rows * 128 + (size_t) bs * nt * 128; };
        q.b_stages = 4;
        const size_t cap = (long long) tiles * splits > 148 ? two_per_sm : (size_t) kTSmemMax;
        while (q.b_stages > 2 && smem(q.b_stages) > cap) q.b_stages--;
        if (smem(q.b_stages) > (size_t) kTSmemMax) throw std::runtime_error("tcgen05 conv: the windows do not fit in shared memory");
        const dim3 grid((unsigned) (n_seg * q.tps), (unsigned) otiles, (unsigned) splits);
        voc_conv_tcw_kernel<<<grid, kTThreads, smem(q.b_stages), s>>>(q);
        if (splits > 1) launch_conv_reduce(a, s);
        return;
    }
    // small grids: split the input-channel chunks across CTAs until about two waves are in flight
    const int tiles = ((a.L + kTM - 1) / kTM) * otiles;  // otiles cover the phases too
    int splits = 1;
    while (tiles * splits * 2 <= 2 * 148 && splits * 2 <= kchunks && splits < 16 &&
           (size_t) splits * 2 * a.cout * a.ldy <= scratch_floats)
        splits *= 2;
    a.splits = splits;
    a.part = scratch;
    TcConv p;
    p.splits = splits;
    p.cps = (kchunks + splits - 1) / splits;
    p.a = a;
    p.w16 = w16;
    p.nt = nt;
    p.otiles = otiles;
    p.kchunks = kchunks;
    p.err = err;
    const int touched = std::min(n_seg, (kTM - 1 + seg - 1) / seg + 1);
    p.win_rows = (kTM + halo * touched + 7) / 8 * 8;
    auto smem = [&](int as, int bs) {
        return (size_t) 1024 + (size_t) as * kTAB + (size_t) bs * nt * 128 + (size_t) p.win_rows * (128 + 8);
    };
    p.a_stages = 3;
    p.b_stages = 3;
    // grids of more than one wave: two CTAs per SM (one's staging and epilogue latency hidden
    // behind the other's work) when two-stage rings make room for them
    const long long ctas = (long long) tiles * splits;
    if (ctas > 148 && smem(2, 2) <= two_per_sm)
        while (smem(p.a_stages, p.b_stages) > two_per_sm) {
            if (p.b_stages > 2) p.b_stages--;
            else p.a_stages--;
        }
    while (smem(p.a_stages, p.b_stages) > (size_t) kTSmemMax) {
        if (p.b_stages > 2) p.b_stages--;
        else if (p.a_stages > 2) p.a_stages--;
        else throw std::runtime_error("tcgen05 conv: the input window does not fit in shared memory");
    }
    const dim3 grid((unsigned) ((a.L + kTM - 1) / kTM), (unsigned) otiles, (unsigned) splits);
    voc_conv_tc_kernel<<<grid, kTThreads, smem(p.a_stages, p.b_stages), s>>>(p);
    if (splits > 1) launch_conv_reduce(a, s);
}

}  // namespace

template <class T> T * Vocoder::dalloc(size_t n) {
    void * p = nullptr;
    VCHECK(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
    allocs_.push_back(p);
    return (T *) p;
}

const GgufTensor & Vocoder::need(const std::string & name) const {
    for (const GgufTensor & t : gg_.tensors)
        if (t.name == name) return t;
    throw std::runtime_error("vocoder: tensor " + name + " missing from the GGUF");
}

float * Vocoder::load_f32(const std::string & name, int64_t expect, bool exp_of, bool recip) {
    const GgufTensor & t = need(name);
    if (t.type != 0 || (expect >= 0 && t.nelem() != expect))
        throw std::runtime_error("vocoder: " + name + " must be F32 with " + std::to_string(expect) + " elements");
    std::vector<float> h((size_t) t.nelem());
    std::memcpy(h.data(), gg_.data(t), h.size() * 4);
    if (exp_of)
        for (float & v : h) v = expf(v);  // SnakeBeta parameters are stored as logarithms
    if (recip)
        for (float & v : h) v = 1.0f / v;  // SnakeBeta's beta: the kernels multiply by 1 / beta
    float * d = dalloc<float>(h.size());
    VCHECK(cudaMemcpyAsync(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice, stream_));
    return d;
}

QMat Vocoder::load_q8(const std::string & name) {
    const GgufTensor & t = need(name);
    if (t.type != GT_Q8_0 && t.type != GT_Q4_K) throw std::runtime_error("vocoder: " + name + " must be Q8_0 or Q4_K");
    const int K = (int) t.ne[0], M = (int) t.rows();
    QMat q;
    q.M = M;
    q.K = K;
    q.KB = K / 32;
    q.MT = (M + 15) / 16;
    uint8_t * raw = nullptr;
    VCHECK(cudaMalloc(&raw, t.nbytes));
    VCHECK(cudaMemcpyAsync(raw, gg_.data(t), t.nbytes, cudaMemcpyHostToDevice, stream_));
    if (t.type == GT_Q4_K) {
        // Q4_K linears run on the tcgen05 dequant-GEMM (its 4-bit tile layout)
        if (K % 256) throw std::runtime_error("vocoder: " + name + " is Q4_K with rows not a multiple of 256");
        UMat u;
        u.M = M; u.MT = (M + 127) / 128; u.K = K; u.KC = K / 64; u.q4 = 1;
        uint8_t * ub = dalloc<uint8_t>((size_t) u.MT * u.KC * kUChunkBytesQ4);
        repack_umma_q4k(raw, M, K, ub, stream_);
        u.blk = ub;
        q.u = u;
    } else {
        uint4 * qs = dalloc<uint4>((size_t) q.MT * q.KB * 32);
        half2 * ds = dalloc<half2>((size_t) q.MT * q.KB * 8);
        repack_q8(raw, M, K, qs, ds, stream_);
        q.qs = qs;
        q.ds = ds;
        if (K % 64 == 0) {
            // the tcgen05 dequant-GEMM's layout as well: the batched decodes' linears run on it
            UMat u;
            u.M = M; u.MT = (M + 127) / 128; u.K = K; u.KC = K / 64; u.q4 = 0;
            uint8_t * ub = dalloc<uint8_t>((size_t) u.MT * u.KC * kUChunkBytes);
            repack_umma(raw, M, K, ub, stream_);
            u.blk = ub;
            q.u = u;
        }
    }
    VCHECK(cudaStreamSynchronize(stream_));
    cudaFree(raw);
    return q;
}

// several Q8_0 / Q4_K matrices of one row length as one tcgen05 matrix: rows stacked in order,
// or (interleave_pairs) a gate and an up matrix in alternating 16-row groups, the layout of the
// GEMM's SwiGLU epilogue (output column j = group 16 + row in group)
QMat Vocoder::load_q8_fused(const std::vector<std::string> & names, bool interleave_pairs) {
    std::vector<const GgufTensor *> parts;
    for (const std::string & n : names) parts.push_back(&need(n));
    const int K = (int) parts[0]->ne[0];
    const bool q4 = parts[0]->type == GT_Q4_K;
    for (const GgufTensor * t : parts) {
        if (t->type != GT_Q8_0 && t->type != GT_Q4_K) throw std::runtime_error("vocoder: " + t->name + " must be Q8_0 or Q4_K");
        if (t->type != parts[0]->type || t->ne[0] != K) throw std::runtime_error("vocoder: " + t->name + " differs from its fused partner");
    }
    if (K % 64 || (q4 && K % 256)) throw std::runtime_error("vocoder: fused matrices need rows of a multiple of 64 (256 for Q4_K)");
    const size_t row_bytes = q4 ? (size_t) (K / 256) * 144 : (size_t) (K / 32) * 34;
    std::vector<const uint8_t *> rows;
    if (interleave_pairs) {
        const int F = (int) parts[0]->rows();
        if (parts.size() != 2 || parts[1]->rows() != F || F % 16) throw std::runtime_error("vocoder: gate/up pair shapes differ");
        for (int p = 0; p < 2 * F; p++) {
            const int grp = p / 32, r = p % 32;
            rows.push_back(gg_.data(*parts[r < 16 ? 0 : 1]) + (size_t) (grp * 16 + (r & 15)) * row_bytes);
        }
    } else {
        for (const GgufTensor * t : parts)
            for (int64_t r = 0; r < t->rows(); r++) rows.push_back(gg_.data(*t) + (size_t) r * row_bytes);
    }
    const int M = (int) rows.size();
    std::vector<uint8_t> raw((size_t) M * row_bytes);
    for (int r = 0; r < M; r++) std::memcpy(raw.data() + (size_t) r * row_bytes, rows[r], row_bytes);
    uint8_t * raw_dev = nullptr;
    VCHECK(cudaMalloc(&raw_dev, raw.size()));
    VCHECK(cudaMemcpyAsync(raw_dev, raw.data(), raw.size(), cudaMemcpyHostToDevice, stream_));
    QMat q;
    q.M = M;
    q.K = K;
    q.KB = K / 32;
    q.MT = (M + 15) / 16;
    UMat u;
    u.M = M; u.MT = (M + 127) / 128; u.K = K; u.KC = K / 64; u.q4 = q4 ? 1 : 0;
    uint8_t * ub = dalloc<uint8_t>((size_t) u.MT * u.KC * umat_chunk_bytes(u.q4));
    if (q4) repack_umma_q4k(raw_dev, M, K, ub, stream_);
    else repack_umma(raw_dev, M, K, ub, stream_);
    u.blk = ub;
    q.u = u;
    VCHECK(cudaStreamSynchronize(stream_));
    cudaFree(raw_dev);
    return q;
}

void Vocoder::linear(const QMat & w, const half * x16, int ldx, int rows, const GemvOut & out, cudaStream_t s) {
    if (w.u.blk && ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(x16) & 15) == 0)
        launch_umma_gemm(w.u, x16, ldx, rows, out, err_, s, false);
    else if (w.qs) launch_gemv(w, x16, ldx, rows, out, scr_, s);
    else throw std::runtime_error("vocoder: a Q4_K linear needs 16-byte aligned activations with a stride multiple of 8");
}

Vocoder::Conv Vocoder::load_conv(const std::string & name, int K, int cin, int cout, int stride) {
    Conv c;
    c.K = K;
    c.cin = cin;
    c.cout = cout;
    const bool transposed = stride > 0;
    const GgufTensor & t = need(name + ".weight");
    if (t.type != GT_F32 || t.ne.size() != 3 || t.ne[0] != K || t.ne[1] != (transposed ? cout : cin) ||
        t.ne[2] != (transposed ? cin : cout))
        throw std::runtime_error("vocoder: unexpected shape or type of " + name + ".weight");
    c.b = load_f32(name + ".bias", cout);
    const float * src = reinterpret_cast<const float *>(gg_.data(t));
    if (!transposed) {
        // [cout][cin][K] -> tap-major [cout][K][cin]
        c.taps = K;
        c.phases = 1;
        std::vector<float> h((size_t) cout * K * cin);
        for (int o = 0; o < cout; o++)
            for (int i = 0; i < cin; i++)
                for (int k = 0; k < K; k++) h[((size_t) o * K + k) * cin + i] = src[((size_t) o * cin + i) * K + k];
        float * d = dalloc<float>(h.size());
        VCHECK(cudaMemcpyAsync(d, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice, stream_));
        c.w = d;
        tile_conv_f16(c, h);
        return c;
    }
    // [cin][cout][K] -> per output phase p: tap-major [cout][taps][cin]; the input step t - m
    // meets weight k = p + m s (zero where k >= K) and sits at tap taps-1-m, so each phase is a
    // causal conv
    c.stride = stride;
    c.phases = stride;
    c.taps = (K + stride - 1) / stride;
    std::vector<float> h((size_t) stride * cout * cin * c.taps, 0.0f);
    for (int p = 0; p < stride; p++)
        for (int o = 0; o < cout; o++)
            for (int i = 0; i < cin; i++)
                for (int m = 0; m < c.taps; m++) {
                    const int k = p + m * stride;
                    if (k < K) h[(((size_t) p * cout + o) * c.taps + (c.taps - 1 - m)) * cin + i] = src[((size_t) i * cout + o) * K + k];
                }
    float * d = dalloc<float>(h.size());
    VCHECK(cudaMemcpyAsync(d, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice, stream_));
    c.w = d;
    tile_conv_f16(c, h);
    return c;
}

void Vocoder::tile_conv_f16(Conv & c, const std::vector<float> & h) {
    const int ncol = c.cout * c.phases;
    c.otiles = (ncol + 255) / 256;
    c.nt = ((ncol + c.otiles - 1) / c.otiles + 31) / 32 * 32;
    c.kchunks = (c.cin + 63) / 64;
    const size_t tile = (size_t) c.nt * 64;  // halves
    std::vector<half> t((size_t) c.otiles * c.kchunks * c.taps * tile, __float2half(0.0f));
    for (int ot = 0; ot < c.otiles; ot++)
        for (int ch = 0; ch < c.kchunks; ch++)
            for (int k = 0; k < c.taps; k++) {
                half * dst = t.data() + (((size_t) ot * c.kchunks + ch) * c.taps + k) * tile;
                for (int n = 0; n < c.nt; n++) {
                        const int g = ot * c.nt + n;
                        if (g >= ncol) continue;
                        const int o = g / c.phases, ph = g % c.phases;
                        for (int i = 0; i < 64; i++) {
                            const int ci = ch * 64 + i;
                            if (ci >= c.cin) continue;
                            // row n: 8-row atoms of 1024 B, 16-byte piece i/8 swizzled by n mod 8
                            const size_t byte = (size_t) (n / 8) * 1024 + (n % 8) * 128 + (size_t) (((i / 8) ^ (n % 8)) * 16) + (i % 8) * 2;
                            dst[byte / 2] = __float2half_rn(h[(((size_t) ph * c.cout + o) * c.taps + k) * c.cin + ci]);
                        }
                }
            }
    c.w16 = dalloc<half>(t.size());
    VCHECK(cudaMemcpyAsync(c.w16, t.data(), t.size() * sizeof(half), cudaMemcpyHostToDevice, stream_));
    // the host vector goes out of scope: the upload must complete first
    VCHECK(cudaStreamSynchronize(stream_));
}

Vocoder::Vocoder(const GgufFile & gg, const ModelConfig & cfg, int device, cudaStream_t stream)
    : gg_(gg), cfg_(cfg), vc_(cfg.voc), device_(device) {
    VCHECK(cudaSetDevice(device));
    if (stream) {
        stream_ = stream;
        own_stream_ = false;
    } else {
        VCHECK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    }
    const GgufTensor & e0 = need("codec.dq.first.0.embed");
    dq_ = (int) e0.ne[0];
    if (e0.ne[1] < cfg_.vs) throw std::runtime_error("vocoder: codebook tables need at least audio_vocab_size rows");
    // tables are read for rows < vs only; keep exactly vs rows of each
    auto table = [&](const std::string & n, float * dst) {
        const GgufTensor & t = need(n);
        if (t.type != 0 || t.ne[0] != dq_) throw std::runtime_error("vocoder: " + n + " must be F32 [dq, rows]");
        VCHECK(cudaMemcpyAsync(dst, gg_.data(t), (size_t) cfg_.vs * dq_ * 4, cudaMemcpyHostToDevice, stream_));
    };
    emb_first_ = dalloc<float>((size_t) cfg_.vs * dq_);
    table("codec.dq.first.0.embed", emb_first_);
    float * rest = dalloc<float>((size_t) std::max(1, cfg_.nc - 1) * cfg_.vs * dq_);
    for (int cb = 1; cb < cfg_.nc; cb++) table("codec.dq.rest." + std::to_string(cb - 1) + ".embed", rest + (size_t) (cb - 1) * cfg_.vs * dq_);
    emb_rest_.assign(1, rest);
    dq_first_out_ = load_q8("codec.dq.first.out_proj.weight");
    dq_rest_out_ = load_q8("codec.dq.rest.out_proj.weight");
    cbdim_ = dq_first_out_.M;
    const GgufTensor & pre = need("codec.dpre.conv.weight");
    latent_ = (int) pre.ne[2];
    dpre_ = load_conv("codec.dpre.conv", (int) pre.ne[0], cbdim_, latent_, 0);
    in_proj_ = load_q8("codec.dtf.in_proj.weight");
    in_proj_b_ = load_f32("codec.dtf.in_proj.bias", vc_.hidden);
    for (int l = 0; l < vc_.n_layer; l++) {
        const std::string p = "codec.dtf.blk." + std::to_string(l);
        Layer L;
        L.attn_norm = load_f32(p + ".attn_norm.weight", vc_.hidden);
        L.qkv = load_q8_fused({ p + ".attn_q.weight", p + ".attn_k.weight", p + ".attn_v.weight" }, false);
        L.o = load_q8(p + ".attn_output.weight");
        L.attn_scale = load_f32(p + ".attn_scale", vc_.hidden);
        L.ffn_norm = load_f32(p + ".ffn_norm.weight", vc_.hidden);
        L.gate_up = load_q8_fused({ p + ".ffn_gate.weight", p + ".ffn_up.weight" }, true);
        L.down = load_q8(p + ".ffn_down.weight");
        L.ffn_scale = load_f32(p + ".ffn_scale", vc_.hidden);
        layers_.push_back(L);
    }
    out_norm_ = load_f32("codec.dtf.norm.weight", vc_.hidden);
    out_proj_ = load_q8("codec.dtf.out_proj.weight");
    out_proj_b_ = load_f32("codec.dtf.out_proj.bias", latent_);
    for (size_t i = 0; i < vc_.ratios.size(); i++) {
        const std::string p = "codec.dup." + std::to_string(i);
        Up u;
        u.ratio = vc_.ratios[i];
        const GgufTensor & ut = need(p + ".up.conv.weight");
        u.up = load_conv(p + ".up.conv", (int) ut.ne[0], latent_, latent_, u.ratio);
        const GgufTensor & dw = need(p + ".dw.weight");
        u.dw.K = (int) dw.ne[1];
        u.dw.cin = u.dw.cout = latent_;
        u.dw.w = load_f32(p + ".dw.weight", (int64_t) latent_ * u.dw.K);
        u.dw.b = load_f32(p + ".dw.bias", latent_);
        u.norm_w = load_f32(p + ".norm.weight", latent_);
        u.norm_b = load_f32(p + ".norm.bias", latent_);
        u.pw1 = load_q8(p + ".pw1.weight");
        u.pw1_b = load_f32(p + ".pw1.bias", u.pw1.M);
        u.pw2 = load_q8(p + ".pw2.weight");
        u.pw2_b = load_f32(p + ".pw2.bias", latent_);
        u.gamma = load_f32(p + ".gamma", latent_);
        ups_.push_back(u);
    }
    const GgufTensor & hd = need("codec.dhead.conv.weight");
    dec_ = (int) hd.ne[2];
    dhead_ = load_conv("codec.dhead.conv", (int) hd.ne[0], latent_, dec_, 0);
    int ch = dec_;
    for (size_t i = 0; i < vc_.rates.size(); i++) {
        const std::string p = "codec.dblk." + std::to_string(i);
        Blk b;
        b.rate = vc_.rates[i];
        b.alpha = load_f32(p + ".alpha", ch, true);
        b.beta = load_f32(p + ".beta", ch, true, true);
        const GgufTensor & ut = need(p + ".up.conv.weight");
        const int co = (int) ut.ne[1];
        b.up = load_conv(p + ".up.conv", (int) ut.ne[0], ch, co, b.rate);
        ch = co;
        for (int j = 0; j < 3; j++) {
            const std::string q = p + ".res." + std::to_string(j);
            Res r;
            r.a1 = load_f32(q + ".a1", ch, true);
            r.b1 = load_f32(q + ".b1", ch, true, true);
            r.c1 = load_conv(q + ".conv1.conv", (int) need(q + ".conv1.conv.weight").ne[0], ch, ch, 0);
            r.a2 = load_f32(q + ".a2", ch, true);
            r.b2 = load_f32(q + ".b2", ch, true, true);
            r.c2 = load_conv(q + ".conv2.conv", (int) need(q + ".conv2.conv.weight").ne[0], ch, ch, 0);
            b.res[j] = r;
        }
        blks_.push_back(b);
    }
    fin_alpha_ = load_f32("codec.dfin.alpha", ch, true);
    fin_beta_ = load_f32("codec.dfin.beta", ch, true, true);
    dfin_ = load_conv("codec.dfin.conv", (int) need("codec.dfin.conv.weight").ne[0], ch, 1, 0);
    int up_total = 1;
    for (int r : vc_.ratios) up_total *= r;
    for (int r : vc_.rates) up_total *= r;
    if (up_total != kSamplesPerFrame)
        throw std::runtime_error("vocoder: the upsampling stages give " + std::to_string(up_total) +
                                 " samples per frame, the C API assumes 1920");
    // dynamic shared memory of the GEMV and tcgen05 GEMM variants and of the widest conv window
    init_kernel_attributes();
    init_umma_attributes();
    {
        int lxp = conv_lxp(std::max({ dpre_.taps, dhead_.taps, dfin_.taps }), 1);
        for (const Up & u : ups_) lxp = std::max(lxp, conv_lxp(u.up.taps, 1));
        const int dil_max[3] = { 1, 3, 9 };
        for (const Blk & b : blks_) {
            lxp = std::max(lxp, conv_lxp(b.up.taps, 1));
            for (int j = 0; j < 3; j++)
                lxp = std::max({ lxp, conv_lxp(b.res[j].c1.taps, dil_max[j]), conv_lxp(b.res[j].c2.taps, 1) });
        }
        raise_conv_smem_limit(conv_smem_bytes(lxp));
    }
    // the carried state of a stream, in decode order: dpre; per ConvNeXt stage its transposed
    // conv and depthwise conv; dhead; per SEANet block its transposed conv and each residual
    // unit's two convs; dfin (a transposed conv carries taps - 1 inputs, a conv (taps - 1) dil)
    {
        auto add = [&](int cin, int P) {
            st_off_.push_back(st_floats_);
            st_floats_ += (size_t) 2 * cin * P;
        };
        add(cbdim_, dpre_.taps - 1);
        for (const Up & u : ups_) {
            add(latent_, u.up.taps - 1);
            add(latent_, u.dw.K - 1);
        }
        add(latent_, dhead_.taps - 1);
        const int dil[3] = { 1, 3, 9 };
        for (const Blk & b : blks_) {
            add(b.up.cin, b.up.taps - 1);
            for (int j = 0; j < 3; j++) {
                add(b.res[j].c1.cin, (b.res[j].c1.taps - 1) * dil[j]);
                add(b.res[j].c2.cin, b.res[j].c2.taps - 1);
            }
        }
        add(dfin_.cin, dfin_.taps - 1);
    }
    err_ = dalloc<int>(1);
    VCHECK(cudaMemsetAsync(err_, 0, sizeof(int), stream_));
    scr_.ws_elems = (size_t) 1 << 20;
    scr_.ws = dalloc<float4>(scr_.ws_elems);
    scr_.n_counters = 4096;
    scr_.counters = dalloc<int>(scr_.n_counters);
    VCHECK(cudaMemsetAsync(scr_.counters, 0, scr_.n_counters * sizeof(int), stream_));
    // every upload above is ordered on stream_ (a plain cudaMemcpy from pageable memory may still
    // be in flight when it returns, and a non-blocking stream does not wait for it)
    VCHECK(cudaStreamSynchronize(stream_));
}

Vocoder::~Vocoder() {
    cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    if (pcm_host_) cudaFreeHost(pcm_host_);
    if (rows_dev_) cudaFree(rows_dev_);
    for (void * p : scratch_allocs_) cudaFree(p);
    for (void * p : stream_allocs_) cudaFree(p);
    for (void * p : allocs_) cudaFree(p);
    if (stream_ && own_stream_) cudaStreamDestroy(stream_);
}

void Vocoder::ensure(int T) {
    if (T <= tcap_) return;
    VCHECK(cudaStreamSynchronize(stream_));
    for (void * p : scratch_allocs_) cudaFree(p);
    scratch_allocs_.clear();
    tcap_ = std::max(T, 64);
    const size_t Tc = (size_t) tcap_;
    // the largest [C][L] activation of the conv stack
    size_t L = Tc, mx = Tc * std::max({ cbdim_, latent_, vc_.hidden });
    for (const Up & u : ups_) {
        L *= u.ratio;
        mx = std::max(mx, (size_t) latent_ * L);
    }
    mx = std::max(mx, (size_t) dec_ * L);
    int ch = dec_;
    for (const Blk & b : blks_) {
        L *= b.rate;
        ch = b.up.cout;
        mx = std::max(mx, (size_t) ch * L);
    }
    act_elems_ = mx;
    size_t up_rows = Tc;
    for (const Up & u : ups_) up_rows *= u.ratio;
    const size_t wide = std::max({ (size_t) vc_.n_head * vc_.hd, (size_t) vc_.ffn, (size_t) 4 * latent_, (size_t) latent_,
                                   (size_t) cbdim_, (size_t) dq_ });
    auto fa = [&](size_t n) { void * p = nullptr; VCHECK(cudaMalloc(&p, std::max<size_t>(n, 16) * 4)); scratch_allocs_.push_back(p); return (float *) p; };
    auto ha = [&](size_t n) { void * p = nullptr; VCHECK(cudaMalloc(&p, std::max<size_t>(n, 16) * 2)); scratch_allocs_.push_back(p); return (half *) p; };
    a_ = fa(act_elems_);
    b_ = fa(act_elems_);
    c_ = fa(act_elems_);
    part_ = fa(2 * act_elems_);
    t32_ = fa(up_rows * wide);
    q_ = fa(Tc * ((size_t) vc_.n_head * vc_.hd + 2 * (size_t) vc_.n_kv * vc_.hd));  // rows of q | k | v
    o_ = fa(up_rows * wide);
    pcm_ = fa(Tc * kSamplesPerFrame);
    fring_ = fa(Tc * 2 * vc_.n_kv * vc_.hd);
    t16_ = ha(up_rows * wide);
    att16_ = ha(Tc * vc_.n_head * vc_.hd);
    f16_ = ha(std::max(up_rows * wide, Tc * (size_t) dq_ * 2));
    void * pc = nullptr;
    VCHECK(cudaMalloc(&pc, Tc * cfg_.nc * sizeof(int)));
    scratch_allocs_.push_back(pc);
    codes_ = (int *) pc;
    if (rope_max_ < tcap_) {
        const std::vector<float2> tab = rope_table(tcap_, vc_.hd, vc_.theta, 1.0f, nullptr);
        void * pr = nullptr;
        VCHECK(cudaMalloc(&pr, tab.size() * sizeof(float2)));
        scratch_allocs_.push_back(pr);
        VCHECK(cudaMemcpyAsync(pr, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice, stream_));
        rope_ = (float2 *) pr;
        rope_max_ = tcap_;
    }
}

void Vocoder::decode(const int * codes, int T, float * pcm) {
    if (T <= 0) return;
    VCHECK(cudaSetDevice(device_));
    ensure(T);
    VCHECK(cudaMemcpyAsync(codes_, codes, (size_t) T * cfg_.nc * sizeof(int), cudaMemcpyHostToDevice, stream_));
    decode_segments(codes_, cfg_.nc, 1, T, nullptr, pcm_);
    VCHECK(cudaMemcpyAsync(pcm, pcm_, (size_t) T * kSamplesPerFrame * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    check_device_error();
}

void Vocoder::check_device_error() {
    int err = 0;
    VCHECK(cudaMemcpyAsync(&err, err_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
    VCHECK(cudaStreamSynchronize(stream_));
    if (err) {
        VCHECK(cudaMemsetAsync(err_, 0, sizeof(int), stream_));
        VCHECK(cudaStreamSynchronize(stream_));
        throw std::runtime_error("vocoder: a bounded wait timed out in the tcgen05 GEMM (device error code " +
                                 std::to_string(err) + ")");
    }
}

void Vocoder::ensure_segments(int S) {
    if (S <= seg_cap_) return;
    VCHECK(cudaStreamSynchronize(stream_));
    const int cap = std::max(S, 256);
    int * d = nullptr;
    VCHECK(cudaMalloc(&d, (size_t) 5 * cap * sizeof(int)));
    std::vector<int> h((size_t) 2 * cap, 0);
    for (int i = 0; i < cap; i++) h[i] = i;
    VCHECK(cudaMemcpyAsync(d + (size_t) 3 * cap, h.data(), h.size() * sizeof(int), cudaMemcpyHostToDevice, stream_));
    VCHECK(cudaStreamSynchronize(stream_));
    if (seg_dev_) cudaFree(seg_dev_);
    seg_dev_ = d;
    seg_ident_ = d + (size_t) 3 * cap;
    seg_cap_ = cap;
}

void Vocoder::decode_segments(const int * codes_dev, int ld_codes, int S, int T, const Segment * segs, float * pcm_dev) {
    if (S <= 0 || T <= 0) return;
    VCHECK(cudaSetDevice(device_));
    const int NF = S * T;  // frames of the whole batch
    ensure(NF);
    ensure_segments(S);
    cudaStream_t s = stream_;
    const int nc = cfg_.nc, H = vc_.hidden, nh = vc_.n_head, nkv = vc_.n_kv, hd = vc_.hd, F = vc_.ffn;
    if (hd > 128 || hd % 32 || nh % nkv) throw std::runtime_error("vocoder: head_dim must be 32..128 (multiple of 32), heads a multiple of kv heads");
    const bool streaming = segs != nullptr;
    const int kvd = nkv * hd;
    // per segment: stream slot, state copy, first position (whole decodes: 0, 1, ... / -1 / 0)
    const int * d_slot = seg_ident_, * d_par = nullptr, * d_pos = seg_ident_ + seg_cap_;
    if (streaming) {
        if (!st_pool_) throw std::runtime_error("vocoder: stream state is not allocated");
        if (T > ring_R_ - vc_.window + 1)
            throw std::runtime_error("vocoder: at most " + std::to_string(ring_R_ - vc_.window + 1) + " new frames per stream and call");
        std::vector<int> h((size_t) 3 * S);
        for (int b = 0; b < S; b++) {
            if (segs[b].pos + T > kMaxStreamFrames) throw std::runtime_error("vocoder: a stream passed " + std::to_string(kMaxStreamFrames) + " frames");
            h[b] = segs[b].slot;
            h[S + b] = segs[b].par;
            h[2 * S + b] = segs[b].pos;
        }
        VCHECK(cudaMemcpyAsync(seg_dev_, h.data(), h.size() * sizeof(int), cudaMemcpyHostToDevice, s));
        d_slot = seg_dev_;
        d_par = seg_dev_ + S;
        d_pos = seg_dev_ + 2 * S;
    }
    int li = 0;  // state layer of the next causal convolution (decode order, see the constructor)

    // quantiser decode -> [NF][cbdim] -> [cbdim][NF]
    half * e_first = f16_, * e_rest = f16_ + (size_t) NF * dq_;
    voc_embed_kernel<<<NF, 128, 0, s>>>(emb_first_, emb_rest_[0], codes_dev, ld_codes, nc, dq_, cfg_.vs, e_first, e_rest);
    linear(dq_first_out_, e_first, dq_, NF, GemvOut{ EPI_STORE, t32_, nullptr, cbdim_ }, s);
    if (nc > 1) linear(dq_rest_out_, e_rest, dq_, NF, GemvOut{ EPI_RESID, t32_, nullptr, cbdim_ }, s);
    auto transpose = [&](const float * in, int R, int C, float * out, const float * add) {
        voc_transpose_kernel<<<dim3((C + 31) / 32, (R + 31) / 32), dim3(32, 8), 0, s>>>(in, R, C, out, add);
    };
    // one causal conv (or the phases of a transposed conv) over x [cin][S seg]: S segments of
    // `seg` steps, each continuing its stream's state of layer li when streaming. The output
    // [cout][S seg phases] holds v = conv + bias (+ res), or SnakeBeta(v) with (sa, sb); y2, when
    // given, receives SnakeBeta(v) with (s2a, s2b)
    struct Act { const float * a = nullptr, * b = nullptr; };
    auto conv = [&](const Conv & c, const float * x, int seg, int dil, float * y, Act act = {}, const float * res = nullptr,
                    float * y2 = nullptr, Act act2 = {}, bool clamp = false) {
        ConvArgs ca;
        ca.x = x; ca.cin = c.cin; ca.L = S * seg;
        ca.w = c.w; ca.taps = c.taps; ca.dil = dil;
        ca.bias = c.b; ca.cout = c.cout;
        ca.y = y; ca.ldy = S * seg * c.phases; ca.ostride = c.phases;
        ca.res = res; ca.sa = act.a; ca.sb = act.b;
        ca.y2 = y2; ca.s2a = act2.a; ca.s2b = act2.b;
        ca.clamp = clamp ? 1 : 0;
        ca.seg_len = seg;
        if (streaming && (c.taps - 1) * dil > 0) {
            ca.st = st_pool_ + st_off_[li];
            ca.st_stride = st_floats_;
            ca.seg_slot = d_slot;
            ca.seg_par = d_par;
        }
        li++;
        launch_conv_tc(ca, c.w16, c.nt, c.otiles, c.kchunks, err_, part_, 2 * act_elems_, s);
    };
    transpose(t32_, NF, cbdim_, a_, nullptr);
    conv(dpre_, a_, T, 1, b_);                                       // [latent][NF]

    // transformer on [NF][latent] rows; keys and values go to each segment's ring (a stream's
    // own ring, or for whole decodes one of T positions per segment)
    transpose(b_, latent_, NF, a_, nullptr);                         // a_ = [NF][latent]
    voc_to_f16_kernel<<<grid_for((size_t) NF * latent_), 256, 0, s>>>(a_, (size_t) NF * latent_, t16_);
    float * h = c_;                                                  // [NF][H]
    linear(in_proj_, t16_, latent_, NF, GemvOut{ EPI_STORE, h, nullptr, H }, s);
    voc_bias_scale_kernel<<<grid_for((size_t) NF * H), 256, 0, s>>>(h, (size_t) NF * H, H, in_proj_b_, nullptr);
    const float scale = 1.0f / std::sqrt((float) hd);
    const float2 * rope = streaming ? srope_ : rope_;
    const int R = streaming ? ring_R_ : T;
    const size_t slot_stride = streaming ? (size_t) vc_.n_layer * ring_R_ * 2 * kvd : (size_t) T * 2 * kvd;
    // per layer: one q/k/v GEMM, the ring append and attention, the o GEMM, the residual add
    // fused with the FFN norm, one gate/up GEMM with the SwiGLU epilogue (f16 out), the down GEMM,
    // the residual add fused with the next norm
    const int QKV = nh * hd + 2 * kvd;
    launch_rmsnorm(h, H, layers_.empty() ? out_norm_ : layers_[0].attn_norm, H, vc_.eps, t16_, H, nullptr, 0, 0, NF, nullptr, s);
    for (size_t l = 0; l < layers_.size(); l++) {
        const Layer & Ly = layers_[l];
        float * ring = streaming ? ring_ + l * (size_t) ring_R_ * 2 * kvd : fring_;
        linear(Ly.qkv, t16_, H, NF, GemvOut{ EPI_STORE, q_, nullptr, QKV }, s);
        voc_kv_ring_append_kernel<<<grid_for((size_t) NF * kvd), 256, 0, s>>>(q_ + nh * hd, q_ + nh * hd + kvd, QKV, S, T, nkv, hd,
                                                                              rope, ring, slot_stride, R, d_slot, d_pos);
        const int warps = NF * nh;
        voc_attn_ring_kernel<<<(warps * 32 + 127) / 128, 128, 0, s>>>(q_, QKV, S, T, nh, nkv, hd, vc_.window, rope, scale, ring,
                                                                        slot_stride, R, d_slot, d_pos, att16_);
        linear(Ly.o, att16_, nh * hd, NF, GemvOut{ EPI_STORE, o_, nullptr, H }, s);
        voc_add_rmsnorm_kernel<<<NF, 256, 0, s>>>(h, o_, Ly.attn_scale, H, Ly.ffn_norm, vc_.eps, t16_);
        linear(Ly.gate_up, t16_, H, NF, GemvOut{ EPI_SWIGLU, nullptr, f16_, F }, s);
        linear(Ly.down, f16_, F, NF, GemvOut{ EPI_STORE, o_, nullptr, H }, s);
        const float * next_norm = l + 1 < layers_.size() ? layers_[l + 1].attn_norm : out_norm_;
        voc_add_rmsnorm_kernel<<<NF, 256, 0, s>>>(h, o_, Ly.ffn_scale, H, next_norm, vc_.eps, t16_);
    }
    linear(out_proj_, t16_, H, NF, GemvOut{ EPI_STORE, o_, nullptr, latent_ }, s);
    voc_bias_scale_kernel<<<grid_for((size_t) NF * latent_), 256, 0, s>>>(o_, (size_t) NF * latent_, latent_, out_proj_b_, nullptr);
    transpose(o_, NF, latent_, a_, nullptr);                         // a_ = [latent][NF]

    // ConvNeXt upsampling stages (L: steps per segment, NL = S L rows in all)
    int L = T;
    float * x = a_;
    float * y = b_;
    for (const Up & u : ups_) {
        conv(u.up, x, L, 1, y);
        L *= u.ratio;
        std::swap(x, y);                                             // x = [latent][S L]
        const int NL = S * L;
        const size_t n = (size_t) NL * latent_;
        const bool dw_state = streaming && u.dw.K > 1;
        voc_depthwise_seg_kernel<<<grid_for(n + (dw_state ? (size_t) S * latent_ * (u.dw.K - 1) : 0)), 256, 0, s>>>(
            x, latent_, S, L, u.dw.w, u.dw.b, u.dw.K, y, dw_state ? st_pool_ + st_off_[li] : nullptr, st_floats_, d_slot, d_par);
        li++;
        transpose(y, latent_, NL, t32_, nullptr);                    // [S L][latent]
        voc_layernorm_kernel<<<NL, 256, 0, s>>>(t32_, latent_, u.norm_w, u.norm_b, 1e-6f, t16_);
        const int F4 = u.pw1.M;
        linear(u.pw1, t16_, latent_, NL, GemvOut{ EPI_STORE, o_, nullptr, F4 }, s);
        voc_bias_gelu_kernel<<<grid_for((size_t) NL * F4), 256, 0, s>>>(o_, (size_t) NL * F4, F4, u.pw1_b, f16_);
        linear(u.pw2, f16_, F4, NL, GemvOut{ EPI_STORE, t32_, nullptr, latent_ }, s);
        voc_bias_scale_kernel<<<grid_for(n), 256, 0, s>>>(t32_, n, latent_, u.pw2_b, u.gamma);
        transpose(t32_, NL, latent_, y, x);                          // y = x + branch^T
        std::swap(x, y);
    }
    // SEANet decoder (src/codec_decoder.cpp:80-97). Every SnakeBeta is applied by the conv that
    // produces its input: Xb holds a block's residual stream, Sb the SnakeBeta of it that the
    // next conv reads, Hb the first conv of a residual unit (already SnakeBeta'd for the second).
    // The second conv of a unit adds Xb in place and also writes the next activation into Sb.
    // A stream's carried state of each conv is its own (already activated) input.
    float * Xb = c_, * Sb = y, * Hb = x;
    auto next_act = [&](size_t bi, int j) -> Act {
        if (j + 1 < 3) return { blks_[bi].res[j + 1].a1, blks_[bi].res[j + 1].b1 };
        if (bi + 1 < blks_.size()) return { blks_[bi + 1].alpha, blks_[bi + 1].beta };
        return { fin_alpha_, fin_beta_ };
    };
    if (blks_.empty()) throw std::runtime_error("vocoder: the decoder has no upsampling blocks");
    conv(dhead_, x, L, 1, Sb, { blks_[0].alpha, blks_[0].beta });
    const int dil[3] = { 1, 3, 9 };
    for (size_t bi = 0; bi < blks_.size(); bi++) {
        const Blk & b = blks_[bi];
        conv(b.up, Sb, L, 1, Xb, {}, nullptr, Hb, { b.res[0].a1, b.res[0].b1 });
        L *= b.rate;
        std::swap(Sb, Hb);
        for (int j = 0; j < 3; j++) {
            const Res & r = b.res[j];
            conv(r.c1, Sb, L, dil[j], Hb, { r.a2, r.b2 });
            conv(r.c2, Hb, L, 1, Xb, {}, Xb, Sb, next_act(bi, j));
        }
    }
    if (L != T * kSamplesPerFrame) throw std::runtime_error("vocoder: unexpected output length");
    conv(dfin_, Sb, L, 1, pcm_dev, {}, nullptr, nullptr, {}, true);
    if (li != (int) st_off_.size()) throw std::runtime_error("vocoder: state layers out of step with the decode");
    VCHECK(cudaGetLastError());
}

// ---------------------------------------------------------------------------------- sessions
void Vocoder::session_create(int sid) {
    std::lock_guard<std::mutex> lk(mu_);
    history_[sid].clear();
}

bool Vocoder::session_free(int sid) {
    std::lock_guard<std::mutex> lk(mu_);
    return history_.erase(sid) > 0;
}

int Vocoder::session_decode(int sid, const int * frames, int n_frames, float * out_pcm) {
    std::lock_guard<std::mutex> lk(mu_);
    const int nc = cfg_.nc, spf = kSamplesPerFrame;
    std::vector<int> & hist = history_[sid];  // an unknown session is created (src/c_api.cpp:1011-1018)
    const int past = (int) hist.size() / nc;
    std::vector<int> all(hist);
    all.insert(all.end(), frames, frames + (size_t) n_frames * nc);
    std::vector<float> audio((size_t) (past + n_frames) * spf);
    decode(all.data(), past + n_frames, audio.data());
    std::memcpy(out_pcm, audio.data() + (size_t) past * spf, (size_t) n_frames * spf * sizeof(float));
    hist.insert(hist.end(), frames, frames + (size_t) n_frames * nc);
    const int cur = (int) hist.size() / nc;
    if (cur > kMaxHistory) hist.erase(hist.begin(), hist.begin() + (size_t) (cur - kMaxHistory) * nc);
    return n_frames * spf;
}

// Every entry's history is taken before any is decoded and the histories are extended in batch
// order afterwards, as in src/c_api.cpp:1066-1162. Entries of equal total length (history + new
// frames) are decoded together as the segments of one batched decode.
int Vocoder::session_decode_batch(int batch, const int * sids, const int * flat_tokens, const int * token_offsets,
                                  const int * n_frames, float * flat_pcm, const int * pcm_offsets, int * out_n_samples) {
    std::lock_guard<std::mutex> lk(mu_);
    const int nc = cfg_.nc, spf = kSamplesPerFrame;
    std::vector<std::vector<int>> codes(batch);
    std::vector<int> past(batch, 0), nfs(batch, 0), poffs(batch, 0);
    std::map<int, std::vector<int>> groups;  // total frames -> entries
    int running_tok = 0, running_pcm = 0;
    for (int b = 0; b < batch; b++) {
        const int nf = std::max(0, n_frames[b]);
        const int off = token_offsets ? token_offsets[b] : running_tok;
        poffs[b] = pcm_offsets ? pcm_offsets[b] : running_pcm;
        const std::vector<int> & hist = history_[sids[b]];  // an unknown session is created (src/c_api.cpp:1085-1093)
        past[b] = (int) hist.size() / nc;
        nfs[b] = nf;
        if (nf > 0) {
            codes[b] = hist;
            codes[b].insert(codes[b].end(), flat_tokens + off, flat_tokens + off + (size_t) nf * nc);
            groups[past[b] + nf].push_back(b);
        }
        running_tok += nf * nc;
        running_pcm += nf * spf;
    }
    std::vector<int> hc;
    std::vector<float> audio;
    for (const auto & kv : groups) {
        const int T = kv.first, S = (int) kv.second.size();
        hc.resize((size_t) S * T * nc);
        for (int i = 0; i < S; i++) std::copy(codes[kv.second[i]].begin(), codes[kv.second[i]].end(), hc.begin() + (size_t) i * T * nc);
        ensure(S * T);
        VCHECK(cudaMemcpyAsync(codes_, hc.data(), hc.size() * sizeof(int), cudaMemcpyHostToDevice, stream_));
        decode_segments(codes_, nc, S, T, nullptr, pcm_);
        audio.resize((size_t) S * T * spf);
        VCHECK(cudaMemcpyAsync(audio.data(), pcm_, audio.size() * sizeof(float), cudaMemcpyDeviceToHost, stream_));
        check_device_error();
        for (int i = 0; i < S; i++) {
            const int b = kv.second[i];
            std::memcpy(flat_pcm + poffs[b], audio.data() + ((size_t) i * T + past[b]) * spf, (size_t) nfs[b] * spf * sizeof(float));
        }
    }
    for (int b = 0; b < batch; b++) {
        if (out_n_samples) out_n_samples[b] = nfs[b] * spf;
        if (nfs[b] == 0) continue;
        std::vector<int> & hist = history_[sids[b]];
        hist.insert(hist.end(), codes[b].begin() + (size_t) past[b] * nc, codes[b].end());
        const int cur = (int) hist.size() / nc;
        if (cur > kMaxHistory) hist.erase(hist.begin(), hist.begin() + (size_t) (cur - kMaxHistory) * nc);
    }
    return batch;
}

int Vocoder::kernels_per_decode(int S, int T) {
    std::lock_guard<std::mutex> lk(mu_);
    VCHECK(cudaSetDevice(device_));
    ensure(S * T);
    ensure_segments(S);
    for (int i = 0; i < 2; i++) decode_segments(codes_, cfg_.nc, S, T, nullptr, pcm_);  // attributes and capacity settled
    VCHECK(cudaStreamSynchronize(stream_));
    cudaGraph_t g = nullptr;
    VCHECK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    try {
        decode_segments(codes_, cfg_.nc, S, T, nullptr, pcm_);
    } catch (...) {
        cudaStreamEndCapture(stream_, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    VCHECK(cudaStreamEndCapture(stream_, &g));
    size_t n = 0;
    VCHECK(cudaGraphGetNodes(g, nullptr, &n));
    std::vector<cudaGraphNode_t> nodes(n);
    VCHECK(cudaGraphGetNodes(g, nodes.data(), &n));
    int kernels = 0;
    for (cudaGraphNode_t nd : nodes) {
        cudaGraphNodeType t;
        VCHECK(cudaGraphNodeGetType(nd, &t));
        kernels += t == cudaGraphNodeTypeKernel;
    }
    cudaGraphDestroy(g);
    return kernels;
}

// ----------------------------------------------------------------------------------- streams
void Vocoder::ensure_streams() {
    if (st_pool_) return;
    VCHECK(cudaSetDevice(device_));
    const char * e = std::getenv("BZB_VOC_STREAMS");
    stream_cap_ = e ? std::max(1, std::atoi(e)) : 256;
    // a stream's ring keeps the attention window plus one call's new frames (at most 56)
    ring_R_ = (vc_.window + 56 + 7) / 8 * 8;
    const size_t kvd = (size_t) vc_.n_kv * vc_.hd;
    auto alloc = [&](size_t bytes) {
        void * p = nullptr;
        VCHECK(cudaMalloc(&p, std::max<size_t>(bytes, 16)));
        stream_allocs_.push_back(p);
        return p;
    };
    st_pool_ = (float *) alloc((size_t) stream_cap_ * st_floats_ * sizeof(float));
    ring_ = (float *) alloc((size_t) stream_cap_ * vc_.n_layer * ring_R_ * 2 * kvd * sizeof(float));
    const std::vector<float2> tab = rope_table(kMaxStreamFrames, vc_.hd, vc_.theta, 1.0f, nullptr);
    srope_ = (float2 *) alloc(tab.size() * sizeof(float2));
    VCHECK(cudaMemcpyAsync(srope_, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice, stream_));
    VCHECK(cudaStreamSynchronize(stream_));
    for (int i = stream_cap_ - 1; i >= 0; i--) free_slots_.push_back(i);
}

void Vocoder::stream_open(int id) {
    std::lock_guard<std::mutex> lk(mu_);
    ensure_streams();
    auto it = streams_.find(id);
    if (it != streams_.end()) {
        it->second.pos = 0;
        it->second.par = -1;
        return;
    }
    if (free_slots_.empty()) throw std::runtime_error("vocoder: all " + std::to_string(stream_cap_) + " stream slots are in use (BZB_VOC_STREAMS)");
    StreamInfo si;
    si.slot = free_slots_.back();
    free_slots_.pop_back();
    streams_[id] = si;
}

bool Vocoder::stream_close(int id) {
    std::lock_guard<std::mutex> lk(mu_);
    auto it = streams_.find(id);
    if (it == streams_.end()) return false;
    free_slots_.push_back(it->second.slot);
    streams_.erase(it);
    return true;
}

std::vector<Vocoder::Segment> Vocoder::stream_segments(int n, const int * ids, const unsigned long long * epochs, int T) {
    ensure_streams();
    std::vector<Segment> segs(n);
    std::map<int, int> seen;
    for (int i = 0; i < n; i++) {
        if (!seen.emplace(ids[i], i).second) throw std::runtime_error("vocoder: stream " + std::to_string(ids[i]) + " listed twice in one call");
        auto it = streams_.find(ids[i]);
        if (it == streams_.end()) {
            if (free_slots_.empty()) throw std::runtime_error("vocoder: all " + std::to_string(stream_cap_) + " stream slots are in use (BZB_VOC_STREAMS)");
            StreamInfo si;
            si.slot = free_slots_.back();
            free_slots_.pop_back();
            if (epochs) si.epoch = epochs[i];
            it = streams_.emplace(ids[i], si).first;
        } else if (epochs && it->second.epoch != epochs[i]) {
            it->second.pos = 0;
            it->second.par = -1;
            it->second.epoch = epochs[i];
        }
        if (it->second.pos + T > kMaxStreamFrames)
            throw std::runtime_error("vocoder: stream " + std::to_string(ids[i]) + " would pass " + std::to_string(kMaxStreamFrames) + " frames");
        segs[i].slot = it->second.slot;
        segs[i].par = it->second.par;
        segs[i].pos = it->second.pos;
    }
    return segs;
}

void Vocoder::advance(int n, const int * ids, int T) {
    for (int i = 0; i < n; i++) {
        StreamInfo & si = streams_[ids[i]];
        si.pos += T;
        si.par = voc_state_next(si.par);
    }
}

void Vocoder::streams_decode(int n, const int * ids, const unsigned long long * epochs, const int * codes, int T,
                             float * pcm) {
    std::lock_guard<std::mutex> lk(mu_);
    if (n <= 0 || T <= 0) return;
    VCHECK(cudaSetDevice(device_));
    const std::vector<Segment> segs = stream_segments(n, ids, epochs, T);
    ensure(n * T);
    VCHECK(cudaMemcpyAsync(codes_, codes, (size_t) n * T * cfg_.nc * sizeof(int), cudaMemcpyHostToDevice, stream_));
    decode_segments(codes_, cfg_.nc, n, T, segs.data(), pcm_);
    advance(n, ids, T);
    VCHECK(cudaMemcpyAsync(pcm, pcm_, (size_t) n * T * kSamplesPerFrame * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    check_device_error();
}

void Vocoder::streams_decode_device(int n, const int * ids, const unsigned long long * epochs, const int * codes_dev,
                                   int ld_codes, int T, float * pcm_dev) {
    std::lock_guard<std::mutex> lk(mu_);
    if (n <= 0 || T <= 0) return;
    const std::vector<Segment> segs = stream_segments(n, ids, epochs, T);
    ensure(n * T);
    decode_segments(codes_dev, ld_codes, n, T, segs.data(), pcm_dev ? pcm_dev : pcm_);
    advance(n, ids, T);
}

void Vocoder::streams_decode_rows_async(int m, const int * ids, const unsigned long long * epochs, const int * frames_dev,
                                        int ld, const int * rows) {
    std::lock_guard<std::mutex> lk(mu_);
    if (m <= 0) return;
    const std::vector<Segment> segs = stream_segments(m, ids, epochs, 1);
    ensure(m);
    const int * codes = frames_dev;
    int ldc = ld;
    if (rows) {
        if (m > rows_cap_) {
            VCHECK(cudaStreamSynchronize(stream_));
            if (rows_dev_) cudaFree(rows_dev_);
            rows_dev_ = nullptr;
            rows_cap_ = std::max(m, 256);
            VCHECK(cudaMalloc(&rows_dev_, (size_t) rows_cap_ * sizeof(int)));
        }
        // a copy from pageable host memory is staged before the call returns
        VCHECK(cudaMemcpyAsync(rows_dev_, rows, (size_t) m * sizeof(int), cudaMemcpyHostToDevice, stream_));
        voc_gather_rows_kernel<<<grid_for((size_t) m * cfg_.nc), 256, 0, stream_>>>(frames_dev, ld, rows_dev_, m, cfg_.nc, codes_);
        codes = codes_;
        ldc = cfg_.nc;
    }
    decode_segments(codes, ldc, m, 1, segs.data(), pcm_);
    const size_t need = (size_t) m * kSamplesPerFrame;
    if (need > pcm_host_cap_) {
        VCHECK(cudaStreamSynchronize(stream_));
        if (pcm_host_) cudaFreeHost(pcm_host_);
        pcm_host_ = nullptr;
        pcm_host_cap_ = std::max(need, (size_t) 64 * kSamplesPerFrame);
        VCHECK(cudaMallocHost(&pcm_host_, pcm_host_cap_ * sizeof(float)));
    }
    VCHECK(cudaMemcpyAsync(pcm_host_, pcm_, need * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    advance(m, ids, 1);
}

int Vocoder::stream_decode(const int * frames, int n_frames, float * out_pcm) {
    std::lock_guard<std::mutex> lk(mu_);
    decode(frames, n_frames, out_pcm);
    return n_frames * kSamplesPerFrame;
}

int Vocoder::stream_decode_batch(int batch, const int * flat_tokens, const int * token_offsets, const int * n_frames,
                                 float * flat_pcm, const int * pcm_offsets, int * out_n_samples) {
    std::lock_guard<std::mutex> lk(mu_);
    const int nc = cfg_.nc, spf = kSamplesPerFrame;
    std::map<int, std::vector<int>> groups;  // frames -> entries, decoded as segments of one batch
    std::vector<int> toks(batch), poffs(batch), nfs(batch);
    int running_tok = 0, running_pcm = 0;
    for (int b = 0; b < batch; b++) {
        nfs[b] = std::max(0, n_frames[b]);
        toks[b] = token_offsets ? token_offsets[b] : running_tok;
        poffs[b] = pcm_offsets ? pcm_offsets[b] : running_pcm;
        if (nfs[b] > 0) groups[nfs[b]].push_back(b);
        if (out_n_samples) out_n_samples[b] = nfs[b] * spf;
        running_tok += nfs[b] * nc;
        running_pcm += nfs[b] * spf;
    }
    std::vector<int> hc;
    std::vector<float> audio;
    for (const auto & kv : groups) {
        const int T = kv.first, S = (int) kv.second.size();
        hc.resize((size_t) S * T * nc);
        for (int i = 0; i < S; i++)
            std::memcpy(hc.data() + (size_t) i * T * nc, flat_tokens + toks[kv.second[i]], (size_t) T * nc * sizeof(int));
        ensure(S * T);
        VCHECK(cudaMemcpyAsync(codes_, hc.data(), hc.size() * sizeof(int), cudaMemcpyHostToDevice, stream_));
        decode_segments(codes_, nc, S, T, nullptr, pcm_);
        audio.resize((size_t) S * T * spf);
        VCHECK(cudaMemcpyAsync(audio.data(), pcm_, audio.size() * sizeof(float), cudaMemcpyDeviceToHost, stream_));
        check_device_error();
        for (int i = 0; i < S; i++)
            std::memcpy(flat_pcm + poffs[kv.second[i]], audio.data() + (size_t) i * T * spf, (size_t) T * spf * sizeof(float));
    }
    return batch;
}

}  // namespace bzb

// ================================================================================= codec encoder
namespace bzb {

namespace {

constexpr int kRvqThreads = 256;  // codebook entries per distance block

// squared distances of frame f's vector to codebook entries [256 chunk, 256 chunk + 256) in f32,
// summed over the dimension in order with separately rounded products (as src/codec.cpp:61-74
// computes them), then the chunk's first minimum
__global__ void __launch_bounds__(kRvqThreads) rvq_dist_kernel(const float * vec, int dim, const float * bookT, int n,
                                                              float * dmin, int * imin, int chunks) {
    extern __shared__ float sv[];
    __shared__ float bd[kRvqThreads / 32];
    __shared__ int bi[kRvqThreads / 32];
    const int f = blockIdx.x, chunk = blockIdx.y;
    for (int k = threadIdx.x; k < dim; k += blockDim.x) sv[k] = vec[(size_t) f * dim + k];
    __syncthreads();
    const int c = chunk * kRvqThreads + threadIdx.x;
    float d = INFINITY;
    int idx = INT_MAX;
    if (c < n) {
        d = 0.0f;
        for (int k = 0; k < dim; k++) {
            const float diff = __fsub_rn(sv[k], __ldg(bookT + (size_t) k * n + c));
            d = __fadd_rn(d, __fmul_rn(diff, diff));
        }
        idx = c;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float od = __shfl_xor_sync(0xffffffffu, d, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (od < d || (od == d && oi < idx)) { d = od; idx = oi; }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { bd[warp] = d; bi[warp] = idx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kRvqThreads / 32; w++)
            if (bd[w] < bd[0] || (bd[w] == bd[0] && bi[w] < bi[0])) { bd[0] = bd[w]; bi[0] = bi[w]; }
        dmin[(size_t) f * chunks + chunk] = bd[0];
        imin[(size_t) f * chunks + chunk] = bi[0];
    }
}

// the first minimum over the chunks becomes the frame's code in column `col`; with `update` the
// chosen entry is subtracted from the residual (the next acoustic stage's input)
__global__ void rvq_pick_kernel(float * res, int dim, const float * bookT, int n, const float * dmin, const int * imin,
                                int chunks, int * codes, int ld_codes, int col, int update) {
    __shared__ int sc;
    const int f = blockIdx.x;
    if (threadIdx.x == 0) {
        float b = dmin[(size_t) f * chunks];
        int bix = imin[(size_t) f * chunks];
        for (int c = 1; c < chunks; c++)
            if (dmin[(size_t) f * chunks + c] < b) { b = dmin[(size_t) f * chunks + c]; bix = imin[(size_t) f * chunks + c]; }
        if (bix == INT_MAX) bix = 0;
        sc = bix;
        codes[(size_t) f * ld_codes + col] = bix;
    }
    __syncthreads();
    if (!update) return;
    for (int k = threadIdx.x; k < dim; k += blockDim.x)
        res[(size_t) f * dim + k] = __fsub_rn(res[(size_t) f * dim + k], __ldg(bookT + (size_t) k * n + sc));
}

}  // namespace

#define ECHECK(x) VCHECK(x)

const GgufTensor & CodecEncoder::need(const std::string & name) const {
    const GgufTensor * t = gg_.find(name);
    if (!t) throw std::runtime_error("codec encoder: tensor " + name + " missing from the GGUF");
    return *t;
}

float * CodecEncoder::upload(const std::vector<float> & h) {
    void * p = nullptr;
    ECHECK(cudaMalloc(&p, std::max<size_t>(h.size(), 1) * sizeof(float)));
    allocs_.push_back(p);
    ECHECK(cudaMemcpyAsync(p, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice, stream_));
    return (float *) p;
}

float * CodecEncoder::load_f32(const std::string & name, int64_t expect) {
    const GgufTensor & t = need(name);
    if (t.type != GT_F32 || (expect >= 0 && t.nelem() != expect))
        throw std::runtime_error("codec encoder: " + name + " must be F32 with " + std::to_string(expect) + " elements");
    const float * src = reinterpret_cast<const float *>(gg_.data(t));
    return upload(std::vector<float>(src, src + t.nelem()));
}

QMat CodecEncoder::load_lin(const std::string & name) {
    const GgufTensor & t = need(name);
    if (t.type != GT_Q8_0 && t.type != GT_Q4_K) throw std::runtime_error("codec encoder: " + name + " must be Q8_0 or Q4_K");
    const int K = (int) t.ne[0], M = (int) t.rows();
    QMat q;
    q.M = M; q.K = K; q.KB = K / 32; q.MT = (M + 15) / 16;
    uint8_t * raw = nullptr;
    ECHECK(cudaMalloc(&raw, t.nbytes));
    ECHECK(cudaMemcpyAsync(raw, gg_.data(t), t.nbytes, cudaMemcpyHostToDevice, stream_));
    auto dal = [&](size_t bytes) { void * p = nullptr; ECHECK(cudaMalloc(&p, bytes)); allocs_.push_back(p); return p; };
    if (t.type == GT_Q4_K) {
        if (K % 256) throw std::runtime_error("codec encoder: " + name + " is Q4_K with rows not a multiple of 256");
        UMat u;
        u.M = M; u.MT = (M + 127) / 128; u.K = K; u.KC = K / 64; u.q4 = 1;
        uint8_t * ub = (uint8_t *) dal((size_t) u.MT * u.KC * kUChunkBytesQ4);
        repack_umma_q4k(raw, M, K, ub, stream_);
        u.blk = ub;
        q.u = u;
    } else {
        q.qs = (uint4 *) dal((size_t) q.MT * q.KB * 32 * sizeof(uint4));
        q.ds = (half2 *) dal((size_t) q.MT * q.KB * 8 * sizeof(half2));
        repack_q8(raw, M, K, const_cast<uint4 *>(q.qs), const_cast<half2 *>(q.ds), stream_);
    }
    ECHECK(cudaStreamSynchronize(stream_));
    cudaFree(raw);
    return q;
}

// [Cout][Cin][K] (ggml [K, Cin, Cout]) with stride s -> tap-major polyphase [Cout][taps][Cin * s]:
// output t reads x[i][s t + k - pad], pad = K - s; with k - pad = s m + r (0 <= r < s) that is phase
// channel i*s + r at step t + m, tap taps-1+m
CodecEncoder::Conv CodecEncoder::load_conv(const std::string & name, int cin, int cout, int stride, bool bias) {
    const GgufTensor & t = need(name + ".weight");
    if (t.type != GT_F32 || t.ne.size() != 3 || t.ne[1] != cin || t.ne[2] != cout)
        throw std::runtime_error("codec encoder: unexpected shape or type of " + name + ".weight");
    const int K = (int) t.ne[0], s = stride;
    if (K < s) throw std::runtime_error("codec encoder: " + name + " has a kernel shorter than its stride");
    Conv c;
    c.cin = cin; c.cout = cout; c.stride = s;
    c.taps = (K + s - 1) / s;
    const int pad = K - s;
    const float * src = reinterpret_cast<const float *>(gg_.data(t));
    std::vector<float> h((size_t) cout * c.taps * cin * s, 0.0f);
    for (int o = 0; o < cout; o++)
        for (int i = 0; i < cin; i++)
            for (int k = 0; k < K; k++) {
                const int rel = k - pad;
                const int m = rel >= 0 ? rel / s : -((-rel + s - 1) / s);
                const int r = rel - m * s, kk = m + c.taps - 1;
                h[((size_t) o * c.taps + kk) * cin * s + (size_t) i * s + r] = src[((size_t) o * cin + i) * K + k];
            }
    c.w = upload(h);
    if (bias) c.b = load_f32(name + ".bias", cout);
    return c;
}

CodecEncoder::CodecEncoder(const GgufFile & gg, const ModelConfig & cfg, int device)
    : gg_(gg), cfg_(cfg), ec_(cfg.enc), device_(device) {
    ECHECK(cudaSetDevice(device));
    ECHECK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    init_kernel_attributes();
    init_umma_attributes();
    const std::vector<int> & rt = ec_.ratios;
    if (rt.size() != 4) throw std::runtime_error("codec encoder: four SEANet ratios expected");
    if (rt[0] * rt[1] * rt[2] * rt[3] * 2 != kSamplesPerFrame) throw std::runtime_error("codec encoder: the ratios do not give 1920 samples per frame");
    const int nf = ec_.nf;
    c0_ = load_conv("codec.enc.0.conv", 1, nf, 1, true);
    const int res_idx[4] = { 1, 4, 7, 10 }, conv_idx[4] = { 3, 6, 9, 12 };
    int ch = nf;
    for (int st = 0; st < 4; st++) {
        const std::string rb = "codec.enc." + std::to_string(res_idx[st]);
        res1_[st] = load_conv(rb + ".block.1.conv", ch, ch / 2, 1, true);
        res3_[st] = load_conv(rb + ".block.3.conv", ch / 2, ch, 1, true);
        strided_[st] = load_conv("codec.enc." + std::to_string(conv_idx[st]) + ".conv", ch, 2 * ch, rt[3 - st], true);
        ch *= 2;
    }
    c14_ = load_conv("codec.enc.14.conv", ch, ec_.hidden, 1, true);
    const int H = ec_.hidden;
    if (ec_.n_head * ec_.hd != H || ec_.hd > 128 || ec_.hd % 32) throw std::runtime_error("codec encoder: unsupported attention shape");
    for (int l = 0; l < ec_.n_layer; l++) {
        const std::string p = "codec.enct.blk." + std::to_string(l);
        Layer L;
        L.an_w = load_f32(p + ".attn_norm.weight", H);
        L.an_b = load_f32(p + ".attn_norm.bias", H);
        L.q = load_lin(p + ".attn_q.weight");
        L.k = load_lin(p + ".attn_k.weight");
        L.v = load_lin(p + ".attn_v.weight");
        L.o = load_lin(p + ".attn_output.weight");
        L.attn_scale = load_f32(p + ".attn_scale", H);
        L.fn_w = load_f32(p + ".ffn_norm.weight", H);
        L.fn_b = load_f32(p + ".ffn_norm.bias", H);
        L.up = load_lin(p + ".ffn_up.weight");
        L.down = load_lin(p + ".ffn_down.weight");
        L.ffn_scale = load_f32(p + ".ffn_scale", H);
        layers_.push_back(L);
    }
    down_ = load_conv("codec.downsample.conv", H, H, 2, false);
    sq_in_ = load_lin("codec.sq.in_proj.weight");
    aq_in_ = load_lin("codec.aq.in_proj.weight");
    if (sq_in_.M != ec_.dim || aq_in_.M != ec_.dim) throw std::runtime_error("codec encoder: quantiser projections do not match codebook_dim");
    // codebooks, transposed to [dim][entries] so that a distance block reads them coalesced
    const int nc = cfg_.nc, n_ac = nc - ec_.n_sem;
    if (ec_.n_sem != 1 || n_ac < 0) throw std::runtime_error("codec encoder: one semantic codebook expected");
    const GgufTensor & b0 = need("codec.sq.0.embed");
    book_n_ = (int) b0.ne[1];
    std::vector<float> books((size_t) nc * ec_.dim * book_n_);
    for (int bi = 0; bi < nc; bi++) {
        const GgufTensor & t = need(bi == 0 ? std::string("codec.sq.0.embed") : "codec.aq." + std::to_string(bi - 1) + ".embed");
        if (t.type != GT_F32 || t.ne[0] != ec_.dim || t.ne[1] != book_n_) throw std::runtime_error("codec encoder: codebook " + t.name + " has an unexpected shape");
        const float * src = reinterpret_cast<const float *>(gg_.data(t));
        float * dst = books.data() + (size_t) bi * ec_.dim * book_n_;
        for (int e = 0; e < book_n_; e++)
            for (int k = 0; k < ec_.dim; k++) dst[(size_t) k * book_n_ + e] = src[(size_t) e * ec_.dim + k];
    }
    books_ = upload(books);
    {
        void * p = nullptr;
        scr_.ws_elems = (size_t) 1 << 20;
        ECHECK(cudaMalloc(&p, scr_.ws_elems * sizeof(float4)));
        allocs_.push_back(p);
        scr_.ws = (float4 *) p;
        scr_.n_counters = 4096;
        ECHECK(cudaMalloc(&p, scr_.n_counters * sizeof(int)));
        allocs_.push_back(p);
        scr_.counters = (int *) p;
        ECHECK(cudaMemsetAsync(scr_.counters, 0, scr_.n_counters * sizeof(int), stream_));
        ECHECK(cudaMalloc(&p, sizeof(int)));
        allocs_.push_back(p);
        err_ = (int *) p;
        ECHECK(cudaMemsetAsync(err_, 0, sizeof(int), stream_));
    }
    // widest conv window: dynamic shared memory of the conv kernel
    int lxp = conv_lxp(c0_.taps, 1);
    for (int st = 0; st < 4; st++)
        lxp = std::max({ lxp, conv_lxp(res1_[st].taps, 1), conv_lxp(res3_[st].taps, 1), conv_lxp(strided_[st].taps, 1) });
    lxp = std::max({ lxp, conv_lxp(c14_.taps, 1), conv_lxp(down_.taps, 1) });
    raise_conv_smem_limit(conv_smem_bytes(lxp));
    ECHECK(cudaStreamSynchronize(stream_));  // the uploads above are ordered on stream_
}

CodecEncoder::~CodecEncoder() {
    cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    for (void * p : scratch_) cudaFree(p);
    for (void * p : allocs_) cudaFree(p);
    if (stream_) cudaStreamDestroy(stream_);
}

void CodecEncoder::ensure(int L) {
    if (L <= lcap_) return;
    ECHECK(cudaStreamSynchronize(stream_));
    for (void * p : scratch_) cudaFree(p);
    scratch_.clear();
    lcap_ = std::max(L, 64 * kSamplesPerFrame);
    const size_t Lc = (size_t) lcap_;
    act_ = std::max((size_t) ec_.nf * Lc, (size_t) 1024);
    const size_t T1 = Lc / (kSamplesPerFrame / 2) + 1, T2 = Lc / kSamplesPerFrame + 1;
    const size_t wide = (size_t) std::max({ ec_.hidden, ec_.ffn, ec_.dim });
    auto fa = [&](size_t n) { void * p = nullptr; ECHECK(cudaMalloc(&p, std::max<size_t>(n, 16) * 4)); scratch_.push_back(p); return (float *) p; };
    auto ha = [&](size_t n) { void * p = nullptr; ECHECK(cudaMalloc(&p, std::max<size_t>(n, 16) * 2)); scratch_.push_back(p); return (half *) p; };
    X_ = fa(act_); E_ = fa(act_); H_ = fa(act_); part_ = fa(2 * act_);
    t32_ = fa(T1 * wide); q_ = fa(T1 * wide); k_ = fa(T1 * wide); v_ = fa(T1 * wide); o_ = fa(T1 * wide); res_ = fa(T1 * wide);
    t16_ = ha(T1 * wide); att16_ = ha(T1 * wide); f16_ = ha(T1 * wide);
    const int chunks = (book_n_ + kRvqThreads - 1) / kRvqThreads;
    dpart_ = fa(T2 * chunks);
    ipart_ = (int *) fa(T2 * chunks);
    codes_ = (int *) fa(T2 * cfg_.nc);
    if (rope_max_ < (int) T1) {
        const std::vector<float2> tab = rope_table((int) T1, ec_.hd, ec_.theta, 1.0f, nullptr);
        void * p = nullptr;
        ECHECK(cudaMalloc(&p, tab.size() * sizeof(float2)));
        scratch_.push_back(p);
        ECHECK(cudaMemcpyAsync(p, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice, stream_));
        rope_ = (float2 *) p;
        rope_max_ = (int) T1;
    }
}

void CodecEncoder::conv(const Conv & c, const float * x, int Lin, float * y, bool elu_out, const float * res, float * y2,
                        bool elu2, cudaStream_t s) {
    ConvArgs ca;
    ca.x = x; ca.cin = c.cin * c.stride; ca.L = Lin / c.stride; ca.istride = c.stride; ca.Lin = Lin;
    ca.w = c.w; ca.taps = c.taps; ca.dil = 1;
    ca.bias = c.b; ca.cout = c.cout;
    ca.y = y; ca.ldy = ca.L; ca.ostride = 1;
    ca.res = res;
    ca.elu1 = elu_out ? 1 : 0;
    ca.y2 = y2; ca.elu2 = elu2 ? 1 : 0;
    launch_conv(ca, 1, part_, 2 * act_, s);
}

int CodecEncoder::encode(const float * pcm, int n, std::vector<int> & codes) {
    std::lock_guard<std::mutex> lk(mu_);
    const int T = n / kSamplesPerFrame;
    codes.assign((size_t) std::max(T, 0) * cfg_.nc, 0);
    if (T <= 0) return 0;
    ECHECK(cudaSetDevice(device_));
    int L = T * kSamplesPerFrame;
    ensure(L);
    cudaStream_t s = stream_;
    // the PCM goes in as a [1][L] input row
    ECHECK(cudaMemcpyAsync(H_, pcm, (size_t) L * sizeof(float), cudaMemcpyHostToDevice, s));
    float * X = X_, * E = E_, * Hb = H_;
    // SEANet (src/codec_conv.cpp:60-77): X the stage's residual stream, E = ELU(X) (the next
    // conv's input), Hb the residual block's middle activation
    conv(c0_, Hb, L, X, false, nullptr, E, true, s);
    for (int st = 0; st < 4; st++) {
        conv(res1_[st], E, L, Hb, true, nullptr, nullptr, false, s);     // ELU(conv(ELU(x)))
        conv(res3_[st], Hb, L, X, false, X, E, true, s);                 // x += conv(...); E = ELU(x)
        conv(strided_[st], E, L, X, false, nullptr, Hb, true, s);        // strided conv of ELU(x)
        L /= strided_[st].stride;
        std::swap(E, Hb);
    }
    conv(c14_, E, L, Hb, false, nullptr, nullptr, false, s);             // [hidden][T1]
    const int T1 = L, H = ec_.hidden, nh = ec_.n_head, hd = ec_.hd, F = ec_.ffn;
    auto transpose = [&](const float * in, int R, int C, float * out) {
        voc_transpose_kernel<<<dim3((C + 31) / 32, (R + 31) / 32), dim3(32, 8), 0, s>>>(in, R, C, out, nullptr);
    };
    auto lin = [&](const QMat & w, const half * x16, int ldx, int rows, const GemvOut & out) {
        if (w.qs) launch_gemv(w, x16, ldx, rows, out, scr_, s);
        else launch_umma_gemm(w.u, x16, ldx, rows, out, err_, s, false);
    };
    // Mimi encoder transformer (src/codec_transformer.cpp:9-45) on [T1][hidden] rows
    transpose(Hb, H, T1, t32_);
    const float scale = 1.0f / std::sqrt((float) hd);
    for (const Layer & Ly : layers_) {
        voc_layernorm_kernel<<<T1, 256, 0, s>>>(t32_, H, Ly.an_w, Ly.an_b, ec_.eps, t16_);
        lin(Ly.q, t16_, H, T1, GemvOut{ EPI_STORE, q_, nullptr, H });
        lin(Ly.k, t16_, H, T1, GemvOut{ EPI_STORE, k_, nullptr, H });
        lin(Ly.v, t16_, H, T1, GemvOut{ EPI_STORE, v_, nullptr, H });
        const int warps = T1 * nh;
        voc_attn_kernel<<<(warps * 32 + 127) / 128, 128, 0, s>>>(q_, k_, v_, T1, nh, nh, hd, ec_.window, rope_, scale, att16_);
        lin(Ly.o, att16_, H, T1, GemvOut{ EPI_STORE, o_, nullptr, H });
        voc_scaled_add_kernel<<<grid_for((size_t) T1 * H), 256, 0, s>>>(t32_, o_, (size_t) T1 * H, H, Ly.attn_scale);
        voc_layernorm_kernel<<<T1, 256, 0, s>>>(t32_, H, Ly.fn_w, Ly.fn_b, ec_.eps, t16_);
        lin(Ly.up, t16_, H, T1, GemvOut{ EPI_STORE, o_, nullptr, F });
        voc_bias_gelu_kernel<<<grid_for((size_t) T1 * F), 256, 0, s>>>(o_, (size_t) T1 * F, F, nullptr, f16_);
        lin(Ly.down, f16_, F, T1, GemvOut{ EPI_STORE, res_, nullptr, H });
        voc_scaled_add_kernel<<<grid_for((size_t) T1 * H), 256, 0, s>>>(t32_, res_, (size_t) T1 * H, H, Ly.ffn_scale);
    }
    // stride-2 downsample, then the quantiser projections on [T2][hidden] rows
    transpose(t32_, T1, H, X);                                           // [hidden][T1]
    conv(down_, X, T1, E, false, nullptr, nullptr, false, s);            // [hidden][T2]
    const int T2 = T1 / 2;
    transpose(E, H, T2, t32_);
    voc_to_f16_kernel<<<grid_for((size_t) T2 * H), 256, 0, s>>>(t32_, (size_t) T2 * H, t16_);
    const int dim = ec_.dim;
    lin(sq_in_, t16_, H, T2, GemvOut{ EPI_STORE, q_, nullptr, dim });   // semantic input
    lin(aq_in_, t16_, H, T2, GemvOut{ EPI_STORE, k_, nullptr, dim });   // acoustic residual
    // nearest codebook entries (src/codec.cpp:104-120)
    const int nc = cfg_.nc, chunks = (book_n_ + kRvqThreads - 1) / kRvqThreads;
    const size_t book_stride = (size_t) dim * book_n_;
    for (int bi = 0; bi < nc; bi++) {
        const float * vec = bi == 0 ? q_ : k_;
        rvq_dist_kernel<<<dim3(T2, chunks), kRvqThreads, dim * sizeof(float), s>>>(vec, dim, books_ + bi * book_stride, book_n_,
                                                                                   dpart_, ipart_, chunks);
        rvq_pick_kernel<<<T2, 128, 0, s>>>(k_, dim, books_ + bi * book_stride, book_n_, dpart_, ipart_, chunks, codes_, nc, bi,
                                           bi > 0 ? 1 : 0);
    }
    ECHECK(cudaGetLastError());
    codes.assign((size_t) T2 * nc, 0);
    ECHECK(cudaMemcpyAsync(codes.data(), codes_, codes.size() * sizeof(int), cudaMemcpyDeviceToHost, s));
    int err = 0;
    ECHECK(cudaMemcpyAsync(&err, err_, sizeof(int), cudaMemcpyDeviceToHost, s));
    ECHECK(cudaStreamSynchronize(s));
    if (err) throw std::runtime_error("codec encoder: a bounded wait timed out in the tcgen05 GEMM");
    return T2;
}

}  // namespace bzb
