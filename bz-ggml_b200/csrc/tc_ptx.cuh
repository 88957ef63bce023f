// Inline PTX for the sm_100a tensor-core pipeline: mbarriers, bulk and tensor (TMA) copies,
// TMEM allocation and loads, tcgen05.mma with shared-memory descriptors, and the Q8_0 int8 ->
// f16 conversion the dequantising producers use. Shared by the dequant-GEMM and the persistent
// depth-decoder kernel.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace bzb {
namespace tc {

constexpr long long kSpinLimit = 1ll << 22;

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void * p) { return (uint32_t) __cvta_generic_to_shared(p); }

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done) : "r"(a), "r"(parity) : "memory");
    return done != 0;
}

// bounded wait for the completion of the mbarrier phase with the given parity; returns false
// when `limit` polls pass (recording error code 1) or as soon as another thread has recorded an
// error, instead of spinning forever. `backoff_ns` > 0 sleeps that long between polls after the
// first few, so that a warp with a long wait ahead leaves the issue slots to the warps doing
// the work (the MMA issuer, whose latency paces the pipeline, polls without pause)
__device__ __forceinline__ bool mbar_wait(uint64_t * bar, uint32_t parity, int * err, long long limit = kSpinLimit,
                                          unsigned backoff_ns = 0) {
    const uint32_t a = smem_u32(bar);
    for (long long i = 0; i < limit; i++) {
        if (mbar_try(a, parity)) return true;
        if ((i & 1023) == 1023 && err && *reinterpret_cast<volatile int *>(err)) return false;
        if (backoff_ns && i >= 4) __nanosleep(backoff_ns);
    }
    if (err) atomicCAS(err, 0, 1);
    return false;
}

// the wait a role uses after a failure to let the copies or MMAs it issued land before the
// CTA releases its shared memory or tensor memory: it does not give up when an error is already
// recorded, only after `limit` polls (recording error code 5)
__device__ __forceinline__ bool mbar_drain(uint64_t * bar, uint32_t parity, int * err, long long limit = kSpinLimit) {
    const uint32_t a = smem_u32(bar);
    for (long long i = 0; i < limit; i++)
        if (mbar_try(a, parity)) return true;
    if (err) atomicCAS(err, 0, 5);
    return false;
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t * slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// K-major operand in the 128-byte swizzle layout: 8-row atoms of 1024 bytes stacked along M/N
// (stride byte offset 1024), descriptor version 1, layout type SWIZZLE_128B
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    return (uint64_t) ((addr & 0x3FFFF) >> 4) | ((uint64_t) 1 << 16) | ((uint64_t) (1024 >> 4) << 32) |
           ((uint64_t) 1 << 46) | ((uint64_t) 2 << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum) : "memory");
}
// the same with A read from tensor memory: row i of the 128-row A tile in TMEM lane i, its K
// values packed two f16 to a 32-bit column (8 columns per K = 16 step)
__device__ __forceinline__ void umma_f16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accum) : "memory");
}
// 16 consecutive 32-bit columns of this thread's TMEM lane (warp-collective; a warp reaches the
// 32 lanes of its quarter, warp % 4)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
                 ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
                   "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void umma_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float * v) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 4 int8 -> two half2 in natural order, scaled
__device__ __forceinline__ void dq4(uint32_t w, half2 s, uint32_t & lo, uint32_t & hi) {
    const uint32_t u = w ^ 0x80808080u;
    uint32_t l = __byte_perm(u, 0x64646464u, 0x5140u);
    uint32_t h = __byte_perm(u, 0x64646464u, 0x7362u);
    const half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    half2 hl = __hmul2(__hsub2(*reinterpret_cast<half2 *>(&l), bias), s);
    half2 hh = __hmul2(__hsub2(*reinterpret_cast<half2 *>(&h), bias), s);
    lo = *reinterpret_cast<uint32_t *>(&hl);
    hi = *reinterpret_cast<uint32_t *>(&hh);
}

// 8 Q4_K values of one word (even values in nibbles 0-3, odd ones in nibbles 4-7) -> 4 f16 pairs
// a q - b: 0x6400 | q is the f16 1024 + q exactly and subtracting 1024 leaves q; a q - b is one
// f32 fused multiply-add (a and b are exact f32 products), rounded once to f16
__device__ __forceinline__ void dq8_nib_f32(uint32_t w, float a, float b, uint32_t o[4]) {
    const half2 k1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
#pragma unroll
    for (int k = 0; k < 4; k++) {
        uint32_t h;
        asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(h) : "r"(w >> (4 * k)), "r"(0x000F000Fu), "r"(0x64006400u));
        const float2 q = __half22float2(__hsub2(*reinterpret_cast<half2 *>(&h), k1024));
        const half2 v = __floats2half2_rn(fmaf(a, q.x, -b), fmaf(a, q.y, -b));
        o[k] = *reinterpret_cast<const uint32_t *>(&v);
    }
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float gelu_tanh_f(float x) {
    const float c = 0.7978845608028654f;
    return 0.5f * x * (1.0f + tanhf(c * x * (1.0f + 0.044715f * x * x)));
}

__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tma_2d(void * dst, const CUtensorMap * map, int x, int y, uint64_t * bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tma_3d(void * dst, const CUtensorMap * map, int x, int y, int z, uint64_t * bar) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)) : "memory");
}

}  // namespace tc
}  // namespace bzb
