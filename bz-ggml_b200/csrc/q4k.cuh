// Q4_K super-block decoding (the GGUF block format: 256 values in 144 bytes). The layout:
// f16 d, f16 dmin, 12 bytes of packed 6-bit scales and mins for eight 32-value sub-blocks,
// then 128 bytes of 4-bit values. Sub-block s covers values 32s..32s+31. Its values sit in the
// low nibbles (s even) or high nibbles (s odd) of bytes 32(s/2)..32(s/2)+31, and
// value = d * scale_s * q - dmin * min_s.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace bzb {

constexpr int kQ4KBlockBytes = 144;
constexpr int kQ4KBlockValues = 256;

// the 6-bit scale and min of sub-block s: the first four sit in the low 6 bits of bytes 0-3
// (scales) and 4-7 (mins); the last four take their low 4 bits from bytes 8-11 and their top 2
// bits from the spare high bits of bytes 0-3 (scales) and 4-7 (mins)
__device__ __forceinline__ void q4k_scale_min(const uint8_t * packed, int s, int & scale, int & mn) {
    if (s < 4) {
        scale = packed[s] & 63;
        mn = packed[s + 4] & 63;
    } else {
        scale = (packed[s + 4] & 0x0F) | ((packed[s - 4] >> 6) << 4);
        mn = (packed[s + 4] >> 4) | ((packed[s] >> 6) << 4);
    }
}

// sub-block s of the super-block at blk as stored: the f16 bits of d and dmin, the 6-bit scale
// and min, and its 32 values q (0..15)
__device__ __forceinline__ void q4k_sub_block_raw(const uint8_t * blk, int s, uint16_t & d, uint16_t & dmin,
                                                  int & scale, int & mn, uint8_t q[32]) {
    d = (uint16_t) (blk[0] | (blk[1] << 8));
    dmin = (uint16_t) (blk[2] | (blk[3] << 8));
    q4k_scale_min(blk + 4, s, scale, mn);
    const uint8_t * qs = blk + 16 + 32 * (s >> 1);
    const int shift = (s & 1) * 4;
#pragma unroll
    for (int i = 0; i < 32; i++) q[i] = (uint8_t) ((qs[i] >> shift) & 0x0F);
}

// sub-block s of the super-block at blk: its f16 scale a = d * scale, min b = dmin * min (f32
// products rounded once to f16) and its 32 values q (0..15)
__device__ __forceinline__ void q4k_sub_block(const uint8_t * blk, int s, half & a, half & b, uint8_t q[32]) {
    uint16_t d = 0, dmin = 0;
    int scale = 0, mn = 0;
    q4k_sub_block_raw(blk, s, d, dmin, scale, mn, q);
    a = __float2half_rn(__half2float(__ushort_as_half(d)) * (float) scale);
    b = __float2half_rn(__half2float(__ushort_as_half(dmin)) * (float) mn);
}

// the f32 scale and min of sub-block hb (0 or 1) from a tcgen05 chunk's 8 bytes of row data
// (f16 d, f16 dmin, u8 scales[2], u8 mins[2]): products of an f16 and a 6-bit integer, exact in f32
__device__ __forceinline__ void q4k_chunk_scale_min(uint2 meta, int hb, float & a, float & b) {
    a = __half2float(__ushort_as_half((unsigned short) (meta.x & 0xFFFFu))) * (float) ((meta.y >> (8 * hb)) & 0xFFu);
    b = __half2float(__ushort_as_half((unsigned short) (meta.x >> 16))) * (float) ((meta.y >> (16 + 8 * hb)) & 0xFFu);
}

}  // namespace bzb
