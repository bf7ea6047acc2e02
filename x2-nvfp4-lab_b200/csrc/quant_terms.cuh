// Multi-term NVFP4 quantisation of activation rows (device helpers shared by
// the prefill quantiser and the decode path's tensor-core variant).
//
// A row with FP32 global scale g = amax/2688 (1 for an all-zero row) is fed
// to the block-scaled tensor cores as J NVFP4 terms: per 16-element block and
// term, s = E4M3_RN((bamax / 6) / g), denom = s * g, code =
// E2M1_RN(r * RN(1/denom)) (0 when denom is 0), then r -= code * denom, so
// term j+1 quantises what terms 1..j left over. Every operation is an
// individually rounded FP32 operation, so the result does not depend on how
// the blocks are spread over threads (the oracle's quantize_rows_split
// performs the same sequence).
#pragma once

#include "nvfp4_common.cuh"

namespace nvfp4 {

__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ uint32_t f32x2_to_e2m1x2(float lo, float hi) {
    uint16_t r;
    asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u16.u8 %0, t;\n\t}"
        : "=h"(r)
        : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float e4m3_byte_to_f32(uint32_t b) {
    const uint32_t h2 = e4m3x2_to_f16x2(static_cast<uint16_t>(b));
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFFu)));
}

// Clear the sign of zero-magnitude E2M1 codes (eight nibbles per word).
__device__ __forceinline__ uint32_t canonical_zero_codes(uint32_t w) {
    const uint32_t m = w & 0x77777777u;
    const uint32_t nz = (m | (m >> 1) | (m >> 2)) & 0x11111111u;
    return m | (w & (nz << 3));
}

// Row global scale from the row's absolute maximum.
__device__ __forceinline__ float row_global_scale(float amax) {
    return amax > 0.0f ? __fdiv_rn(amax, 2688.0f) : 1.0f;
}

// Quantise one 16-element block (v, overwritten by the residual) into the
// next term: c0 holds elements 0..7 (element 2i in the low nibble of byte i),
// c1 elements 8..15; returns the term's E4M3 scale byte.
__device__ __forceinline__ uint32_t quantize_block_term(float (&v)[16], float g, uint32_t &c0, uint32_t &c1) {
    float bamax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) bamax = fmaxf(bamax, fabsf(v[i]));
    const float target = __fdiv_rn(__fdiv_rn(bamax, 6.0f), g);
    const uint32_t sb = f32x2_to_e4m3x2(target, 0.0f) & 0xFFu;
    const float denom = __fmul_rn(e4m3_byte_to_f32(sb), g);
    const float inv = denom != 0.0f ? __frcp_rn(denom) : 0.0f;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int e0 = 8 * p + 2 * i;
            const uint32_t cc = f32x2_to_e2m1x2(__fmul_rn(v[e0], inv), __fmul_rn(v[e0 + 1], inv)) & 0xFFu;
            word |= cc << (8 * i);
        }
        word = canonical_zero_codes(word);
        if (p == 0) c0 = word; else c1 = word;
        uint32_t h[4];
        e2m1x8_to_f16x8(word, h);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 d = __half22float2(*reinterpret_cast<const __half2 *>(&h[i]));
            const int e0 = 8 * p + 2 * i;
            v[e0] = __fsub_rn(v[e0], __fmul_rn(d.x, denom));
            v[e0 + 1] = __fsub_rn(v[e0 + 1], __fmul_rn(d.y, denom));
        }
    }
    return sb;
}

// Byte offset of B row n (< 128), 16-element block b of a tcgen05
// scale-factor atom sequence [K/64][512 B].
__device__ __forceinline__ size_t sf_atom_byte(int n, int b) {
    return (size_t)(b >> 2) * 512 + (n & 31) * 16 + (n >> 5) * 4 + (b & 3);
}

}  // namespace nvfp4
