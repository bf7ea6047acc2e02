// Device helpers shared by the NVFP4 MoE kernels (sm_100a only).
//
// NVFP4 storage follows the lab's checkpoint-native layout
// (native_nvfp4/kernels/nvfp4_gemv.cl:10-27,74-75):
//   * packed   : row-major bytes, byte b of a row holds column 2b in its low
//                nibble and column 2b+1 in its high nibble, E2M1 code
//                {0,.5,1,1.5,2,3,4,6} with bit 3 the sign;
//   * scales   : one E4M3 byte per 16 consecutive columns of a row;
//   * global   : one FP32 divisor per projection (the kernel multiplies by
//                its inverse).
// Scale bytes in a bank are sanitised at upload (sign cleared, 0x7F -> 0) so
// the hardware E4M3 conversion reproduces the lab's decoding rule exactly.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "the NVFP4 MoE kernels target sm_100a only"
#endif

namespace nvfp4 {

// One 32-bit word of packed E2M1 (8 columns) -> four f16x2 words; word j
// holds columns 2j (low half) and 2j+1 (high half). Exact conversion.
__device__ __forceinline__ void e2m1x8_to_f16x8(uint32_t w, uint32_t (&h)[4]) {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
        : "r"(w));
}

// Two sanitised E4M3 scale bytes (low byte first) -> f16x2. Exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t s) {
    uint32_t r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(s));
    return r;
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// Broadcast the low / high f16 of a f16x2 into both halves.
__device__ __forceinline__ uint32_t f16x2_lo_lo(uint32_t v) {
    return __byte_perm(v, v, 0x1010);
}
__device__ __forceinline__ uint32_t f16x2_hi_hi(uint32_t v) {
    return __byte_perm(v, v, 0x3232);
}

// D += A(16x16, row) * B(16x8, col), f16 inputs, f32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                          uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Streaming 128-bit load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ldg_stream128(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint16_t ldg_u16(const void *p) {
    return __ldg(reinterpret_cast<const unsigned short *>(p));
}

__device__ __forceinline__ uint4 ldcg128(const void *p) {
    return __ldcg(reinterpret_cast<const uint4 *>(p));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits16) {
    return __uint_as_float(bits16 << 16);
}

// Packed FP32 pairs (sm_100a f32x2 arithmetic): element lo in the low word.
// Each element is rounded to nearest even exactly as add.rn.f32 / mul.rn.f32
// round it (subnormals kept), so a pair of independent chains gives the same
// bits as two scalar chains.
__device__ __forceinline__ unsigned long long f32x2_pack(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}

__device__ __forceinline__ void f32x2_unpack(unsigned long long v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

__device__ __forceinline__ unsigned long long f32x2_mul_rn(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ unsigned long long f32x2_add_rn(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// Round-to-nearest-even FP32 -> BF16 bits (finite inputs; NaN stays NaN).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float v) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// Top-k comparison used by routing: larger value wins, lower id on ties.
__device__ __forceinline__ bool route_better(float v, int id, float bv, int bid) {
    return v > bv || (v == bv && id < bid);
}

// Byte offset of column k of token row j inside a swizzled f16 activation
// tile. k = q*128 + 32*c + 8*v + e (q chunk, c lane quarter, v 16-byte slot,
// e element). The slot index is XORed with (c >> 1) and the token stride is
// 32 mod 128 bytes so that the LDS.128 of one MMA B-fragment load (8 lanes
// per phase: two tokens x four quarters) touches eight distinct 16-byte bank
// groups.
__host__ __device__ __forceinline__ int act_tile_stride_bytes(int k_cols) {
    int base = 2 * k_cols;
    return base + ((32 - (base % 128)) + 128) % 128;
}

__device__ __forceinline__ int act_tile_offset(int token_stride, int j, int q, int c,
                                               int v) {
    return j * token_stride + q * 256 + c * 64 + ((v ^ (c >> 1)) << 4);
}

}  // namespace nvfp4
