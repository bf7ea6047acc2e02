// tcgen05 (5th-generation tensor core) helpers for sm_100a kernels: tensor
// memory allocation, shared-memory matrix descriptors, the block-scaled
// NVFP4 MMA (kind::mxf4nvf4, E2M1 x E2M1 with E4M3 scales per 16 elements),
// scale-factor copies into tensor memory, commits to mbarriers and
// tensor-memory loads and stores. Every helper but st_sf_atoms issues exactly
// one PTX instruction; the caller owns ordering (fences) and elected-thread
// rules.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace nvfp4 {
namespace tc {

// ---------------------------------------------------------------- TMEM

// Allocate `ncols` tensor-memory columns (a power of two >= 32); the base
// address is written to shared memory at `slot`. Executed by one full warp.
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(slot))),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Order this thread's generic-proxy shared-memory accesses before later
// async-proxy (TMA, tcgen05) accesses of the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------- smem descriptors

// K-major operand tile in shared memory with the 128-byte swizzle: rows of
// 128 bytes, 8-row atoms 1024 bytes apart (stride byte offset), the tile
// base 1024-byte aligned. `addr` is the shared-memory byte address of the
// first row's first 16-byte unit of the K slice (advance by 32 bytes per
// 64 FP4 elements inside the 128-byte row).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);           // start address, bits [0,14)
    d |= static_cast<uint64_t>(1u) << 16;                        // leading byte offset (unused for SW128 K-major)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;                // stride byte offset, bits [32,46)
    d |= static_cast<uint64_t>(1u) << 46;                        // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2u) << 61;                        // layout: 128-byte swizzle
    return d;
}

// Scale-factor atom source for tcgen05.cp 32x128b: 32 rows of 16 bytes,
// no swizzle, 8-row core matrices 128 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sf(uint32_t addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(128u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    return d;
}

// Instruction descriptor of kind::mxf4nvf4 with E2M1 A and B, E4M3 scale
// factors, FP32 accumulation, both operands K-major, M = 128 and N = `n`.
__host__ __device__ constexpr uint32_t idesc_mxf4nvf4(uint32_t n) {
    return (1u << 7)              // A format: E2M1
           | (1u << 10)           // B format: E2M1
           | ((n >> 3) << 17)     // N / 8
           | (0u << 23)           // scale format: UE4M3
           | ((128u >> 4) << 24); // M / 16
}

// Instruction descriptor of kind::f16 with BF16 A and B, FP32 accumulation,
// both operands K-major, M = 128 and N = `n`.
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t n) {
    return (1u << 4)              // D format: F32
           | (1u << 7)            // A format: BF16
           | (1u << 10)           // B format: BF16
           | ((n >> 3) << 17)     // N / 8
           | ((128u >> 4) << 24); // M / 16
}

// D[tmem d] (+)= A[smem a] * B[smem b]^T, BF16 operands (K 16 per instruction).
__device__ __forceinline__ void mma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem d] (+)= A[smem a] * B[smem b]^T with per-16 block scales read from
// tensor memory at `sfa` and `sfb`. Issued by one thread.
__device__ __forceinline__ void mma_mxf4nvf4(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                             uint32_t sfb, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
        : "memory");
}

// Copy one 512-byte scale-factor atom (32 rows x 16 bytes) from shared
// memory into 4 tensor-memory columns, replicated to all four 32-lane
// sub-partitions. Issued by one thread.
__device__ __forceinline__ void cp_sf_atom(uint32_t tmem_col_addr, uint64_t src_desc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem_col_addr), "l"(src_desc) : "memory");
}

// Arrive once on `bar` when every tcgen05 operation this thread issued so
// far has completed.
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (32 * (warp % 4) + t) of columns [col, col + 32).
__device__ __forceinline__ void ld_32x32b_x32(uint32_t addr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(addr));
}

// Four consecutive accumulator columns of the warp's 32 lanes.
__device__ __forceinline__ void ld_32x32b_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Store 32 consecutive 32-bit columns of the warp's 32 lanes (register c to
// column c of the address).
__device__ __forceinline__ void st_32x32b_x32(uint32_t addr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        :
        : "r"(addr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void st_32x32b_x16(uint32_t addr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        :
        : "r"(addr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Scale-factor atoms of 32 rows x 16 bytes, `n` of them from shared memory
// at `src` (atom a at src + a * stride), written by one warp into its lane
// quarter as the layout tcgen05.cp .32x128b.warpx4 gives: lane r, columns
// 4a..4a+3 = bytes r*16 .. r*16+15 of atom a (every lane quarter holds the
// same 32 rows). `taddr` carries the warp's lane quarter in bits 16+.
// kPairs (N == 8): the source holds two runs of four atoms (P then Q) and
// the columns receive them interleaved, P0 Q0 P1 Q1 ..., which is the
// scale-factor layout of one 256-row operand made of a P row block and a Q
// row block (row r's scales in column r / 32 of each 64-wide K step).
template <int N, bool kPairs = false>
__device__ __forceinline__ void st_sf_atoms(uint32_t taddr, const uint8_t *src, int stride, int lane) {
    static_assert(N == 4 || N == 8, "one 16- or 32-column store");
    static_assert(!kPairs || N == 8, "pairs interleave two runs of four");
    uint32_t r[4 * N];
#pragma unroll
    for (int a = 0; a < N; ++a) {
        const int from = kPairs ? (a & 1) * 4 + (a >> 1) : a;
        uint4 v;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(src + from * stride + lane * 16))));
        r[4 * a] = v.x;
        r[4 * a + 1] = v.y;
        r[4 * a + 2] = v.z;
        r[4 * a + 3] = v.w;
    }
    if constexpr (N == 8)
        st_32x32b_x32(taddr, r);
    else
        st_32x32b_x16(taddr, r);
}

}  // namespace tc
}  // namespace nvfp4
