// TMA, mbarrier and tensor-map helpers for sm_100a kernels.
//
// Every wait on an mbarrier is bounded: after kSpinLimit polls the waiting
// thread records a timeout in a caller-supplied error word and gives up, so
// a kernel can never spin forever on a barrier that is not completed.
// Every copy here lands in the issuing CTA's own shared memory only.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nvfp4 {

constexpr uint32_t kSpinLimit = 1u << 26;          // polls before a drain wait gives up
constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // wall-clock bound of one wait (1 s)
constexpr int kErrWaitTimeout = 1;
// Codes recorded by a wait that gave up (kernel, barrier).
enum WaitSite : int {
    kSiteGateUpEmpty = 11,
    kSiteGateUpFull = 12,
    kSiteDownEmpty = 21,
    kSiteDownFull = 22,
    kSiteGemmEmpty = 31,
    kSiteGemmFull = 32,
    kSiteGemmAccEmpty = 33,
    kSiteGemmAccFull = 34,
    kSiteEpPeerTile = 41,   // expert-parallel combine: a peer's partial tile
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete. Gives up after
// kWaitLimitNs of wall-clock time, recording `site` (a nonzero code naming
// the wait) in *err unless an earlier failure is recorded there, or at once
// when another thread already recorded a failure. Returns false on giving up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int site = kErrWaitTimeout) {
    unsigned long long t0 = 0;
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u) {
            if (*reinterpret_cast<volatile int *>(err) != 0) return false;
            const unsigned long long now = global_ns();
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > kWaitLimitNs) {
                atomicCAS(err, 0, site);
                return false;
            }
        }
    }
}

// 2D tiled TMA load into this CTA's shared memory, completing on `bar`.
// Coordinates are {x (innermost, elements), y}.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Contiguous global -> shared bulk copy (both addresses 16-byte aligned,
// bytes a multiple of 16), completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// 4-byte global -> shared copy (cp.async.ca).
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// 16-byte global -> shared copy that bypasses L1 (cp.async.cg).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Arrive on `bar` once every cp.async this thread issued so far has landed.
// The arrival is not pre-counted: the barrier's init count must include it.
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// Wait until at most N of this thread's committed cp.async groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Named barrier over `count` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Programmatic dependent launch controls (no-ops without the launch attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Host: encode a 2D uint8 tensor map over a row-major array of `rows` rows
// holding `row_bytes` valid bytes each at a row pitch of `pitch` bytes (a
// multiple of 16), with a box of [box_rows, box_bytes] and the given swizzle.
cudaError_t make_tensor_map_u8(CUtensorMap *map, const void *base, uint64_t row_bytes, uint64_t pitch,
                               uint64_t rows, uint32_t box_bytes, uint32_t box_rows, CUtensorMapSwizzle swizzle);

}  // namespace nvfp4
