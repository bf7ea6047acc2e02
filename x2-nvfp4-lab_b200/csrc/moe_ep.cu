// Expert parallelism, two ways of adding the ranks' partial sums:
//  * finalize_bf16_kernel: out = BF16(sum + residual) after a collective
//    (NCCL all-reduce) has added NVFP4_MOE_PARTIAL_F32 partials;
//  * moe_combine_ep_kernel: the decode combine fused with the reduction over
//    NVLink peer memory. Every rank maps every other rank's partial buffer
//    and flag array (CUDA IPC); a CTA computes its local partial tile and
//    stores it; the rank's CTAs count their tiles in, and the last one makes
//    them all visible to the peers with one system-scope fence and raises the
//    rank's flag in every peer's array (a system-scope fence per tile cost
//    ~14 us per call); every CTA then waits (bounded by wall-clock time) for
//    every peer's flag with acquire loads and adds the ranks' tiles in rank
//    order, so every rank writes the same BF16 output. One rank alone needs
//    neither fence nor flag.
// Partial buffers alternate between two parities by call number: a rank can
// start call e+1 while a peer still reads its call-e tile, never call e+2
// (that needs the peer's flags of call e+1, raised after its call e ended).
// The grid (hidden/256 x tokens CTAs of 256 threads, at most 16 x 64) is
// always co-resident, so no CTA waits for a peer tile whose CTA cannot run.
#include "internal.h"
#include "moe_decode.cuh"
#include "nvfp4_common.cuh"
#include "tma_util.cuh"

#include <algorithm>
#include <cstring>
#include <memory>

struct nvfp4_ep {
    nvfp4_runtime *runtime = nullptr;
    int rank = 0, world = 1, max_tokens = 0, hidden = 0;
    size_t part_bytes = 0;      // one parity's partial buffer
    size_t max_tiles = 0;
    uint8_t *local = nullptr;   // [2][part_bytes] partials, then flags [world][max_tiles] u32
    uint8_t *peer[nvfp4::kMaxEpRanks] = {};
    bool opened = false;
    unsigned epoch = 0;
    int *err = nullptr;         // device error word
    int *host_err = nullptr;    // pinned host-mapped error word (host address)
    int *host_err_dev = nullptr;  // its device address
    ~nvfp4_ep() {
        for (int p = 0; p < world; ++p)
            if (peer[p] && p != rank) cudaIpcCloseMemHandle(peer[p]);
        if (host_err) {
            runtime->error_words.erase(std::remove_if(runtime->error_words.begin(), runtime->error_words.end(),
                                                      [&](const auto &w) { return w.second == err; }),
                                       runtime->error_words.end());
            cudaFreeHost(host_err);
        }
        if (err) cudaFree(err);
        if (local) cudaFree(local);
    }
    size_t flags_offset() const { return 2 * part_bytes; }
};

namespace nvfp4 {
namespace {

__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(256) moe_combine_ep_kernel(DownArgs a, EpArgs e) {
    pdl_wait();
    const DecodeScratch &s = a.s;
    const int H = a.H, T = a.T;
    const int t = blockIdx.y;
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    __shared__ int s_ok;
    float v = 0.0f;
    if (h < H) {
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            const int pos = s.inv_pos[t * kTopK + k];
            if (pos >= 0) v += s.ypart[(size_t)pos * H + h];
        }
        if (a.shared_here) v += s.ypart[(size_t)(T * kTopK + t) * H + h];
        if (a.residual && e.rank == 0) v += bf16_bits_to_f32(static_cast<const uint16_t *>(a.residual)[(size_t)t * H + h]);
        e.part[e.rank][(size_t)t * H + h] = v;
    }
    __syncthreads();
    if (e.world > 1) {
        if (threadIdx.x == 0) {
            // Publish: the last of this rank's CTAs to count its tile in
            // releases them all (system scope) and raises the rank's flag in
            // every peer's array (slot `rank`).
            __threadfence();
            if (atomicAdd(e.ticket, 1u) == gridDim.x * gridDim.y - 1) {
                *e.ticket = 0u;  // the next call's count (read by no other CTA of this call)
                __threadfence_system();
                for (int p = 0; p < e.world; ++p)
                    if (p != e.rank) *reinterpret_cast<volatile unsigned *>(e.flags_peer[p] + e.rank) = e.epoch;
            }
            // Collect every peer's flag of this call.
            int ok = *reinterpret_cast<volatile int *>(e.err) == 0;
            const unsigned long long t0 = global_ns();
            for (int p = 0; p < e.world && ok; ++p) {
                if (p == e.rank) continue;
                for (uint32_t i = 0;; ++i) {
                    if ((int)(ld_acquire_sys_u32(e.flags_local + p) - e.epoch) >= 0) break;
                    if ((i & 63u) == 63u && global_ns() - t0 > kWaitLimitNs) {
                        atomicCAS(e.err, 0, kSiteEpPeerTile);
                        ok = 0;
                        break;
                    }
                }
            }
            s_ok = ok;
        }
        __syncthreads();
        if (!s_ok) {
            if (threadIdx.x == 0 && e.host_err) *reinterpret_cast<volatile int *>(e.host_err) = kSiteEpPeerTile;
            return;
        }
    }
    if (h >= H) return;
    float acc = 0.0f;
    for (int p = 0; p < e.world; ++p) acc += p == e.rank ? v : __ldcg(e.part[p] + (size_t)t * H + h);
    static_cast<uint16_t *>(a.out)[(size_t)t * H + h] = f32_to_bf16_bits(acc);
}

// Four consecutive elements per thread (hidden is a multiple of 16).
__global__ void __launch_bounds__(256) finalize_bf16_kernel(const float *sum, const uint16_t *residual, uint16_t *out,
                                                            size_t n4) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = reinterpret_cast<const float4 *>(sum)[i];
        float f[4] = {v.x, v.y, v.z, v.w};
        if (residual) {
            const uint2 r = reinterpret_cast<const uint2 *>(residual)[i];
            f[0] += bf16_bits_to_f32(r.x & 0xFFFFu);
            f[1] += bf16_bits_to_f32(r.x >> 16);
            f[2] += bf16_bits_to_f32(r.y & 0xFFFFu);
            f[3] += bf16_bits_to_f32(r.y >> 16);
        }
        const uint32_t lo = f32_to_bf16_bits(f[0]) | (static_cast<uint32_t>(f32_to_bf16_bits(f[1])) << 16);
        const uint32_t hi = f32_to_bf16_bits(f[2]) | (static_cast<uint32_t>(f32_to_bf16_bits(f[3])) << 16);
        reinterpret_cast<uint2 *>(out)[i] = make_uint2(lo, hi);
    }
}

}  // namespace

cudaError_t launch_combine_ep(const DownArgs &a, const EpArgs &e, cudaStream_t stream) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((a.H + 255) / 256, a.T);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, moe_combine_ep_kernel, a, e);
}

// Arguments of the next fused combine on this context (advances the call
// number). False if the context cannot serve `tokens` x `hidden`.
bool ep_next_call(nvfp4_ep *ep, int tokens, int hidden, EpArgs *out) {
    if (!ep || !ep->opened || tokens < 1 || tokens > ep->max_tokens || hidden != ep->hidden) return false;
    ++ep->epoch;
    EpArgs e{};
    const size_t parity = (ep->epoch & 1u) * ep->part_bytes;
    for (int p = 0; p < ep->world; ++p) {
        e.part[p] = reinterpret_cast<float *>(ep->peer[p] + parity);
        e.flags_peer[p] = reinterpret_cast<unsigned *>(ep->peer[p] + ep->flags_offset());
    }
    e.flags_local = reinterpret_cast<unsigned *>(ep->local + ep->flags_offset());
    e.ticket = reinterpret_cast<unsigned *>(ep->local + ep->flags_offset() +
                                            static_cast<size_t>(ep->world) * ep->max_tiles * sizeof(unsigned));
    e.epoch = ep->epoch;
    e.rank = ep->rank;
    e.world = ep->world;
    e.tiles = ((hidden + 255) / 256) * tokens;
    e.err = ep->err;
    e.host_err = ep->host_err_dev;
    *out = e;
    return true;
}

}  // namespace nvfp4

using namespace nvfp4;

extern "C" NVFP4_API nvfp4_status nvfp4_ep_create(nvfp4_runtime *runtime, int rank, int world, int max_tokens,
                                                 int hidden, nvfp4_ep **out) {
    if (!runtime || !out || world < 1 || world > kMaxEpRanks || rank < 0 || rank >= world || max_tokens < 1 ||
        max_tokens > kDecodeMaxTokens || hidden < 16 || hidden % 16 != 0)
        return fail_invalid("expert-parallel context: 1..8 ranks, 1..64 tokens, hidden a positive multiple of 16");
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        auto ep = std::make_unique<nvfp4_ep>();
        ep->runtime = runtime;
        ep->rank = rank;
        ep->world = world;
        ep->max_tokens = max_tokens;
        ep->hidden = hidden;
        ep->part_bytes = ((static_cast<size_t>(max_tokens) * hidden * sizeof(float)) + 255) & ~size_t(255);
        ep->max_tiles = static_cast<size_t>((hidden + 255) / 256) * max_tokens;
        const size_t bytes = 2 * ep->part_bytes + static_cast<size_t>(world) * ep->max_tiles * sizeof(unsigned) + 256;
        check_cuda(cudaMalloc(&ep->local, bytes), "cudaMalloc(expert-parallel buffers)");
        check_cuda(cudaMemset(ep->local, 0, bytes), "cudaMemset(expert-parallel buffers)");
        check_cuda(cudaMalloc(&ep->err, sizeof(int)), "cudaMalloc(expert-parallel error word)");
        check_cuda(cudaMemset(ep->err, 0, sizeof(int)), "cudaMemset(expert-parallel error word)");
        check_cuda(cudaHostAlloc(reinterpret_cast<void **>(&ep->host_err), sizeof(int), cudaHostAllocMapped),
                   "cudaHostAlloc(expert-parallel error word)");
        *ep->host_err = 0;
        check_cuda(cudaHostGetDevicePointer(reinterpret_cast<void **>(&ep->host_err_dev), ep->host_err, 0),
                   "cudaHostGetDevicePointer(expert-parallel error word)");
        runtime->error_words.emplace_back(ep->host_err, ep->err);
        ep->peer[rank] = ep->local;
        *out = ep.release();
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_ep_ipc_handle(nvfp4_ep *ep, void *handle) {
    if (!ep || !handle) return fail_invalid("invalid expert-parallel handle query");
    try {
        cudaIpcMemHandle_t h;
        check_cuda(cudaIpcGetMemHandle(&h, ep->local), "cudaIpcGetMemHandle");
        static_assert(sizeof(h) == NVFP4_EP_HANDLE_BYTES, "IPC handle size");
        std::memcpy(handle, &h, sizeof(h));
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_ep_open_peers(nvfp4_ep *ep, const void *handles) {
    if (!ep || !handles || ep->opened) return fail_invalid("invalid or repeated expert-parallel peer opening");
    try {
        for (int p = 0; p < ep->world; ++p) {
            if (p == ep->rank) continue;
            cudaIpcMemHandle_t h;
            std::memcpy(&h, static_cast<const uint8_t *>(handles) + static_cast<size_t>(p) * sizeof(h), sizeof(h));
            void *ptr = nullptr;
            check_cuda(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
            ep->peer[p] = static_cast<uint8_t *>(ptr);
        }
        ep->opened = true;
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API void nvfp4_ep_destroy(nvfp4_ep *ep) {
    if (!ep) return;
    if (ep->runtime) {
        std::lock_guard<std::mutex> lock(ep->runtime->queue_mutex);
        cudaStreamSynchronize(ep->runtime->stream);
        cudaDeviceSynchronize();
        delete ep;
        return;
    }
    delete ep;
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_finalize_bf16(nvfp4_runtime *runtime, const float *sum_f32,
                                                         const void *residual_bf16, void *out_bf16, int tokens,
                                                         int hidden, void *stream) {
    if (!runtime || !sum_f32 || !out_bf16 || tokens < 1 || hidden < 16 || hidden % 16 != 0)
        return fail_invalid("invalid finalize arguments (hidden must be a positive multiple of 16)");
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        const size_t n4 = static_cast<size_t>(tokens) * hidden / 4;
        const int grid = static_cast<int>((n4 + 255) / 256 < 4096 ? (n4 + 255) / 256 : 4096);
        runtime->direct_call(static_cast<cudaStream_t>(stream), [&](cudaStream_t s) {
            finalize_bf16_kernel<<<grid, 256, 0, s>>>(sum_f32, static_cast<const uint16_t *>(residual_bf16),
                                                      static_cast<uint16_t *>(out_bf16), n4);
            check_cuda(cudaGetLastError(), "finalize_bf16_kernel");
        });
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}
