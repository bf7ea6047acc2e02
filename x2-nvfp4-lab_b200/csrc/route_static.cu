// Router + top-8 + dispatch entry point that allocates nothing.
//
// Some callers cannot allocate device memory at the point where they route
// tokens: a serving loop whose device memory is planned and owned up front by
// the host framework (every buffer handed to libraries is carved from that
// plan, and a library that calls cudaMalloc breaks the plan or stalls the
// loop on the allocator's implicit synchronisation), or an embedder that
// forbids allocation on its latency-critical path. For them this entry point
// runs the same routing kernel as the MoE bank but keeps its internal
// working memory (router logits, FP16 token copy, per-expert tables, the
// last-block ticket) in one fixed-size array that lives in the library's own
// device globals. Inputs and outputs remain the caller's buffers.
//
// Limits: tokens <= 64, experts in [8, 256], hidden a multiple of 128 and at
// most 4096. The array (kRouteStaticScratchBytes, 1 MiB) is part of the
// library image: every GPU on which the library is loaded holds it until the
// process exits.
//
// Sharing: every call, on every stream, uses the same array, which keeps
// whatever the last call left in it. The call clears the words that have to
// start at zero (the last-block tickets) before launching. Two calls whose
// kernels overlap on the GPU -- different streams without ordering, or
// several threads -- race on the array and produce garbage; order them.
//
// Set-up: the first call on each device looks up the array's device address
// with cudaGetSymbolAddress (with that device current) and caches it. Make
// that first call before any stream capture begins. The cache assumes the
// device's primary context lives as long as the process: after
// cudaDeviceReset the cached address is stale, so a process that resets a
// device must not call this entry point on it again.
#include "internal.h"
#include "moe_decode.cuh"

#include <mutex>

using namespace nvfp4;

namespace {

constexpr size_t kRouteStaticScratchBytes = 1u << 20;
constexpr int kRouteStaticMaxHidden = 4096;
constexpr int kRouteStaticCarveIntermediate = 128;  // the routing kernel never touches `act`
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_route_scratch[kRouteStaticScratchBytes];

std::mutex g_setup_mutex;
void *g_scratch_address[kMaxDevices] = {};

// Device address of g_route_scratch on the current device (looked up once).
cudaError_t scratch_address(void **out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_address[dev]) {
        void *ptr = nullptr;
        err = cudaGetSymbolAddress(&ptr, g_route_scratch);
        if (err != cudaSuccess) return err;
        g_scratch_address[dev] = ptr;
    }
    *out = g_scratch_address[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" NVFP4_API nvfp4_status nvfp4_moe_route_static_scratch(
    const void *router_bf16, const void *x_bf16, int tokens, int experts, int hidden, int32_t *ids,
    float *weights, int32_t *counts, int32_t *perm, void *stream) {
    if (!router_bf16 || !x_bf16 || !ids || !weights)
        return fail_invalid("router, x, ids and weights are required");
    if (tokens < 1 || tokens > kDecodeMaxTokens)
        return fail_invalid("static-scratch routing takes 1 to 64 tokens per call");
    if (experts < 8 || experts > 256)
        return fail_invalid("static-scratch routing takes 8 to 256 experts");
    if (hidden <= 0 || hidden % 128 != 0 || hidden > kRouteStaticMaxHidden)
        return fail_invalid("static-scratch routing needs hidden to be a multiple of 128, at most 4096");
    const size_t tables = decode_route_scratch_bytes(experts, hidden);
    const size_t inv_bytes = 3 * (static_cast<size_t>(experts) + 1) * sizeof(float);
    if (tables + inv_bytes > kRouteStaticScratchBytes)
        return fail_invalid("routing working set exceeds the 1 MiB static scratch array");
    try {
        void *base = nullptr;
        check_cuda(scratch_address(&base), "cudaGetSymbolAddress(g_route_scratch)");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        DecodeScratch ds{};
        decode_scratch_carve(ds, base, experts, hidden, kRouteStaticCarveIntermediate);
        // Caller-owned outputs replace the scratch copies.
        ds.ids = ids;
        ds.weights = weights;
        if (counts) ds.counts = counts;
        if (perm) ds.perm = perm;
        float *inv_scales = reinterpret_cast<float *>(static_cast<unsigned char *>(base) + tables);
        // The tickets must start at zero; the inverse-scale table only feeds
        // internal per-expert coefficients, zero is a valid value.
        check_cuda(cudaMemsetAsync(ds.ticket, 0, kRouteTickets * sizeof(unsigned), s),
                   "cudaMemsetAsync(tickets)");
        check_cuda(cudaMemsetAsync(inv_scales, 0, inv_bytes, s), "cudaMemsetAsync(inverse scales)");
        RouteArgs ra{};
        ra.router = static_cast<const uint16_t *>(router_bf16);
        ra.x = x_bf16;
        ra.x_is_f32 = 0;
        ra.T = tokens;
        ra.E = experts;
        ra.H = hidden;
        ra.inv_scales = inv_scales;
        ra.bias = nullptr;
        ra.e_first = 0;
        ra.e_count = experts;
        ra.shared_here = 1;
        ra.s = ds;
        check_cuda(launch_route(ra, s), "moe_route_kernel(static scratch)");
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}
