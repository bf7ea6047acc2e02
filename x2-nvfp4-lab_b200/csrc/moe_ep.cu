// Expert parallelism: the last step after the partial sums of the ranks'
// expert ranges have been reduced (NVFP4_MOE_PARTIAL_F32 forwards, then a
// collective sum over the ranks): out = BF16(sum + residual).
#include "internal.h"
#include "nvfp4_common.cuh"

namespace nvfp4 {
namespace {

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
}  // namespace nvfp4

using namespace nvfp4;

extern "C" NVFP4_API nvfp4_status nvfp4_moe_finalize_bf16(nvfp4_runtime *runtime, const float *sum_f32,
                                                         const void *residual_bf16, void *out_bf16, int tokens,
                                                         int hidden, void *stream) {
    if (!runtime || !sum_f32 || !out_bf16 || tokens < 1 || hidden < 16 || hidden % 16 != 0)
        return fail_invalid("invalid finalize arguments (hidden must be a positive multiple of 16)");
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        const size_t n4 = static_cast<size_t>(tokens) * hidden / 4;
        const int grid = static_cast<int>((n4 + 255) / 256 < 4096 ? (n4 + 255) / 256 : 4096);
        runtime->profiled_call("moe_finalize", static_cast<cudaStream_t>(stream), [&](cudaStream_t s) {
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
