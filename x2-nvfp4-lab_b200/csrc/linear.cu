// Dense NVFP4 linear: the lab's nvfp4_matrix objects and its A16 linear entry
// points (native_nvfp4/runtime/nvfp4_runtime.h:208-217,238-270; implemented at
// nvfp4_runtime.cpp:1705-1735,2106-2270) on sm_100a. This is the weight path
// behind the lab's vLLM NvFp4LinearKernel provider
// (vllm_nvfp4_opencl/linear.py:15-70): FP32 activations, checkpoint-native
// NVFP4 weights, FP32 output,
//
//   dst[v, r] = (1 / weight_global_scale) *
//               sum_c E2M1(W[r, c]) * E4M3(S[r, c / 16]) * x[v, c].
//
// Storage (device, owned by the matrix): packed E2M1 rows padded to a 16-byte
// pitch, scale rows padded to a 16-byte pitch, both zero-filled beyond the
// row, scale bytes sanitised at upload like the bank's (sign cleared, 0x7F ->
// 0: the lab's decoding rule, nvfp4_gemv.cl:14-27).
//
// Kernels. Every call runs the tensor-core kernel (linear_tc.cu: the
// activations as six NVFP4 terms, the weights streamed through tcgen05
// block-scaled MMAs, within ~2e-6 of the output scale) except calls with the
// scalar kernel kind, which run the CUDA-core kernel below on the FP32
// activations themselves.
//
// CUDA-core kernel: a weight stream bound by HBM for a few vectors. Each warp owns four
// rows at a time; lane l takes the 32-column chunks l, l+32, ... of the rows
// (one 16-byte packed load and one 2-byte scale load per chunk and row), two
// chunks of every row loaded before any arithmetic so that eight 16-byte
// loads per lane are in flight. The
// E2M1 codes and the E4M3 scales convert exactly to FP16, their product is
// exact in FP16 (at most five significant bits, magnitude in [2^-10, 2688]),
// and each product multiplies the FP32 activation in an FP32 FMA; the lanes'
// partial sums meet in an xor butterfly and the row sum is scaled by the
// inverse global scale. The activations of up to eight vectors per pass sit
// in shared memory, each 32-column chunk's float4 groups rotated by the chunk
// index so that a warp's LDS.128 hits distinct bank groups.

#include "internal.h"
#include "linear_tc.cuh"
#include "nvfp4_common.cuh"

#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <limits>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

struct nvfp4_matrix {
    nvfp4_runtime *runtime = nullptr;
    int rows = 0;
    int cols = 0;
    int packed_pitch = 0;  // bytes per packed row (multiple of 16)
    int scale_pitch = 0;   // bytes per scale row (multiple of 16)
    uint8_t *packed = nullptr;
    uint8_t *scales = nullptr;
    float inv_global = 0.0f;
    nvfp4::LinearTcState tc;               // tensor-core path: scale atoms, activation terms, tensor maps
    volatile int *host_err = nullptr;      // pinned, device-mapped wait-timeout word (read at synchronize)

    ~nvfp4_matrix() {
        nvfp4::free_linear_tc(tc);
        if (host_err) cudaFreeHost(const_cast<int *>(host_err));
        if (packed) cudaFree(packed);
        if (scales) cudaFree(scales);
    }
};

namespace nvfp4 {
namespace {

constexpr int kLinThreads = 256;
constexpr int kLinWarps = kLinThreads / 32;
constexpr int kLinRowsPerWarp = 4;
constexpr int kLinChunksInFlight = 2;  // 32-column chunks per lane loaded before any math
constexpr int kLinMaxCols = 49152;
constexpr size_t kLinSmemBudget = 200 * 1024;  // activation bytes of one pass

struct LinearArgs {
    const uint8_t *packed;
    const uint8_t *scales;
    const float *x;  // [vectors, cols]
    float *dst;      // [vectors, rows]
    int rows;
    int cols;
    int chunks;  // packed_pitch / 16: 32 columns per chunk
    int packed_pitch;
    int scale_pitch;
    int v0;       // first vector of this pass
    int vectors;  // vectors of the call
    float inv_global;
};

// Shared-memory slot of activation (v, col), col < chunks * 32.
__device__ __forceinline__ int xs_index(int chunks, int v, int col) {
    const int c = col >> 5, g = (col >> 2) & 7, e = col & 3;
    return (v * chunks + c) * 32 + (((g + c) & 7) << 2) + e;
}

__device__ __forceinline__ float2 f16x2_to_f32x2(uint32_t h) {
    __half2 v;
    memcpy(&v, &h, sizeof(v));
    return __half22float2(v);
}

template <int V>
__global__ void __launch_bounds__(kLinThreads) nvfp4_linear_kernel(LinearArgs a) {
    extern __shared__ __align__(16) float xs[];
    const int xcols = a.chunks * 32;
    for (int i = threadIdx.x; i < V * xcols; i += kLinThreads) {
        const int v = i / xcols, col = i - v * xcols;
        const int gv = a.v0 + v;
        const float val = (gv < a.vectors && col < a.cols) ? a.x[static_cast<size_t>(gv) * a.cols + col] : 0.0f;
        xs[xs_index(a.chunks, v, col)] = val;
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int stride = gridDim.x * kLinWarps * kLinRowsPerWarp;
    for (int r0 = (blockIdx.x * kLinWarps + warp) * kLinRowsPerWarp; r0 < a.rows; r0 += stride) {
        float acc[kLinRowsPerWarp][V];
#pragma unroll
        for (int j = 0; j < kLinRowsPerWarp; ++j)
#pragma unroll
            for (int v = 0; v < V; ++v) acc[j][v] = 0.0f;

        for (int cb = lane; cb < a.chunks; cb += 32 * kLinChunksInFlight) {
            // Every load of the row group's chunks is issued before any math
            // (kLinRowsPerWarp x kLinChunksInFlight 16-byte loads per lane in
            // flight); chunks past the row re-read the row's last chunk and
            // are not added.
            uint4 qq[kLinChunksInFlight][kLinRowsPerWarp];
            uint16_t ss[kLinChunksInFlight][kLinRowsPerWarp];
#pragma unroll
            for (int u = 0; u < kLinChunksInFlight; ++u) {
                const size_t cc = static_cast<size_t>(min(cb + 32 * u, a.chunks - 1));
#pragma unroll
                for (int j = 0; j < kLinRowsPerWarp; ++j) {
                    // A missing row re-reads the last row; its sum is not stored.
                    const size_t r = static_cast<size_t>(min(r0 + j, a.rows - 1));
                    qq[u][j] = ldg_stream128(a.packed + r * a.packed_pitch + cc * 16);
                    ss[u][j] = ldg_u16(a.scales + r * a.scale_pitch + cc * 2);
                }
            }
#pragma unroll
            for (int u = 0; u < kLinChunksInFlight; ++u) {
            const int c = cb + 32 * u;
            if (c >= a.chunks) break;
            const uint4 *q = qq[u];
            uint32_t sc[kLinRowsPerWarp];
#pragma unroll
            for (int j = 0; j < kLinRowsPerWarp; ++j) sc[j] = e4m3x2_to_f16x2(ss[u][j]);
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {  // word wi: columns c*32 + 8*wi .. +7
                float w[kLinRowsPerWarp][8];
#pragma unroll
                for (int j = 0; j < kLinRowsPerWarp; ++j) {
                    const uint32_t word = wi == 0 ? q[j].x : wi == 1 ? q[j].y : wi == 2 ? q[j].z : q[j].w;
                    const uint32_t s2 = wi < 2 ? f16x2_lo_lo(sc[j]) : f16x2_hi_hi(sc[j]);
                    uint32_t h[4];
                    e2m1x8_to_f16x8(word, h);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float2 f = f16x2_to_f32x2(hmul2_u32(h[k], s2));
                        w[j][2 * k] = f.x;
                        w[j][2 * k + 1] = f.y;
                    }
                }
                const int col = c * 32 + wi * 8;
#pragma unroll
                for (int v = 0; v < V; ++v) {
                    const float4 x0 = *reinterpret_cast<const float4 *>(&xs[xs_index(a.chunks, v, col)]);
                    const float4 x1 = *reinterpret_cast<const float4 *>(&xs[xs_index(a.chunks, v, col + 4)]);
#pragma unroll
                    for (int j = 0; j < kLinRowsPerWarp; ++j) {
                        float s = acc[j][v];
                        s = fmaf(w[j][0], x0.x, s);
                        s = fmaf(w[j][1], x0.y, s);
                        s = fmaf(w[j][2], x0.z, s);
                        s = fmaf(w[j][3], x0.w, s);
                        s = fmaf(w[j][4], x1.x, s);
                        s = fmaf(w[j][5], x1.y, s);
                        s = fmaf(w[j][6], x1.z, s);
                        s = fmaf(w[j][7], x1.w, s);
                        acc[j][v] = s;
                    }
                }
            }
            }
        }
#pragma unroll
        for (int j = 0; j < kLinRowsPerWarp; ++j) {
#pragma unroll
            for (int v = 0; v < V; ++v) {
                float s = acc[j][v];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                const int r = r0 + j, gv = a.v0 + v;
                if (lane == 0 && r < a.rows && gv < a.vectors)
                    a.dst[static_cast<size_t>(gv) * a.rows + r] = s * a.inv_global;
            }
        }
    }
}

template <int V>
void launch_pass(const LinearArgs &a, int sm_count, cudaStream_t stream) {
    // The shared-memory limit is a per-device function attribute: set once on
    // each device this process launches on.
    static std::atomic<uint64_t> configured{0};
    int device = 0;
    check_cuda(cudaGetDevice(&device), "cudaGetDevice");
    const uint64_t bit = device < 64 ? (uint64_t{1} << device) : 0;
    if (!bit || !(configured.load(std::memory_order_acquire) & bit)) {
        check_cuda(cudaFuncSetAttribute(nvfp4_linear_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(kLinSmemBudget)),
                   "cudaFuncSetAttribute(nvfp4_linear_kernel)");
        configured.fetch_or(bit, std::memory_order_acq_rel);
    }
    const size_t smem = static_cast<size_t>(V) * a.chunks * 32 * sizeof(float);
    int per_sm = 0;
    check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, nvfp4_linear_kernel<V>, kLinThreads, smem),
               "cudaOccupancyMaxActiveBlocksPerMultiprocessor(nvfp4_linear_kernel)");
    const int rows_per_cta = kLinWarps * kLinRowsPerWarp;
    const int need = (a.rows + rows_per_cta - 1) / rows_per_cta;
    const int grid = std::max(1, std::min(need, std::max(1, sm_count) * std::max(1, per_sm)));
    nvfp4_linear_kernel<V><<<grid, kLinThreads, smem, stream>>>(a);
    check_cuda(cudaGetLastError(), "nvfp4_linear_kernel");
}

// All passes of one call. The tensor-core kernel (linear_tc.cu) serves every
// call except those that ask for the scalar kernel kind, which run the
// CUDA-core kernel above on the FP32 activations themselves: up to eight
// vectors per pass (fewer when the activations of eight would exceed the
// shared-memory budget).
void launch_linear(const nvfp4_matrix &m, const float *x, int vectors, float *dst, int sm_count,
                   cudaStream_t stream, bool tensor_cores = true) {
    // The tensor-core kernel reads the activations as 16-byte vectors.
    if (tensor_cores && (reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
        check_cuda(launch_linear_tc(m.tc, x, vectors, m.rows, m.cols, m.inv_global, dst, sm_count, stream),
                   "linear_tc_kernel");
        return;
    }
    LinearArgs a{};
    a.packed = m.packed;
    a.scales = m.scales;
    a.x = x;
    a.dst = dst;
    a.rows = m.rows;
    a.cols = m.cols;
    a.chunks = m.packed_pitch / 16;
    a.packed_pitch = m.packed_pitch;
    a.scale_pitch = m.scale_pitch;
    a.vectors = vectors;
    a.inv_global = m.inv_global;
    const size_t xcol_bytes = static_cast<size_t>(a.chunks) * 32 * sizeof(float);
    int vmax = 8;
    while (vmax > 1 && static_cast<size_t>(vmax) * xcol_bytes > kLinSmemBudget) vmax >>= 1;
    for (int v0 = 0; v0 < vectors;) {
        const int rem = vectors - v0;
        int V = 1;
        while (V < rem && V < vmax) V <<= 1;
        a.v0 = v0;
        switch (V) {
            case 1: launch_pass<1>(a, sm_count, stream); break;
            case 2: launch_pass<2>(a, sm_count, stream); break;
            case 4: launch_pass<4>(a, sm_count, stream); break;
            default: launch_pass<8>(a, sm_count, stream); break;
        }
        v0 += V;
    }
}

bool valid_kind(nvfp4_kernel_kind kind) {
    return kind == NVFP4_KERNEL_SCALAR || kind == NVFP4_KERNEL_SUBGROUP || kind == NVFP4_KERNEL_TILED ||
           kind == NVFP4_KERNEL_ROW_TILED;
}

// The reference's kernel-kind rules (nvfp4_runtime.cpp:2116-2129): the tiled
// kernel needs more than one vector, the row-tiled kernel exactly one. Every
// kind runs the kernel above on this backend.
bool kind_matches(nvfp4_kernel_kind kind, int vectors) {
    return !(kind == NVFP4_KERNEL_TILED && vectors == 1) && !(kind == NVFP4_KERNEL_ROW_TILED && vectors != 1);
}

bool sizes_fit(const nvfp4_matrix *m, int vectors, size_t *in_bytes, size_t *out_bytes) {
    const size_t in = static_cast<size_t>(vectors) * static_cast<size_t>(m->cols);
    const size_t out = static_cast<size_t>(vectors) * static_cast<size_t>(m->rows);
    if (in > std::numeric_limits<size_t>::max() / sizeof(float) ||
        out > std::numeric_limits<size_t>::max() / sizeof(float))
        return false;
    *in_bytes = in * sizeof(float);
    *out_bytes = out * sizeof(float);
    return true;
}

struct DeviceScratch {
    void *p = nullptr;
    ~DeviceScratch() {
        if (p) cudaFree(p);
    }
};

struct EventLease {
    nvfp4_runtime *rt;
    cudaEvent_t e;
    explicit EventLease(nvfp4_runtime *r) : rt(r), e(r->acquire_event()) {}
    ~EventLease() { rt->release_event(e); }
};

uint64_t elapsed_ns(cudaEvent_t a, cudaEvent_t b) {
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, a, b) != cudaSuccess) return 0;
    return static_cast<uint64_t>(static_cast<double>(ms) * 1.0e6);
}

}  // namespace
}  // namespace nvfp4

using namespace nvfp4;

extern "C" NVFP4_API nvfp4_status nvfp4_matrix_upload(nvfp4_runtime *runtime, const uint8_t *packed,
                                                      size_t packed_bytes, const uint8_t *scales_e4m3,
                                                      size_t scale_bytes, int rows, int cols,
                                                      float weight_global_scale, nvfp4_matrix **out_matrix) {
    if (!runtime || !packed || !scales_e4m3 || !out_matrix || rows <= 0 || cols <= 0 || cols % 16 != 0 ||
        weight_global_scale == 0.0f)
        return fail_invalid("invalid native NVFP4 matrix arguments");
    const size_t row_packed = static_cast<size_t>(cols / 2), row_scales = static_cast<size_t>(cols / 16);
    if (packed_bytes != static_cast<size_t>(rows) * row_packed ||
        scale_bytes != static_cast<size_t>(rows) * row_scales)
        return fail_invalid("packed/scales byte counts do not match rows and cols");
    if (cols > kLinMaxCols) return fail_invalid("NVFP4 linear supports at most 49152 columns on this backend");
    *out_matrix = nullptr;
    try {
        auto m = std::make_unique<nvfp4_matrix>();
        m->runtime = runtime;
        m->rows = rows;
        m->cols = cols;
        m->packed_pitch = static_cast<int>((row_packed + 15) / 16 * 16);
        m->scale_pitch = static_cast<int>((row_scales + 15) / 16 * 16);
        m->inv_global = 1.0f / weight_global_scale;
        std::vector<uint8_t> sanitized(static_cast<size_t>(rows) * m->scale_pitch, 0);
        for (size_t r = 0; r < static_cast<size_t>(rows); ++r) {
            const uint8_t *src = scales_e4m3 + r * row_scales;
            uint8_t *dst = sanitized.data() + r * m->scale_pitch;
            for (size_t c = 0; c < row_scales; ++c) {
                const uint8_t b = src[c] & 0x7Fu;
                dst[c] = b == 0x7Fu ? 0u : b;
            }
        }
        const size_t packed_total = static_cast<size_t>(rows) * m->packed_pitch;
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        check_cuda(cudaMalloc(&m->packed, packed_total), "cudaMalloc(matrix packed)");
        check_cuda(cudaMalloc(&m->scales, sanitized.size()), "cudaMalloc(matrix scales)");
        check_cuda(cudaMemsetAsync(m->packed, 0, packed_total, runtime->stream), "cudaMemsetAsync(matrix packed)");
        check_cuda(cudaMemcpy2DAsync(m->packed, m->packed_pitch, packed, row_packed, row_packed, rows,
                                     cudaMemcpyHostToDevice, runtime->stream),
                   "cudaMemcpy2DAsync(matrix packed)");
        check_cuda(cudaMemcpyAsync(m->scales, sanitized.data(), sanitized.size(), cudaMemcpyHostToDevice,
                                   runtime->stream),
                   "cudaMemcpyAsync(matrix scales)");
        check_cuda(init_linear_tc(m->tc, m->packed, m->packed_pitch, m->scales, m->scale_pitch, rows, cols,
                                  runtime->stream),
                   "tensor-core linear set-up");
        int *host_err = nullptr;
        check_cuda(cudaHostAlloc(reinterpret_cast<void **>(&host_err), sizeof(int), cudaHostAllocMapped),
                   "cudaHostAlloc(matrix error word)");
        m->host_err = host_err;
        *host_err = 0;
        check_cuda(cudaHostGetDevicePointer(reinterpret_cast<void **>(&m->tc.host_err_dev), host_err, 0),
                   "cudaHostGetDevicePointer(matrix error word)");
        check_cuda(cudaStreamSynchronize(runtime->stream), "cudaStreamSynchronize(matrix upload)");
        runtime->error_words.emplace_back(m->host_err, m->tc.err);
        *out_matrix = m.release();
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API void nvfp4_matrix_destroy(nvfp4_matrix *matrix) {
    if (!matrix) return;
    if (matrix->runtime) {
        std::lock_guard<std::mutex> lock(matrix->runtime->queue_mutex);
        cudaStreamSynchronize(matrix->runtime->stream);
        auto &words = matrix->runtime->error_words;
        words.erase(std::remove_if(words.begin(), words.end(),
                                   [&](const std::pair<volatile int *, int *> &w) { return w.second == matrix->tc.err; }),
                    words.end());
    }
    delete matrix;
}

extern "C" NVFP4_API nvfp4_status nvfp4_linear_f32(nvfp4_runtime *runtime, const nvfp4_matrix *matrix,
                                                   const float *x, int vectors, float *dst,
                                                   nvfp4_kernel_kind kernel_kind) {
    if (!runtime || !matrix || matrix->runtime != runtime || !x || !dst || vectors <= 0 || !valid_kind(kernel_kind))
        return fail_invalid("invalid linear arguments or mismatched runtime/matrix");
    if (kernel_kind == NVFP4_KERNEL_TILED && vectors == 1)
        return fail_invalid("the tiled kernel requires more than one vector");
    if (kernel_kind == NVFP4_KERNEL_ROW_TILED && vectors != 1)
        return fail_invalid("the row-tiled kernel requires one vector");
    size_t in_bytes = 0, out_bytes = 0;
    if (!sizes_fit(matrix, vectors, &in_bytes, &out_bytes)) return fail_invalid("linear buffer size overflow");
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        cudaStream_t s = runtime->stream;
        DeviceScratch dx, dy;
        check_cuda(cudaMalloc(&dx.p, in_bytes), "cudaMalloc(linear input)");
        check_cuda(cudaMalloc(&dy.p, out_bytes), "cudaMalloc(linear output)");
        EventLease e0(runtime), e1(runtime), e2(runtime), e3(runtime);
        check_cuda(cudaEventRecord(e0.e, s), "cudaEventRecord");
        check_cuda(cudaMemcpyAsync(dx.p, x, in_bytes, cudaMemcpyHostToDevice, s), "cudaMemcpyAsync(linear input)");
        check_cuda(cudaEventRecord(e1.e, s), "cudaEventRecord");
        launch_linear(*matrix, static_cast<const float *>(dx.p), vectors, static_cast<float *>(dy.p),
                      runtime->sm_count, s, kernel_kind != NVFP4_KERNEL_SCALAR);
        check_cuda(cudaEventRecord(e2.e, s), "cudaEventRecord");
        check_cuda(cudaMemcpyAsync(dst, dy.p, out_bytes, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync(linear output)");
        check_cuda(cudaEventRecord(e3.e, s), "cudaEventRecord");
        check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize(linear)");
        raise_device_timeouts(runtime);
        runtime->last_profile = {elapsed_ns(e0.e, e1.e), elapsed_ns(e1.e, e2.e), elapsed_ns(e2.e, e3.e)};
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

namespace {

nvfp4_status check_device_linear(nvfp4_runtime *runtime, const nvfp4_matrix *matrix, const nvfp4_buffer *x,
                                 int vectors, const nvfp4_buffer *dst, nvfp4_kernel_kind kernel_kind,
                                 const char *invalid_message) {
    if (!runtime || !matrix || matrix->runtime != runtime || !x || x->runtime != runtime || !dst ||
        dst->runtime != runtime || vectors <= 0 || !valid_kind(kernel_kind))
        return fail_invalid(invalid_message);
    if (!kind_matches(kernel_kind, vectors))
        return fail_invalid(kernel_kind == NVFP4_KERNEL_TILED ? "the tiled kernel requires more than one vector"
                                                              : "the row-tiled kernel requires one vector");
    size_t in_bytes = 0, out_bytes = 0;
    if (!sizes_fit(matrix, vectors, &in_bytes, &out_bytes)) return fail_invalid("device linear buffer size overflow");
    if (x->bytes < in_bytes || dst->bytes < out_bytes)
        return fail_invalid("device linear buffer capacity is too small");
    return NVFP4_STATUS_OK;
}

}  // namespace

extern "C" NVFP4_API nvfp4_status nvfp4_linear_device_f32(nvfp4_runtime *runtime, const nvfp4_matrix *matrix,
                                                          const nvfp4_buffer *x, int vectors, nvfp4_buffer *dst,
                                                          nvfp4_kernel_kind kernel_kind) {
    const nvfp4_status st = check_device_linear(runtime, matrix, x, vectors, dst, kernel_kind,
                                                "invalid device linear arguments or mismatched runtime");
    if (st != NVFP4_STATUS_OK) return st;
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        cudaStream_t s = runtime->stream;
        EventLease e0(runtime), e1(runtime);
        check_cuda(cudaEventRecord(e0.e, s), "cudaEventRecord");
        launch_linear(*matrix, static_cast<const float *>(x->data), vectors, static_cast<float *>(dst->data),
                      runtime->sm_count, s, kernel_kind != NVFP4_KERNEL_SCALAR);
        check_cuda(cudaEventRecord(e1.e, s), "cudaEventRecord");
        check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize(device linear)");
        raise_device_timeouts(runtime);
        runtime->last_profile = {0, elapsed_ns(e0.e, e1.e), 0};
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_linear_device_enqueue_f32(nvfp4_runtime *runtime,
                                                                  const nvfp4_matrix *matrix,
                                                                  const nvfp4_buffer *x, int vectors,
                                                                  nvfp4_buffer *dst,
                                                                  nvfp4_kernel_kind kernel_kind) {
    const nvfp4_status st = check_device_linear(runtime, matrix, x, vectors, dst, kernel_kind,
                                                "invalid enqueued device linear arguments");
    if (st != NVFP4_STATUS_OK) return st;
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        runtime->profiled("nvfp4_linear", nullptr, [&](cudaStream_t s) {
            launch_linear(*matrix, static_cast<const float *>(x->data), vectors, static_cast<float *>(dst->data),
                          runtime->sm_count, s, kernel_kind != NVFP4_KERNEL_SCALAR);
        });
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_linear_ptr_f32(nvfp4_runtime *runtime, const nvfp4_matrix *matrix,
                                                       const float *x, int vectors, float *dst, void *stream) {
    if (!runtime || !matrix || matrix->runtime != runtime || !x || !dst || vectors <= 0)
        return fail_invalid("invalid linear arguments or mismatched runtime/matrix");
    size_t in_bytes = 0, out_bytes = 0;
    if (!sizes_fit(matrix, vectors, &in_bytes, &out_bytes)) return fail_invalid("linear buffer size overflow");
    // The kernel reads the matrix on the runtime's device: activations and
    // outputs allocated on another GPU are rejected here rather than read
    // across devices (host or managed memory the device can reach is left
    // to the caller).
    for (const void *p : {static_cast<const void *>(x), static_cast<const void *>(dst)}) {
        cudaPointerAttributes attr{};
        if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
            cudaGetLastError();
            return fail_invalid("linear: cannot query the device of x or dst");
        }
        if (attr.type == cudaMemoryTypeDevice && attr.device != runtime->device) {
            const std::string msg = "linear: x and dst must be on the matrix's device (cuda:" +
                                    std::to_string(runtime->device) + "), got cuda:" + std::to_string(attr.device);
            return fail_invalid(msg.c_str());
        }
    }
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        runtime->direct_call(static_cast<cudaStream_t>(stream), [&](cudaStream_t s) {
            runtime->profiled_kernel("nvfp4_linear", s, [&](cudaStream_t ks) {
                launch_linear(*matrix, x, vectors, dst, runtime->sm_count, ks);
            });
        });
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}
