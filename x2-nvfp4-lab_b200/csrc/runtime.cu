// Runtime, device buffers, tracing and graph primitives of the C ABI.
//
// Mirrors the lab runtime's object model (native_nvfp4/runtime/nvfp4_runtime.cpp
// :173-329 runtime, :1594-1703 buffers, :1273-1386 synchronize and trace,
// :2637-2818 graph primitives) on CUDA: one in-order stream per runtime
// instead of one OpenCL queue, cudaMalloc instead of SVM, CUDA event pairs
// instead of OpenCL profiling events.
#include "internal.h"
#include "nvfp4_common.cuh"

#include <algorithm>
#include <cstring>
#include <limits>
#include <memory>

namespace nvfp4 {

namespace {
thread_local std::string g_last_error;

void copy_fixed(char *dst, size_t cap, const std::string &src) {
    const size_t n = std::min(cap - 1, src.size());
    std::memcpy(dst, src.data(), n);
    dst[n] = '\0';
}
}  // namespace

const std::string &last_error_ref() { return g_last_error; }
void set_last_error(const std::string &message) { g_last_error = message; }
void clear_last_error() { g_last_error.clear(); }

nvfp4_status fail_invalid(const char *message) {
    g_last_error = message;
    return NVFP4_STATUS_INVALID_ARGUMENT;
}

nvfp4_status fail_exception(const std::exception &error) {
    g_last_error = error.what();
    if (dynamic_cast<const cuda_error *>(&error)) return NVFP4_STATUS_CUDA_ERROR;
    if (dynamic_cast<const invalid_argument_error *>(&error)) return NVFP4_STATUS_INVALID_ARGUMENT;
    return NVFP4_STATUS_INTERNAL_ERROR;
}

// ------------------------------------------------------------ kernels

namespace {

__global__ void add_f32_kernel(const float *a, const float *b, float *dst, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        dst[i] = a[i] + b[i];
}

__global__ void weighted_accumulate_f32_kernel(const float *src, float scale, float *dst, int n,
                                               int reset) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float prev = reset ? 0.0f : dst[i];
        dst[i] = prev + scale * src[i];
    }
}

__global__ void silu_mul_f32_kernel(const float *gate, const float *up, float *dst, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = gate[i];
        dst[i] = v / (1.0f + expf(-v)) * up[i];
    }
}

// One CTA per row. FP32 sum of squares (thread-strided partial sums, then a
// fixed tree), scaled by rsqrt(mean + eps), times the weight.
template <bool BF16>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const void *x, const void *weight, void *dst,
                                                      int cols, float eps) {
    __shared__ float red[8];
    const int row = blockIdx.x;
    float ss = 0.0f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        float v;
        if (BF16)
            v = bf16_bits_to_f32(static_cast<const uint16_t *>(x)[(size_t)row * cols + c]);
        else
            v = static_cast<const float *>(x)[(size_t)row * cols + c];
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
    const float inv = rsqrtf(tot / (float)cols + eps);
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        const size_t o = (size_t)row * cols + c;
        if (BF16) {
            const float v = bf16_bits_to_f32(static_cast<const uint16_t *>(x)[o]);
            const float w = bf16_bits_to_f32(static_cast<const uint16_t *>(weight)[c]);
            static_cast<uint16_t *>(dst)[o] = f32_to_bf16_bits(v * inv * w);
        } else {
            const float v = static_cast<const float *>(x)[o];
            static_cast<float *>(dst)[o] = v * inv * static_cast<const float *>(weight)[c];
        }
    }
}

// Warp per row, FP64 accumulation of bf16(W) * x, rounded to FP32 once.
__global__ void __launch_bounds__(256) bf16_gemv_kernel(const uint16_t *w, const float *x,
                                                        float *dst, int rows, int cols) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    double acc = 0.0;
    for (int c = lane; c < cols; c += 32)
        acc = fma((double)bf16_bits_to_f32(w[(size_t)row * cols + c]), (double)x[c], acc);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) dst[row] = (float)acc;
}

int elementwise_grid(int n, int sms) {
    const int g = (n + 255) / 256;
    return std::max(1, std::min(g, sms * 8));
}

}  // namespace

cudaError_t launch_rmsnorm_bf16(const void *x, const void *weight, void *dst, int rows, int cols, float epsilon,
                                cudaStream_t stream) {
    rmsnorm_kernel<true><<<rows, 256, 0, stream>>>(x, weight, dst, cols, epsilon);
    return cudaGetLastError();
}

}  // namespace nvfp4

using namespace nvfp4;

// ------------------------------------------------------------ runtime

cudaEvent_t nvfp4_runtime::acquire_event() {
    if (!event_pool.empty()) {
        cudaEvent_t e = event_pool.back();
        event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    check_cuda(cudaEventCreate(&e), "cudaEventCreate");
    return e;
}

void nvfp4_runtime::release_event(cudaEvent_t event) {
    if (event) event_pool.push_back(event);
}

extern "C" NVFP4_API const char *nvfp4_last_error(void) { return last_error_ref().c_str(); }

extern "C" NVFP4_API nvfp4_status nvfp4_runtime_create(const char *kernel_source_path,
                                                       nvfp4_runtime **out_runtime) {
    (void)kernel_source_path;
    if (!out_runtime) return fail_invalid("out_runtime is required");
    *out_runtime = nullptr;
    try {
        auto holder = std::make_unique<nvfp4_runtime>();
        int count = 0;
        check_cuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
        if (count <= 0) throw cuda_error("cudaGetDeviceCount", cudaErrorNoDevice);
        check_cuda(cudaGetDevice(&holder->device), "cudaGetDevice");
        cudaDeviceProp prop{};
        check_cuda(cudaGetDeviceProperties(&prop, holder->device), "cudaGetDeviceProperties");
        if (prop.major < 10)
            throw cuda_error("device check (sm_100a kernels need compute capability 10.x)",
                             cudaErrorNoKernelImageForDevice);
        holder->device_name = prop.name;
        holder->sm_count = prop.multiProcessorCount;
        check_cuda(cudaStreamCreateWithFlags(&holder->stream, cudaStreamNonBlocking),
                   "cudaStreamCreateWithFlags");
        clear_last_error();
        *out_runtime = holder.release();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API void nvfp4_runtime_destroy(nvfp4_runtime *runtime) {
    if (!runtime) return;
    {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        if (runtime->stream) cudaStreamSynchronize(runtime->stream);
        for (auto &ev : runtime->pending) {
            if (ev.start) cudaEventDestroy(ev.start);
            if (ev.end) cudaEventDestroy(ev.end);
        }
        for (cudaEvent_t e : runtime->event_pool) cudaEventDestroy(e);
        if (runtime->epoch_event) cudaEventDestroy(runtime->epoch_event);
        if (runtime->stream) cudaStreamDestroy(runtime->stream);
    }
    delete runtime;
}

extern "C" NVFP4_API const char *nvfp4_runtime_device_name(const nvfp4_runtime *runtime) {
    return runtime ? runtime->device_name.c_str() : "";
}

extern "C" NVFP4_API void *nvfp4_runtime_stream(const nvfp4_runtime *runtime) {
    return runtime ? static_cast<void *>(runtime->stream) : nullptr;
}

extern "C" NVFP4_API int nvfp4_runtime_sm_count(const nvfp4_runtime *runtime) {
    return runtime ? runtime->sm_count : 0;
}

extern "C" NVFP4_API nvfp4_status nvfp4_runtime_query_device(const nvfp4_runtime *runtime,
                                                             nvfp4_device_info *out_info) {
    if (!runtime || !out_info) return fail_invalid("runtime and out_info are required");
    try {
        cudaDeviceProp prop{};
        check_cuda(cudaGetDeviceProperties(&prop, runtime->device), "cudaGetDeviceProperties");
        nvfp4_device_info info{};
        copy_fixed(info.platform_name, sizeof(info.platform_name), "NVIDIA CUDA");
        copy_fixed(info.device_name, sizeof(info.device_name), prop.name);
        copy_fixed(info.device_version, sizeof(info.device_version),
                   "sm_" + std::to_string(prop.major) + std::to_string(prop.minor));
        int driver = 0;
        check_cuda(cudaDriverGetVersion(&driver), "cudaDriverGetVersion");
        copy_fixed(info.driver_version, sizeof(info.driver_version), std::to_string(driver));
        info.global_memory_bytes = prop.totalGlobalMem;
        info.max_allocation_bytes = prop.totalGlobalMem;
        info.global_cache_bytes = static_cast<uint64_t>(prop.l2CacheSize);
        info.local_memory_bytes = prop.sharedMemPerBlockOptin;
        info.compute_units = static_cast<uint32_t>(prop.multiProcessorCount);
        int clock_khz = 0;
        cudaDeviceGetAttribute(&clock_khz, cudaDevAttrClockRate, runtime->device);
        info.max_clock_mhz = static_cast<uint32_t>(clock_khz / 1000);
        info.svm_capabilities = 0;
        *out_info = info;
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_runtime_last_profile(const nvfp4_runtime *runtime,
                                                             nvfp4_profile *out_profile) {
    if (!runtime || !out_profile) return fail_invalid("runtime and out_profile are required");
    std::lock_guard<std::mutex> lock(runtime->queue_mutex);
    *out_profile = runtime->last_profile;
    clear_last_error();
    return NVFP4_STATUS_OK;
}

namespace nvfp4 {

void raise_device_timeouts(nvfp4_runtime *runtime) {
    int timed_out = 0;
    for (auto &word : runtime->error_words) {
        if (*word.first != 0) {
            timed_out = *word.first;
            *word.first = 0;
            check_cuda(cudaMemsetAsync(word.second, 0, sizeof(int), runtime->stream),
                       "cudaMemsetAsync(device error word)");
        }
    }
    if (timed_out) {
        check_cuda(cudaStreamSynchronize(runtime->stream), "cudaStreamSynchronize");
        throw std::runtime_error(
            "an MoE bank kernel gave up waiting on a pipeline barrier (wait site " + std::to_string(timed_out) +
            "); outputs since the previous synchronize are invalid");
    }
}

}  // namespace nvfp4

extern "C" NVFP4_API nvfp4_status nvfp4_runtime_synchronize(nvfp4_runtime *runtime) {
    if (!runtime) return fail_invalid("runtime is required");
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        check_cuda(cudaStreamSynchronize(runtime->stream), "cudaStreamSynchronize");
        std::vector<pending_event> events = std::move(runtime->pending);
        runtime->pending.clear();
        runtime->last_trace.clear();
        uint64_t kernel_ns = 0;
        cudaError_t first_error = cudaSuccess;
        for (pending_event &ev : events) {
            float ms = 0.0f, start_ms = 0.0f;
            cudaError_t err = cudaEventSynchronize(ev.end);
            if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, ev.start, ev.end);
            if (err == cudaSuccess) {
                kernel_ns += static_cast<uint64_t>(ms * 1.0e6);
                if (ev.traced && runtime->epoch_valid &&
                    cudaEventElapsedTime(&start_ms, runtime->epoch_event, ev.start) == cudaSuccess) {
                    nvfp4_trace_event trace{};
                    copy_fixed(trace.scope, sizeof(trace.scope), ev.scope);
                    copy_fixed(trace.operation, sizeof(trace.operation), ev.operation);
                    trace.queued_ns = ev.queued_ns;
                    trace.submit_ns = ev.queued_ns;
                    trace.start_ns = runtime->epoch_host_ns + static_cast<uint64_t>(start_ms * 1.0e6);
                    trace.end_ns = trace.start_ns + static_cast<uint64_t>(ms * 1.0e6);
                    runtime->last_trace.push_back(trace);
                }
            } else if (first_error == cudaSuccess) {
                first_error = err;
            }
            runtime->release_event(ev.start);
            runtime->release_event(ev.end);
        }
        if (runtime->epoch_valid) {
            runtime->release_event(runtime->epoch_event);
            runtime->epoch_event = nullptr;
            runtime->epoch_valid = false;
        }
        check_cuda(first_error, "cudaEventElapsedTime(profile)");
        runtime->last_profile = {0, kernel_ns, 0};
        raise_device_timeouts(runtime);
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_runtime_trace_set_enabled(nvfp4_runtime *runtime,
                                                                  int enabled) {
    if (!runtime || (enabled != 0 && enabled != 1))
        return fail_invalid("runtime and boolean trace state are required");
    std::lock_guard<std::mutex> lock(runtime->queue_mutex);
    runtime->trace_enabled = enabled != 0;
    runtime->trace_scope.clear();
    if (runtime->trace_enabled) runtime->last_trace.clear();
    clear_last_error();
    return NVFP4_STATUS_OK;
}

extern "C" NVFP4_API nvfp4_status nvfp4_runtime_trace_set_scope(nvfp4_runtime *runtime,
                                                                const char *scope) {
    if (!runtime || !scope) return fail_invalid("runtime and trace scope are required");
    const size_t length = std::strlen(scope);
    if (length >= NVFP4_TRACE_SCOPE_CAPACITY)
        return fail_invalid("trace scope exceeds NVFP4_TRACE_SCOPE_CAPACITY");
    std::lock_guard<std::mutex> lock(runtime->queue_mutex);
    if (!runtime->trace_enabled) return fail_invalid("trace scope requires tracing to be enabled");
    runtime->trace_scope.assign(scope, length);
    clear_last_error();
    return NVFP4_STATUS_OK;
}

extern "C" NVFP4_API size_t nvfp4_runtime_trace_count(const nvfp4_runtime *runtime) {
    if (!runtime) return 0;
    std::lock_guard<std::mutex> lock(runtime->queue_mutex);
    return runtime->last_trace.size();
}

extern "C" NVFP4_API nvfp4_status nvfp4_runtime_trace_read(const nvfp4_runtime *runtime,
                                                           size_t index,
                                                           nvfp4_trace_event *out_event) {
    if (!runtime || !out_event) return fail_invalid("runtime and trace output are required");
    std::lock_guard<std::mutex> lock(runtime->queue_mutex);
    if (index >= runtime->last_trace.size()) return fail_invalid("trace event index is out of range");
    *out_event = runtime->last_trace[index];
    clear_last_error();
    return NVFP4_STATUS_OK;
}

// ------------------------------------------------------------ buffers

extern "C" NVFP4_API nvfp4_status nvfp4_buffer_create(nvfp4_runtime *runtime, size_t bytes,
                                                      nvfp4_buffer **out_buffer) {
    if (!runtime || bytes == 0 || !out_buffer) return fail_invalid("invalid device-buffer arguments");
    *out_buffer = nullptr;
    try {
        auto holder = std::make_unique<nvfp4_buffer>();
        holder->runtime = runtime;
        holder->bytes = bytes;
        check_cuda(cudaMalloc(&holder->data, bytes), "cudaMalloc(device_buffer)");
        clear_last_error();
        *out_buffer = holder.release();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API void nvfp4_buffer_destroy(nvfp4_buffer *buffer) {
    if (!buffer) return;
    if (buffer->data) {
        if (buffer->runtime) {
            std::lock_guard<std::mutex> lock(buffer->runtime->queue_mutex);
            cudaStreamSynchronize(buffer->runtime->stream);
        }
        cudaFree(buffer->data);
    }
    delete buffer;
}

extern "C" NVFP4_API void *nvfp4_buffer_device_pointer(const nvfp4_buffer *buffer) {
    return buffer ? buffer->data : nullptr;
}

extern "C" NVFP4_API size_t nvfp4_buffer_bytes(const nvfp4_buffer *buffer) {
    return buffer ? buffer->bytes : 0;
}

extern "C" NVFP4_API nvfp4_status nvfp4_buffer_upload(nvfp4_buffer *buffer, size_t offset,
                                                      const void *data, size_t bytes) {
    if (!buffer || !buffer->runtime || !data || bytes == 0 || offset > buffer->bytes ||
        bytes > buffer->bytes - offset)
        return fail_invalid("invalid device-buffer upload");
    try {
        nvfp4_runtime *rt = buffer->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        cudaEvent_t a = rt->acquire_event(), b = rt->acquire_event();
        check_cuda(cudaEventRecord(a, rt->stream), "cudaEventRecord");
        check_cuda(cudaMemcpyAsync(static_cast<uint8_t *>(buffer->data) + offset, data, bytes,
                                   cudaMemcpyHostToDevice, rt->stream),
                   "cudaMemcpyAsync(buffer_upload)");
        check_cuda(cudaEventRecord(b, rt->stream), "cudaEventRecord");
        check_cuda(cudaEventSynchronize(b), "cudaEventSynchronize(buffer_upload)");
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, a, b);
        rt->release_event(a);
        rt->release_event(b);
        rt->last_profile = {static_cast<uint64_t>(ms * 1.0e6), 0, 0};
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_buffer_download(const nvfp4_buffer *buffer, size_t offset,
                                                        void *data, size_t bytes) {
    if (!buffer || !buffer->runtime || !data || bytes == 0 || offset > buffer->bytes ||
        bytes > buffer->bytes - offset)
        return fail_invalid("invalid device-buffer download");
    try {
        nvfp4_runtime *rt = buffer->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        cudaEvent_t a = rt->acquire_event(), b = rt->acquire_event();
        check_cuda(cudaEventRecord(a, rt->stream), "cudaEventRecord");
        check_cuda(cudaMemcpyAsync(data, static_cast<const uint8_t *>(buffer->data) + offset, bytes,
                                   cudaMemcpyDeviceToHost, rt->stream),
                   "cudaMemcpyAsync(buffer_download)");
        check_cuda(cudaEventRecord(b, rt->stream), "cudaEventRecord");
        check_cuda(cudaEventSynchronize(b), "cudaEventSynchronize(buffer_download)");
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, a, b);
        rt->release_event(a);
        rt->release_event(b);
        rt->last_profile = {0, 0, static_cast<uint64_t>(ms * 1.0e6)};
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_buffer_copy_enqueue(const nvfp4_buffer *source,
                                                            size_t source_offset,
                                                            nvfp4_buffer *destination,
                                                            size_t destination_offset,
                                                            size_t bytes) {
    if (!source || !destination || !source->runtime || destination->runtime != source->runtime ||
        bytes == 0 || source_offset > source->bytes || bytes > source->bytes - source_offset ||
        destination_offset > destination->bytes || bytes > destination->bytes - destination_offset)
        return fail_invalid("invalid device-buffer copy range");
    try {
        nvfp4_runtime *rt = source->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        rt->profiled("buffer_copy", nullptr, [&](cudaStream_t s) {
            check_cuda(cudaMemcpyAsync(static_cast<uint8_t *>(destination->data) + destination_offset,
                                       static_cast<const uint8_t *>(source->data) + source_offset,
                                       bytes, cudaMemcpyDeviceToDevice, s),
                       "cudaMemcpyAsync(buffer_copy)");
        });
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

// ------------------------------------------------------ graph primitives

namespace {
bool same_runtime(const nvfp4_runtime *rt, const nvfp4_buffer *b) { return b && b->runtime == rt; }
}  // namespace

extern "C" NVFP4_API nvfp4_status nvfp4_add_device_enqueue_f32(nvfp4_runtime *runtime,
                                                               const nvfp4_buffer *a,
                                                               const nvfp4_buffer *b, int elements,
                                                               nvfp4_buffer *dst) {
    const size_t bytes = elements > 0 ? static_cast<size_t>(elements) * sizeof(float) : 0;
    if (!runtime || !same_runtime(runtime, a) || !same_runtime(runtime, b) ||
        !same_runtime(runtime, dst) || elements <= 0 || a->bytes < bytes || b->bytes < bytes ||
        dst->bytes < bytes)
        return fail_invalid("invalid enqueued add buffers or element count");
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        runtime->profiled("add", nullptr, [&](cudaStream_t s) {
            add_f32_kernel<<<elementwise_grid(elements, runtime->sm_count), 256, 0, s>>>(
                static_cast<const float *>(a->data), static_cast<const float *>(b->data),
                static_cast<float *>(dst->data), elements);
            check_cuda(cudaGetLastError(), "add_f32_kernel");
        });
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_weighted_accumulate_device_enqueue_f32(
    nvfp4_runtime *runtime, const nvfp4_buffer *source, float scale, nvfp4_buffer *dst,
    int elements, int reset) {
    const size_t bytes = elements > 0 ? static_cast<size_t>(elements) * sizeof(float) : 0;
    if (!runtime || !same_runtime(runtime, source) || !same_runtime(runtime, dst) ||
        elements <= 0 || source->bytes < bytes || dst->bytes < bytes || (reset != 0 && reset != 1))
        return fail_invalid("invalid weighted-accumulate buffers or arguments");
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        runtime->profiled("weighted_accumulate", nullptr, [&](cudaStream_t s) {
            weighted_accumulate_f32_kernel<<<elementwise_grid(elements, runtime->sm_count), 256, 0, s>>>(
                static_cast<const float *>(source->data), scale, static_cast<float *>(dst->data),
                elements, reset);
            check_cuda(cudaGetLastError(), "weighted_accumulate_f32_kernel");
        });
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_silu_mul_device_enqueue_f32(nvfp4_runtime *runtime,
                                                                    const nvfp4_buffer *gate,
                                                                    const nvfp4_buffer *up,
                                                                    int elements, nvfp4_buffer *dst) {
    const size_t bytes = elements > 0 ? static_cast<size_t>(elements) * sizeof(float) : 0;
    if (!runtime || !same_runtime(runtime, gate) || !same_runtime(runtime, up) ||
        !same_runtime(runtime, dst) || elements <= 0 || gate->bytes < bytes || up->bytes < bytes ||
        dst->bytes < bytes)
        return fail_invalid("invalid enqueued SiLU-multiply buffers or element count");
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        runtime->profiled("silu_mul", nullptr, [&](cudaStream_t s) {
            silu_mul_f32_kernel<<<elementwise_grid(elements, runtime->sm_count), 256, 0, s>>>(
                static_cast<const float *>(gate->data), static_cast<const float *>(up->data),
                static_cast<float *>(dst->data), elements);
            check_cuda(cudaGetLastError(), "silu_mul_f32_kernel");
        });
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

namespace {
nvfp4_status rmsnorm_enqueue(nvfp4_runtime *runtime, const nvfp4_buffer *x,
                             const nvfp4_buffer *weight, int rows, int cols, float epsilon,
                             nvfp4_buffer *dst, bool bf16) {
    const size_t elem = bf16 ? 2 : 4;
    if (!runtime || !same_runtime(runtime, x) || !same_runtime(runtime, weight) ||
        !same_runtime(runtime, dst) || rows <= 0 || cols <= 0 || epsilon < 0.0f ||
        static_cast<size_t>(rows) > std::numeric_limits<size_t>::max() / static_cast<size_t>(cols) / elem)
        return fail_invalid("invalid enqueued RMSNorm arguments");
    const size_t bytes = static_cast<size_t>(rows) * cols * elem;
    if (x->bytes < bytes || weight->bytes < static_cast<size_t>(cols) * elem || dst->bytes < bytes)
        return fail_invalid("enqueued RMSNorm buffer capacity is too small");
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        runtime->profiled(bf16 ? "rmsnorm_bf16" : "rmsnorm", nullptr, [&](cudaStream_t s) {
            if (bf16)
                rmsnorm_kernel<true><<<rows, 256, 0, s>>>(x->data, weight->data, dst->data, cols, epsilon);
            else
                rmsnorm_kernel<false><<<rows, 256, 0, s>>>(x->data, weight->data, dst->data, cols, epsilon);
            check_cuda(cudaGetLastError(), "rmsnorm_kernel");
        });
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}
}  // namespace

extern "C" NVFP4_API nvfp4_status nvfp4_rmsnorm_device_enqueue_f32(nvfp4_runtime *runtime,
                                                                   const nvfp4_buffer *x,
                                                                   const nvfp4_buffer *weight,
                                                                   int rows, int cols, float epsilon,
                                                                   nvfp4_buffer *dst) {
    return rmsnorm_enqueue(runtime, x, weight, rows, cols, epsilon, dst, false);
}

extern "C" NVFP4_API nvfp4_status nvfp4_rmsnorm_device_enqueue_bf16(nvfp4_runtime *runtime,
                                                                    const nvfp4_buffer *x,
                                                                    const nvfp4_buffer *weight,
                                                                    int rows, int cols, float epsilon,
                                                                    nvfp4_buffer *dst) {
    return rmsnorm_enqueue(runtime, x, weight, rows, cols, epsilon, dst, true);
}

extern "C" NVFP4_API nvfp4_status nvfp4_rmsnorm_ptr_bf16(nvfp4_runtime *runtime, const void *x_bf16,
                                                         const void *weight_bf16, int rows, int cols, float epsilon,
                                                         void *dst_bf16, void *stream) {
    if (!runtime || !x_bf16 || !weight_bf16 || !dst_bf16 || rows <= 0 || cols <= 0 || epsilon < 0.0f)
        return fail_invalid("invalid RMSNorm arguments");
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        runtime->direct_call(static_cast<cudaStream_t>(stream), [&](cudaStream_t s) {
            rmsnorm_kernel<true><<<rows, 256, 0, s>>>(x_bf16, weight_bf16, dst_bf16, cols, epsilon);
            check_cuda(cudaGetLastError(), "rmsnorm_kernel");
        });
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_bf16_gemv_device_enqueue(nvfp4_runtime *runtime,
                                                                 const nvfp4_buffer *weights,
                                                                 const nvfp4_buffer *x, int rows,
                                                                 int cols, nvfp4_buffer *dst) {
    if (!runtime || !same_runtime(runtime, weights) || !same_runtime(runtime, x) ||
        !same_runtime(runtime, dst) || rows <= 0 || cols <= 0 ||
        static_cast<size_t>(rows) > std::numeric_limits<size_t>::max() / static_cast<size_t>(cols) / 2)
        return fail_invalid("invalid BF16 GEMV arguments");
    if (weights->bytes < static_cast<size_t>(rows) * cols * 2 ||
        x->bytes < static_cast<size_t>(cols) * 4 || dst->bytes < static_cast<size_t>(rows) * 4)
        return fail_invalid("BF16 GEMV buffer capacity is too small");
    try {
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        runtime->profiled("bf16_gemv", nullptr, [&](cudaStream_t s) {
            bf16_gemv_kernel<<<(rows + 7) / 8, 256, 0, s>>>(static_cast<const uint16_t *>(weights->data),
                                                          static_cast<const float *>(x->data),
                                                          static_cast<float *>(dst->data), rows, cols);
            check_cuda(cudaGetLastError(), "bf16_gemv_kernel");
        });
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}
