// Host-side internals shared by the translation units of libnvfp4_moe_cuda.so.
#pragma once

#include "../../include/nvfp4_runtime.h"

#include <cuda_runtime.h>

#include <chrono>
#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace nvfp4 {

// Failure of a CUDA runtime call; mapped to NVFP4_STATUS_CUDA_ERROR.
struct cuda_error : std::runtime_error {
    cuda_error(const char *operation, cudaError_t code)
        : std::runtime_error(std::string(operation) + " failed: " + cudaGetErrorName(code) + " (" +
                             cudaGetErrorString(code) + ")") {}
};

// Invalid caller input detected after the entry point's own argument checks.
struct invalid_argument_error : std::runtime_error {
    using std::runtime_error::runtime_error;
};

inline void check_cuda(cudaError_t code, const char *operation) {
    if (code != cudaSuccess) throw cuda_error(operation, code);
}

const std::string &last_error_ref();
void set_last_error(const std::string &message);
void clear_last_error();
nvfp4_status fail_invalid(const char *message);
nvfp4_status fail_exception(const std::exception &error);

// Operations beyond this many between two synchronize calls run unprofiled.
constexpr size_t kMaxPendingEvents = 1u << 16;

// One enqueued operation whose device duration is harvested at synchronize.
struct pending_event {
    cudaEvent_t start = nullptr;
    cudaEvent_t end = nullptr;
    bool traced = false;
    std::string scope;
    std::string operation;
    uint64_t queued_ns = 0;
};

}  // namespace nvfp4

struct nvfp4_runtime {
    int device = 0;
    int sm_count = 0;
    std::string device_name;
    cudaStream_t stream = nullptr;
    mutable std::mutex queue_mutex;
    bool trace_enabled = false;
    std::string trace_scope;
    std::vector<nvfp4::pending_event> pending;
    std::vector<cudaEvent_t> event_pool;
    std::vector<nvfp4_trace_event> last_trace;
    nvfp4_profile last_profile{0, 0, 0};
    // Device-side timeout words of the banks on this runtime: a pinned
    // host-mapped copy that kernels store to, and the device word they poll.
    std::vector<std::pair<volatile int *, int *>> error_words;
    cudaEvent_t epoch_event = nullptr;      // device-time origin of the trace
    uint64_t epoch_host_ns = 0;             // host clock when epoch was recorded
    bool epoch_valid = false;

    cudaEvent_t acquire_event();
    void release_event(cudaEvent_t event);
    // Record an event pair around `launch` on `on_stream` (the runtime stream
    // when null). Caller holds queue_mutex. Nothing is recorded while the
    // stream is being captured into a CUDA graph.
    template <typename F>
    void profiled(const char *operation, cudaStream_t on_stream, F &&launch);
    // Per-kernel pairs when tracing, one pair per API call otherwise.
    template <typename F>
    void profiled_kernel(const char *operation, cudaStream_t on_stream, F &&launch) {
        if (trace_enabled) profiled(operation, on_stream, launch);
        else launch(on_stream ? on_stream : stream);
    }
    // Serving entry points (raw-pointer and expert-parallel forwards, the
    // finalize step): no per-call event pair, which would sit between the
    // caller's previous kernel and this call's first one; with tracing
    // enabled every kernel still gets its own pair (profiled_kernel).
    template <typename F>
    void direct_call(cudaStream_t on_stream, F &&launch) {
        launch(on_stream ? on_stream : stream);
    }
    template <typename F>
    void profiled_call(const char *operation, cudaStream_t on_stream, F &&launch) {
        if (trace_enabled) launch(on_stream ? on_stream : stream);
        else profiled(operation, on_stream, launch);
    }
};

struct nvfp4_buffer {
    nvfp4_runtime *runtime = nullptr;
    void *data = nullptr;
    size_t bytes = 0;
};

namespace nvfp4 {

// After the runtime stream has drained: throws when a kernel of a bank on
// this runtime recorded a bounded wait that ran out (its wait-site code is
// in the message) and clears the words. Caller holds queue_mutex.
void raise_device_timeouts(nvfp4_runtime *runtime);

// The BF16 RMSNorm kernel of nvfp4_rmsnorm_ptr_bf16 (runtime.cu), one CTA per row.
cudaError_t launch_rmsnorm_bf16(const void *x, const void *weight, void *dst, int rows, int cols, float epsilon,
                                cudaStream_t stream);

inline uint64_t host_now_ns() {
    return static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                     std::chrono::steady_clock::now().time_since_epoch())
                                     .count());
}

}  // namespace nvfp4

template <typename F>
void nvfp4_runtime::profiled(const char *operation, cudaStream_t on_stream, F &&launch) {
    cudaStream_t s = on_stream ? on_stream : stream;
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &capture) != cudaSuccess) capture = cudaStreamCaptureStatusNone;
    if (pending.size() >= nvfp4::kMaxPendingEvents || capture != cudaStreamCaptureStatusNone) {
        launch(s);
        return;
    }
    nvfp4::pending_event ev;
    ev.queued_ns = nvfp4::host_now_ns();
    if (!epoch_valid) {
        epoch_event = acquire_event();
        nvfp4::check_cuda(cudaEventRecord(epoch_event, s), "cudaEventRecord(epoch)");
        epoch_host_ns = ev.queued_ns;
        epoch_valid = true;
    }
    ev.start = acquire_event();
    ev.end = acquire_event();
    nvfp4::check_cuda(cudaEventRecord(ev.start, s), "cudaEventRecord(start)");
    launch(s);
    nvfp4::check_cuda(cudaEventRecord(ev.end, s), "cudaEventRecord(end)");
    ev.traced = trace_enabled;
    if (ev.traced) {
        ev.scope = trace_scope;
        ev.operation = operation;
    }
    pending.push_back(std::move(ev));
}
