/*
 * nvfp4_runtime.h - C ABI of the B200 (sm_100a) NVFP4 mixture-of-experts bank.
 *
 * This is a drop-in replacement for the MoE-bank slice of the lab runtime's
 * C ABI (native_nvfp4/runtime/nvfp4_runtime.h in hotschmoe/x2-nvfp4-lab).
 * Every symbol marked "reference:" keeps the reference's name, argument order,
 * argument meaning and status codes; the line cited is the declaration it
 * replaces. Symbols marked "additive:" have no reference counterpart; they
 * follow the same conventions (status return, thread-local last error,
 * asynchronous enqueue on the runtime's in-order stream).
 *
 * Conventions shared by every entry point
 *  - Functions return nvfp4_status; on failure nvfp4_last_error() returns a
 *    thread-local message. It is cleared by the next successful call.
 *  - "enqueue" functions are asynchronous on the runtime's single in-order
 *    CUDA stream; results are valid after nvfp4_runtime_synchronize().
 *  - Host arrays passed to upload functions are copied before the call
 *    returns; the caller may free them afterwards.
 *  - A runtime must outlive every buffer and bank created from it.
 *  - There is no CPU execution path: every compute entry point launches CUDA
 *    kernels built for sm_100a and fails with NVFP4_STATUS_CUDA_ERROR when no
 *    such device is present.
 */
#ifndef NVFP4_RUNTIME_H
#define NVFP4_RUNTIME_H

#include <stddef.h>
#include <stdint.h>

#define NVFP4_API __attribute__((visibility("default")))

#ifdef __cplusplus
extern "C" {
#endif

/* reference: nvfp4_runtime.h:21,23,25 (opaque handles). */
typedef struct nvfp4_runtime nvfp4_runtime;
typedef struct nvfp4_moe_bank nvfp4_moe_bank;
typedef struct nvfp4_buffer nvfp4_buffer;
typedef struct nvfp4_ep nvfp4_ep;
/* reference: nvfp4_runtime.h:22 (dense NVFP4 weight matrix). */
typedef struct nvfp4_matrix nvfp4_matrix;

/* reference: nvfp4_runtime.h:33-39. Code 2 keeps its slot; on this backend it
 * reports a CUDA runtime error instead of an OpenCL one. */
typedef enum nvfp4_status {
    NVFP4_STATUS_OK = 0,
    NVFP4_STATUS_INVALID_ARGUMENT = 1,
    NVFP4_STATUS_OPENCL_ERROR = 2,
    NVFP4_STATUS_CUDA_ERROR = 2,
    NVFP4_STATUS_IO_ERROR = 3,
    NVFP4_STATUS_INTERNAL_ERROR = 4,
} nvfp4_status;

/* reference: nvfp4_runtime.h:41-46. The linear entry points keep the
 * reference's rules for these kinds (TILED needs more than one vector,
 * ROW_TILED exactly one); every kind runs the same sm_100a kernel. */
typedef enum nvfp4_kernel_kind {
    NVFP4_KERNEL_SCALAR = 0,
    NVFP4_KERNEL_SUBGROUP = 1,
    NVFP4_KERNEL_TILED = 2,
    NVFP4_KERNEL_ROW_TILED = 3,
} nvfp4_kernel_kind;

/* reference: nvfp4_runtime.h:48-52. kernel_ns is the summed device time of
 * the operations enqueued since the previous synchronize. */
typedef struct nvfp4_profile {
    uint64_t upload_ns;
    uint64_t kernel_ns;
    uint64_t download_ns;
} nvfp4_profile;

/* reference: nvfp4_runtime.h:54-66. */
enum {
    NVFP4_TRACE_SCOPE_CAPACITY = 96,
    NVFP4_TRACE_OPERATION_CAPACITY = 64,
};

typedef struct nvfp4_trace_event {
    char scope[NVFP4_TRACE_SCOPE_CAPACITY];
    char operation[NVFP4_TRACE_OPERATION_CAPACITY];
    uint64_t queued_ns;
    uint64_t submit_ns;
    uint64_t start_ns;
    uint64_t end_ns;
} nvfp4_trace_event;

/* reference: nvfp4_runtime.h:75-87. svm_capabilities is always 0 here. */
typedef struct nvfp4_device_info {
    char platform_name[256];
    char device_name[256];
    char device_version[256];
    char driver_version[256];
    uint64_t global_memory_bytes;
    uint64_t max_allocation_bytes;
    uint64_t global_cache_bytes;
    uint64_t local_memory_bytes;
    uint32_t compute_units;
    uint32_t max_clock_mhz;
    uint32_t svm_capabilities;
} nvfp4_device_info;

/* ---------------------------------------------------------------- runtime */

/* reference: nvfp4_runtime.h:91-93. kernel_source_path is accepted for
 * signature compatibility and ignored (kernels are compiled ahead of time);
 * it may be NULL. Binds the current CUDA device and creates one in-order
 * non-blocking stream. */
NVFP4_API nvfp4_status nvfp4_runtime_create(
    const char * kernel_source_path,
    nvfp4_runtime ** out_runtime);

/* reference: nvfp4_runtime.h:95-100. */
NVFP4_API void nvfp4_runtime_destroy(nvfp4_runtime * runtime);
NVFP4_API const char * nvfp4_runtime_device_name(const nvfp4_runtime * runtime);
NVFP4_API const char * nvfp4_last_error(void);
NVFP4_API nvfp4_status nvfp4_runtime_last_profile(
    const nvfp4_runtime * runtime,
    nvfp4_profile * out_profile);

/* reference: nvfp4_runtime.h:102-104. */
NVFP4_API nvfp4_status nvfp4_runtime_query_device(
    const nvfp4_runtime * runtime,
    nvfp4_device_info * out_info);

/* reference: nvfp4_runtime.h:106. Waits for the stream, then publishes
 * last_profile.kernel_ns and (when tracing) the completed trace. */
NVFP4_API nvfp4_status nvfp4_runtime_synchronize(nvfp4_runtime * runtime);

/* reference: nvfp4_runtime.h:111-122. Trace timestamps come from CUDA event
 * pairs around each enqueued operation. */
NVFP4_API nvfp4_status nvfp4_runtime_trace_set_enabled(
    nvfp4_runtime * runtime,
    int enabled);
NVFP4_API nvfp4_status nvfp4_runtime_trace_set_scope(
    nvfp4_runtime * runtime,
    const char * scope);
NVFP4_API size_t nvfp4_runtime_trace_count(
    const nvfp4_runtime * runtime);
NVFP4_API nvfp4_status nvfp4_runtime_trace_read(
    const nvfp4_runtime * runtime,
    size_t index,
    nvfp4_trace_event * out_event);

/* additive: the runtime's cudaStream_t, so a host framework can order its
 * own work against the runtime's queue. */
NVFP4_API void * nvfp4_runtime_stream(const nvfp4_runtime * runtime);

/* additive: number of streaming multiprocessors of the bound device. */
NVFP4_API int nvfp4_runtime_sm_count(const nvfp4_runtime * runtime);

/* ---------------------------------------------------------------- buffers */

/* reference: nvfp4_runtime.h:179-203. Device memory from cudaMalloc. */
NVFP4_API nvfp4_status nvfp4_buffer_create(
    nvfp4_runtime * runtime,
    size_t bytes,
    nvfp4_buffer ** out_buffer);
NVFP4_API void nvfp4_buffer_destroy(nvfp4_buffer * buffer);
NVFP4_API nvfp4_status nvfp4_buffer_upload(
    nvfp4_buffer * buffer,
    size_t offset,
    const void * data,
    size_t bytes);
NVFP4_API nvfp4_status nvfp4_buffer_download(
    const nvfp4_buffer * buffer,
    size_t offset,
    void * data,
    size_t bytes);
NVFP4_API nvfp4_status nvfp4_buffer_copy_enqueue(
    const nvfp4_buffer * source,
    size_t source_offset,
    nvfp4_buffer * destination,
    size_t destination_offset,
    size_t bytes);

/* additive: the buffer's device address and its size in bytes. */
NVFP4_API void * nvfp4_buffer_device_pointer(const nvfp4_buffer * buffer);
NVFP4_API size_t nvfp4_buffer_bytes(const nvfp4_buffer * buffer);

/* ------------------------------------------------------ graph primitives */

/* reference: nvfp4_runtime.h:345-350. dst[i] = a[i] + b[i]. */
NVFP4_API nvfp4_status nvfp4_add_device_enqueue_f32(
    nvfp4_runtime * runtime,
    const nvfp4_buffer * a,
    const nvfp4_buffer * b,
    int elements,
    nvfp4_buffer * dst);

/* reference: nvfp4_runtime.h:352-358. dst = (reset ? 0 : dst) + scale*source. */
NVFP4_API nvfp4_status nvfp4_weighted_accumulate_device_enqueue_f32(
    nvfp4_runtime * runtime,
    const nvfp4_buffer * source,
    float scale,
    nvfp4_buffer * dst,
    int elements,
    int reset);

/* reference: nvfp4_runtime.h:360-365. dst = gate*sigmoid(gate)*up. */
NVFP4_API nvfp4_status nvfp4_silu_mul_device_enqueue_f32(
    nvfp4_runtime * runtime,
    const nvfp4_buffer * gate,
    const nvfp4_buffer * up,
    int elements,
    nvfp4_buffer * dst);

/* reference: nvfp4_runtime.h:367-374. Row-wise FP32 RMSNorm. */
NVFP4_API nvfp4_status nvfp4_rmsnorm_device_enqueue_f32(
    nvfp4_runtime * runtime,
    const nvfp4_buffer * x,
    const nvfp4_buffer * weight,
    int rows,
    int cols,
    float epsilon,
    nvfp4_buffer * dst);

/* reference: nvfp4_runtime.h:384-390. dst[r] = sum_c bf16(W[r,c]) * x[c]
 * with x FP32; products accumulate in FP64 and round to FP32 once. */
NVFP4_API nvfp4_status nvfp4_bf16_gemv_device_enqueue(
    nvfp4_runtime * runtime,
    const nvfp4_buffer * weights,
    const nvfp4_buffer * x,
    int rows,
    int cols,
    nvfp4_buffer * dst);

/* additive: BF16 RMSNorm over [rows, cols] with an FP32 statistic and a BF16
 * weight, BF16 output (the pre-norm of the resident layer stack). */
NVFP4_API nvfp4_status nvfp4_rmsnorm_device_enqueue_bf16(
    nvfp4_runtime * runtime,
    const nvfp4_buffer * x,
    const nvfp4_buffer * weight,
    int rows,
    int cols,
    float epsilon,
    nvfp4_buffer * dst);

/* additive: the same BF16 RMSNorm on raw device pointers (x, dst BF16
 * [rows, cols], weight BF16 [cols]), enqueued on `stream` (a cudaStream_t;
 * NULL selects the runtime's stream): the per-layer pre-norm of a resident
 * layer stack driven from a host framework's tensors (the lab's full-model
 * driver, native_nvfp4/bench_moe_full_model.py:388-395, norms each layer's
 * input before its bank). Statistic per row: FP32 fmaf partial sums of 256
 * column-strided threads, xor butterfly per warp, warp sums in order, then
 * rsqrtf(mean + epsilon). */
NVFP4_API nvfp4_status nvfp4_rmsnorm_ptr_bf16(
    nvfp4_runtime * runtime,
    const void * x_bf16,
    const void * weight_bf16,
    int rows,
    int cols,
    float epsilon,
    void * dst_bf16,
    void * stream);

/* ------------------------------------------------------- dense NVFP4 linear
 * dst[v, r] = sum_c E2M1(W[r, c]) * E4M3(S[r, c/16]) * x[v, c] /
 * weight_global_scale, x FP32 [vectors, cols] and dst FP32 [vectors, rows],
 * both row-major (the weight path of the lab's vLLM NvFp4LinearKernel
 * provider, vllm_nvfp4_opencl/linear.py:15-70; bias stays the adapter's job).
 * Products of weight and scale are exact; the sum is FP32. */

/* reference: nvfp4_runtime.h:208-217 (nvfp4_runtime.cpp:1705-1735). The
 * compressed-tensors representation: packed [rows, cols/2] E2M1 pairs (low
 * nibble = even column), scales_e4m3 [rows, cols/16]; cols a multiple of 16.
 * Copied to device memory before returning (scale bytes sanitised: sign
 * cleared, 0x7F -> 0). This backend supports cols <= 49152. */
NVFP4_API nvfp4_status nvfp4_matrix_upload(
    nvfp4_runtime * runtime,
    const uint8_t * packed,
    size_t packed_bytes,
    const uint8_t * scales_e4m3,
    size_t scale_bytes,
    int rows,
    int cols,
    float weight_global_scale,
    nvfp4_matrix ** out_matrix);

/* reference: nvfp4_runtime.h:238 (nvfp4_runtime.cpp:2106-2108). Drains the
 * runtime stream first. */
NVFP4_API void nvfp4_matrix_destroy(nvfp4_matrix * matrix);

/* reference: nvfp4_runtime.h:240-248 (nvfp4_runtime.cpp:2110-2183).
 * Synchronous, host x and dst; last_profile gets the upload, kernel and
 * download times. On this backend NVFP4_KERNEL_SCALAR runs a CUDA-core kernel
 * on the FP32 activations; every other kind (and nvfp4_linear_ptr_f32) runs
 * the tcgen05 kernel, the activations as six NVFP4 terms per vector (within
 * ~2e-6 of the output scale). Calls on one matrix share its activation-term
 * buffers and must not overlap on the GPU. */
NVFP4_API nvfp4_status nvfp4_linear_f32(
    nvfp4_runtime * runtime,
    const nvfp4_matrix * matrix,
    const float * x,
    int vectors,
    float * dst,
    nvfp4_kernel_kind kernel_kind);

/* reference: nvfp4_runtime.h:250-256 (nvfp4_runtime.cpp:2185-2231).
 * Device buffers; waits for the kernel; last_profile.kernel_ns. */
NVFP4_API nvfp4_status nvfp4_linear_device_f32(
    nvfp4_runtime * runtime,
    const nvfp4_matrix * matrix,
    const nvfp4_buffer * x,
    int vectors,
    nvfp4_buffer * dst,
    nvfp4_kernel_kind kernel_kind);

/* reference: nvfp4_runtime.h:258-264 (nvfp4_runtime.cpp:2233-2270).
 * Enqueued on the runtime stream. */
NVFP4_API nvfp4_status nvfp4_linear_device_enqueue_f32(
    nvfp4_runtime * runtime,
    const nvfp4_matrix * matrix,
    const nvfp4_buffer * x,
    int vectors,
    nvfp4_buffer * dst,
    nvfp4_kernel_kind kernel_kind);

/* additive: the same linear on raw device pointers (x FP32 [vectors, cols],
 * dst FP32 [vectors, rows]) enqueued on `stream` (a cudaStream_t; NULL
 * selects the runtime's stream): the path of the torch-facing provider,
 * whose activations are already device tensors. */
NVFP4_API nvfp4_status nvfp4_linear_ptr_f32(
    nvfp4_runtime * runtime,
    const nvfp4_matrix * matrix,
    const float * x,
    int vectors,
    float * dst,
    void * stream);

/* ------------------------------------------------------------- MoE bank */

/* reference: nvfp4_runtime.h:392-403 (implemented at
 * native_nvfp4/runtime/nvfp4_runtime.cpp:1780-1856). Expert indices
 * [0, experts) are routed; index `experts` is the always-on shared expert.
 * experts in [8,256]; hidden and intermediate positive multiples of 16;
 * router_bytes == experts*hidden*2; shared_gate_bytes == hidden*2.
 * This backend additionally needs hidden and intermediate to be multiples
 * of 128 and reports INVALID_ARGUMENT otherwise. */
NVFP4_API nvfp4_status nvfp4_moe_bank_create(
    nvfp4_runtime * runtime,
    const uint16_t * router_bf16,
    size_t router_bytes,
    const uint16_t * shared_gate_bf16,
    size_t shared_gate_bytes,
    int experts,
    int hidden,
    int intermediate,
    nvfp4_moe_bank ** out_bank);

/* reference: nvfp4_runtime.h:405-414 (nvfp4_runtime.cpp:1858-1911).
 * projection: 0=gate [intermediate,hidden], 1=up [intermediate,hidden],
 * 2=down [hidden,intermediate]. packed is row-major E2M1 pairs (low nibble =
 * even column), scales_e4m3 one byte per 16 columns. weight_global_scale is a
 * divisor: dequantised w = E2M1 * E4M3(scale) / weight_global_scale.
 * Scale bytes are stored with the sign bit cleared and 0x7F mapped to 0, the
 * reference's scale-decoding rule (nvfp4_gemv.cl:14-27). Synchronises the
 * runtime stream before writing, as the reference does. */
NVFP4_API nvfp4_status nvfp4_moe_bank_upload_projection(
    nvfp4_moe_bank * bank,
    int expert,
    int projection,
    const uint8_t * packed,
    size_t packed_bytes,
    const uint8_t * scales_e4m3,
    size_t scale_bytes,
    float weight_global_scale);

/* reference: nvfp4_runtime.h:416-419 (nvfp4_runtime.cpp:1913-2074).
 * Single-token decode: x FP32 [hidden], dst FP32 [hidden] =
 * sum_k w_k * expert_k(x) + sigmoid(shared_gate . x) * shared(x), without
 * the residual. Requires every routed and shared projection uploaded. */
NVFP4_API nvfp4_status nvfp4_moe_bank_decode_device_enqueue_f32(
    nvfp4_moe_bank * bank,
    const nvfp4_buffer * x,
    nvfp4_buffer * dst);

/* reference: nvfp4_runtime.h:421 (nvfp4_runtime.cpp:2076-2082). Drains the
 * stream first. */
NVFP4_API void nvfp4_moe_bank_destroy(nvfp4_moe_bank * bank);

/* additive: upload one projection from DEVICE memory (same layout and
 * semantics as nvfp4_moe_bank_upload_projection). Enqueued on the runtime
 * stream; the source must stay valid until the next synchronize. */
NVFP4_API nvfp4_status nvfp4_moe_bank_upload_projection_device(
    nvfp4_moe_bank * bank,
    int expert,
    int projection,
    const void * packed_device,
    size_t packed_bytes,
    const void * scales_device,
    size_t scale_bytes,
    float weight_global_scale);

/* additive: flags for the batched forward. */
enum {
    NVFP4_MOE_ADD_RESIDUAL = 1u << 0,
    /* dst is FP32 [tokens, hidden] and receives this bank's partial sum: the
     * experts of its range (nvfp4_moe_bank_set_expert_range), plus the
     * residual when NVFP4_MOE_ADD_RESIDUAL is set. Summing the partials of
     * banks whose ranges cover every expert once (and one of which computes
     * the shared expert) gives the layer output. */
    NVFP4_MOE_PARTIAL_F32 = 1u << 1,
    /* x is normalised first (RMSNorm with the bank's weight and epsilon,
     * nvfp4_moe_bank_set_pre_norm) and the experts see the normalised rows;
     * the residual is added as given. Up to 32 tokens the routing kernel
     * normalises its staged copy of x; larger calls normalise each slice into
     * the slice's dst rows first (dst must not overlap x or the residual).
     * The bits equal those of nvfp4_rmsnorm_ptr_bf16 followed by a forward
     * without the flag. */
    NVFP4_MOE_PRE_NORM = 1u << 2,
};

/* additive: batched layer forward with BF16 I/O. x and residual are BF16
 * [tokens, hidden] buffers, dst BF16 [tokens, hidden]:
 *   dst = (flags & NVFP4_MOE_ADD_RESIDUAL ? residual : 0)
 *         + sum_k w_k * expert_k(x) + sigmoid(shared_gate . x) * shared(x).
 * residual may be NULL when the flag is clear. tokens >= 1. */
NVFP4_API nvfp4_status nvfp4_moe_bank_forward_device_enqueue_bf16(
    nvfp4_moe_bank * bank,
    const nvfp4_buffer * x,
    const nvfp4_buffer * residual,
    int tokens,
    int flags,
    nvfp4_buffer * dst);

/* additive: the same forward on raw device pointers, enqueued on `stream`
 * (a cudaStream_t; NULL selects the runtime's stream). For host frameworks
 * whose tensors are not nvfp4_buffer objects. The batched forwards are the
 * serving path: they record no per-call profiling events (the lab's decode
 * entry point does), so nvfp4_runtime_last_profile covers them only while
 * tracing is enabled, when every kernel is timed. */
NVFP4_API nvfp4_status nvfp4_moe_bank_forward_ptr_bf16(
    nvfp4_moe_bank * bank,
    const void * x_bf16,
    const void * residual_bf16,
    void * dst_bf16,
    int tokens,
    int flags,
    void * stream);

/* additive: one layer call on HOST buffers, end to end -- the sequence the
 * lab's callers run as nvfp4_buffer_upload, the bank enqueue,
 * nvfp4_runtime_synchronize and nvfp4_buffer_download
 * (vllm_nvfp4_opencl/runtime.py:370-377, nvfp4_runtime.h:140-160,416-419),
 * in one call: x is copied to device staging on the runtime stream, the
 * forward is enqueued behind it, the result reaches dst and the stream is
 * synchronised once (device timeouts are reported as by
 * nvfp4_runtime_synchronize). x_host, residual_host, dst_host: BF16
 * [tokens, hidden] in host memory; page-locked memory (cudaHostAlloc,
 * torch pin_memory) makes the copies asynchronous DMA, pageable memory works
 * through the driver's staging. Calls of up to 64 tokens (one pass of the
 * decode kernels) read a page-locked residual and store into a page-locked
 * dst across the bus from the combining kernel itself, each value once, when
 * the driver reports the whole span as one mapped allocation; otherwise
 * both go through device staging and copies. flags: NVFP4_MOE_ADD_RESIDUAL
 * and NVFP4_MOE_PRE_NORM. The first call (and any larger call) allocates the
 * device staging for 3 x tokens x hidden x 2 bytes, kept by the bank. */
NVFP4_API nvfp4_status nvfp4_moe_bank_forward_host_bf16(
    nvfp4_moe_bank * bank,
    const void * x_host,
    const void * residual_host,
    void * dst_host,
    int tokens,
    int flags);

/* additive: routing introspection of the most recent forward or decode.
 * Call after nvfp4_runtime_synchronize(). Any output pointer may be NULL.
 *   ids      int32 [tokens, 9]  top-8 ids by descending logit (lowest id on
 *                               ties), slot 8 = experts (the shared expert)
 *   weights  float [tokens, 9]  renormalised top-8 softmax, slot 8 = sigmoid
 *   counts   int32 [experts]    tokens routed to each expert
 *   perm     int32 [tokens*8]   dispatch permutation: flat (token*8 + k)
 *                               indices grouped by expert ascending, tokens
 *                               ascending within an expert
 * max_tokens bounds the ids/weights/perm writes; *out_tokens receives the
 * token count of the last call. */
NVFP4_API nvfp4_status nvfp4_moe_bank_last_routing(
    nvfp4_moe_bank * bank,
    int max_tokens,
    int32_t * ids,
    float * weights,
    int32_t * counts,
    int32_t * perm,
    int * out_tokens);

/* additive: router logits of the most recent forward or decode, FP32
 * [tokens, experts + 1]; column `experts` holds the shared-gate logit. */
NVFP4_API nvfp4_status nvfp4_moe_bank_last_logits(
    nvfp4_moe_bank * bank,
    int max_tokens,
    float * logits,
    int * out_tokens);

/* additive: FP32 per-expert router logit bias [experts] (the skewed-routing
 * configuration). Routing uses logit_e = fp32(router_e . x) + bias_e; pass
 * NULL to clear. Synchronises the runtime stream before writing. */
NVFP4_API nvfp4_status nvfp4_moe_bank_set_router_bias(
    nvfp4_moe_bank * bank,
    const float * bias,
    int experts);

/* additive: bank geometry and resident device bytes. */
NVFP4_API nvfp4_status nvfp4_moe_bank_info(
    const nvfp4_moe_bank * bank,
    int * experts,
    int * hidden,
    int * intermediate,
    size_t * resident_bytes);

/* additive: activation terms of the prefill path (calls above 64 tokens).
 * The prefill expert GEMMs run on FP4 tensor cores: each activation row is
 * fed as the sum of `terms` NVFP4 rows (term j+1 quantises what terms 1..j
 * left over; all share the row's FP32 global scale amax/2688). x_terms
 * applies to the layer input, act_terms to SiLU(gate)*up. 1 = plain NVFP4
 * activations (fastest); the default 4/3 keeps the layer within 2e-3
 * relative RMSE of FP32 activations. Takes effect at the next forward. */
NVFP4_API nvfp4_status nvfp4_moe_bank_set_prefill_terms(
    nvfp4_moe_bank * bank,
    int x_terms,
    int act_terms);

/* additive: expert parallelism (no counterpart in the lab, which runs one
 * device). Later forwards and decodes compute only routed experts
 * [first, first + count) and the shared expert when shared_here is 1; routing
 * still covers every expert (ids, counts and permutation are those of the
 * whole layer). Only the projections of the computed experts need to be
 * uploaded. The default is every expert and the shared expert. */
NVFP4_API nvfp4_status nvfp4_moe_bank_set_expert_range(
    nvfp4_moe_bank * bank,
    int first,
    int count,
    int shared_here);

/* additive: expert parallelism with the reduction fused into the combine
 * (no counterpart in the lab, which runs one device). One context per rank
 * (one process per GPU): nvfp4_ep_create allocates this rank's partial
 * buffers and flags, nvfp4_ep_ipc_handle exports them (NVFP4_EP_HANDLE_BYTES
 * bytes), every rank gathers all ranks' handles in rank order (any host
 * collective) and passes them to nvfp4_ep_open_peers. Then
 * nvfp4_moe_bank_forward_ep_bf16, called on every rank with the same tokens
 * (up to max_tokens <= 64) on banks whose expert ranges cover every expert
 * once, writes the whole layer's BF16 output on every rank: the combine adds
 * the ranks' partial tiles over NVLink peer memory (each wait bounded; a
 * timeout is reported by nvfp4_runtime_synchronize as INTERNAL). The
 * residual, when flagged, is added once. Calls must alternate no further
 * than one call ahead between ranks, which stream order on each rank
 * guarantees. */
#define NVFP4_EP_HANDLE_BYTES 64
NVFP4_API nvfp4_status nvfp4_ep_create(
    nvfp4_runtime * runtime,
    int rank,
    int world,
    int max_tokens,
    int hidden,
    nvfp4_ep ** out_ep);
NVFP4_API nvfp4_status nvfp4_ep_ipc_handle(
    nvfp4_ep * ep,
    void * handle);
NVFP4_API nvfp4_status nvfp4_ep_open_peers(
    nvfp4_ep * ep,
    const void * handles);
NVFP4_API nvfp4_status nvfp4_moe_bank_forward_ep_bf16(
    nvfp4_moe_bank * bank,
    nvfp4_ep * ep,
    const void * x_bf16,
    const void * residual_bf16,
    void * dst_bf16,
    int tokens,
    int flags,
    void * stream);
NVFP4_API void nvfp4_ep_destroy(nvfp4_ep * ep);

/* additive: out = BF16(sum + residual) over [tokens, hidden], with sum FP32
 * (the reduced partial sums of expert-parallel banks) and residual BF16 or
 * NULL; device pointers, enqueued on `stream` (NULL: the runtime's stream). */
NVFP4_API nvfp4_status nvfp4_moe_finalize_bf16(
    nvfp4_runtime * runtime,
    const float * sum_f32,
    const void * residual_bf16,
    void * out_bf16,
    int tokens,
    int hidden,
    void * stream);

/* additive: expert-GEMV kernels of the decode path (calls of up to 64
 * tokens). TENSOR_CORE (default) streams the weights through tcgen05
 * block-scaled NVFP4 MMAs with the activations as four NVFP4 terms per row
 * (relative RMSE about 1e-4 against FP32 activations); it serves calls of 4
 * to 64 tokens on banks with hidden a multiple of 256 up to 2048 and
 * intermediate 256 or 512, and other calls use IN_REGISTER, which decodes
 * E2M1/E4M3 to f16 in registers and keeps the activations in f16 (faster
 * below 4 tokens). FUSED_TOKEN is TENSOR_CORE except for one-token calls of
 * a bank that computes every expert, which run the whole layer (router,
 * top-8, gate/up, down, combine) as one persistent cooperative kernel with
 * bounded grid barriers; it is opt-in because the three-launch path measures
 * faster on B200 (27.7 against 28.7 us per call). Takes effect at the next
 * forward. */
#define NVFP4_DECODE_KERNELS_TENSOR_CORE 0
#define NVFP4_DECODE_KERNELS_IN_REGISTER 1
#define NVFP4_DECODE_KERNELS_FUSED_TOKEN 2
NVFP4_API nvfp4_status nvfp4_moe_bank_set_decode_kernels(
    nvfp4_moe_bank * bank,
    int kernels);

/* additive: the RMSNorm that forwards with NVFP4_MOE_PRE_NORM apply to x
 * (the per-layer pre-norm of a resident layer stack, fused into the layer;
 * the lab's full-model driver runs it as a separate rmsnorm_device call,
 * native_nvfp4/bench_moe_full_model.py:388-395). weight_bf16 is a device
 * pointer to BF16 [hidden], copied into the bank (NULL: ones); epsilon >= 0.
 * Synchronises the device. */
NVFP4_API nvfp4_status nvfp4_moe_bank_set_pre_norm(
    nvfp4_moe_bank * bank,
    const void * weight_bf16,
    float epsilon);

/* additive: allocate the prefill working memory for calls of up to
 * max_tokens tokens (capped at 16384 per pass) now, so that later forwards
 * neither allocate nor synchronise (needed before CUDA-graph capture). */
NVFP4_API nvfp4_status nvfp4_moe_bank_reserve_prefill(
    nvfp4_moe_bank * bank,
    int max_tokens);

/* additive: the prefill path's activation quantiser on its own. src is BF16
 * (src_is_f16 = 0) or FP16 [rows, cols] device memory, cols a multiple of
 * 64. Outputs (device):
 *   codes        uint8 [terms, rows, cols/2]  E2M1 pairs, low nibble = even
 *                column, zero magnitude always with a clear sign bit
 *   scale_words  uint32 [terms, rows, cols/64] four E4M3 block scales per
 *                word, lowest byte = lowest block
 *   row_scales   float [rows] g = amax/2688 (1 for an all-zero row)
 * Per term and 16-column block: s = E4M3_RN((blockamax/6)/g), d = s*g,
 * code = E2M1_RN(r * RN(1/d)) (0 when d is 0), r -= code*d. stream is a
 * cudaStream_t (NULL = legacy default stream). */
NVFP4_API nvfp4_status nvfp4_quantize_rows_enqueue(
    const void * src,
    int src_is_f16,
    int rows,
    int cols,
    int terms,
    void * codes,
    void * scale_words,
    void * row_scales,
    void * stream);

/* ------------------------------------------------ allocation-free routing */

/* No counterpart in the reference. Router logits, top-8 selection with the
 * lowest id on ties, renormalised weights, the sigmoid shared-expert gate and
 * the dispatch permutation for up to 64 tokens -- the same kernel the MoE
 * bank runs first -- for callers that must not allocate device memory while
 * they route (their device memory is planned and owned by the host framework,
 * or allocation is forbidden on their latency-critical path). The kernel's
 * working memory is one 1 MiB array in the library's device globals instead
 * of memory from cudaMalloc; this function allocates nothing.
 *   router_bf16  device BF16 [experts + 1, hidden]; the last row is the
 *                shared-expert gate
 *   x_bf16       device BF16 [tokens, hidden]
 *   ids          device int32 [tokens, 9]  (slot 8 = experts)
 *   weights      device float [tokens, 9]  (slot 8 = sigmoid gate)
 *   counts       device int32 [experts] or NULL
 *   perm         device int32 [tokens * 8] or NULL
 *   stream       cudaStream_t (NULL = legacy default stream)
 * Limits: 1 <= tokens <= 64, 8 <= experts <= 256, hidden a multiple of 128
 * and at most 4096; larger sizes return NVFP4_STATUS_INVALID_ARGUMENT.
 * Every call shares the one array and it keeps the previous call's
 * contents; calls whose kernels overlap on the GPU race and must be ordered.
 * The first call on each device looks up the array's address; make it before
 * any stream capture. The looked-up address is kept for the process: do not
 * call this entry point on a device after cudaDeviceReset on it. */
NVFP4_API nvfp4_status nvfp4_moe_route_static_scratch(
    const void * router_bf16,
    const void * x_bf16,
    int tokens,
    int experts,
    int hidden,
    int32_t * ids,
    float * weights,
    int32_t * counts,
    int32_t * perm,
    void * stream);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_RUNTIME_H */
