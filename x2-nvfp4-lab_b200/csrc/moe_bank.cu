// MoE bank entry points of the C ABI.
//
// Storage mirrors the lab's contiguous bank (native_nvfp4/runtime/
// nvfp4_runtime.cpp:392-429,1780-1856): for each projection one array of
// (experts+1) matrices, expert `experts` being the shared expert, plus one
// FP32 inverse-global-scale table [3][experts+1] indexed
// projection*(experts+1)+expert. The BF16 router and the shared-expert gate
// row are stored as one [(experts+1), hidden] matrix so that the routing
// kernel treats the shared gate as router row `experts`.
#include "internal.h"
#include "moe_decode.cuh"
#include "moe_prefill.cuh"
#include "moe_token.cuh"

#include <cmath>
#include <cstring>
#include <limits>
#include <memory>

using namespace nvfp4;

namespace nvfp4 {
bool ep_next_call(nvfp4_ep *ep, int tokens, int hidden, EpArgs *out);  // moe_ep.cu
}

struct nvfp4_moe_bank {
    nvfp4_runtime *runtime = nullptr;
    int experts = 0;
    int hidden = 0;
    int intermediate = 0;
    uint8_t *packed[3] = {nullptr, nullptr, nullptr};
    uint8_t *scales[3] = {nullptr, nullptr, nullptr};
    float *inv_scales = nullptr;   // device [3][experts+1]
    uint16_t *router = nullptr;    // device [(experts+1)][hidden]
    float *router_bias = nullptr;  // device [experts] or null
    void *scratch = nullptr;
    DecodeScratch ds{};
    StreamMaps maps{};             // TMA descriptors over packed/scales
    std::vector<uint8_t> uploaded;
    size_t uploaded_projections = 0;
    int last_tokens = 0;
    int last_path = 0;             // 1 = decode path (routing record valid)
    size_t resident_bytes = 0;
    int *host_error = nullptr;     // pinned host-mapped timeout word (DecodeScratch::host_error)
    // Prefill path (token batches above the decode limit).
    uint8_t *sf_atoms[3] = {nullptr, nullptr, nullptr};  // weight scales in tcgen05 atom layout
    float wnorm_max = 0.0f;        // max L2 norm of the routed router rows
    void *pscratch = nullptr;
    PrefillScratch ps{};
    PrefillMaps pmaps{};
    int prefill_tokens = 0;        // token capacity of pscratch
    int terms_x = 4, terms_act = 3;
    int scratch_terms_x = 0, scratch_terms_act = 0;
    // Decode expert-GEMV variant: NVFP4_DECODE_KERNELS_TENSOR_CORE (calls of
    // 4 to kDecodeMaxTokens tokens on shapes with prefill kernels),
    // NVFP4_DECODE_KERNELS_IN_REGISTER, or NVFP4_DECODE_KERNELS_FUSED_TOKEN
    // (tensor-core, and one-token calls as one persistent kernel).
    int decode_kernels = NVFP4_DECODE_KERNELS_TENSOR_CORE;
    // Expert parallelism: routed experts [e_first, e_first + e_count) and the
    // shared expert (when shared_here) are computed by this bank.
    int e_first = 0, e_count = 0, shared_here = 1;
    bool tc_ready = false;         // tc_maps built
    DecodeTcMaps tc_maps{};
    // RMSNorm applied to x by forwards with NVFP4_MOE_PRE_NORM (the layer
    // stack's pre-norm): the bank's own copy of the BF16 weight [hidden].
    uint16_t *norm_w = nullptr;
    float norm_eps = 1e-6f;
    // Device staging of nvfp4_moe_bank_forward_host_bf16: x, residual and
    // output rows of the largest call so far.
    uint8_t *io_stage = nullptr;
    size_t io_stage_bytes = 0;
    // Barrier words of the one-token kernel (moe_token.cu), zeroed at creation.
    unsigned *token_sync = nullptr;

    ~nvfp4_moe_bank() {
        if (token_sync) cudaFree(token_sync);
        if (io_stage) cudaFree(io_stage);
        if (host_error) cudaFreeHost(host_error);
        if (norm_w) cudaFree(norm_w);
        for (int p = 0; p < 3; ++p)
            if (sf_atoms[p]) cudaFree(sf_atoms[p]);
        if (pscratch) cudaFree(pscratch);
        for (int p = 0; p < 3; ++p) {
            if (packed[p]) cudaFree(packed[p]);
            if (scales[p]) cudaFree(scales[p]);
        }
        if (inv_scales) cudaFree(inv_scales);
        if (router) cudaFree(router);
        if (router_bias) cudaFree(router_bias);
        if (scratch) cudaFree(scratch);
    }

    size_t rows(int projection) const { return projection < 2 ? intermediate : hidden; }
    size_t cols(int projection) const { return projection < 2 ? hidden : intermediate; }
    size_t per_packed() const { return static_cast<size_t>(hidden) * intermediate / 2; }
    size_t per_scales() const { return static_cast<size_t>(hidden) * intermediate / 16; }
    // Device row pitch of a projection's scale bytes: cols/16 rounded up to
    // 16 so every row starts on a 16-byte boundary (a TMA requirement); the
    // padding bytes stay zero.
    size_t scale_pitch(int projection) const { return (cols(projection) / 16 + 15) & ~size_t(15); }
    size_t scales_per_expert(int projection) const { return rows(projection) * scale_pitch(projection); }
    // Every projection this bank computes has been uploaded.
    bool owned_uploaded() const {
        const size_t slots = static_cast<size_t>(experts) + 1;
        for (int p = 0; p < 3; ++p) {
            for (int e = e_first; e < e_first + e_count; ++e)
                if (!uploaded[p * slots + e]) return false;
            if (shared_here && !uploaded[p * slots + experts]) return false;
        }
        return true;
    }
};

namespace {

// Copy `rows` rows of `cols` scale bytes into a pitched destination,
// clearing the sign bit and mapping 0x7F to 0 (the lab's decoding rule).
__global__ void sanitize_scales_kernel(uint8_t *dst, size_t pitch, const uint8_t *src, size_t rows, size_t cols) {
    const size_t n = rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, c = i - r * cols;
        const uint8_t b = src[i] & 0x7Fu;
        dst[r * pitch + c] = b == 0x7Fu ? 0u : b;
    }
}

// True when [p, p + bytes) lies inside one page-locked host allocation that
// kernels on the current device can store to: both ends are mapped host
// memory of the same CUDA buffer, bytes - 1 apart on the device side. *dev
// receives the device address of p. Pageable memory, registrations the
// driver cannot identify, and spans crossing allocations answer false.
bool mapped_host_span(void *p, size_t bytes, void **dev) {
    using GetAttrFn = CUresult (*)(void *, CUpointer_attribute, CUdeviceptr);
    static GetAttrFn get_attr = [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuPointerGetAttribute", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return static_cast<GetAttrFn>(nullptr);
        }
        return reinterpret_cast<GetAttrFn>(fn);
    }();
    if (!get_attr || bytes == 0) return false;
    char *last = static_cast<char *>(p) + (bytes - 1);
    cudaPointerAttributes a{}, b{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess || cudaPointerGetAttributes(&b, last) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (a.type != cudaMemoryTypeHost || b.type != cudaMemoryTypeHost || !a.devicePointer || !b.devicePointer ||
        static_cast<char *>(b.devicePointer) - static_cast<char *>(a.devicePointer) !=
            static_cast<ptrdiff_t>(bytes - 1))
        return false;
    unsigned long long id_a = 0, id_b = 0;
    if (get_attr(&id_a, CU_POINTER_ATTRIBUTE_BUFFER_ID, reinterpret_cast<CUdeviceptr>(a.devicePointer)) !=
            CUDA_SUCCESS ||
        get_attr(&id_b, CU_POINTER_ATTRIBUTE_BUFFER_ID, reinterpret_cast<CUdeviceptr>(b.devicePointer)) !=
            CUDA_SUCCESS ||
        id_a == 0 || id_a != id_b)
        return false;
    *dev = a.devicePointer;
    return true;
}

void mark_uploaded(nvfp4_moe_bank *bank, int expert, int projection) {
    const size_t slots = static_cast<size_t>(bank->experts) + 1;
    const size_t index = static_cast<size_t>(projection) * slots + expert;
    if (!bank->uploaded[index]) {
        bank->uploaded[index] = 1;
        ++bank->uploaded_projections;
    }
}

nvfp4_status check_upload_args(const nvfp4_moe_bank *bank, int expert, int projection,
                               const void *packed, size_t packed_bytes, const void *scales,
                               size_t scale_bytes, float weight_global_scale) {
    if (!bank || !bank->runtime || !packed || !scales || expert < 0 || expert > bank->experts ||
        projection < 0 || projection > 2 || weight_global_scale == 0.0f ||
        !std::isfinite(weight_global_scale))
        return fail_invalid("invalid MoE bank projection upload arguments");
    if (packed_bytes != bank->per_packed() || scale_bytes != bank->per_scales())
        return fail_invalid("MoE bank projection byte counts do not match dimensions");
    return NVFP4_STATUS_OK;
}

// Enqueue the three decode-path kernels for `tokens` <= kDecodeMaxTokens,
// each between a pair of profiling events (trace operations moe_route,
// moe_gate_up, moe_down). Caller holds the runtime's queue mutex.
// Below kDecodeTcMinTokens tokens the in-register GEMVs finish first (they
// split the few active experts into more, smaller work items); from there on
// the tensor-core GEMVs stream the weights faster (layer call on one B200,
// E 256, H 2048, I 512, L2 flushed: 42.0 vs 43.1 us at 3 tokens, 50.2 vs
// 49.1 at 4, 72.8 vs 61.4 at 8).
constexpr int kDecodeTcMinTokens = 4;

bool use_tensor_core_decode(const nvfp4_moe_bank *bank, int tokens) {
    return bank->decode_kernels != NVFP4_DECODE_KERNELS_IN_REGISTER && bank->tc_ready &&
           tokens >= kDecodeTcMinTokens && tokens <= kDecodeMaxTokens;
}

// One-token calls of a bank that computes every expert run as one persistent
// kernel (moe_token.cu) when the bank's decode kernels are FUSED_TOKEN.
bool use_token_kernel(const nvfp4_moe_bank *bank, int tokens, const EpArgs *ep) {
    return tokens == 1 && !ep && bank->token_sync && bank->decode_kernels == NVFP4_DECODE_KERNELS_FUSED_TOKEN &&
           bank->e_first == 0 && bank->e_count == bank->experts && bank->shared_here &&
           token_supported(bank->runtime->sm_count, bank->experts, bank->hidden, bank->intermediate,
                           static_cast<int>(bank->scale_pitch(0)), static_cast<int>(bank->scale_pitch(2)));
}

void enqueue_decode(nvfp4_moe_bank *bank, const void *x, int x_is_f32, const void *residual,
                    void *out, int out_f32, int tokens, cudaStream_t stream, const EpArgs *ep = nullptr,
                    bool pre_norm = false, bool residual_early = false) {
    const int E = bank->experts, H = bank->hidden, I = bank->intermediate;
    const int sms = bank->runtime->sm_count;
    nvfp4_runtime *rt = bank->runtime;
    if (use_token_kernel(bank, tokens, ep)) {
        TokenArgs ta{};
        ta.router = bank->router;
        ta.bias = bank->router_bias;
        ta.x = x;
        ta.x_is_f32 = x_is_f32;
        ta.norm_w = pre_norm && !x_is_f32 ? bank->norm_w : nullptr;
        ta.norm_eps = bank->norm_eps;
        ta.residual = residual;
        ta.out = out;
        ta.out_f32 = out_f32;
        for (int p = 0; p < 3; ++p) {
            ta.packed[p] = bank->packed[p];
            ta.scales[p] = bank->scales[p];
            ta.scale_pitch[p] = static_cast<int>(bank->scale_pitch(p));
        }
        ta.inv_scales = bank->inv_scales;
        ta.E = E;
        ta.H = H;
        ta.I = I;
        ta.act = bank->ds.ypart;
        ta.sync = bank->token_sync;
        ta.s = bank->ds;
        rt->profiled_kernel("moe_token", stream, [&](cudaStream_t s) {
            check_cuda(launch_token(ta, sms, s), "moe_token_kernel");
        });
        return;
    }
    const bool tc = use_tensor_core_decode(bank, tokens);
    RouteArgs ra{};
    ra.router = bank->router;
    ra.x = x;
    ra.x_is_f32 = x_is_f32;
    ra.T = tokens;
    ra.E = E;
    ra.H = H;
    ra.inv_scales = bank->inv_scales;
    ra.bias = bank->router_bias;
    ra.e_first = bank->e_first;
    ra.e_count = bank->e_count;
    ra.shared_here = bank->shared_here;
    ra.quantize_x = tc ? 1 : 0;
    ra.norm_w = pre_norm && !x_is_f32 ? bank->norm_w : nullptr;
    ra.norm_eps = bank->norm_eps;
    ra.s = bank->ds;
    rt->profiled_kernel("moe_route", stream, [&](cudaStream_t s) {
        check_cuda(launch_route(ra, s, true), "moe_route_kernel");
    });

    DownArgs da{};
    da.down_packed = bank->packed[2];
    da.down_scales = bank->scales[2];
    da.residual = residual;
    da.residual_early = residual_early ? 1 : 0;
    da.out = out;
    da.out_f32 = out_f32;
    da.shared_here = bank->shared_here;
    da.T = tokens;
    da.E = E;
    da.H = H;
    da.I = I;
    da.s = bank->ds;

    if (tc) {
        DecodeTcArgs ta{};
        ta.inv_scales = bank->inv_scales;
        ta.E = E;
        ta.H = H;
        ta.I = I;
        ta.T = tokens;
        ta.shared_last = bank->shared_here ? 1 : 0;
        ta.s = bank->ds;
        ta.sfa[0] = bank->sf_atoms[0];
        ta.sfa[1] = bank->sf_atoms[1];
        ta.sfb = bank->ds.xsf_tc;
        rt->profiled_kernel("moe_gate_up", stream, [&](cudaStream_t s) {
            check_cuda(launch_gate_up_tc(bank->pmaps.w[0], bank->pmaps.w[1], bank->tc_maps, ta, tokens, sms, s),
                       "moe_gate_up_tc_kernel");
        });
        // Above kDecodeTcMaxTokens tokens the activation quantiser and the
        // down kernel walk the down groups (an expert's two token halves
        // merged where they fit one tile).
        DecodeScratch dv = bank->ds;
        if (tokens > kDecodeTcMaxTokens) {
            dv.n_active = dv.n_down;
            dv.active_expert = dv.down_expert;
            dv.tok_start = dv.down_start;
            dv.tok_count = dv.down_count;
        }
        rt->profiled_kernel("moe_quantize_act", stream, [&](cudaStream_t s) {
            check_cuda(launch_quantize_act_tc(dv, tokens, I, s), "quantize_act_tc_kernel");
        });
        ta.s = dv;
        ta.sfa[0] = bank->sf_atoms[2];
        ta.sfa[1] = bank->sf_atoms[2];
        ta.sfb = bank->ds.asf_tc;
        rt->profiled_kernel("moe_down", stream, [&](cudaStream_t s) {
            check_cuda(launch_down_tc(bank->pmaps.w[2], bank->tc_maps, ta, tokens, sms, s),
                       "moe_down_tc_kernel");
            if (!ep) check_cuda(launch_combine(da, s), "moe_combine_kernel");
        });
        if (ep)
            rt->profiled_kernel("moe_combine_ep", stream, [&](cudaStream_t s) {
                check_cuda(launch_combine_ep(da, *ep, s), "moe_combine_ep_kernel");
            });
        return;
    }

    GateUpArgs ga{};
    ga.gate_packed = bank->packed[0];
    ga.gate_scales = bank->scales[0];
    ga.up_packed = bank->packed[1];
    ga.up_scales = bank->scales[1];
    ga.inv_scales = bank->inv_scales;
    ga.E = E;
    ga.H = H;
    ga.I = I;
    ga.s = bank->ds;
    rt->profiled_kernel("moe_gate_up", stream, [&](cudaStream_t s) {
        check_cuda(launch_gate_up_tma(bank->maps, ga, tokens, sms, s), "moe_gate_up_tma_kernel");
    });

    rt->profiled_kernel("moe_down", stream, [&](cudaStream_t s) {
        check_cuda(launch_down_tma(bank->maps, da, sms, s, ep == nullptr), "moe_down_tma_kernel");
    });
    if (ep)
        rt->profiled_kernel("moe_combine_ep", stream, [&](cudaStream_t s) {
            check_cuda(launch_combine_ep(da, *ep, s), "moe_combine_ep_kernel");
        });
}

bool prefill_supported(const nvfp4_moe_bank *bank) {
    return bank->hidden % 256 == 0 && bank->intermediate % 256 == 0;
}

// Make the prefill scratch hold `tokens` tokens at the bank's term counts.
// Reallocation drains the runtime stream first; it is a no-op when the
// scratch is already large enough (reserve it up front for graph capture).
void ensure_prefill(nvfp4_moe_bank *bank, int tokens) {
    if (tokens <= bank->prefill_tokens && bank->scratch_terms_x == bank->terms_x &&
        bank->scratch_terms_act == bank->terms_act)
        return;
    const int cap = tokens > bank->prefill_tokens ? ((tokens + 255) / 256) * 256 : bank->prefill_tokens;
    nvfp4_runtime *rt = bank->runtime;
    check_cuda(cudaStreamSynchronize(rt->stream), "cudaStreamSynchronize(prefill scratch)");
    check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize(prefill scratch)");
    if (bank->pscratch) {
        cudaFree(bank->pscratch);
        bank->pscratch = nullptr;
        bank->prefill_tokens = 0;
    }
    const int E = bank->experts, H = bank->hidden, I = bank->intermediate;
    const size_t bytes = prefill_scratch_bytes(cap, E, H, I, bank->terms_x, bank->terms_act);
    check_cuda(cudaMalloc(&bank->pscratch, bytes), "cudaMalloc(MoE bank prefill scratch)");
    check_cuda(cudaMemsetAsync(bank->pscratch, 0, bytes, rt->stream), "cudaMemsetAsync(MoE bank prefill scratch)");
    check_cuda(cudaStreamSynchronize(rt->stream), "cudaStreamSynchronize(prefill scratch)");
    prefill_scratch_carve(bank->ps, bank->pscratch, cap, E, H, I, bank->terms_x, bank->terms_act);
    bank->ps.error = bank->ds.error;
    bank->ps.host_error = bank->ds.host_error;
    check_cuda(make_prefill_act_maps(bank->pmaps, bank->ps, bank->terms_x, bank->terms_act),
               "cuTensorMapEncodeTiled(MoE bank prefill activations)");
    bank->prefill_tokens = cap;
    bank->scratch_terms_x = bank->terms_x;
    bank->scratch_terms_act = bank->terms_act;
}

// Prefill-path launches for `tokens` <= bank->prefill_tokens (BF16 in/out).
void enqueue_prefill(nvfp4_moe_bank *bank, const void *x, const void *residual, void *out, int out_f32, int tokens,
                     cudaStream_t stream) {
    const int E = bank->experts, H = bank->hidden, I = bank->intermediate;
    const int sms = bank->runtime->sm_count;
    nvfp4_runtime *rt = bank->runtime;
    bank->ps.e_first = bank->e_first;
    bank->ps.e_count = bank->e_count;
    bank->ps.shared_here = bank->shared_here;
    const PrefillScratch &ps = bank->ps;
    PrefillRouteArgs ra{};
    ra.router = bank->router;
    ra.x = static_cast<const uint16_t *>(x);
    ra.bias = bank->router_bias;
    ra.inv_scales = bank->inv_scales;
    ra.wnorm_max = bank->wnorm_max;
    ra.T = tokens;
    ra.E = E;
    ra.H = H;
    rt->profiled_kernel("moe_route_logits", stream, [&](cudaStream_t s) {
        check_cuda(launch_prefill_route(ra, ps, 0, s, &bank->pmaps), "prefill_logits_tc_kernel");
    });
    rt->profiled_kernel("moe_route_select", stream, [&](cudaStream_t s) {
        check_cuda(launch_prefill_route(ra, ps, 1, s), "prefill_select_kernel");
    });
    rt->profiled_kernel("moe_dispatch", stream, [&](cudaStream_t s) {
        check_cuda(launch_prefill_route(ra, ps, 2, s), "prefill dispatch kernels");
    });
    rt->profiled_kernel("moe_quantize_x", stream, [&](cudaStream_t s) {
        check_cuda(launch_quantize_x_prefill(x, tokens, ps, bank->terms_x, s), "quantize_blocks_kernel(x)");
    });
    GemmArgs ga{};
    ga.sfa[0] = bank->sf_atoms[0];
    ga.sfa[1] = bank->sf_atoms[1];
    ga.sfb = ps.xsf;
    ga.Rb = ps.max_rows;
    ga.J = bank->terms_x;
    ga.K = H;
    ga.M = I;
    ga.E = E;
    ga.inv_scales = bank->inv_scales;
    ga.proj = 0;
    ga.s = ps;
    rt->profiled_kernel("moe_gate_up", stream, [&](cudaStream_t s) {
        check_cuda(launch_gemm_gate_up(bank->pmaps, ga, sms, s), "moe_gemm_kernel(gate/up)");
    });
    rt->profiled_kernel("moe_quantize_act", stream, [&](cudaStream_t s) {
        check_cuda(launch_quantize_act_prefill(ps, bank->terms_act, s), "quantize_blocks_kernel(act)");
    });
    GemmArgs gd = ga;
    gd.sfa[0] = bank->sf_atoms[2];
    gd.sfa[1] = bank->sf_atoms[2];
    gd.sfb = ps.asf;
    gd.Rb = ps.max_rows;
    gd.J = bank->terms_act;
    gd.K = I;
    gd.M = H;
    gd.proj = 2;
    rt->profiled_kernel("moe_down", stream, [&](cudaStream_t s) {
        check_cuda(launch_gemm_down(bank->pmaps, gd, sms, s), "moe_gemm_kernel(down)");
    });
    rt->profiled_kernel("moe_combine", stream, [&](cudaStream_t s) {
        check_cuda(launch_prefill_combine(ps, tokens, residual, out, out_f32, s), "prefill_combine_kernel");
    });
}

constexpr int kPrefillMaxSlice = 16384;

// Forwards with NVFP4_MOE_PRE_NORM: up to this many tokens the routing kernel
// normalises its staged tokens (one launch fewer); larger calls run the
// RMSNorm kernel first (every routing CTA would repeat the work of its
// token block: measured per layer call, L2 flushed, 104.5 vs 107.1 us at 32
// tokens, 221.3 vs 213.1 us at 64).
constexpr int kFusedNormMaxTokens = 32;

// Batched BF16 forward: the decode path up to kDecodeMaxTokens tokens, the
// prefill path above it (in slices of at most kPrefillMaxSlice tokens), or
// decode-path slices when the bank's shape has no prefill kernels.
void enqueue_forward_bf16(nvfp4_moe_bank *bank, const void *x, const void *residual, void *out,
                          int tokens, cudaStream_t stream, int out_f32 = 0, bool pre_norm = false) {
    const size_t row_bytes = static_cast<size_t>(bank->hidden) * 2;
    const size_t out_row_bytes = static_cast<size_t>(bank->hidden) * (out_f32 ? 4 : 2);
    const bool prefill = tokens > kDecodeMaxTokens && prefill_supported(bank);
    const int slice = prefill ? (tokens < kPrefillMaxSlice ? tokens : kPrefillMaxSlice) : kDecodeMaxTokens;
    if (prefill) ensure_prefill(bank, slice);
    for (int t0 = 0; t0 < tokens; t0 += slice) {
        const int n = tokens - t0 < slice ? tokens - t0 : slice;
        const uint8_t *xs = static_cast<const uint8_t *>(x) + t0 * row_bytes;
        const uint8_t *rs = residual ? static_cast<const uint8_t *>(residual) + t0 * row_bytes : nullptr;
        uint8_t *os = static_cast<uint8_t *>(out) + t0 * out_row_bytes;
        if (pre_norm && (prefill || n > kFusedNormMaxTokens)) {
            // The slice's normalised rows go to its own output rows (BF16,
            // within the slice's output bytes): only the first kernels read
            // them as x, before the combine overwrites them.
            check_cuda(launch_rmsnorm_bf16(xs, bank->norm_w, os, n, bank->hidden, bank->norm_eps, stream),
                       "rmsnorm_kernel");
            if (prefill)
                enqueue_prefill(bank, os, rs, os, out_f32, n, stream);
            else
                enqueue_decode(bank, os, 0, rs, os, out_f32, n, stream);
        } else if (prefill) {
            enqueue_prefill(bank, xs, rs, os, out_f32, n, stream);
        } else {
            enqueue_decode(bank, xs, 0, rs, os, out_f32, n, stream, nullptr, pre_norm);
        }
    }
    bank->last_tokens = tokens;
    bank->last_path = tokens <= kDecodeMaxTokens ? 1 : (prefill && tokens <= slice ? 2 : 0);
}

}  // namespace

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_create(nvfp4_runtime *runtime,
                                                        const uint16_t *router_bf16,
                                                        size_t router_bytes,
                                                        const uint16_t *shared_gate_bf16,
                                                        size_t shared_gate_bytes, int experts,
                                                        int hidden, int intermediate,
                                                        nvfp4_moe_bank **out_bank) {
    if (!runtime || !router_bf16 || !shared_gate_bf16 || !out_bank || experts < 8 ||
        experts > 256 || hidden <= 0 || intermediate <= 0 || hidden % 16 != 0 ||
        intermediate % 16 != 0 ||
        router_bytes != static_cast<size_t>(experts) * hidden * sizeof(uint16_t) ||
        shared_gate_bytes != static_cast<size_t>(hidden) * sizeof(uint16_t))
        return fail_invalid("invalid MoE bank creation arguments");
    if (hidden % 128 != 0 || intermediate % 128 != 0)
        return fail_invalid("this CUDA backend needs hidden and intermediate to be multiples of 128");
    *out_bank = nullptr;
    try {
        auto holder = std::make_unique<nvfp4_moe_bank>();
        holder->runtime = runtime;
        holder->experts = experts;
        holder->e_count = experts;
        holder->hidden = hidden;
        holder->intermediate = intermediate;
        const size_t slots = static_cast<size_t>(experts) + 1;
        if (static_cast<size_t>(hidden) >
            std::numeric_limits<size_t>::max() / static_cast<size_t>(intermediate) / slots)
            throw std::overflow_error("MoE bank dimensions overflow size_t");
        const size_t elements = slots * static_cast<size_t>(hidden) * intermediate;
        std::lock_guard<std::mutex> lock(runtime->queue_mutex);
        size_t scale_bytes_all = 0;
        for (int p = 0; p < 3; ++p) {
            const size_t sb = slots * holder->scales_per_expert(p);
            scale_bytes_all += sb;
            check_cuda(cudaMalloc(&holder->packed[p], elements / 2), "cudaMalloc(MoE bank packed)");
            check_cuda(cudaMalloc(&holder->scales[p], sb), "cudaMalloc(MoE bank scales)");
            check_cuda(cudaMemsetAsync(holder->packed[p], 0, elements / 2, runtime->stream),
                       "cudaMemsetAsync(MoE bank packed)");
            check_cuda(cudaMemsetAsync(holder->scales[p], 0, sb, runtime->stream), "cudaMemsetAsync(MoE bank scales)");
        }
        check_cuda(cudaMalloc(&holder->inv_scales, 3 * slots * sizeof(float)),
                   "cudaMalloc(MoE bank inverse scales)");
        check_cuda(cudaMemsetAsync(holder->inv_scales, 0, 3 * slots * sizeof(float), runtime->stream),
                   "cudaMemsetAsync(MoE bank inverse scales)");
        const size_t router_all = slots * static_cast<size_t>(hidden) * sizeof(uint16_t);
        check_cuda(cudaMalloc(&holder->router, router_all), "cudaMalloc(MoE bank router)");
        // Host-to-device copies go through the runtime stream: a synchronous
        // cudaMemcpy from pageable memory may return before its DMA lands and
        // is not ordered with the (non-blocking) runtime stream.
        check_cuda(cudaMemcpyAsync(holder->router, router_bf16, router_bytes, cudaMemcpyHostToDevice,
                                   runtime->stream),
                   "cudaMemcpy(MoE bank router)");
        check_cuda(cudaMemcpyAsync(reinterpret_cast<uint8_t *>(holder->router) + router_bytes,
                              shared_gate_bf16, shared_gate_bytes, cudaMemcpyHostToDevice, runtime->stream),
                   "cudaMemcpy(MoE bank shared gate)");
        const size_t scratch = decode_scratch_bytes(experts, hidden, intermediate);
        check_cuda(cudaMalloc(&holder->scratch, scratch), "cudaMalloc(MoE bank scratch)");
        check_cuda(cudaMemsetAsync(holder->scratch, 0, scratch, runtime->stream),
                   "cudaMemsetAsync(MoE bank scratch)");
        decode_scratch_carve(holder->ds, holder->scratch, experts, hidden, intermediate);
        check_cuda(cudaMalloc(&holder->token_sync, token_sync_bytes()), "cudaMalloc(MoE bank token barriers)");
        check_cuda(cudaMemsetAsync(holder->token_sync, 0, token_sync_bytes(), runtime->stream),
                   "cudaMemsetAsync(MoE bank token barriers)");
        check_cuda(cudaHostAlloc(reinterpret_cast<void **>(&holder->host_error), sizeof(int), cudaHostAllocMapped),
                   "cudaHostAlloc(MoE bank error word)");
        *holder->host_error = 0;
        check_cuda(cudaHostGetDevicePointer(reinterpret_cast<void **>(&holder->ds.host_error), holder->host_error, 0),
                   "cudaHostGetDevicePointer(MoE bank error word)");
        check_cuda(make_stream_maps(holder->maps, holder->packed, holder->scales, experts, hidden, intermediate),
                   "cuTensorMapEncodeTiled(MoE bank)");
        for (int p = 0; p < 3; ++p) {
            const size_t ab = slots * holder->rows(p) * (holder->cols(p) / 16);
            check_cuda(cudaMalloc(&holder->sf_atoms[p], ab), "cudaMalloc(MoE bank scale atoms)");
            check_cuda(cudaMemsetAsync(holder->sf_atoms[p], 0, ab, runtime->stream),
                       "cudaMemsetAsync(MoE bank scale atoms)");
        }
        check_cuda(make_prefill_weight_maps(holder->pmaps, holder->packed, experts, hidden, intermediate),
                   "cuTensorMapEncodeTiled(MoE bank prefill)");
        check_cuda(make_prefill_router_map(holder->pmaps, holder->router, experts, hidden),
                   "cuTensorMapEncodeTiled(MoE bank router)");
        if (prefill_supported(holder.get()) && decode_tc_supported(hidden, intermediate)) {
            check_cuda(make_decode_tc_maps(holder->tc_maps, holder->ds, hidden, intermediate),
                       "cuTensorMapEncodeTiled(MoE bank decode terms)");
            holder->tc_ready = true;
        }
        {
            // Largest routed router-row norm: bounds the approximate-logit
            // error of the prefill router (rounded up by a relative 1e-6).
            double mx = 0.0;
            for (int e = 0; e < experts; ++e) {
                double ss = 0.0;
                for (int k = 0; k < hidden; ++k) {
                    uint32_t bits = static_cast<uint32_t>(router_bf16[static_cast<size_t>(e) * hidden + k]) << 16;
                    float w;
                    std::memcpy(&w, &bits, 4);
                    ss += static_cast<double>(w) * w;
                }
                mx = ss > mx ? ss : mx;
            }
            holder->wnorm_max = static_cast<float>(std::sqrt(mx) * (1.0 + 1e-6));
        }
        check_cuda(cudaStreamSynchronize(runtime->stream), "cudaStreamSynchronize(MoE bank create)");
        holder->uploaded.assign(slots * 3, 0);
        holder->resident_bytes = 3 * (elements / 2) + scale_bytes_all + 3 * (elements / 16) +
                                 3 * slots * sizeof(float) + router_all;
        runtime->error_words.emplace_back(holder->host_error, holder->ds.error);
        clear_last_error();
        *out_bank = holder.release();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_upload_projection(
    nvfp4_moe_bank *bank, int expert, int projection, const uint8_t *packed, size_t packed_bytes,
    const uint8_t *scales_e4m3, size_t scale_bytes, float weight_global_scale) {
    const nvfp4_status st = check_upload_args(bank, expert, projection, packed, packed_bytes,
                                              scales_e4m3, scale_bytes, weight_global_scale);
    if (st != NVFP4_STATUS_OK) return st;
    try {
        nvfp4_runtime *rt = bank->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        check_cuda(cudaStreamSynchronize(rt->stream), "cudaStreamSynchronize(MoE bank upload)");
        const size_t pp = bank->per_packed(), ps = bank->per_scales();
        std::vector<uint8_t> clean(scales_e4m3, scales_e4m3 + ps);
        for (uint8_t &b : clean) {
            b &= 0x7Fu;
            if (b == 0x7Fu) b = 0u;
        }
        // Copies are ordered on the runtime stream (see nvfp4_moe_bank_create);
        // pageable sources are staged before each call returns.
        check_cuda(cudaMemcpyAsync(bank->packed[projection] + static_cast<size_t>(expert) * pp, packed, pp,
                                   cudaMemcpyHostToDevice, rt->stream),
                   "cudaMemcpy(MoE bank packed upload)");
        const size_t scols = bank->cols(projection) / 16, pitch = bank->scale_pitch(projection);
        check_cuda(cudaMemcpy2DAsync(bank->scales[projection] + static_cast<size_t>(expert) *
                                                                    bank->scales_per_expert(projection),
                                     pitch, clean.data(), scols, scols, bank->rows(projection),
                                     cudaMemcpyHostToDevice, rt->stream),
                   "cudaMemcpy2D(MoE bank scale upload)");
        check_cuda(launch_scale_atoms(bank->sf_atoms[projection], bank->scales[projection], pitch,
                                      (int)bank->rows(projection), (int)scols, expert * (int)bank->rows(projection),
                                      rt->stream),
                   "scale_atoms_kernel");
        const float inv = 1.0f / weight_global_scale;
        const size_t slots = static_cast<size_t>(bank->experts) + 1;
        check_cuda(cudaMemcpyAsync(bank->inv_scales + static_cast<size_t>(projection) * slots + expert, &inv,
                                   sizeof(float), cudaMemcpyHostToDevice, rt->stream),
                   "cudaMemcpy(MoE bank inverse scale)");
        check_cuda(cudaStreamSynchronize(rt->stream), "cudaStreamSynchronize(MoE bank upload)");
        mark_uploaded(bank, expert, projection);
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_upload_projection_device(
    nvfp4_moe_bank *bank, int expert, int projection, const void *packed_device,
    size_t packed_bytes, const void *scales_device, size_t scale_bytes, float weight_global_scale) {
    const nvfp4_status st = check_upload_args(bank, expert, projection, packed_device, packed_bytes,
                                              scales_device, scale_bytes, weight_global_scale);
    if (st != NVFP4_STATUS_OK) return st;
    try {
        nvfp4_runtime *rt = bank->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        const size_t pp = bank->per_packed(), ps = bank->per_scales();
        check_cuda(cudaMemcpyAsync(bank->packed[projection] + static_cast<size_t>(expert) * pp,
                                   packed_device, pp, cudaMemcpyDeviceToDevice, rt->stream),
                   "cudaMemcpyAsync(MoE bank packed upload)");
        const int grid = static_cast<int>((ps + 255) / 256 < 4096 ? (ps + 255) / 256 : 4096);
        sanitize_scales_kernel<<<grid, 256, 0, rt->stream>>>(
            bank->scales[projection] + static_cast<size_t>(expert) * bank->scales_per_expert(projection),
            bank->scale_pitch(projection), static_cast<const uint8_t *>(scales_device), bank->rows(projection),
            bank->cols(projection) / 16);
        check_cuda(cudaGetLastError(), "sanitize_scales_kernel");
        check_cuda(launch_scale_atoms(bank->sf_atoms[projection], bank->scales[projection],
                                      bank->scale_pitch(projection), (int)bank->rows(projection),
                                      (int)(bank->cols(projection) / 16), expert * (int)bank->rows(projection),
                                      rt->stream),
                   "scale_atoms_kernel");
        const float inv = 1.0f / weight_global_scale;
        const size_t slots = static_cast<size_t>(bank->experts) + 1;
        // cudaMemcpyAsync from pageable memory stages the value before returning.
        check_cuda(cudaMemcpyAsync(bank->inv_scales + static_cast<size_t>(projection) * slots + expert,
                                   &inv, sizeof(float), cudaMemcpyHostToDevice, rt->stream),
                   "cudaMemcpyAsync(MoE bank inverse scale)");
        mark_uploaded(bank, expert, projection);
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_decode_device_enqueue_f32(nvfp4_moe_bank *bank,
                                                                           const nvfp4_buffer *x,
                                                                           nvfp4_buffer *dst) {
    if (!bank || !bank->runtime || !x || x->runtime != bank->runtime || !dst ||
        dst->runtime != bank->runtime ||
        x->bytes < static_cast<size_t>(bank->hidden) * sizeof(float) ||
        dst->bytes < static_cast<size_t>(bank->hidden) * sizeof(float))
        return fail_invalid("invalid MoE bank decode buffers");
    if (!bank->owned_uploaded())
        return fail_invalid("MoE bank decode requires every routed and shared projection of its expert range");
    try {
        nvfp4_runtime *rt = bank->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        rt->profiled_call("moe_bank_decode", nullptr, [&](cudaStream_t s) {
            enqueue_decode(bank, x->data, 1, nullptr, dst->data, 1, 1, s);
        });
        bank->last_tokens = 1;
        bank->last_path = 1;
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_forward_ptr_bf16(nvfp4_moe_bank *bank,
                                                                 const void *x_bf16,
                                                                 const void *residual_bf16,
                                                                 void *dst_bf16, int tokens, int flags,
                                                                 void *stream) {
    if (!bank || !bank->runtime || !x_bf16 || !dst_bf16 || tokens <= 0 ||
        (flags & ~static_cast<int>(NVFP4_MOE_ADD_RESIDUAL | NVFP4_MOE_PARTIAL_F32 | NVFP4_MOE_PRE_NORM)) != 0 ||
        ((flags & NVFP4_MOE_ADD_RESIDUAL) && !residual_bf16) || ((flags & NVFP4_MOE_PRE_NORM) && !bank->norm_w))
        return fail_invalid("invalid MoE bank forward arguments");
    if (!bank->owned_uploaded())
        return fail_invalid("MoE bank forward requires every routed and shared projection of its expert range");
    try {
        nvfp4_runtime *rt = bank->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        const void *res = (flags & NVFP4_MOE_ADD_RESIDUAL) ? residual_bf16 : nullptr;
        rt->direct_call(static_cast<cudaStream_t>(stream), [&](cudaStream_t s) {
            enqueue_forward_bf16(bank, x_bf16, res, dst_bf16, tokens, s, (flags & NVFP4_MOE_PARTIAL_F32) ? 1 : 0,
                                 (flags & NVFP4_MOE_PRE_NORM) != 0);
        });
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_forward_ep_bf16(nvfp4_moe_bank *bank, nvfp4_ep *ep,
                                                                 const void *x_bf16, const void *residual_bf16,
                                                                 void *dst_bf16, int tokens, int flags,
                                                                 void *stream) {
    if (!bank || !bank->runtime || !ep || !x_bf16 || !dst_bf16 || tokens < 1 || tokens > kDecodeMaxTokens ||
        (flags & ~static_cast<int>(NVFP4_MOE_ADD_RESIDUAL)) != 0 ||
        ((flags & NVFP4_MOE_ADD_RESIDUAL) && !residual_bf16))
        return fail_invalid("invalid expert-parallel forward arguments (1..64 tokens)");
    if (!bank->owned_uploaded())
        return fail_invalid("MoE bank forward requires every routed and shared projection of its expert range");
    try {
        nvfp4_runtime *rt = bank->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        EpArgs e{};
        if (!ep_next_call(ep, tokens, bank->hidden, &e))
            return fail_invalid("expert-parallel context not opened, or its token or hidden size does not fit");
        const void *res = (flags & NVFP4_MOE_ADD_RESIDUAL) ? residual_bf16 : nullptr;
        rt->direct_call(static_cast<cudaStream_t>(stream), [&](cudaStream_t s) {
            enqueue_decode(bank, x_bf16, 0, res, dst_bf16, 0, tokens, s, &e);
        });
        bank->last_tokens = tokens;
        bank->last_path = 1;
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_forward_device_enqueue_bf16(
    nvfp4_moe_bank *bank, const nvfp4_buffer *x, const nvfp4_buffer *residual, int tokens,
    int flags, nvfp4_buffer *dst) {
    if (!bank || !bank->runtime || !x || x->runtime != bank->runtime || !dst ||
        dst->runtime != bank->runtime || tokens <= 0)
        return fail_invalid("invalid MoE bank forward buffers");
    const size_t bytes = static_cast<size_t>(tokens) * bank->hidden * 2;
    const size_t dst_bytes = bytes * ((flags & NVFP4_MOE_PARTIAL_F32) ? 2 : 1);
    if (x->bytes < bytes || dst->bytes < dst_bytes)
        return fail_invalid("MoE bank forward buffer capacity is too small");
    if (flags & NVFP4_MOE_ADD_RESIDUAL) {
        if (!residual || residual->runtime != bank->runtime || residual->bytes < bytes)
            return fail_invalid("MoE bank forward residual buffer is missing or too small");
    }
    return nvfp4_moe_bank_forward_ptr_bf16(bank, x->data, residual ? residual->data : nullptr,
                                          dst->data, tokens, flags, nullptr);
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_forward_host_bf16(nvfp4_moe_bank *bank, const void *x_host,
                                                                  const void *residual_host, void *out_host,
                                                                  int tokens, int flags) {
    if (!bank || !bank->runtime || !x_host || !out_host || tokens <= 0 ||
        (flags & ~static_cast<int>(NVFP4_MOE_ADD_RESIDUAL | NVFP4_MOE_PRE_NORM)) != 0 ||
        ((flags & NVFP4_MOE_ADD_RESIDUAL) && !residual_host) || ((flags & NVFP4_MOE_PRE_NORM) && !bank->norm_w))
        return fail_invalid("invalid MoE bank host forward arguments");
    if (!bank->owned_uploaded())
        return fail_invalid("MoE bank forward requires every routed and shared projection of its expert range");
    try {
        nvfp4_runtime *rt = bank->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        const size_t bytes = static_cast<size_t>(tokens) * bank->hidden * 2;
        if (bank->io_stage_bytes < 3 * bytes) {
            // Grow once to the largest call; the old staging may still be read
            // by queued work, so drain the stream before freeing it.
            check_cuda(cudaStreamSynchronize(rt->stream), "cudaStreamSynchronize(host forward staging)");
            if (bank->io_stage) check_cuda(cudaFree(bank->io_stage), "cudaFree(host forward staging)");
            bank->io_stage = nullptr;
            bank->io_stage_bytes = 0;
            check_cuda(cudaMalloc(reinterpret_cast<void **>(&bank->io_stage), 3 * bytes),
                       "cudaMalloc(host forward staging)");
            bank->io_stage_bytes = 3 * bytes;
        }
        uint8_t *dx = bank->io_stage, *dr = bank->io_stage + bytes, *dstage = bank->io_stage + 2 * bytes;
        cudaStream_t s = rt->stream;
        const bool res = (flags & NVFP4_MOE_ADD_RESIDUAL) != 0;
        const bool pre_norm = (flags & NVFP4_MOE_PRE_NORM) != 0;
        // A call that runs as one pass of the decode kernels reads a
        // page-locked residual and stores its output rows into a page-locked
        // dst over the bus itself: the combining kernel reads each residual
        // value once (before it waits on the down kernel) and stores each
        // output value once, and no kernel reads dst back. Pageable buffers,
        // and every buffer of other calls, go through the device staging.
        const bool decode = tokens <= kDecodeMaxTokens && !(pre_norm && tokens > kFusedNormMaxTokens);
        void *res_dev = nullptr, *out_dev = nullptr;
        const bool res_direct =
            decode && res && mapped_host_span(const_cast<void *>(residual_host), bytes, &res_dev);
        const bool out_direct = decode && mapped_host_span(out_host, bytes, &out_dev);
        check_cuda(cudaMemcpyAsync(dx, x_host, bytes, cudaMemcpyHostToDevice, s), "cudaMemcpyAsync(x)");
        if (res && !res_direct)
            check_cuda(cudaMemcpyAsync(dr, residual_host, bytes, cudaMemcpyHostToDevice, s),
                       "cudaMemcpyAsync(residual)");
        const void *rsrc = !res ? nullptr : res_direct ? res_dev : static_cast<const void *>(dr);
        void *dout = out_direct ? out_dev : static_cast<void *>(dstage);
        rt->direct_call(s, [&](cudaStream_t ks) {
            if (decode) {
                enqueue_decode(bank, dx, 0, rsrc, dout, 0, tokens, ks, nullptr, pre_norm, res_direct);
                bank->last_tokens = tokens;
                bank->last_path = 1;
            } else {
                enqueue_forward_bf16(bank, dx, rsrc, dout, tokens, ks, 0, pre_norm);
            }
        });
        if (!out_direct)
            check_cuda(cudaMemcpyAsync(out_host, dstage, bytes, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync(out)");
        check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize(host forward)");
        raise_device_timeouts(rt);
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_last_routing(nvfp4_moe_bank *bank, int max_tokens,
                                                              int32_t *ids, float *weights,
                                                              int32_t *counts, int32_t *perm,
                                                              int *out_tokens) {
    if (!bank || !bank->runtime || max_tokens < 0) return fail_invalid("invalid routing query");
    if (bank->last_tokens == 0) return fail_invalid("no forward has run on this bank");
    if (!bank->last_path)
        return fail_invalid("routing record is kept for calls that ran as one decode or prefill pass");
    try {
        nvfp4_runtime *rt = bank->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        check_cuda(cudaStreamSynchronize(rt->stream), "cudaStreamSynchronize(last_routing)");
        const int T = bank->last_tokens < max_tokens ? bank->last_tokens : max_tokens;
        const bool pre = bank->last_path == 2;
        const int *src_ids = pre ? bank->ps.ids : bank->ds.ids;
        const float *src_w = pre ? bank->ps.weights : bank->ds.weights;
        const int *src_counts = pre ? bank->ps.counts : bank->ds.counts;
        const int *src_perm = pre ? bank->ps.perm : bank->ds.perm;
        if (ids)
            check_cuda(cudaMemcpy(ids, src_ids, sizeof(int32_t) * T * kSlots, cudaMemcpyDeviceToHost),
                       "cudaMemcpy(routing ids)");
        if (weights)
            check_cuda(cudaMemcpy(weights, src_w, sizeof(float) * T * kSlots, cudaMemcpyDeviceToHost),
                       "cudaMemcpy(routing weights)");
        if (counts)
            check_cuda(cudaMemcpy(counts, src_counts, sizeof(int32_t) * bank->experts, cudaMemcpyDeviceToHost),
                       "cudaMemcpy(routing counts)");
        if (perm && T == bank->last_tokens)
            check_cuda(cudaMemcpy(perm, src_perm, sizeof(int32_t) * T * kTopK, cudaMemcpyDeviceToHost),
                       "cudaMemcpy(routing perm)");
        if (out_tokens) *out_tokens = bank->last_tokens;
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_last_logits(nvfp4_moe_bank *bank, int max_tokens,
                                                             float *logits, int *out_tokens) {
    if (!bank || !bank->runtime || max_tokens < 0 || !logits) return fail_invalid("invalid logits query");
    if (bank->last_tokens == 0) return fail_invalid("no forward has run on this bank");
    if (bank->last_path != 1)
        return fail_invalid("router logits are kept for calls of at most 64 tokens");
    try {
        nvfp4_runtime *rt = bank->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        check_cuda(cudaStreamSynchronize(rt->stream), "cudaStreamSynchronize(last_logits)");
        const int T = bank->last_tokens < max_tokens ? bank->last_tokens : max_tokens;
        check_cuda(cudaMemcpy(logits, bank->ds.logits, sizeof(float) * T * (bank->experts + 1),
                              cudaMemcpyDeviceToHost),
                   "cudaMemcpy(router logits)");
        if (out_tokens) *out_tokens = bank->last_tokens;
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_set_router_bias(nvfp4_moe_bank *bank,
                                                                 const float *bias, int experts) {
    if (!bank || !bank->runtime || (bias && experts != bank->experts))
        return fail_invalid("router bias must have one value per routed expert");
    try {
        nvfp4_runtime *rt = bank->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        check_cuda(cudaStreamSynchronize(rt->stream), "cudaStreamSynchronize(router bias)");
        if (!bias) {
            if (bank->router_bias) cudaFree(bank->router_bias);
            bank->router_bias = nullptr;
        } else {
            if (!bank->router_bias)
                check_cuda(cudaMalloc(&bank->router_bias, sizeof(float) * bank->experts),
                           "cudaMalloc(router bias)");
            check_cuda(cudaMemcpyAsync(bank->router_bias, bias, sizeof(float) * bank->experts,
                                       cudaMemcpyHostToDevice, rt->stream),
                       "cudaMemcpy(router bias)");
            check_cuda(cudaStreamSynchronize(rt->stream), "cudaStreamSynchronize(router bias)");
        }
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_info(const nvfp4_moe_bank *bank, int *experts,
                                                      int *hidden, int *intermediate,
                                                      size_t *resident_bytes) {
    if (!bank) return fail_invalid("bank is required");
    if (experts) *experts = bank->experts;
    if (hidden) *hidden = bank->hidden;
    if (intermediate) *intermediate = bank->intermediate;
    if (resident_bytes) *resident_bytes = bank->resident_bytes;
    clear_last_error();
    return NVFP4_STATUS_OK;
}

extern "C" NVFP4_API void nvfp4_moe_bank_destroy(nvfp4_moe_bank *bank) {
    if (bank && bank->runtime) {
        std::lock_guard<std::mutex> lock(bank->runtime->queue_mutex);
        if (bank->runtime->stream) cudaStreamSynchronize(bank->runtime->stream);
        auto &words = bank->runtime->error_words;
        for (size_t i = 0; i < words.size(); ++i) {
            if (words[i].second == bank->ds.error) {
                words.erase(words.begin() + static_cast<std::ptrdiff_t>(i));
                break;
            }
        }
    }
    delete bank;
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_set_prefill_terms(nvfp4_moe_bank *bank, int x_terms,
                                                                   int act_terms) {
    if (!bank || !bank->runtime || x_terms < 1 || x_terms > kMaxTerms || act_terms < 1 || act_terms > kMaxTerms)
        return fail_invalid("prefill activation terms must be between 1 and 4");
    std::lock_guard<std::mutex> lock(bank->runtime->queue_mutex);
    bank->terms_x = x_terms;
    bank->terms_act = act_terms;
    clear_last_error();
    return NVFP4_STATUS_OK;
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_set_expert_range(nvfp4_moe_bank *bank, int first, int count,
                                                                  int shared_here) {
    if (!bank || !bank->runtime || first < 0 || count < 1 || first + count > bank->experts ||
        (shared_here != 0 && shared_here != 1))
        return fail_invalid("expert range must lie within [0, experts) and hold at least one expert");
    std::lock_guard<std::mutex> lock(bank->runtime->queue_mutex);
    bank->e_first = first;
    bank->e_count = count;
    bank->shared_here = shared_here;
    clear_last_error();
    return NVFP4_STATUS_OK;
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_set_decode_kernels(nvfp4_moe_bank *bank, int kernels) {
    if (!bank || !bank->runtime ||
        (kernels != NVFP4_DECODE_KERNELS_TENSOR_CORE && kernels != NVFP4_DECODE_KERNELS_IN_REGISTER &&
         kernels != NVFP4_DECODE_KERNELS_FUSED_TOKEN))
        return fail_invalid("decode kernels must be NVFP4_DECODE_KERNELS_TENSOR_CORE, _IN_REGISTER or _FUSED_TOKEN");
    std::lock_guard<std::mutex> lock(bank->runtime->queue_mutex);
    bank->decode_kernels = kernels;
    clear_last_error();
    return NVFP4_STATUS_OK;
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_set_pre_norm(nvfp4_moe_bank *bank, const void *weight_bf16,
                                                               float epsilon) {
    if (!bank || !bank->runtime || !(epsilon >= 0.0f)) return fail_invalid("invalid pre-norm arguments");
    try {
        nvfp4_runtime *rt = bank->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        const size_t bytes = static_cast<size_t>(bank->hidden) * 2;
        // Calls already enqueued may still read the previous weight.
        check_cuda(cudaStreamSynchronize(rt->stream), "cudaStreamSynchronize(pre-norm)");
        check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize(pre-norm)");
        if (!bank->norm_w) check_cuda(cudaMalloc(&bank->norm_w, bytes), "cudaMalloc(pre-norm weight)");
        if (weight_bf16) {
            check_cuda(cudaMemcpyAsync(bank->norm_w, weight_bf16, bytes, cudaMemcpyDefault, rt->stream),
                       "cudaMemcpyAsync(pre-norm weight)");
        } else {
            const std::vector<uint16_t> ones(bank->hidden, 0x3F80u);  // BF16 1.0
            check_cuda(cudaMemcpyAsync(bank->norm_w, ones.data(), bytes, cudaMemcpyHostToDevice, rt->stream),
                       "cudaMemcpyAsync(pre-norm weight)");
        }
        check_cuda(cudaStreamSynchronize(rt->stream), "cudaStreamSynchronize(pre-norm)");
        bank->norm_eps = epsilon;
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_moe_bank_reserve_prefill(nvfp4_moe_bank *bank, int max_tokens) {
    if (!bank || !bank->runtime || max_tokens < 1) return fail_invalid("invalid prefill reservation");
    if (!prefill_supported(bank))
        return fail_invalid("the prefill path needs hidden and intermediate to be multiples of 256");
    try {
        nvfp4_runtime *rt = bank->runtime;
        std::lock_guard<std::mutex> lock(rt->queue_mutex);
        ensure_prefill(bank, max_tokens < kPrefillMaxSlice ? max_tokens : kPrefillMaxSlice);
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}

extern "C" NVFP4_API nvfp4_status nvfp4_quantize_rows_enqueue(const void *src, int src_is_f16, int rows, int cols,
                                                              int terms, void *codes, void *scale_words,
                                                              void *row_scales, void *stream) {
    if (!src || !codes || !scale_words || !row_scales || rows < 1 || cols < 64 || cols % 64 != 0 || terms < 1 ||
        terms > kMaxTerms || (src_is_f16 != 0 && src_is_f16 != 1))
        return fail_invalid("invalid row quantisation arguments");
    try {
        check_cuda(launch_quantize_rows(src, src_is_f16, rows, cols, terms, static_cast<uint8_t *>(codes),
                                        static_cast<uint32_t *>(scale_words), static_cast<float *>(row_scales), rows,
                                        static_cast<cudaStream_t>(stream)),
                   "quantize_blocks_kernel");
        clear_last_error();
        return NVFP4_STATUS_OK;
    } catch (const std::exception &error) {
        return fail_exception(error);
    }
}
