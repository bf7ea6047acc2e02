// Decode-path kernels of the NVFP4 MoE layer (tokens <= kDecodeMaxTokens).
//
// Three launches per layer on one stream:
//   1. moe_route_kernel    router + shared-gate logits (FP64 fixed-order dot),
//                          then, in the last CTA to finish, top-8 + softmax
//                          renormalisation + sigmoid shared gate + dispatch
//                          (per-expert histogram, offsets, stable permutation,
//                          compacted active-expert work list).
//   2. moe_gate_up_kernel  gate and up NVFP4 GEMVs of every (active expert,
//                          32-row tile), SiLU(gate)*up fused in the epilogue.
//   3. moe_down_kernel     down NVFP4 GEMV of every active expert for a
//                          16-row slice of the output, weighted combine over
//                          experts and the residual add fused in the epilogue.
// The lab runs the same layer as seven launches (nvfp4_runtime.cpp:1943-2066:
// router GEMV, shared-gate GEMV, top-8, gate/up, SiLU, down, reduce).
#pragma once

#include "nvfp4_common.cuh"

namespace nvfp4 {

constexpr int kDecodeMaxTokens = 64;
constexpr int kTopK = 8;
constexpr int kSlots = kTopK + 1;  // slot 8 is the shared expert

// Device scratch of one bank for the decode path. All pointers are device
// addresses; sizes are for kDecodeMaxTokens tokens and E routed experts.
struct DecodeScratch {
    float *logits;          // [T][E+1], column E = shared-gate logit
    __half *x_f16;          // [T][H]
    int *ids;               // [T][9]
    float *weights;         // [T][9]
    int *counts;            // [E]
    int *offsets;           // [E+1]
    int *perm;              // [T*8]
    int *n_active;          // [1]
    int *active_expert;     // [E+1]
    int *tok_start;         // [E+1]
    int *tok_count;         // [E+1]
    int *tok_list;          // [T*9]
    int *pos_tab;           // [(E+1)][kDecodeMaxTokens]
    float *coef_tab;        // [(E+1)][kDecodeMaxTokens]
    uint32_t *ntile_mask;   // [E+1]
    __half *act;            // [T*9][I]
    unsigned *ticket;       // [1]
};

struct RouteArgs {
    const uint16_t *router;   // [(E+1)][H] BF16, row E = shared gate
    const void *x;            // [T][H] BF16 or FP32
    int x_is_f32;
    int T, E, H;
    const float *inv_scales;  // [3][E+1]
    const float *bias;        // [E] router logit bias or nullptr
    int e_first, e_count;     // locally computed routed experts
    int shared_here;          // 1 if the shared expert is computed here
    DecodeScratch s;
};

struct GateUpArgs {
    const uint8_t *gate_packed, *gate_scales, *up_packed, *up_scales;
    const float *inv_scales;
    int E, H, I;
    DecodeScratch s;
};

struct DownArgs {
    const uint8_t *down_packed, *down_scales;
    const void *residual;     // BF16 [T][H] or nullptr
    void *out;                // BF16 or FP32 [T][H]
    int out_f32;
    int T, E, H, I;
    DecodeScratch s;
};

// Launch helpers (defined in moe_decode.cu).
cudaError_t launch_route(const RouteArgs &a, cudaStream_t stream);
cudaError_t launch_gate_up(const GateUpArgs &a, int T, int grid_cap, cudaStream_t stream);
cudaError_t launch_down(const DownArgs &a, int grid_cap, cudaStream_t stream);

// Scratch byte size for a bank of E experts, hidden H, intermediate I.
size_t decode_scratch_bytes(int E, int H, int I);
size_t decode_scratch_carve(DecodeScratch &s, void *base, int E, int H, int I);

}  // namespace nvfp4
