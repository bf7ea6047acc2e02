// Decode-path kernels of the NVFP4 MoE layer (tokens <= kDecodeMaxTokens).
//
// Per layer call, one stream, programmatic dependent launch between kernels
// (each one's prologue overlaps its predecessor's tail):
//   moe_route_kernel        router + shared-gate logits (FP32, fixed order),
//                           top-8 + softmax renormalisation + sigmoid shared
//                           gate per 4-token block, then dispatch (per-expert
//                           histogram, offsets, stable permutation, compacted
//                           active-expert list).
// then one of two expert-GEMV variants:
//   in-register decode (any shape):
//     moe_gate_up_tma_kernel  gate and up NVFP4 GEMVs of every (active expert,
//                             32-row tile), E2M1/E4M3 decoded to f16 in
//                             registers, mma.sync against f16 tokens,
//                             SiLU(gate)*up fused;
//     moe_down_tma_kernel     down GEMV of every (active expert, 64-row tile),
//                             scaled per (token, slot); in calls of up to
//                             kFusedCombineMaxTokens tokens the CTA that
//                             finishes an output tile's last group also
//                             combines that tile (no combine launch);
//   tensor-core (calls of 4 to kDecodeMaxTokens tokens on the shapes
//   decode_tc_supported accepts; the routing kernel also writes x as four
//   NVFP4 terms per token):
//     moe_gate_up_tc_kernel   gate/up on tcgen05 block-scaled MMA; the four
//                             terms of every token are four B rows (N), so the
//                             weights stream once;
//     quantize_act_tc_kernel  activations -> four terms per slot row;
//     moe_down_tc_kernel      down, scaled per (token, slot);
// and finally (unless the down kernel combined)
//   moe_combine_kernel      sum of the nine slots + residual.
// The lab runs the same layer as seven launches (nvfp4_runtime.cpp:1943-2066:
// router GEMV, shared-gate GEMV, top-8, gate/up, SiLU, down, reduce).
#pragma once

#include "nvfp4_common.cuh"

#include <cuda.h>

namespace nvfp4 {

constexpr int kDecodeMaxTokens = 64;
constexpr int kTopK = 8;
constexpr int kSlots = kTopK + 1;  // slot 8 is the shared expert
constexpr int kRouteTickets = 1 + kDecodeMaxTokens / 4;
constexpr int kDecodeTcMaxTokens = 32;  // tensor-core variant: 4 terms x 32 tokens = one 128-row B tile
constexpr int kDecodeTcTerms = 4;

// Device scratch of one bank for the decode path. All pointers are device
// addresses; sizes are for kDecodeMaxTokens tokens and E routed experts.
// The fields the routing kernel touches come first (decode_route_scratch_bytes
// covers exactly them); the expert-GEMV buffers follow.
struct DecodeScratch {
    float *logits;          // [T][E+1], column E = shared-gate logit
    __half *x_f16;          // [T][H]
    int *ids;               // [T][9]
    float *weights;         // [T][9]
    int *counts;            // [E]
    int *offsets;           // [E+1]
    int *perm;              // [T*8]
    int *inv_pos;           // [T*8] position of (token, slot) in perm order, -1 if not computed here
    int *n_active;          // [1]
    // Active groups: one per computed expert; tensor-core calls of more than
    // kDecodeTcMaxTokens tokens split each expert by token half (tokens
    // 0-31, then 32-63), every half-0 group listed before every half-1 group.
    int *n_half0;           // [1] groups of the first token half (tensor-core calls above 32 tokens)
    int *active_expert;     // [2(E+1)]
    int *tok_start;         // [2(E+1)]
    int *tok_count;         // [2(E+1)]
    // Tensor-core calls above kDecodeTcMaxTokens tokens: the down kernel's
    // groups (an expert's tokens together up to kDecodeTcMaxTokens, else one
    // group per token half; B rows are the group's own slot rows, so one tile
    // serves any 32 of them). slot_group and coef_tab then index these.
    int *n_down;            // [1]
    int *down_expert;       // [2(E+1)]
    int *down_start;        // [2(E+1)]
    int *down_count;        // [2(E+1)]
    int *tok_list;          // [T*9]
    float *coef_tab;        // [2(E+1)][kDecodeMaxTokens]
    unsigned *ticket;       // [kRouteTickets] dispatch ticket, then one per 4-token block
    int *error;             // [1] device-side wait timeout flag
    int *slot_group;        // [T*9] active-group index of each dispatch position, -1 if not computed here
    __half *act;            // [T*9][I]      SiLU(gate)*up per (token, slot)
    float *ypart;           // [T*9][H]      scaled down-projection per (token, slot)
    unsigned *tile_count;   // [H/64]        finished groups per 64-row output tile (zeroed by routing)
    // Tensor-core variant: activation terms. Row 4*t + j of a B tile is term j
    // of token (or slot) t; scale bytes are stored in tcgen05 atom layout
    // [K/64][512 B] per 128-row tile: byte (n%32)*16 + (n/32)*4 + (k/16)%4.
    uint8_t *xq_tc;         // [256][H/2]               terms of x by token (rows 128h.. : token half h)
    uint8_t *xsf_tc;        // [2][H/64][512]           their scale atoms, one 128-row tile per half
    float *gx_tc;           // [kDecodeMaxTokens]       global scale of each token row
    uint8_t *aq_tc;         // [T*9*4][I/2]             terms of the activations by slot
    uint8_t *asf_tc;        // [2(E+1)][I/64][512]      scale atoms per active group (rows from tok_start)
    float *ga_tc;           // [T*9]                    global scale of each slot row
    int *host_error;        // pinned host-mapped word the host reads at synchronize, or nullptr
};

// TMA descriptors over a bank's packed and scale arrays (gate, up, down).
struct StreamMaps {
    CUtensorMap packed[3];
    CUtensorMap scales[3];       // box of 64 scale bytes (four 256-column boxes)
    CUtensorMap scales_half[3];  // box of 32 scale bytes (two 256-column boxes)
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
    int quantize_x;           // 1: also write x as four NVFP4 terms (tensor-core variant)
    const uint16_t *norm_w;   // BF16 [H] RMSNorm weight applied to x first, or nullptr (BF16 x only)
    float norm_eps;
    DecodeScratch s;
};

struct GateUpArgs {
    const uint8_t *gate_packed, *gate_scales, *up_packed, *up_scales;
    const float *inv_scales;
    int E, H, I;
    DecodeScratch s;
};

// Tensor maps of the tensor-core variant's activation terms (128-row boxes,
// 128-byte swizzle).
struct DecodeTcMaps {
    CUtensorMap xq;
    CUtensorMap aq;
};

// Where a combining kernel writes: out = residual + the nine slot partials.
struct CombineOut {
    const void *residual;     // BF16 [T][H] or nullptr
    void *out;                // BF16 or FP32 [T][H]
    int out_f32;
    int shared_here;          // 1 if the shared expert's slot is summed here
    int T, H;
};

struct DecodeTcArgs {
    const uint8_t *sfa[2];    // weight scale atoms: gate, up (MODE 0) or down (MODE 1)
    const uint8_t *sfb;       // activation scale atoms (xsf_tc or asf_tc)
    const float *inv_scales;  // [3][E+1]
    int E, H, I;
    int shared_last;          // 1: the shared expert is computed here (always the last active group)
    int T;                    // tokens of the call (above kDecodeTcMaxTokens: groups by token half)
    DecodeScratch s;
};

// Output rows h..h+3 (h % 4 == 0) of token t: the slot partials summed in
// slot order, then the shared slot, then the residual (the order of
// moe_combine_kernel, so every combining kernel gives the same bits). The
// partials may come from other CTAs of the running grid and are read
// through L2.
__device__ __forceinline__ void combine_quad(const CombineOut &c, const DecodeScratch &s, int t, int h) {
    const int H = c.H;
    int pos[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) pos[k] = s.inv_pos[t * kTopK + k];
    const size_t o = (size_t)t * H + h;
    float r[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (c.residual) {
        const uint16_t *res = static_cast<const uint16_t *>(c.residual) + o;
#pragma unroll
        for (int q = 0; q < 4; ++q) r[q] = bf16_bits_to_f32(res[q]);
    }
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int k = 0; k <= kTopK; ++k) {
        const int p = k < kTopK ? pos[k] : (c.shared_here ? c.T * kTopK + t : -1);
        if (p >= 0) {
            const float4 y = __ldcg(reinterpret_cast<const float4 *>(s.ypart + (size_t)p * H + h));
            v[0] += y.x;
            v[1] += y.y;
            v[2] += y.z;
            v[3] += y.w;
        }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        if (c.residual) v[q] += r[q];
        if (c.out_f32)
            static_cast<float *>(c.out)[o + q] = v[q];
        else
            static_cast<uint16_t *>(c.out)[o + q] = f32_to_bf16_bits(v[q]);
    }
}

struct DownArgs {
    const uint8_t *down_packed, *down_scales;
    const void *residual;     // BF16 [T][H] or nullptr
    void *out;                // BF16 or FP32 [T][H]
    int out_f32;
    int shared_here;          // 1 if the shared expert's slot is summed here
    int T, E, H, I;
    int fuse_combine;         // in-register down kernel: the last CTA of each output tile also combines it
    // The residual was written before the call was enqueued (the caller's
    // page-locked host rows): moe_combine_kernel reads it before waiting on
    // the down kernel, so its latency overlaps the down GEMV.
    int residual_early;
    DecodeScratch s;
};

// Calls of up to this many tokens combine inside the in-register down
// kernel (one tile of at most 16 x 64 outputs per finishing CTA); larger
// calls launch the combine kernel.
constexpr int kFusedCombineMaxTokens = 16;

// Expert-parallel combine fused with the cross-rank reduction (moe_ep.cu).
// Each rank writes its partial tile into its own buffer (mapped by every
// peer), raises one flag per peer for that tile, waits (bounded) until every
// peer's flag for the tile has arrived, then sums all ranks' tiles in rank
// order, so every rank produces the same BF16 output.
constexpr int kMaxEpRanks = 8;
struct EpArgs {
    float *part[kMaxEpRanks];          // each rank's partial buffer of this call's parity, [T][H] FP32
    unsigned *flags_peer[kMaxEpRanks]; // each rank's flag array [world][tiles]
    unsigned *flags_local;             // this rank's flag array
    unsigned *ticket;                  // this rank's tile count of the call (zero between calls)
    unsigned epoch;                    // call number, >= 1
    int rank, world, tiles;
    int *err;                          // device error word
    int *host_err;                     // host-mapped error word or nullptr
};
cudaError_t launch_combine_ep(const DownArgs &a, const EpArgs &e, cudaStream_t stream);

// Launch helpers (defined in moe_decode.cu). `dependent`: a programmatic
// dependent launch (the kernel fetches the router before it waits for the
// preceding kernel; use it only when the preceding stream operation is a
// kernel launch).
cudaError_t launch_route(const RouteArgs &a, cudaStream_t stream, bool dependent = false);

// TMA-pipelined expert GEMVs (moe_stream.cu).
cudaError_t make_stream_maps(StreamMaps &m, uint8_t *const packed[3], uint8_t *const scales[3], int E, int H,
                             int I);
cudaError_t launch_gate_up_tma(const StreamMaps &m, const GateUpArgs &a, int T, int sms, cudaStream_t stream);
cudaError_t launch_down_tma(const StreamMaps &m, const DownArgs &a, int sms, cudaStream_t stream,
                            bool with_combine = true);
cudaError_t launch_combine(const DownArgs &a, cudaStream_t stream);

// Tensor-core variant (moe_decode_tc.cu): shapes it serves (H and I
// multiples of 256, H <= 2048, I of 256 or 512).
bool decode_tc_supported(int H, int I);
cudaError_t make_decode_tc_maps(DecodeTcMaps &m, const DecodeScratch &s, int H, int I);
cudaError_t launch_quantize_act_tc(const DecodeScratch &s, int T, int I, cudaStream_t stream);
cudaError_t launch_gate_up_tc(const CUtensorMap &w_gate, const CUtensorMap &w_up, const DecodeTcMaps &m,
                              const DecodeTcArgs &a, int T, int sms, cudaStream_t stream);
cudaError_t launch_down_tc(const CUtensorMap &w_down, const DecodeTcMaps &m, const DecodeTcArgs &a, int T, int sms,
                           cudaStream_t stream);

// Scratch byte size for a bank of E experts, hidden H, intermediate I, and
// the prefix of it that the routing kernel alone uses.
size_t decode_scratch_bytes(int E, int H, int I);
size_t decode_route_scratch_bytes(int E, int H);
size_t decode_scratch_carve(DecodeScratch &s, void *base, int E, int H, int I);

}  // namespace nvfp4
