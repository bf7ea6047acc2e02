// Prefill path of the NVFP4 MoE layer (token batches above the decode
// limit), built on tcgen05 block-scaled NVFP4 MMA.
//
// Numerics. The expert GEMMs run kind::mxf4nvf4 (E2M1 x E2M1 with E4M3
// scales per 16 elements, FP32 accumulation in tensor memory). Activations
// enter as a sum of J NVFP4 "terms" per row: term 1 quantises the row, term
// j+1 quantises what terms 1..j left over, all terms sharing the row's FP32
// global scale g = amax/2688. J = 1 is plain NVFP4 activation quantisation;
// every extra term cuts the activation error about elevenfold (J = 3 or 4
// holds the layer within the BF16-grade parity tolerance). The GEMM adds the
// J products in one accumulator (the terms are extra K).
//
// Launch sequence (one stream):
//   1. prefill_logits_tc_kernel approximate router logits (tcgen05 kind::f16,
//                               BF16 operands; prefill_logits_kernel with
//                               mma.sync on shapes the tcgen05 tiles skip)
//   2. prefill_select_kernel    exact FP32 fixed-order logits of the
//                               candidates near the top-8 boundary, top-8,
//                               weights, shared gate; per-64-token masks
//   3. prefill_scan_kernel      counts, offsets, active groups, tile table
//   4. prefill_place_kernel     dispatch permutation and per-slot tables
//   5. quantize_blocks_kernel   x -> J NVFP4 terms (per token, written to
//                               each of its slot rows)
//   6. moe_gemm_kernel<0,...>   act = SiLU(gate) * up, FP16 [slot rows][I]
//   7. quantize_blocks_kernel   act -> J NVFP4 terms (per slot row)
//   8. moe_gemm_kernel<1,...>   y = coef * W_down act, FP16 [slot rows][H]
//   9. prefill_combine_kernel   out = sum of nine slots (+ residual), BF16
#pragma once

#include "moe_decode.cuh"

#include <cuda.h>

namespace nvfp4 {

constexpr int kPrefillTileN = 128;   // slot rows per GEMM column tile
constexpr int kPrefillTileM = 128;   // weight rows per GEMM tile
constexpr int kMaxTerms = 4;

// Slot rows of the prefill path are "padded positions": each active expert
// group (routed experts with tokens, then the shared expert) starts on a
// multiple of 128 rows, so every GEMM column tile is one 128-row block and
// its activation scale factors can be stored in tcgen05 atom layout. The
// routing ABI's dispatch permutation stays unpadded.
//
// Device scratch of the prefill path for up to `max_tokens` tokens.
struct PrefillScratch {
    int max_tokens;
    int max_rows;            // padded slot-row capacity: max_tokens*9 + (E+1)*128, rounded to 128
    int E, H, I;
    float *approx;           // [T][Rp] approximate logits, Rp = round_up(E+1, 64)
    int *ids;                // [T][9]
    float *weights;          // [T][9]
    unsigned long long *blk_mask;  // [E][mask_stride] token bits per 64-token block
    int *blk_base;           // [E][mask_stride] rank of each block's first token within the expert
    int mask_stride;         // 64-token blocks of max_tokens
    unsigned *ticket;        // [1] completion counter of the dispatch scan
    int *counts;             // [E]
    int *offsets;            // [E+1] unpadded (routing ABI)
    int *epstart;            // [E+1] padded first row of each expert (index E = shared expert)
    int *rows_used;          // [1] padded rows in use
    int *n_active;           // [1]
    int *active_expert;      // [E+1]
    int *tok_start;          // [E+1] padded first row of each active group
    int *tok_count;          // [E+1]
    int *n_tiles;            // [1] column tiles
    int *tile_group;         // [max tiles] active-group index of a column tile
    int *tile_n0;            // [max tiles] first slot row of a column tile
    int *perm;               // [T*8] unpadded dispatch permutation (routing ABI)
    int *inv_pos;            // [T*8] padded row of each (token, slot)
    int *tok_list;           // [rows] token of each padded slot row
    float *coef;             // [rows] routing weight * inverse down global scale
    uint8_t *xq;             // [Jx][rows][H/2] codes of each slot row's token
    uint8_t *xsf;            // [Jx][rows/128][H/64][512] scale atoms of the slot rows
    float *gx;               // [T]
    __half *act;             // [rows][I]
    uint8_t *aq;             // [Ja][rows][I/2]
    uint8_t *asf;            // [Ja][rows/128][I/64][512] scale atoms
    float *ga;               // [rows]
    __half *ypart;           // [rows][H]
    int *error;              // device error word (shared with the decode scratch)
    int *host_error;         // host-mapped error word or nullptr
    int max_tiles;
    // Experts computed here (expert parallelism): routed [e_first,
    // e_first + e_count) and the shared expert when shared_here. Routing and
    // the routing ABI's counts, offsets and permutation cover every expert.
    int e_first, e_count, shared_here;
};

// TMA descriptors of one prefill scratch (activation terms) and a bank's
// weights (128-row boxes).
struct PrefillMaps {
    CUtensorMap w[3];        // packed weights, box {128 B, 128 rows}, 128-byte swizzle
    CUtensorMap xq;          // [Jx*rows][H/2], box {128 B, 128 rows}
    CUtensorMap aq;          // [Ja*rows][I/2], box {128 B, 128 rows}
    CUtensorMap router;      // BF16 router as bytes [(E+1)][2H], box {128 B, 64 rows}
};

struct PrefillRouteArgs {
    const uint16_t *router;   // [(E+1)][H]
    const uint16_t *x;        // [T][H] BF16
    const float *bias;        // [E] or nullptr
    const float *inv_scales;  // [3][E+1]
    float wnorm_max;          // max over router rows of the L2 norm (host-computed bound)
    int T, E, H;
};

struct GemmArgs {
    const uint8_t *sfa[2];    // weight scale atoms of the A projections
    const uint8_t *sfb;       // [J][rows/128][K/64][512] scale atoms of the slot rows
    int Rb;                   // rows per term of the B tensors (the padded slot-row capacity)
    int J;                    // activation terms
    int K;                    // reduction length
    int M;                    // weight rows per expert
    int E;
    const float *inv_scales;  // [3][E+1]
    int proj;                 // first projection index (0 gate/up, 2 down)
    PrefillScratch s;
};

size_t prefill_scratch_bytes(int T, int E, int H, int I, int Jx, int Ja);
void prefill_scratch_carve(PrefillScratch &s, void *base, int T, int E, int H, int I, int Jx, int Ja);

cudaError_t make_prefill_weight_maps(PrefillMaps &m, uint8_t *const packed[3], int E, int H, int I);
cudaError_t make_prefill_router_map(PrefillMaps &m, const uint16_t *router, int E, int H);
cudaError_t make_prefill_act_maps(PrefillMaps &m, const PrefillScratch &s, int Jx, int Ja);

// Weight scale bytes [rows][K/16] (pitched) -> the tcgen05 scale-factor atom
// layout [rows/128][K/64][512 B]: byte (r%32)*16 + ((r%128)/32)*4 + (k/16)%4.
cudaError_t launch_scale_atoms(uint8_t *atoms, const uint8_t *scales, size_t pitch, int rows, int k16, int row0,
                               cudaStream_t stream);

// Routing in three parts: 0 approximate logits, 1 exact selection, 2 dispatch.
// Part 0 runs on tcgen05 when `maps` is given (H a multiple of 64).
cudaError_t launch_prefill_route(const PrefillRouteArgs &a, const PrefillScratch &s, int part, cudaStream_t stream,
                                 const PrefillMaps *maps = nullptr);
cudaError_t launch_quantize_rows(const void *src, int src_is_f16, int rows, int cols, int terms, uint8_t *codes,
                                 uint32_t *sf, float *g, int rows_stride, cudaStream_t stream);
// Prefill forms: token rows of x (codes by token, scale atoms scattered to
// each token's nine slot rows) and slot rows of the activations (codes and
// atoms by slot row; rows past rows_used are skipped).
cudaError_t launch_quantize_x_prefill(const void *x, int T, const PrefillScratch &s, int terms, cudaStream_t stream);
cudaError_t launch_quantize_act_prefill(const PrefillScratch &s, int terms, cudaStream_t stream);
cudaError_t launch_gemm_gate_up(const PrefillMaps &m, const GemmArgs &a, int sms, cudaStream_t stream);
cudaError_t launch_gemm_down(const PrefillMaps &m, const GemmArgs &a, int sms, cudaStream_t stream);
// out: BF16 [T][H], or FP32 when out_f32 (a partial sum for expert
// parallelism); residual (BF16) is added when given.
cudaError_t launch_prefill_combine(const PrefillScratch &s, int T, const void *residual, void *out, int out_f32,
                                   cudaStream_t stream);

}  // namespace nvfp4
