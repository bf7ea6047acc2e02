// Dense NVFP4 linear on tcgen05 block-scaled MMA (the tensor-core form of the
// lab's nvfp4_linear entry points; linear.cu holds the matrix objects and the
// CUDA-core kernel).
#pragma once

#include "nvfp4_common.cuh"

#include <cuda.h>

namespace nvfp4 {

// Activation terms per vector: six NVFP4 terms (term j + 1 quantises what
// terms 0..j left over; quant_terms.cuh) bring the activations to within
// ~2e-6 of the output scale, under the lab's GEMV gate of 2e-5.
constexpr int kLinTcTerms = 6;
// Vectors per pass: their terms are the N rows of one 128-row B tile.
constexpr int kLinTcVectors = 128 / kLinTcTerms;  // 21
constexpr int kLinTcStageK = 256;                   // columns per pipeline stage

// Per-matrix device state of the tensor-core path (owned by nvfp4_matrix).
struct LinearTcState {
    int kstages = 0;          // ceil(cols / 256)
    int tiles = 0;            // ceil(rows / 128)
    uint8_t *w_atoms = nullptr;  // [tiles][4 * kstages][512 B] weight scale atoms (zero beyond cols / rows)
    uint8_t *xq = nullptr;       // [128][kstages * 128 B] activation term codes, B row 6v + j
    uint8_t *x_atoms = nullptr;  // [4 * kstages][512 B] their scale atoms
    float *gx = nullptr;         // [kLinTcVectors] each vector's global scale
    int *err = nullptr;          // device wait-timeout word
    int *host_err_dev = nullptr; // device view of the host-mapped word
    CUtensorMap map_w;           // packed weights: box 128 B x 128 rows, 128-byte swizzle
    CUtensorMap map_x;           // xq: box 128 B x 128 rows, 128-byte swizzle
};

// Upload-time set-up: scale atoms from the sanitised scale rows, the
// activation-term buffers and both tensor maps. `state` receives device
// allocations the caller frees with free_linear_tc.
cudaError_t init_linear_tc(LinearTcState &state, const uint8_t *packed, int packed_pitch, const uint8_t *scales,
                           int scale_pitch, int rows, int cols, cudaStream_t stream);
void free_linear_tc(LinearTcState &state);

// One call (every pass of up to kLinTcVectors vectors): quantise the pass's
// activations into terms, then stream the weights through the MMAs.
// dst[v][r] = inv_global * sum_c W[r, c] * x[v, c].
cudaError_t launch_linear_tc(const LinearTcState &state, const float *x, int vectors, int rows, int cols,
                             float inv_global, float *dst, int sm_count, cudaStream_t stream);

}  // namespace nvfp4
