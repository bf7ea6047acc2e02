// One-token layer call in one persistent kernel (moe_token.cu).
#pragma once

#include "moe_decode.cuh"

namespace nvfp4 {

struct TokenArgs {
    const uint16_t *router;      // [(E+1)][H] BF16, row E = shared gate
    const float *bias;           // [E] router logit bias or nullptr
    const void *x;               // [H] BF16 or FP32
    int x_is_f32;
    const uint16_t *norm_w;      // [H] BF16 RMSNorm weight applied to x first, or nullptr (BF16 x only)
    float norm_eps;
    const void *residual;        // [H] BF16 or nullptr
    void *out;                   // [H] BF16, or FP32 when out_f32
    int out_f32;
    const uint8_t *packed[3];    // gate, up, down banks
    const uint8_t *scales[3];
    int scale_pitch[3];          // bytes per scale row (multiples of 16)
    const float *inv_scales;     // [3][E+1]
    int E, H, I;
    float *act;                  // [9][I] FP32 exchange buffer (SiLU(gate)*up)
    unsigned *sync;              // token_sync_bytes() of zeroed barrier words, owned by the bank
    DecodeScratch s;             // logits, ids, weights, counts, perm, error words
};

// Barrier words the kernel needs (zeroed once at allocation; the kernel
// leaves them at rest after every call).
size_t token_sync_bytes();
size_t token_smem_bytes(int sms, int H, int I, int gate_pitch, int down_pitch);
// Shapes the kernel serves on a grid of `sms` CTAs: H a multiple of 256 up
// to 2048, I a multiple of 128 up to 1024, 8..256 experts, and the CTA's
// rows fitting in shared memory.
bool token_supported(int sms, int E, int H, int I, int gate_pitch, int down_pitch);
cudaError_t launch_token(const TokenArgs &a, int sms, cudaStream_t stream);

}  // namespace nvfp4
