// Prefill path: routing, dispatch, activation quantisation and combine
// kernels (the tcgen05 expert GEMMs are in moe_gemm.cu).
#include "moe_prefill.cuh"
#include "quant_terms.cuh"
#include "tcgen05_util.cuh"
#include "tma_util.cuh"

#include <atomic>
#include <cfloat>

namespace nvfp4 {

namespace {

constexpr int kLogitsTile = 64;       // tokens x router rows per CTA of the logits kernel
constexpr int kSelectWarps = 8;       // tokens per CTA of the select kernel
constexpr int kMaxCandidates = 64;
// Margin of the approximate logits. Both the tensor-core logit and the exact
// one are FP32 sums of the same exactly representable BF16 x BF16 products
// p_k; any FP32 summation order of H terms, even with truncating adds, stays
// within 2 * H * 2^-24 * sum|p| of the true sum, and sum|p| <= |w| * |x|.
// delta = H * 2^-21 * |w| * |x| is twice the resulting bound on
// |approx - exact|, so every expert of the exact top-8 has an approximate
// logit >= (approximate 8th largest) - 2 * delta.
constexpr float kMarginPerColumn = 1.0f / 2097152.0f;  // 2^-21

__device__ __forceinline__ unsigned float_order_key(float v) {
    v = (v == 0.0f) ? 0.0f : v;
    const unsigned b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ------------------------------------------------------ approximate logits
//
// approx[t][e] = sum_k x[t,k] * W[e,k] with BF16 tensor-core MMAs (FP32
// accumulation, order unspecified). A CTA covers 64 tokens x 64 router rows;
// 64-column chunks of both are staged in shared memory (cp.async, double
// buffered, rows padded to 144 bytes so fragment loads are conflict-free).
// Warp w computes tokens 16w..16w+15 against all 64 rows; lane (g, c) reads
// columns [16c, 16c+16) of its rows, and the four k16 steps of a chunk map
// the MMA's k-slots {2c, 2c+1, 2c+8, 2c+9} to columns 16c + 4i + {0,1,2,3},
// the same mapping on both operands.
constexpr int kLogitsPitch = 144;

// Approximate logits on tcgen05 (kind::f16, BF16 x BF16 -> FP32 in tensor
// memory): one CTA per tile of 128 tokens x 64 router rows, all of K = H in
// 64-column stages through a 6-deep TMA ring. Warp 0 issues the TMA loads
// (token rows and router rows as 128-byte swizzled boxes), warp 1 the MMAs
// (four M128 N64 K16 per stage), warps 2-5 move the accumulator to `approx`.
// The order of the FP32 additions differs from the exact logits; the
// candidate margin of the selection bounds any order.
constexpr int kLtTokens = 128, kLtRows = 64, kLtStages = 6;
constexpr int kLtStageBytes = kLtTokens * 128 + kLtRows * 128;
constexpr size_t kLtSmem = 1024 + (size_t)kLtStages * kLtStageBytes + 256;

__global__ void __launch_bounds__(192, 1)
    prefill_logits_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                             PrefillRouteArgs a, float *approx, int Rp, int *err, int *host_err) {
    extern __shared__ uint8_t lt_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(lt_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)kLtStages * kLtStageBytes);
    uint64_t *empty = full + kLtStages;
    uint64_t *acc_full = empty + kLtStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
    int *acc_ok = reinterpret_cast<int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * kLtTokens, e0 = blockIdx.y * kLtRows;
    const int kstages = a.H / 64;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kLtStages; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, 1);
        }
        mbar_init(acc_full, 1);
        fence_barrier_init();
        prefetch_tensormap(&tm_x);
        prefetch_tensormap(&tm_w);
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, 64);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            for (int ks = 0; ks < kstages; ++ks, ++it) {
                const int st = it % kLtStages;
                if (!mbar_wait(empty + st, ((it / kLtStages) & 1u) ^ 1u, err, kSiteGemmEmpty)) {
                    // Drain the loads in flight (bounded) before the CTA exits.
                    const uint32_t first = it > (uint32_t)kLtStages ? it - kLtStages : 0u;
                    for (uint32_t k = first; k < it; ++k) {
                        const unsigned long long w0 = global_ns();
                        while (!mbar_try_wait(full + (k % kLtStages), (k / kLtStages) & 1u) &&
                               global_ns() - w0 < kWaitLimitNs) {
                        }
                    }
                    break;
                }
                uint8_t *stage = smem + (size_t)st * kLtStageBytes;
                mbar_arrive_expect_tx(full + st, kLtStageBytes);
                tma_load_2d(stage, &tm_x, full + st, ks * 128, t0);
                tma_load_2d(stage + kLtTokens * 128, &tm_w, full + st, ks * 128, e0);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_bf16(kLtRows);
            const uint32_t base = smem_u32(smem);
            bool ok = true;
            for (int ks = 0; ks < kstages && ok; ++ks) {
                const int st = ks % kLtStages;
                if (!mbar_wait(full + st, (ks / kLtStages) & 1u, err, kSiteGemmFull)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t sb = base + (uint32_t)st * kLtStageBytes;
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    tc::mma_bf16(tmem, tc::smem_desc_sw128(sb + 32 * k), tc::smem_desc_sw128(sb + kLtTokens * 128 + 32 * k),
                                 idesc, (ks | k) != 0 ? 1u : 0u);
                tc::commit(empty + st);
            }
            tc::commit(acc_full);
            // Every MMA has completed before tensor memory is freed (bounded).
            const unsigned long long w0 = global_ns();
            while (!mbar_try_wait(acc_full, 0) && global_ns() - w0 < kWaitLimitNs) {
            }
        }
        __syncwarp();
    } else {
        const int sub = warp & 3;
        if (threadIdx.x == 64) *acc_ok = mbar_wait(acc_full, 0, err, kSiteGemmAccFull) ? 1 : 0;
        named_barrier(1, 128);
        if (*reinterpret_cast<volatile int *>(acc_ok)) {
            tc::fence_after_sync();
            const int t = t0 + 32 * sub + lane;
#pragma unroll
            for (int c0 = 0; c0 < kLtRows; c0 += 32) {
                uint32_t r[32];
                tc::ld_32x32b_x32(tmem + ((uint32_t)(32 * sub) << 16) + c0, r);
                tc::wait_ld();
                if (t < a.T) {
#pragma unroll
                    for (int n = 0; n < 32; ++n) {
                        const int e = e0 + c0 + n;
                        if (e < a.E) approx[(size_t)t * Rp + e] = __uint_as_float(r[n]);
                    }
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 64);
    }
    if (threadIdx.x == 0 && *reinterpret_cast<volatile int *>(err) != 0 && host_err)
        *reinterpret_cast<volatile int *>(host_err) = *reinterpret_cast<volatile int *>(err);
}

constexpr int kLogitsStages = 4;      // cp.async ring depth (64 columns of x and of the router per stage)
constexpr int kLogitsStageBytes = 2 * kLogitsTile * kLogitsPitch;

__global__ void __launch_bounds__(128) prefill_logits_kernel(PrefillRouteArgs a, float *approx, int Rp) {
    extern __shared__ __align__(16) uint8_t logits_smem[];  // [kLogitsStages][x tile | router tile]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, c = lane & 3;
    const int R = a.E + 1, H = a.H;
    const int t0 = blockIdx.x * kLogitsTile, e0 = blockIdx.y * kLogitsTile;
    const int chunks = H / 64;
    // Stage kc holds columns [64 kc, 64 kc + 64) of the CTA's 64 tokens and
    // 64 router rows; three stages are in flight while one is multiplied.
    auto load = [&](int kc) {
        if (kc < chunks) {
            uint8_t *sx = logits_smem + (size_t)(kc % kLogitsStages) * kLogitsStageBytes;
            uint8_t *sw = sx + kLogitsTile * kLogitsPitch;
            const int k = kc * 64;
            for (int i = tid; i < kLogitsTile * 8; i += 128) {
                const int r = i >> 3, u = i & 7;
                cp_async16(sx + r * kLogitsPitch + u * 16, a.x + (size_t)min(t0 + r, a.T - 1) * H + k + u * 8);
                cp_async16(sw + r * kLogitsPitch + u * 16, a.router + (size_t)min(e0 + r, R - 1) * H + k + u * 8);
            }
        }
        cp_async_commit();  // an empty group past the end keeps the group count uniform
    };
    float acc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[n][r] = 0.0f;
#pragma unroll
    for (int kc = 0; kc < kLogitsStages - 1; ++kc) load(kc);
    for (int kc = 0; kc < chunks; ++kc) {
        load(kc + kLogitsStages - 1);
        cp_async_wait_group<kLogitsStages - 1>();
        __syncthreads();
        const uint8_t *bx = logits_smem + (size_t)(kc % kLogitsStages) * kLogitsStageBytes;
        const uint8_t *bw = bx + kLogitsTile * kLogitsPitch;
        const uint4 xa0 = *reinterpret_cast<const uint4 *>(bx + (16 * warp + g) * kLogitsPitch + 32 * c);
        const uint4 xa1 = *reinterpret_cast<const uint4 *>(bx + (16 * warp + g) * kLogitsPitch + 32 * c + 16);
        const uint4 xb0 = *reinterpret_cast<const uint4 *>(bx + (16 * warp + g + 8) * kLogitsPitch + 32 * c);
        const uint4 xb1 = *reinterpret_cast<const uint4 *>(bx + (16 * warp + g + 8) * kLogitsPitch + 32 * c + 16);
        const uint32_t A[8] = {xa0.x, xa0.y, xa0.z, xa0.w, xa1.x, xa1.y, xa1.z, xa1.w};
        const uint32_t B[8] = {xb0.x, xb0.y, xb0.z, xb0.w, xb1.x, xb1.y, xb1.z, xb1.w};
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            const uint4 w0 = *reinterpret_cast<const uint4 *>(bw + (8 * n + g) * kLogitsPitch + 32 * c);
            const uint4 w1 = *reinterpret_cast<const uint4 *>(bw + (8 * n + g) * kLogitsPitch + 32 * c + 16);
            const uint32_t W[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
                mma_bf16_16816(acc[n], A[2 * i], B[2 * i], A[2 * i + 1], B[2 * i + 1], W[2 * i], W[2 * i + 1]);
        }
        __syncthreads();  // the stage is refilled by a later iteration's load
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int t = t0 + 16 * warp + g + (r >= 2 ? 8 : 0);
            const int e = e0 + 8 * n + 2 * c + (r & 1);
            if (t < a.T && e < R) approx[(size_t)t * Rp + e] = acc[n][r];
        }
    }
}

// Exact router logit of row `row` for token row `x` in the lab's FP32 order
// (lane l owns columns j*128 + 4l + e; product and sum rounded separately;
// xor butterfly 16..1), identical to the decode routing kernel's order.
__device__ __forceinline__ float exact_logit(const uint16_t *w, const uint16_t *x, int H, int lane) {
    float acc = 0.0f;
    for (int k = lane * 4; k < H; k += 128) {
        const uint2 wv = __ldg(reinterpret_cast<const uint2 *>(w + k));
        const uint2 xv = __ldg(reinterpret_cast<const uint2 *>(x + k));
        acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(wv.x & 0xFFFFu), bf16_bits_to_f32(xv.x & 0xFFFFu)));
        acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(wv.x >> 16), bf16_bits_to_f32(xv.x >> 16)));
        acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(wv.y & 0xFFFFu), bf16_bits_to_f32(xv.y & 0xFFFFu)));
        acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(wv.y >> 16), bf16_bits_to_f32(xv.y >> 16)));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
    return acc;
}

// Four exact logits at once (independent chains, identical per-row order).
__device__ __forceinline__ void exact_logit4(const uint16_t *router, const int (&rows)[4], const uint16_t *x, int H,
                                             int lane, float (&out)[4]) {
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int k = lane * 4; k < H; k += 128) {
        const uint2 xv = __ldg(reinterpret_cast<const uint2 *>(x + k));
        const float x0 = bf16_bits_to_f32(xv.x & 0xFFFFu), x1 = bf16_bits_to_f32(xv.x >> 16);
        const float x2 = bf16_bits_to_f32(xv.y & 0xFFFFu), x3 = bf16_bits_to_f32(xv.y >> 16);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const uint2 wv = __ldg(reinterpret_cast<const uint2 *>(router + (size_t)rows[r] * H + k));
            acc[r] = __fadd_rn(acc[r], __fmul_rn(bf16_bits_to_f32(wv.x & 0xFFFFu), x0));
            acc[r] = __fadd_rn(acc[r], __fmul_rn(bf16_bits_to_f32(wv.x >> 16), x1));
            acc[r] = __fadd_rn(acc[r], __fmul_rn(bf16_bits_to_f32(wv.y & 0xFFFFu), x2));
            acc[r] = __fadd_rn(acc[r], __fmul_rn(bf16_bits_to_f32(wv.y >> 16), x3));
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) acc[r] = __fadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], off));
        out[r] = acc[r];
    }
}

// One warp per token: approximate top-8 boundary, exact logits of every
// expert within twice the margin of it (a superset of the exact top-8), then
// the exact top-8 (lowest id on ties), renormalised softmax weights and the
// sigmoid shared gate -- the same selection and weight arithmetic as the
// decode routing kernel. Also records the token in its 64-token block's
// per-expert bit masks for dispatch.
__global__ void __launch_bounds__(kSelectWarps * 32) prefill_select_kernel(PrefillRouteArgs a, PrefillScratch s,
                                                                          int Rp) {
    __shared__ int s_cand[kSelectWarps][kMaxCandidates];
    __shared__ float s_val[kSelectWarps][kMaxCandidates];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * kSelectWarps + warp;
    if (t >= a.T) return;
    const int E = a.E, H = a.H;
    const uint16_t *x = a.x + (size_t)t * H;

    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = lane + 32 * i;
        float val = -FLT_MAX;
        if (e < E) {
            val = s.approx[(size_t)t * Rp + e];
            if (a.bias) val += a.bias[e];
        }
        v[i] = val;
    }
    // 8th largest approximate logit.
    float a8 = -FLT_MAX;
    {
        unsigned taken = 0;
        for (int slot = 0; slot < kTopK; ++slot) {
            float bv = -FLT_MAX;
            int bi = -1;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (!((taken >> i) & 1u) && lane + 32 * i < E && (bi < 0 || v[i] > bv)) {
                    bv = v[i];
                    bi = i;
                }
            const unsigned key = bi < 0 ? 0u : float_order_key(bv);
            const unsigned kmax = __reduce_max_sync(0xffffffffu, key);
            const unsigned owner = __ffs(__ballot_sync(0xffffffffu, key == kmax && bi >= 0)) - 1;
            if (lane == (int)owner) taken |= 1u << bi;
            a8 = __shfl_sync(0xffffffffu, bv, owner);
        }
    }
    // |x| for the margin.
    float ss = 0.0f;
    for (int k = lane * 4; k < H; k += 128) {
        const uint2 xv = __ldg(reinterpret_cast<const uint2 *>(x + k));
        const float x0 = bf16_bits_to_f32(xv.x & 0xFFFFu), x1 = bf16_bits_to_f32(xv.x >> 16);
        const float x2 = bf16_bits_to_f32(xv.y & 0xFFFFu), x3 = bf16_bits_to_f32(xv.y >> 16);
        ss += x0 * x0 + x1 * x1 + x2 * x2 + x3 * x3;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float delta = kMarginPerColumn * (float)H * a.wnorm_max * sqrtf(ss) * 1.0001f + 1e-30f;
    const float thresh = a8 - 2.0f * delta;

    // Candidate list (expert ids ascending within each lane's stride).
    int n = 0;
    bool overflow = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = lane + 32 * i;
        const bool cand = e < E && v[i] >= thresh;
        const unsigned m = __ballot_sync(0xffffffffu, cand);
        const int idx = n + __popc(m & ((1u << lane) - 1u));
        if (cand && idx < kMaxCandidates) s_cand[warp][idx] = e;
        n += __popc(m);
    }
    if (n > kMaxCandidates) {
        overflow = true;
        n = 0;
    }
    __syncwarp();
    // Exact logits; on overflow every expert is evaluated in a streaming
    // top-8 (rare: it needs a very flat logit distribution).
    float top_v[kTopK];
    int top_i[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        top_v[k] = -FLT_MAX;
        top_i[k] = 0x7fffffff;
    }
    if (!overflow) {
        // Candidates four at a time; the shared-gate row rides along in the
        // first group's spare slot when there is one.
        for (int i0 = 0; i0 < n; i0 += 4) {
            int rows[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) rows[r] = i0 + r < n ? s_cand[warp][i0 + r] : E;
            float val[4];
            exact_logit4(a.router, rows, x, H, lane, val);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                if (i0 + r < n) {
                    float v2 = val[r];
                    if (a.bias) v2 = __fadd_rn(v2, a.bias[rows[r]]);
                    if (lane == 0) s_val[warp][i0 + r] = v2;
                }
            }
        }
        __syncwarp();
        // Top-8 of the candidates: lane holds candidates lane and lane+32.
        float cv[2];
        int ci[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int idx = lane + 32 * h;
            cv[h] = idx < n ? s_val[warp][idx] : -FLT_MAX;
            ci[h] = idx < n ? s_cand[warp][idx] : 0x7fffffff;
        }
        for (int slot = 0; slot < kTopK; ++slot) {
            float bv = -FLT_MAX;
            int bi = 0x7fffffff;
#pragma unroll
            for (int h = 0; h < 2; ++h)
                if (ci[h] != 0x7fffffff && (cv[h] > bv || (cv[h] == bv && ci[h] < bi))) {
                    bv = cv[h];
                    bi = ci[h];
                }
            const unsigned key = bi == 0x7fffffff ? 0u : float_order_key(bv);
            const unsigned kmax = __reduce_max_sync(0xffffffffu, key);
            const unsigned imin = __reduce_min_sync(0xffffffffu, key == kmax ? (unsigned)bi : 0xffffffffu);
            const int owner_h = (ci[0] == (int)imin) ? 0 : 1;
            const bool mine = (ci[0] == (int)imin) || (ci[1] == (int)imin);
            const unsigned ob = __ballot_sync(0xffffffffu, mine);
            const int owner = __ffs(ob) - 1;
            const float val = __shfl_sync(0xffffffffu, mine ? cv[owner_h] : 0.0f, owner);
            if (mine) ci[owner_h] = 0x7fffffff;
            top_v[slot] = val;
            top_i[slot] = (int)imin;
        }
    } else {
        for (int e = 0; e < E; ++e) {
            float val = exact_logit(a.router + (size_t)e * H, x, H, lane);
            if (a.bias) val = __fadd_rn(val, a.bias[e]);
            // Insert into the running top-8 (every lane keeps the same copy).
            if (val > top_v[kTopK - 1]) {
                int p = kTopK - 1;
                while (p > 0 && val > top_v[p - 1]) {
                    top_v[p] = top_v[p - 1];
                    top_i[p] = top_i[p - 1];
                    --p;
                }
                top_v[p] = val;
                top_i[p] = e;
            }
        }
    }
    const float sl = exact_logit(a.router + (size_t)E * H, x, H, lane);
    if (lane == 0) {
        float den = 0.0f;
#pragma unroll
        for (int slot = 0; slot < kTopK; ++slot) den += expf(top_v[slot] - top_v[0]);
        for (int slot = 0; slot < kTopK; ++slot) {
            s.ids[t * kSlots + slot] = top_i[slot];
            s.weights[t * kSlots + slot] = expf(top_v[slot] - top_v[0]) / den;
        }
        s.ids[t * kSlots + kTopK] = E;
        s.weights[t * kSlots + kTopK] = 1.0f / (1.0f + expf(-sl));
    }
    if (lane < kTopK) {
        const int e = top_i[lane];
        atomicOr(&s.blk_mask[(size_t)e * s.mask_stride + (t >> 6)], 1ull << (t & 63));
    }
}

// prefill_select_kernel with the token held in registers: lane l keeps its
// CH column chunks of x (columns 128q + 4l .. +3, the order of the exact
// logit), so x is read once per token instead of once per group of four
// exact rows; the weight loads of four chunks of four rows are in flight
// together; the shared gate's row is the last entry of the row list
// (candidates, then row E) instead of a separate pass; the softmax
// exponentials run one per lane. Every rounded operation and every
// summation order is the one of prefill_select_kernel, so the ids, weights
// and gates are the same bits (the rare overflow case, more than
// kMaxCandidates candidates, runs prefill_select_kernel's streaming loop).
template <int CH>
__global__ void __launch_bounds__(kSelectWarps * 32) prefill_select_reg_kernel(PrefillRouteArgs a, PrefillScratch s,
                                                                              int Rp) {
    __shared__ int s_cand[kSelectWarps][kMaxCandidates];
    __shared__ float s_val[kSelectWarps][kMaxCandidates];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * kSelectWarps + warp;
    if (t >= a.T) return;
    const int E = a.E, H = a.H;
    const uint16_t *x = a.x + (size_t)t * H;

    uint2 xr[CH];
#pragma unroll
    for (int q = 0; q < CH; ++q) xr[q] = __ldg(reinterpret_cast<const uint2 *>(x + 128 * q + 4 * lane));
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = lane + 32 * i;
        float val = -FLT_MAX;
        if (e < E) {
            val = s.approx[(size_t)t * Rp + e];
            if (a.bias) val += a.bias[e];
        }
        v[i] = val;
    }
    // 8th largest approximate logit.
    float a8 = -FLT_MAX;
    {
        unsigned taken = 0;
#pragma unroll 1
        for (int slot = 0; slot < kTopK; ++slot) {
            float bv = -FLT_MAX;
            int bi = -1;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (!((taken >> i) & 1u) && lane + 32 * i < E && (bi < 0 || v[i] > bv)) {
                    bv = v[i];
                    bi = i;
                }
            const unsigned key = bi < 0 ? 0u : float_order_key(bv);
            const unsigned kmax = __reduce_max_sync(0xffffffffu, key);
            const unsigned owner = __ffs(__ballot_sync(0xffffffffu, key == kmax && bi >= 0)) - 1;
            if (lane == (int)owner) taken |= 1u << bi;
            a8 = __shfl_sync(0xffffffffu, bv, owner);
        }
    }
    // |x| for the margin (the same per-lane partial sums and butterfly).
    float ss = 0.0f;
#pragma unroll
    for (int q = 0; q < CH; ++q) {
        const float x0 = bf16_bits_to_f32(xr[q].x & 0xFFFFu), x1 = bf16_bits_to_f32(xr[q].x >> 16);
        const float x2 = bf16_bits_to_f32(xr[q].y & 0xFFFFu), x3 = bf16_bits_to_f32(xr[q].y >> 16);
        ss += x0 * x0 + x1 * x1 + x2 * x2 + x3 * x3;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float delta = kMarginPerColumn * (float)H * a.wnorm_max * sqrtf(ss) * 1.0001f + 1e-30f;
    const float thresh = a8 - 2.0f * delta;

    int n = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = lane + 32 * i;
        const bool cand = e < E && v[i] >= thresh;
        const unsigned m = __ballot_sync(0xffffffffu, cand);
        const int idx = n + __popc(m & ((1u << lane) - 1u));
        if (cand && idx < kMaxCandidates) s_cand[warp][idx] = e;
        n += __popc(m);
    }
    if (n > kMaxCandidates) {
        float top_v[kTopK];
        int top_i[kTopK];
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            top_v[k] = -FLT_MAX;
            top_i[k] = 0x7fffffff;
        }
        for (int e = 0; e < E; ++e) {
            float val = exact_logit(a.router + (size_t)e * H, x, H, lane);
            if (a.bias) val = __fadd_rn(val, a.bias[e]);
            if (val > top_v[kTopK - 1]) {
                int p = kTopK - 1;
                while (p > 0 && val > top_v[p - 1]) {
                    top_v[p] = top_v[p - 1];
                    top_i[p] = top_i[p - 1];
                    --p;
                }
                top_v[p] = val;
                top_i[p] = e;
            }
        }
        const float sl_o = exact_logit(a.router + (size_t)E * H, x, H, lane);
        if (lane == 0) {
            float den = 0.0f;
#pragma unroll
            for (int slot = 0; slot < kTopK; ++slot) den += expf(top_v[slot] - top_v[0]);
            for (int slot = 0; slot < kTopK; ++slot) {
                s.ids[t * kSlots + slot] = top_i[slot];
                s.weights[t * kSlots + slot] = expf(top_v[slot] - top_v[0]) / den;
            }
            s.ids[t * kSlots + kTopK] = E;
            s.weights[t * kSlots + kTopK] = 1.0f / (1.0f + expf(-sl_o));
        }
        if (lane < kTopK) {
            const int e = top_i[lane];
            atomicOr(&s.blk_mask[(size_t)e * s.mask_stride + (t >> 6)], 1ull << (t & 63));
        }
        return;
    }
    __syncwarp();
    // Exact logits of the candidates, then of row E (the shared gate), four
    // rows at a time.
    float sl = 0.0f;
#pragma unroll 1
    for (int i0 = 0; i0 <= n; i0 += 4) {
        int rows[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) rows[r] = i0 + r < n ? s_cand[warp][i0 + r] : E;
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int q0 = 0; q0 < CH; q0 += 4) {
            uint2 wv[4][4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    wv[r][u] = __ldg(reinterpret_cast<const uint2 *>(a.router + (size_t)rows[r] * H + 128 * (q0 + u) +
                                                                     4 * lane));
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint2 xv = xr[q0 + u];
                const float x0 = bf16_bits_to_f32(xv.x & 0xFFFFu), x1 = bf16_bits_to_f32(xv.x >> 16);
                const float x2 = bf16_bits_to_f32(xv.y & 0xFFFFu), x3 = bf16_bits_to_f32(xv.y >> 16);
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    acc[r] = __fadd_rn(acc[r], __fmul_rn(bf16_bits_to_f32(wv[r][u].x & 0xFFFFu), x0));
                    acc[r] = __fadd_rn(acc[r], __fmul_rn(bf16_bits_to_f32(wv[r][u].x >> 16), x1));
                    acc[r] = __fadd_rn(acc[r], __fmul_rn(bf16_bits_to_f32(wv[r][u].y & 0xFFFFu), x2));
                    acc[r] = __fadd_rn(acc[r], __fmul_rn(bf16_bits_to_f32(wv[r][u].y >> 16), x3));
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1)
                acc[r] = __fadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], off));
            if (i0 + r < n) {
                float v2 = acc[r];
                if (a.bias) v2 = __fadd_rn(v2, a.bias[rows[r]]);
                if (lane == 0) s_val[warp][i0 + r] = v2;
            } else if (i0 + r == n) {
                sl = acc[r];
            }
        }
    }
    __syncwarp();
    // Top-8 of the candidates (lane holds candidates lane and lane + 32);
    // lane `slot` keeps the slot-th pick.
    float cv[2];
    int ci[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int idx = lane + 32 * h;
        cv[h] = idx < n ? s_val[warp][idx] : -FLT_MAX;
        ci[h] = idx < n ? s_cand[warp][idx] : 0x7fffffff;
    }
    float my_v = 0.0f, top0 = 0.0f;
    int my_i = 0;
#pragma unroll 1
    for (int slot = 0; slot < kTopK; ++slot) {
        float bv = -FLT_MAX;
        int bi = 0x7fffffff;
#pragma unroll
        for (int h = 0; h < 2; ++h)
            if (ci[h] != 0x7fffffff && (cv[h] > bv || (cv[h] == bv && ci[h] < bi))) {
                bv = cv[h];
                bi = ci[h];
            }
        const unsigned key = bi == 0x7fffffff ? 0u : float_order_key(bv);
        const unsigned kmax = __reduce_max_sync(0xffffffffu, key);
        const unsigned imin = __reduce_min_sync(0xffffffffu, key == kmax ? (unsigned)bi : 0xffffffffu);
        const int owner_h = (ci[0] == (int)imin) ? 0 : 1;
        const bool mine = (ci[0] == (int)imin) || (ci[1] == (int)imin);
        const unsigned ob = __ballot_sync(0xffffffffu, mine);
        const int owner = __ffs(ob) - 1;
        const float val = __shfl_sync(0xffffffffu, mine ? cv[owner_h] : 0.0f, owner);
        if (mine) ci[owner_h] = 0x7fffffff;
        if (slot == 0) top0 = val;
        if (lane == slot) {
            my_v = val;
            my_i = (int)imin;
        }
    }
    // Softmax over the picks relative to the largest, the denominator added
    // in slot order; one exponential per lane.
    const float my_e = lane < kTopK ? expf(my_v - top0) : 0.0f;
    float den = 0.0f;
#pragma unroll
    for (int slot = 0; slot < kTopK; ++slot) den += __shfl_sync(0xffffffffu, my_e, slot);
    if (lane < kTopK) {
        s.ids[t * kSlots + lane] = my_i;
        s.weights[t * kSlots + lane] = my_e / den;
        atomicOr(&s.blk_mask[(size_t)my_i * s.mask_stride + (t >> 6)], 1ull << (t & 63));
    } else if (lane == kTopK) {
        s.ids[t * kSlots + kTopK] = E;
        s.weights[t * kSlots + kTopK] = 1.0f / (1.0f + expf(-sl));
    }
}

// Exclusive prefix sum over the 256 threads of a CTA; *total gets the sum.
__device__ __forceinline__ int block_excl_scan256(int v, int *warp_sums, int *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inc = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += o;
    }
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int w = lane < 8 ? warp_sums[lane] : 0;
        int winc = w;
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, winc, off);
            if (lane >= off) winc += o;
        }
        if (lane < 8) warp_sums[8 + lane] = winc - w;
        if (lane == 7) warp_sums[16] = winc;
    }
    __syncthreads();
    const int ex = warp_sums[8 + warp] + inc - v;
    *total = warp_sums[16];
    __syncthreads();
    return ex;
}

// One CTA per routed expert: rank bases of its 64-token blocks (prefix sum
// of the block masks' popcounts) and its token count. The last CTA to finish
// then builds the cross-expert tables: unpadded offsets (routing ABI),
// padded group starts, the compacted active groups (routed experts with
// tokens, then the shared expert) and the GEMM column-tile table.
__global__ void __launch_bounds__(256) prefill_scan_kernel(PrefillScratch s, int T) {
    __shared__ int warp_sums[17];
    __shared__ int s_last;
    const int E = s.E;
    const int nb = (T + 63) / 64;
    const int e = blockIdx.x;
    int total = 0;
    for (int b0 = 0; b0 < nb; b0 += 256) {
        const int b = b0 + threadIdx.x;
        const int c = b < nb ? __popcll(s.blk_mask[(size_t)e * s.mask_stride + b]) : 0;
        int chunk = 0;
        const int ex = block_excl_scan256(c, warp_sums, &chunk);
        if (b < nb) s.blk_base[(size_t)e * s.mask_stride + b] = total + ex;
        total += chunk;
    }
    if (threadIdx.x == 0) {
        s.counts[e] = total;
        __threadfence();
        s_last = atomicAdd(s.ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    const int i = threadIdx.x;
    const int cnt = i < E ? __ldcg(s.counts + i) : 0;
    // Only the experts computed here get padded rows, groups and tiles.
    const bool own = i >= s.e_first && i < s.e_first + s.e_count;
    const int ocnt = own ? cnt : 0;
    const int ntile = (ocnt + kPrefillTileN - 1) / kPrefillTileN;
    int n_off = 0, n_act = 0, n_tiles = 0, n_pad = 0;
    const int off = block_excl_scan256(cnt, warp_sums, &n_off);
    const int ai = block_excl_scan256(ocnt > 0 ? 1 : 0, warp_sums, &n_act);
    const int tile0 = block_excl_scan256(ntile, warp_sums, &n_tiles);
    const int pst = block_excl_scan256(ntile * kPrefillTileN, warp_sums, &n_pad);
    if (i < E) {
        s.offsets[i] = off;
        s.epstart[i] = pst;
        if (ocnt > 0) {
            s.active_expert[ai] = i;
            s.tok_start[ai] = pst;
            s.tok_count[ai] = cnt;
            for (int j = 0; j < ntile; ++j) {
                s.tile_group[tile0 + j] = ai;
                s.tile_n0[tile0 + j] = pst + j * kPrefillTileN;
            }
        }
    }
    const int shared_tiles = s.shared_here ? (T + kPrefillTileN - 1) / kPrefillTileN : 0;
    for (int j = i; j < shared_tiles; j += blockDim.x) {
        s.tile_group[n_tiles + j] = n_act;
        s.tile_n0[n_tiles + j] = n_pad + j * kPrefillTileN;
    }
    if (i == 0) {
        s.offsets[E] = n_off;
        s.epstart[E] = n_pad;
        if (s.shared_here) {
            s.active_expert[n_act] = E;
            s.tok_start[n_act] = n_pad;
            s.tok_count[n_act] = T;
        }
        *s.n_active = n_act + (s.shared_here ? 1 : 0);
        *s.n_tiles = n_tiles + shared_tiles;
        *s.rows_used = n_pad + shared_tiles * kPrefillTileN;
        *s.ticket = 0u;
    }
}

// Thread per (token, slot): rank among the expert's tokens (tokens
// ascending), giving the unpadded dispatch position (routing ABI) and the
// padded slot row used by the GEMMs.
__global__ void prefill_place_kernel(PrefillScratch s, int T, const float *inv_scales) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int E = s.E;
    const float *inv_down = inv_scales + 2 * (size_t)(E + 1);
    if (i < T * kTopK) {
        const int t = i / kTopK, k = i - t * kTopK;
        const int e = s.ids[t * kSlots + k];
        const int b = t >> 6;
        const unsigned long long m = s.blk_mask[(size_t)e * s.mask_stride + b];
        const int rank = s.blk_base[(size_t)e * s.mask_stride + b] + __popcll(m & ((1ull << (t & 63)) - 1ull));
        s.perm[s.offsets[e] + rank] = i;
        if (e < s.e_first || e >= s.e_first + s.e_count) {
            s.inv_pos[i] = -1;  // computed on another rank
            return;
        }
        const int row = s.epstart[e] + rank;
        s.tok_list[row] = t;
        s.inv_pos[i] = row;
        s.coef[row] = s.weights[t * kSlots + k] * inv_down[e];
    } else if (i < T * kSlots && s.shared_here) {
        const int t = i - T * kTopK;
        const int row = s.epstart[E] + t;
        s.tok_list[row] = t;
        s.coef[row] = s.weights[t * kSlots + kTopK] * inv_down[E];
    }
}

// ------------------------------------------------------- quantisation

// Where a quantised row's scale words go.
//   kWords: compact words [J][rows_stride][cols/64] (the standalone ABI)
//   kTokenAtoms: row r is token r; its codes and words go to each of the
//     token's nine padded slot rows (inv_pos, shared row), words in tcgen05
//     scale-atom layout
//   kRowAtoms: row r is a padded slot row; words go to its own atoms, and
//     rows at or past *rows_used are skipped
enum QuantMode : int { kWords = 0, kTokenAtoms = 1, kRowAtoms = 2 };

struct QuantTargets {
    uint8_t *codes;           // [J][rows_stride][cols/2]
    uint32_t *words;          // kWords
    uint8_t *atoms;           // [J][atom_blocks][cols/64][512]
    float *g;                 // [rows]
    int rows_stride;
    int atom_blocks;
    const int *inv_pos;       // kTokenAtoms
    const int *shared_row0;   // kTokenAtoms: padded first row of the shared expert
    const int *rows_used;     // kRowAtoms
};

__device__ __forceinline__ size_t atom_offset(int j, int atom_blocks, int words_per_row, int p, int word) {
    return ((size_t)(j * atom_blocks + p / 128) * words_per_row + word) * 512 + (p % 32) * 16 + ((p % 128) / 32) * 4;
}

// One thread per 16-element block of a row (the row's threads reduce its
// absolute maximum first), terms in a loop that is not unrolled: a lean
// kernel keeps many rows in flight. Per term: s = E4M3_RN((bamax / 6) / g);
// denom = s * g; code = E2M1_RN(r * RN(1/denom)) (0 when denom is 0);
// r -= code * denom (quant_terms.cuh).
constexpr int kQuantThreads = 256;

template <int MODE>
__global__ void __launch_bounds__(kQuantThreads) quantize_blocks_kernel(const void *src, int src_kind, int rows,
                                                                       int cols, int terms, int row_threads,
                                                                       QuantTargets q) {
    __shared__ float s_warp_max[kQuantThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rows_per_cta = blockDim.x / row_threads;
    const int lr = threadIdx.x / row_threads;           // row within the CTA
    const int tr = threadIdx.x - lr * row_threads;      // thread within the row
    const int r = blockIdx.x * rows_per_cta + lr;
    bool valid = r < rows;
    if (MODE == kRowAtoms && valid && r >= *q.rows_used) valid = false;
    const int nb = cols / 16;
    const int wpr = cols / 64;
    const int esz = src_kind == 2 ? 4 : 2;
    const uint8_t *row = static_cast<const uint8_t *>(src) + (size_t)(valid ? r : 0) * cols * esz;
    auto load_block = [&](int b, float (&v)[16]) {
        if (src_kind == 2) {
            const float4 *p = reinterpret_cast<const float4 *>(row + (size_t)b * 64);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 f = __ldg(p + i);
                v[4 * i] = f.x;
                v[4 * i + 1] = f.y;
                v[4 * i + 2] = f.z;
                v[4 * i + 3] = f.w;
            }
            return;
        }
        const uint4 *p = reinterpret_cast<const uint4 *>(row + (size_t)b * 32);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint4 u = __ldg(p + i);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                if (src_kind == 1) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[h]));
                    v[8 * i + 2 * h] = f.x;
                    v[8 * i + 2 * h + 1] = f.y;
                } else {
                    v[8 * i + 2 * h] = bf16_bits_to_f32(w[h] & 0xFFFFu);
                    v[8 * i + 2 * h + 1] = bf16_bits_to_f32(w[h] >> 16);
                }
            }
        }
    };
    // Row absolute maximum: the row's threads (whole warps when a row spans
    // several; a lane group of a warp otherwise) reduce it.
    float amax = 0.0f;
    if (valid)
        for (int b = tr; b < nb; b += row_threads) {
            float v[16];
            load_block(b, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
        }
    const int span = row_threads < 32 ? row_threads : 32;
    for (int off = span >> 1; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if (row_threads > 32) {
        if (lane == 0) s_warp_max[warp] = amax;
        __syncthreads();
        const int w0 = (lr * row_threads) >> 5, nw = row_threads >> 5;
        amax = 0.0f;
#pragma unroll 1
        for (int w = 0; w < nw; ++w) amax = fmaxf(amax, s_warp_max[w0 + w]);
    }
    if (!valid) return;
    const float g = row_global_scale(amax);
    if (tr == 0) q.g[r] = g;
    int dst[kSlots];
    int ndst = 1;
    dst[0] = r;
    if (MODE == kTokenAtoms) {
        ndst = 0;
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            const int p = q.inv_pos[r * kTopK + k];
            if (p >= 0) dst[ndst++] = p;  // -1: the slot is computed on another rank
        }
        if (q.shared_row0) dst[ndst++] = *q.shared_row0 + r;
    }
    for (int b = tr; b < nb; b += row_threads) {
        float v[16];
        load_block(b, v);
#pragma unroll 1
        for (int j = 0; j < terms; ++j) {
            uint32_t c0, c1;
            const uint8_t sc = static_cast<uint8_t>(quantize_block_term(v, g, c0, c1));
#pragma unroll 1
            for (int d = 0; d < ndst; ++d) {
                const int p = dst[d];
                const size_t prow = (size_t)j * q.rows_stride + p;
                *reinterpret_cast<uint2 *>(q.codes + prow * (cols / 2) + (size_t)b * 8) = make_uint2(c0, c1);
                if (MODE == kWords)
                    reinterpret_cast<uint8_t *>(q.words)[(prow * wpr + (b >> 2)) * 4 + (b & 3)] = sc;
                else
                    q.atoms[atom_offset(j, q.atom_blocks, wpr, p, b >> 2) + (b & 3)] = sc;
            }
        }
    }
}

// ------------------------------------------------------------- combine

// out[t][h] = sum over routed slots k = 0..7 of ypart[inv_pos[t*8+k]][h],
// then the shared slot, then the BF16 residual (the decode combine order).
// Each thread handles 8 consecutive h.
__global__ void __launch_bounds__(256) prefill_combine_kernel(PrefillScratch s, int T, const uint16_t *residual,
                                                              void *out, int out_f32) {
    const int t = blockIdx.y;
    const int H = s.H;
    const int h = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (h >= H) return;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    auto add_row = [&](int pos) {
        const uint4 u = __ldg(reinterpret_cast<const uint4 *>(s.ypart + (size_t)pos * H + h));
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
            acc[2 * i] += f.x;
            acc[2 * i + 1] += f.y;
        }
    };
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        const int pos = s.inv_pos[t * kTopK + k];
        if (pos >= 0) add_row(pos);  // -1: the slot's expert is computed on another rank
    }
    if (s.shared_here) add_row(s.epstart[s.E] + t);
    uint32_t o[4];
    if (residual) {
        const uint4 u = __ldg(reinterpret_cast<const uint4 *>(residual + (size_t)t * H + h));
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            acc[2 * i] += bf16_bits_to_f32(w[i] & 0xFFFFu);
            acc[2 * i + 1] += bf16_bits_to_f32(w[i] >> 16);
        }
    }
    if (out_f32) {
        float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(out) + (size_t)t * H + h);
        dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
        return;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = f32_to_bf16_bits(acc[2 * i]) | (f32_to_bf16_bits(acc[2 * i + 1]) << 16);
    *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(out) + (size_t)t * H + h) = make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void scale_atoms_kernel(uint8_t *atoms, const uint8_t *scales, size_t pitch, int rows, int k16,
                                   int row0) {
    const size_t n = (size_t)rows * k16;
    const int kb64 = k16 / 4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int rl = (int)(i / k16), k = (int)(i - (size_t)rl * k16);
        const int r = row0 + rl;
        const size_t dst = ((size_t)(r / 128) * kb64 + k / 4) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (k % 4);
        atoms[dst] = scales[(size_t)r * pitch + k];
    }
}

}  // namespace

static int prefill_rows(int T, int E) {
    const long long rows = (long long)T * kSlots + (long long)(E + 1) * kPrefillTileN;
    return (int)((rows + kPrefillTileN - 1) / kPrefillTileN * kPrefillTileN);
}

size_t prefill_scratch_bytes(int T, int E, int H, int I, int Jx, int Ja) {
    PrefillScratch s{};
    prefill_scratch_carve(s, nullptr, T, E, H, I, Jx, Ja);
    return reinterpret_cast<size_t>(s.ypart) + (size_t)s.max_rows * H * 2 + 1024;
}

void prefill_scratch_carve(PrefillScratch &s, void *base, int T, int E, int H, int I, int Jx, int Ja) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 1023) & ~size_t(1023);
        return static_cast<uint8_t *>(base) + o;
    };
    const size_t Tz = (size_t)T;
    const int R = E + 1, Rp = (R + 63) / 64 * 64, nb = (T + 63) / 64;
    const size_t P = (size_t)prefill_rows(T, E);
    s.max_tokens = T;
    s.max_rows = (int)P;
    s.E = E;
    s.H = H;
    s.I = I;
    s.max_tiles = (int)(P / kPrefillTileN);
    s.approx = reinterpret_cast<float *>(take(Tz * Rp * 4));
    s.ids = reinterpret_cast<int *>(take(Tz * kSlots * 4));
    s.weights = reinterpret_cast<float *>(take(Tz * kSlots * 4));
    s.mask_stride = nb;
    s.blk_mask = reinterpret_cast<unsigned long long *>(take((size_t)nb * E * 8));
    s.blk_base = reinterpret_cast<int *>(take((size_t)nb * E * 4));
    s.ticket = reinterpret_cast<unsigned *>(take(4));
    s.counts = reinterpret_cast<int *>(take((size_t)E * 4));
    s.offsets = reinterpret_cast<int *>(take((size_t)R * 4));
    s.epstart = reinterpret_cast<int *>(take((size_t)R * 4));
    s.rows_used = reinterpret_cast<int *>(take(4));
    s.n_active = reinterpret_cast<int *>(take(4));
    s.active_expert = reinterpret_cast<int *>(take((size_t)R * 4));
    s.tok_start = reinterpret_cast<int *>(take((size_t)R * 4));
    s.tok_count = reinterpret_cast<int *>(take((size_t)R * 4));
    s.n_tiles = reinterpret_cast<int *>(take(4));
    s.tile_group = reinterpret_cast<int *>(take((size_t)s.max_tiles * 4));
    s.tile_n0 = reinterpret_cast<int *>(take((size_t)s.max_tiles * 4));
    s.perm = reinterpret_cast<int *>(take(Tz * kTopK * 4));
    s.inv_pos = reinterpret_cast<int *>(take(Tz * kTopK * 4));
    s.tok_list = reinterpret_cast<int *>(take(P * 4));
    s.coef = reinterpret_cast<float *>(take(P * 4));
    s.xq = take((size_t)Jx * P * H / 2);
    s.xsf = take((size_t)Jx * P * (H / 16));
    s.gx = reinterpret_cast<float *>(take(Tz * 4));
    s.act = reinterpret_cast<__half *>(take(P * I * 2));
    s.aq = take((size_t)Ja * P * I / 2);
    s.asf = take((size_t)Ja * P * (I / 16));
    s.ga = reinterpret_cast<float *>(take(P * 4));
    s.ypart = reinterpret_cast<__half *>(take(P * H * 2));
}

cudaError_t make_prefill_weight_maps(PrefillMaps &m, uint8_t *const packed[3], int E, int H, int I) {
    const uint64_t slots = static_cast<uint64_t>(E) + 1;
    for (int p = 0; p < 3; ++p) {
        const uint64_t rows = slots * (p < 2 ? I : H);
        const uint64_t k = p < 2 ? H : I;
        cudaError_t err = make_tensor_map_u8(&m.w[p], packed[p], k / 2, k / 2, rows, 128, kPrefillTileM,
                                             CU_TENSOR_MAP_SWIZZLE_128B);
        if (err != cudaSuccess) return err;
    }
    return cudaSuccess;
}

cudaError_t make_prefill_act_maps(PrefillMaps &m, const PrefillScratch &s, int Jx, int Ja) {
    const uint64_t P = (uint64_t)s.max_rows;
    cudaError_t err = make_tensor_map_u8(&m.xq, s.xq, s.H / 2, s.H / 2, Jx * P, 128, kPrefillTileN,
                                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (err != cudaSuccess) return err;
    return make_tensor_map_u8(&m.aq, s.aq, s.I / 2, s.I / 2, Ja * P, 128, kPrefillTileN, CU_TENSOR_MAP_SWIZZLE_128B);
}

cudaError_t launch_scale_atoms(uint8_t *atoms, const uint8_t *scales, size_t pitch, int rows, int k16, int row0,
                               cudaStream_t stream) {
    const size_t n = (size_t)rows * k16;
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    scale_atoms_kernel<<<grid, 256, 0, stream>>>(atoms, scales, pitch, rows, k16, row0);
    return cudaGetLastError();
}

cudaError_t make_prefill_router_map(PrefillMaps &m, const uint16_t *router, int E, int H) {
    return make_tensor_map_u8(&m.router, router, (uint64_t)H * 2, (uint64_t)H * 2, (uint64_t)E + 1, 128, kLtRows,
                              CU_TENSOR_MAP_SWIZZLE_128B);
}

cudaError_t launch_prefill_route(const PrefillRouteArgs &a, const PrefillScratch &s, int part, cudaStream_t stream,
                                 const PrefillMaps *maps) {
    const int R = a.E + 1, Rp = (R + 63) / 64 * 64;
    cudaError_t err = cudaSuccess;
    if (part == 0) {
        err = cudaMemsetAsync(s.blk_mask, 0, (size_t)s.mask_stride * a.E * 8, stream);
        if (err != cudaSuccess) return err;
        if (maps && a.H % 64 == 0) {
            CUtensorMap tm_x;
            err = make_tensor_map_u8(&tm_x, a.x, (uint64_t)a.H * 2, (uint64_t)a.H * 2, (uint64_t)a.T, 128, kLtTokens,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
            if (err != cudaSuccess) return err;
            static std::atomic<uint64_t> done_tc{0};
            int dev = 0;
            err = cudaGetDevice(&dev);
            if (err != cudaSuccess) return err;
            const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
            if (!bit || !(done_tc.load() & bit)) {
                err = cudaFuncSetAttribute(prefill_logits_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kLtSmem);
                if (err != cudaSuccess) return err;
                done_tc.fetch_or(bit);
            }
            const dim3 grid((a.T + kLtTokens - 1) / kLtTokens, (a.E + kLtRows - 1) / kLtRows);
            prefill_logits_tc_kernel<<<grid, 192, kLtSmem, stream>>>(tm_x, maps->router, a, s.approx, Rp, s.error,
                                                                      s.host_error);
            return cudaGetLastError();
        }
        constexpr size_t smem = (size_t)kLogitsStages * kLogitsStageBytes;
        static std::atomic<uint64_t> done{0};
        int dev = 0;
        err = cudaGetDevice(&dev);
        if (err != cudaSuccess) return err;
        const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
        if (!bit || !(done.load() & bit)) {
            err = cudaFuncSetAttribute(prefill_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (err != cudaSuccess) return err;
            done.fetch_or(bit);
        }
        prefill_logits_kernel<<<dim3((a.T + kLogitsTile - 1) / kLogitsTile, (R + kLogitsTile - 1) / kLogitsTile), 128,
                                smem, stream>>>(a, s.approx, Rp);
    } else if (part == 1) {
        const int blocks = (a.T + kSelectWarps - 1) / kSelectWarps;
        if (a.H == 2048)
            prefill_select_reg_kernel<16><<<blocks, kSelectWarps * 32, 0, stream>>>(a, s, Rp);
        else if (a.H == 1024)
            prefill_select_reg_kernel<8><<<blocks, kSelectWarps * 32, 0, stream>>>(a, s, Rp);
        else if (a.H == 512)
            prefill_select_reg_kernel<4><<<blocks, kSelectWarps * 32, 0, stream>>>(a, s, Rp);
        else
            prefill_select_kernel<<<blocks, kSelectWarps * 32, 0, stream>>>(a, s, Rp);
    } else {
        prefill_scan_kernel<<<a.E, 256, 0, stream>>>(s, a.T);
        err = cudaGetLastError();
        if (err != cudaSuccess) return err;
        const int n = a.T * kSlots;
        prefill_place_kernel<<<(n + 255) / 256, 256, 0, stream>>>(s, a.T, a.inv_scales);
    }
    return cudaGetLastError();
}

template <int MODE>
static cudaError_t launch_quantize_mode(const void *src, int src_kind, int rows, int cols, int terms,
                                        const QuantTargets &q, cudaStream_t stream) {
    if (cols % 64 != 0 || rows <= 0 || terms < 1 || terms > kMaxTerms) return cudaErrorInvalidValue;
    // Threads per row: one per 16-element block, a power of two up to the CTA.
    const int nb = cols / 16;
    int row_threads = 4;
    while (row_threads < nb && row_threads < kQuantThreads) row_threads <<= 1;
    const int rows_per_cta = kQuantThreads / row_threads;
    const int grid = (rows + rows_per_cta - 1) / rows_per_cta;
    quantize_blocks_kernel<MODE><<<grid, kQuantThreads, 0, stream>>>(src, src_kind, rows, cols, terms, row_threads, q);
    return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const void *src, int src_is_f16, int rows, int cols, int terms, uint8_t *codes,
                                 uint32_t *sf, float *g, int rows_stride, cudaStream_t stream) {
    QuantTargets q{};
    q.codes = codes;
    q.words = sf;
    q.g = g;
    q.rows_stride = rows_stride;
    return launch_quantize_mode<kWords>(src, src_is_f16, rows, cols, terms, q, stream);
}

cudaError_t launch_quantize_x_prefill(const void *x, int T, const PrefillScratch &s, int terms, cudaStream_t stream) {
    QuantTargets q{};
    q.codes = s.xq;
    q.atoms = s.xsf;
    q.g = s.gx;
    q.rows_stride = s.max_rows;
    q.atom_blocks = s.max_rows / kPrefillTileN;
    q.inv_pos = s.inv_pos;
    q.shared_row0 = s.shared_here ? s.epstart + s.E : nullptr;
    return launch_quantize_mode<kTokenAtoms>(x, 0, T, s.H, terms, q, stream);
}

cudaError_t launch_quantize_act_prefill(const PrefillScratch &s, int terms, cudaStream_t stream) {
    QuantTargets q{};
    q.codes = s.aq;
    q.atoms = s.asf;
    q.g = s.ga;
    q.rows_stride = s.max_rows;
    q.atom_blocks = s.max_rows / kPrefillTileN;
    q.rows_used = s.rows_used;
    return launch_quantize_mode<kRowAtoms>(s.act, 1, s.max_rows, s.I, terms, q, stream);
}

cudaError_t launch_prefill_combine(const PrefillScratch &s, int T, const void *residual, void *out, int out_f32,
                                   cudaStream_t stream) {
    const dim3 grid((s.H / 8 + 255) / 256, T);
    prefill_combine_kernel<<<grid, 256, 0, stream>>>(s, T, static_cast<const uint16_t *>(residual), out, out_f32);
    return cudaGetLastError();
}

}  // namespace nvfp4
