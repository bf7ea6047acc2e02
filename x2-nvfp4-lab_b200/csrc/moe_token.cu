// One-token layer call in one persistent kernel (moe_token_kernel).
//
// The lab runs a single-token MoE layer as seven dependent launches
// (native_nvfp4/runtime/nvfp4_runtime.cpp:1943-2066: router GEMV, shared-gate
// GEMV, top-8, gate/up, SiLU, down, reduce); the batched decode path here
// needs three. At one token every stage is short and the launches, their
// ramps and their tails are most of the time, so this kernel does the whole
// layer in one cooperative grid of one CTA per SM:
//
//   1. router   every warp of the grid owns at most one router row (row E is
//               the shared gate) and computes its FP32 logit in the fixed
//               order of the routing kernel (lane l: columns j*128 + 4l + e,
//               j then e ascending, product and sum each rounded, then an xor
//               butterfly 16..1, the bias last), so logits are bit-identical
//               to the batched path's and to the oracle's;
//      grid barrier 1 (bounded);
//   2. top-8    every CTA selects the eight experts itself from the 257
//               logits in L2 (largest first, lowest id on ties, -0 == +0),
//               the renormalised softmax and the sigmoid shared gate;
//   3. gate/up  the (slot, row) pairs of the nine slots' gate and up
//               projections are split into one contiguous range per CTA; the
//               CTA's rows arrive in shared memory by bulk copies issued as
//               soon as their expert is known -- the shared expert's rows
//               (slot 8) at kernel entry, before routing resolves -- and every
//               lane keeps its columns of x in registers; SiLU(gate)*up goes
//               to an FP32 exchange buffer [9][I];
//      grid barrier 2 (bounded);
//   4. down     each CTA owns a range of output rows for all nine slots; the
//               down-projection rows of those output rows were bulk-copied
//               into shared memory right after routing (the shared expert's
//               at entry), so they are resident when the barrier opens;
//   5. combine  the CTA sums its output rows' nine routing-weighted slot
//               results in slot order (nvfp4_gemv.cl:1443-1457), adds the
//               residual and stores BF16 (or FP32 for the lab's ABI).
//
// Every weight byte is read once, by one CTA, into shared memory; a lane
// decodes its 16-byte units (32 columns, two E4M3 block scales) exactly to
// f16 and accumulates in FP32 against FP32 activations.
//
// Safety: the grid is launched cooperatively (every CTA is resident), each
// grid barrier and each bulk-copy wait is bounded by wall-clock time and
// records a wait-site code in the bank's error word, and every CTA passes
// every barrier even after a failure, so the barrier words return to their
// resting state by the end of the call.
#include "internal.h"
#include "moe_decode.cuh"
#include "moe_token.cuh"
#include "tma_util.cuh"

#include <atomic>
#include <cfloat>

namespace nvfp4 {

namespace {

constexpr int kTokenThreads = 256;
constexpr int kTokenWarps = kTokenThreads / 32;
// Barrier words: [0] count of barrier 1, [32] its generation, [64] count of
// barrier 2, [96] its generation (separate 128-byte lines).
constexpr int kSyncWords = 128;

enum TokenWaitSite : int {
    kSiteTokenLogits = 51,
    kSiteTokenAct = 52,
    kSiteTokenGateUp = 53,
    kSiteTokenDown = 54,
};

__device__ __forceinline__ unsigned token_order_key(float v) {
    v = (v == 0.0f) ? 0.0f : v;
    const unsigned b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float token_from_order_key(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_u32(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid-wide barrier over gridDim.x CTAs. `g0` is the generation thread 0
// read at kernel entry (it cannot advance before this CTA arrives). After
// the CTA's __syncthreads, thread 0 arrives on the count with a gpu-scope
// acquire-release add (which also publishes the CTA's earlier writes), and either --
// last to arrive -- resets the count and advances the generation with a
// release store, or polls the generation with acquire loads, bounded by
// kWaitLimitNs. After a failure recorded in *err (by this wait or any other)
// the CTA still arrives but no longer waits. Returns false when the CTA
// passed without the barrier having opened.
__device__ bool grid_barrier(unsigned *count, unsigned *gen, unsigned g0, int *err, int site, int *s_flag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        unsigned arrived;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(arrived) : "l"(count) : "memory");
        if (arrived + 1u == gridDim.x) {
            asm volatile("st.relaxed.gpu.global.u32 [%0], 0;" ::"l"(count) : "memory");
            st_release_u32(gen, g0 + 1u);
        } else {
            unsigned long long t0 = 0;
            for (unsigned i = 0;; ++i) {
                if (ld_acquire_u32(gen) != g0) break;
                if ((i & 63u) == 63u) {
                    if (*reinterpret_cast<volatile int *>(err) != 0) {
                        ok = 0;
                        break;
                    }
                    const unsigned long long now = global_ns();
                    if (t0 == 0) {
                        t0 = now;
                    } else if (now - t0 > kWaitLimitNs) {
                        atomicCAS(err, 0, site);
                        ok = 0;
                        break;
                    }
                }
            }
        }
        *s_flag = ok;
    }
    __syncthreads();
    return *s_flag != 0;
}

// Two f16 products added to an FP32 accumulator with the sm_100
// mixed-precision FMA (f16 inputs, f32 addend and result, one rounding):
// acc = fma(a.lo, b.lo, acc); acc = fma(a.hi, b.hi, acc).
__device__ __forceinline__ float fma2_f16_f32(uint32_t a, uint32_t b, float acc) {
    asm("{\n\t.reg .f16 a0, a1, b0, b1;\n\t"
        "mov.b32 {a0, a1}, %1;\n\tmov.b32 {b0, b1}, %2;\n\t"
        "fma.rn.f32.f16 %0, a0, b0, %0;\n\tfma.rn.f32.f16 %0, a1, b1, %0;\n\t}"
        : "+f"(acc)
        : "r"(a), "r"(b));
    return acc;
}

// Dot product of one 16-byte unit of a row (32 columns: two E4M3 blocks of
// 16) with 32 activations held as 16 f16x2 words: the E2M1 codes convert
// exactly to f16, each block's products accumulate in FP32 (two chains per
// block), and the block sums are scaled by their E4M3 scales in FP32. The
// E2M1 x activation products are exact, so the sums carry only the FP32
// rounding of the additions.
__device__ __forceinline__ float unit_dot_h(uint4 w, uint16_t sc, const uint32_t *xh, float acc) {
    const uint32_t s2 = e4m3x2_to_f16x2(sc);
    const float2 s = __half22float2(*reinterpret_cast<const __half2 *>(&s2));
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    float p[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t h[4];
        e2m1x8_to_f16x8(words[j], h);
#pragma unroll
        for (int m = 0; m < 4; ++m) p[j] = fma2_f16_f32(h[m], xh[4 * j + m], p[j]);
    }
    acc = fmaf(p[0] + p[1], s.x, acc);
    return fmaf(p[2] + p[3], s.y, acc);
}

__device__ __forceinline__ uint32_t f32x2_to_f16x2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

struct TokenLayout {
    int NR;            // max (slot, row) gate/up pairs per CTA
    int NH;            // max output rows per CTA
    size_t x_s, act_s, gpk, upk, gsc, usc, dpk, dsc, y_s, total;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline TokenLayout token_layout(int G, int H, int I, int gpitch, int dpitch) {
    TokenLayout L{};
    L.NR = (kSlots * I + G - 1) / G;
    L.NH = (H + G - 1) / G;
    size_t o = 0;
    L.x_s = o;   o = align_up(o + sizeof(float) * H, 128);
    L.act_s = o; o = align_up(o + sizeof(__half) * kSlots * I, 128);
    L.gpk = o;   o = align_up(o + (size_t)L.NR * (H / 2), 128);
    L.upk = o;   o = align_up(o + (size_t)L.NR * (H / 2), 128);
    L.gsc = o;   o = align_up(o + (size_t)L.NR * gpitch, 128);
    L.usc = o;   o = align_up(o + (size_t)L.NR * gpitch, 128);
    L.dpk = o;   o = align_up(o + (size_t)kSlots * L.NH * (I / 2), 128);
    L.dsc = o;   o = align_up(o + (size_t)kSlots * L.NH * dpitch, 128);
    L.y_s = o;   o = align_up(o + sizeof(float) * kSlots * L.NH, 128);
    L.total = o;
    return L;
}

// XN: activations each lane keeps (as f16x2 words) for the gate/up rows,
// H / (lanes per row); 64 for H = 2048, 32 for H <= 1024.
template <int XN>
__global__ void __launch_bounds__(kTokenThreads, 1) moe_token_kernel(TokenArgs a) {
    extern __shared__ __align__(128) uint8_t tsm[];
    __shared__ uint64_t bars[4];  // gate/up shared, gate/up routed, down shared, down routed
    __shared__ int s_ids[kSlots];
    __shared__ float s_w[kSlots];
    __shared__ float s_ginv[kSlots], s_uinv[kSlots], s_coef[kSlots];  // per slot: gate, up, weight x down
    __shared__ float s_red[kTokenWarps];
    __shared__ float s_logits[257];
    __shared__ float s_inv;
    __shared__ int s_flag;
    __shared__ int s_drain;

    const int H = a.H, I = a.I, E = a.E, R = E + 1;
    const int G = gridDim.x, c = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gpitch = a.scale_pitch[0], dpitch = a.scale_pitch[2];
    const TokenLayout L = token_layout(G, H, I, gpitch, dpitch);
    float *x_s = reinterpret_cast<float *>(tsm + L.x_s);
    __half *act_s = reinterpret_cast<__half *>(tsm + L.act_s);
    uint8_t *gpk = tsm + L.gpk, *upk = tsm + L.upk, *gsc = tsm + L.gsc, *usc = tsm + L.usc;
    uint8_t *dpk = tsm + L.dpk, *dsc = tsm + L.dsc;
    float *y_s = reinterpret_cast<float *>(tsm + L.y_s);
    int *err = a.s.error;

    // This CTA's gate/up pairs [u0, u1) over (slot, row) = (u / I, u % I),
    // and its output rows [h0, h1).
    const int U = kSlots * I;
    const int u0 = (int)((long long)U * c / G), u1 = (int)((long long)U * (c + 1) / G);
    const int h0 = (int)((long long)H * c / G), h1 = (int)((long long)H * (c + 1) / G);
    const int nh = h1 - h0;
    const int shared_u0 = max(u0, (kSlots - 1) * I);  // first pair of slot 8 in range
    const int routed_end = min(u1, (kSlots - 1) * I);
    const bool have_gu_shared = shared_u0 < u1, have_gu_routed = u0 < routed_end;
    // Routed pairs split at a slot boundary into at most two segments.
    const int mid = have_gu_routed ? min(routed_end, (u0 / I + 1) * I) : u0;

    const size_t gp_row = H / 2, dp_row = I / 2;
    auto gate_up_bytes = [&](int v0, int v1) { return (uint32_t)((v1 - v0) * 2 * (gp_row + gpitch)); };
    const uint32_t down_slot_bytes = (uint32_t)(nh * (dp_row + dpitch));
    // Copy `j` of gate/up pairs [v0, v1) (one slot) of expert e: j = 0/1 the
    // gate/up codes, 2/3 their scales, into local pair index v0 - u0.
    auto copy_gate_up = [&](int j, int v0, int v1, int e, uint64_t *bar) {
        const int r0 = v0 % I, n = v1 - v0, li = v0 - u0;
        const size_t row0 = (size_t)e * I + r0;
        if (j < 2)
            bulk_g2s((j == 0 ? gpk : upk) + li * gp_row, a.packed[j] + row0 * gp_row, (uint32_t)(n * gp_row), bar);
        else
            bulk_g2s((j == 2 ? gsc : usc) + (size_t)li * gpitch, a.scales[j - 2] + row0 * gpitch,
                     (uint32_t)(n * gpitch), bar);
    };
    // Copy `j` (0 codes, 1 scales) of the down rows [h0, h1) of slot `slot`.
    auto copy_down = [&](int j, int slot, int e, uint64_t *bar) {
        const size_t row0 = (size_t)e * H + h0;
        if (j == 0)
            bulk_g2s(dpk + (size_t)slot * L.NH * dp_row, a.packed[2] + row0 * dp_row, (uint32_t)(nh * dp_row), bar);
        else
            bulk_g2s(dsc + (size_t)slot * L.NH * dpitch, a.scales[2] + row0 * dpitch, (uint32_t)(nh * dpitch), bar);
    };

    // ---- entry -------------------------------------------------------------
    // Thread 0: the barrier generations (neither can advance before this CTA
    // arrives, so plain loads whose latency hides behind the router work),
    // the copy barriers and every expected byte count -- the routed counts do
    // not depend on which experts are picked.
    unsigned gen0 = 0, gen1 = 0;
    if (threadIdx.x == 0) {
        gen0 = ld_relaxed_u32(a.sync + 32);
        gen1 = ld_relaxed_u32(a.sync + 96);
#pragma unroll
        for (int i = 0; i < 4; ++i) mbar_init(&bars[i], 1);
        fence_barrier_init();
        if (have_gu_shared) mbar_arrive_expect_tx(&bars[0], gate_up_bytes(shared_u0, u1));
        if (have_gu_routed) mbar_arrive_expect_tx(&bars[1], gate_up_bytes(u0, routed_end));
        if (nh > 0) {
            mbar_arrive_expect_tx(&bars[2], down_slot_bytes);
            mbar_arrive_expect_tx(&bars[3], down_slot_bytes * kTopK);
        }
    }
    __syncthreads();
    // The last warp (no router row on grids of 37 or more CTAs) fetches the
    // shared expert's rows now, before routing resolves.
    if (warp == kTokenWarps - 1) {
        if (have_gu_shared && lane < 4) copy_gate_up(lane, shared_u0, u1, E, &bars[0]);
        if (nh > 0 && lane >= 4 && lane < 6) copy_down(lane - 4, kSlots - 1, E, &bars[2]);
    }

    // Router row of this warp (row E is the shared gate): every load in flight
    // before x is ready.
    const int row = warp * G + c;
    const int chunks = H / 128;  // <= 16
    uint2 wr[16];
    if (row < R) {
        const uint2 *src = reinterpret_cast<const uint2 *>(a.router + (size_t)row * H) + lane;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (j < chunks) wr[j] = __ldg(src + 32 * j);
    }
    const float bias = (a.bias && row < E) ? __ldg(a.bias + row) : 0.0f;

    // x -> shared memory as FP32, normalised first with the bits of the
    // standalone RMSNorm when a norm weight is given (256 column-strided fmaf
    // partial sums, xor butterfly per warp, the eight warp sums in order,
    // rsqrtf, bf16(x * inv * w)).
    if (a.x_is_f32) {
        const float *xf = static_cast<const float *>(a.x);
        for (int i = threadIdx.x; i < H; i += kTokenThreads) x_s[i] = __ldg(xf + i);
    } else {
        const uint16_t *xb = static_cast<const uint16_t *>(a.x);
        for (int i = threadIdx.x; i < H; i += kTokenThreads) x_s[i] = bf16_bits_to_f32(__ldg(xb + i));
    }
    if (a.norm_w) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < H; i += kTokenThreads) ss = fmaf(x_s[i], x_s[i], ss);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (lane == 0) s_red[warp] = ss;
        __syncthreads();
        if (threadIdx.x == 0) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < kTokenWarps; ++w) tot += s_red[w];
            s_inv = rsqrtf(tot / (float)H + a.norm_eps);
        }
        __syncthreads();
        const float inv = s_inv;
        for (int i = threadIdx.x; i < H; i += kTokenThreads)
            x_s[i] = bf16_bits_to_f32(f32_to_bf16_bits(x_s[i] * inv * bf16_bits_to_f32(__ldg(a.norm_w + i))));
    }
    __syncthreads();

    if (row < R) {
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (j < chunks) {
                const float4 xv = *reinterpret_cast<const float4 *>(x_s + j * 128 + lane * 4);
                acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(wr[j].x & 0xFFFFu), xv.x));
                acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(wr[j].x >> 16), xv.y));
                acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(wr[j].y & 0xFFFFu), xv.z));
                acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(wr[j].y >> 16), xv.w));
            }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
        if (lane == 0) {
            if (a.bias && row < E) acc = __fadd_rn(acc, bias);
            a.s.logits[row] = acc;
        }
    }

    // This lane's columns of x (f16x2) for the gate/up rows: LR lanes per row,
    // lane group q of RPW rows per warp pass, 16-byte units lr + LR*k.
    const int LR = H / XN, RPW = 32 / LR, q = lane / LR, lr = lane % LR;
    uint32_t xh[XN / 2];
#pragma unroll
    for (int k = 0; k < XN / 32; ++k) {
        const int unit = lr + LR * k;
#pragma unroll
        for (int m = 0; m < 16; ++m)
            xh[16 * k + m] = f32x2_to_f16x2(x_s[unit * 32 + 2 * m], x_s[unit * 32 + 2 * m + 1]);
    }

    grid_barrier(a.sync, a.sync + 32, gen0, err, kSiteTokenLogits, &s_flag);

    // ---- top-8, in every warp ------------------------------------------------
    // The CTA reads the logits from L2 once (one request per line), then each
    // warp selects the same eight experts from shared memory (largest first,
    // lowest id on ties, -0 == +0) and issues its share of the routed rows'
    // copies at once.
    for (int e = threadIdx.x; e < R; e += kTokenThreads) s_logits[e] = __ldcg(a.s.logits + e);
    __syncthreads();
    {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = lane + 32 * i;
            v[i] = e < E ? s_logits[e] : -FLT_MAX;
        }
        unsigned taken = 0;
        float my_v = 0.0f;
        int my_i = 0;
#pragma unroll 1
        for (int slot = 0; slot < kTopK; ++slot) {
            float bv = -FLT_MAX;
            int bi = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int e = lane + 32 * i;
                if (e < E && !((taken >> i) & 1u) && v[i] > bv) {
                    bv = v[i];
                    bi = e;
                }
            }
            const unsigned key = token_order_key(bv);
            const unsigned kmax = __reduce_max_sync(0xffffffffu, key);
            const unsigned imin = __reduce_min_sync(0xffffffffu, key == kmax ? (unsigned)bi : 0xffffffffu);
            bi = (int)imin;
            bv = token_from_order_key(kmax);
            if (lane == slot) {
                my_v = bv;
                my_i = bi;
            }
            if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        }
        // Routed copies: 8 gate/up (two segments x four arrays) and 16 down
        // (eight slots x codes/scales), three per warp, lane 0 issuing; the
        // expert of each comes from the lane that holds its slot.
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            const int j = 3 * warp + t;
            const int seg = j >> 2;
            const int v0 = seg == 0 ? u0 : mid, v1 = seg == 0 ? mid : routed_end;
            const int src = j < 8 ? (v1 > v0 ? (v0 / I) & 7 : 0) : ((j - 8) >> 1) & 7;
            const int e = __shfl_sync(0xffffffffu, my_i, src);
            if (lane == 0) {
                if (j < 8) {
                    if (have_gu_routed && v1 > v0) copy_gate_up(j & 3, v0, v1, e, &bars[1]);
                } else if (nh > 0) {
                    copy_down((j - 8) & 1, (j - 8) >> 1, e, &bars[3]);
                }
            }
        }
        if (warp == 0) {
            const float sl = s_logits[E];
            const float top0 = __shfl_sync(0xffffffffu, my_v, 0);
            const float my_e = lane < kTopK ? expf(my_v - top0) : 0.0f;
            float den = 0.0f;
#pragma unroll
            for (int slot = 0; slot < kTopK; ++slot) den += __shfl_sync(0xffffffffu, my_e, slot);
            // Dispatch order of the eight picks (ids ascending), for the record.
            int rank_in = 0;
#pragma unroll
            for (int slot = 0; slot < kTopK; ++slot) rank_in += __shfl_sync(0xffffffffu, my_i, slot) < my_i;
            if (lane < kTopK) {
                const float w = my_e / den;
                s_ids[lane] = my_i;
                s_w[lane] = w;
                if (c == 0) {
                    a.s.ids[lane] = my_i;
                    a.s.weights[lane] = w;
                    a.s.perm[rank_in] = lane;
                }
            } else if (lane == kTopK) {
                const float w = 1.0f / (1.0f + expf(-sl));
                s_ids[kTopK] = E;
                s_w[kTopK] = w;
                if (c == 0) {
                    a.s.ids[kTopK] = E;
                    a.s.weights[kTopK] = w;
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x < kSlots) {
        const int e = s_ids[threadIdx.x];
        s_ginv[threadIdx.x] = __ldg(a.inv_scales + e);
        s_uinv[threadIdx.x] = __ldg(a.inv_scales + R + e);
        s_coef[threadIdx.x] = s_w[threadIdx.x] * __ldg(a.inv_scales + 2 * R + e);
    }
    if (c == 0)
        for (int e = threadIdx.x; e < E; e += kTokenThreads) {
            int n = 0;
#pragma unroll
            for (int slot = 0; slot < kTopK; ++slot) n += s_ids[slot] == e;
            a.s.counts[e] = n;
        }
    __syncthreads();

    // ---- gate/up: shared-expert pairs first (already resident), then routed ----
    // One rolled loop over the CTA's pairs in that order (pair index t:
    // t < n_sh the shared pairs from shared_u0, then the routed ones from
    // u0); the routed copies are waited for when a warp first reaches them.
    bool ok = true;
    {
        const int n_sh = have_gu_shared ? u1 - shared_u0 : 0;
        const int n_all = n_sh + (have_gu_routed ? routed_end - u0 : 0);
        if (have_gu_shared) ok = mbar_wait(&bars[0], 0, err, kSiteTokenGateUp);
        bool routed_ready = false;
#pragma unroll 1
        for (int base = warp * RPW; base < n_all; base += kTokenWarps * RPW) {
            if (have_gu_routed && base + RPW > n_sh && !routed_ready) {
                ok = mbar_wait(&bars[1], 0, err, kSiteTokenGateUp) && ok;
                routed_ready = true;
            }
            const int t = base + q;
            const int v = t < n_sh ? shared_u0 + t : u0 + (t - n_sh);
            float g = 0.0f, u = 0.0f;
            const int slot = v / I;
            if (t < n_all && ok) {
                const int li = v - u0;
                const uint8_t *gr = gpk + li * gp_row, *ur = upk + li * gp_row;
                const uint8_t *gs = gsc + (size_t)li * gpitch, *us = usc + (size_t)li * gpitch;
#pragma unroll
                for (int k = 0; k < XN / 32; ++k) {
                    const int unit = lr + LR * k;
                    const uint4 gw = *reinterpret_cast<const uint4 *>(gr + unit * 16);
                    const uint4 uw = *reinterpret_cast<const uint4 *>(ur + unit * 16);
                    const uint16_t gsv = *reinterpret_cast<const uint16_t *>(gs + unit * 2);
                    const uint16_t usv = *reinterpret_cast<const uint16_t *>(us + unit * 2);
                    g = unit_dot_h(gw, gsv, xh + 16 * k, g);
                    u = unit_dot_h(uw, usv, xh + 16 * k, u);
                }
            }
#pragma unroll
            for (int off = LR / 2; off >= 1; off >>= 1) {
                g += __shfl_xor_sync(0xffffffffu, g, off);
                u += __shfl_xor_sync(0xffffffffu, u, off);
            }
            if (t < n_all && lr == 0) {
                g *= s_ginv[slot];
                u *= s_uinv[slot];
                a.act[slot * I + v % I] = g / (1.0f + expf(-g)) * u;
            }
        }
        // A warp with no routed pair of its own still consumes the phase.
        if (have_gu_routed && !routed_ready) ok = mbar_wait(&bars[1], 0, err, kSiteTokenGateUp) && ok;
    }

    grid_barrier(a.sync + 64, a.sync + 96, gen1, err, kSiteTokenAct, &s_flag);

    // ---- down: the act vectors as f16 (rotated 16-byte groups) -----------------
    {
        const int per_slot = I / 4;  // float4 per slot
        const float4 *src = reinterpret_cast<const float4 *>(a.act);
        for (int idx = threadIdx.x; idx < kSlots * per_slot; idx += kTokenThreads) {
            const int slot = idx / per_slot, f = idx - slot * per_slot, unit = f >> 3, g4 = f & 7;
            const float4 t = __ldcg(src + idx);
            // Unit (32 columns = 64 bytes of f16) holds four 16-byte groups;
            // group g = float4 pair (2g, 2g+1), stored at position
            // (g + unit / 2) & 3, so the 16-byte loads of eight consecutive
            // units hit eight distinct bank groups.
            uint2 hv;
            hv.x = f32x2_to_f16x2(t.x, t.y);
            hv.y = f32x2_to_f16x2(t.z, t.w);
            uint8_t *dst = reinterpret_cast<uint8_t *>(act_s + slot * I + unit * 32);
            *reinterpret_cast<uint2 *>(dst + (((g4 >> 1) + (unit >> 1)) & 3) * 16 + (g4 & 1) * 8) = hv;
        }
    }
    __syncthreads();
    if (nh > 0) {
        ok = mbar_wait(&bars[2], 0, err, kSiteTokenDown) && ok;
        ok = mbar_wait(&bars[3], 0, err, kSiteTokenDown) && ok;
    }
    if (ok && nh > 0) {
        // Rows d = slot * nh + (h - h0), slot-major; each warp a contiguous
        // range, LD lanes per row (one 16-byte unit each), two rows per lane
        // at a time (RPD rows per half-pass).
        const int LD = I / 32 < 32 ? I / 32 : 32, RPD = 32 / LD, qd = lane / LD, ld = lane % LD;
        const int D = kSlots * nh;
        const int d0 = D * warp / kTokenWarps, d1 = D * (warp + 1) / kTokenWarps;
#pragma unroll 1
        for (int base = d0; base < d1; base += 2 * RPD) {
            float acc[2] = {0.0f, 0.0f};
            int dd[2], slots[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                dd[r] = base + qd + r * RPD;
                slots[r] = dd[r] < d1 ? dd[r] / nh : 0;
            }
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (dd[r] < d1) {
                    const int hl = dd[r] - slots[r] * nh;
                    const uint8_t *ar = reinterpret_cast<const uint8_t *>(act_s + slots[r] * I + ld * 32);
                    uint32_t av[16];
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        const uint4 t = *reinterpret_cast<const uint4 *>(ar + ((g + (ld >> 1)) & 3) * 16);
                        av[4 * g] = t.x;
                        av[4 * g + 1] = t.y;
                        av[4 * g + 2] = t.z;
                        av[4 * g + 3] = t.w;
                    }
                    const uint8_t *pr = dpk + ((size_t)slots[r] * L.NH + hl) * dp_row;
                    const uint8_t *sr = dsc + ((size_t)slots[r] * L.NH + hl) * dpitch;
                    acc[r] = unit_dot_h(*reinterpret_cast<const uint4 *>(pr + ld * 16),
                                        *reinterpret_cast<const uint16_t *>(sr + ld * 2), av, 0.0f);
                }
            }
#pragma unroll
            for (int off = LD / 2; off >= 1; off >>= 1) {
                acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], off);
                acc[1] += __shfl_xor_sync(0xffffffffu, acc[1], off);
            }
            if (ld == 0) {
#pragma unroll
                for (int r = 0; r < 2; ++r)
                    if (dd[r] < d1) y_s[slots[r] * L.NH + (dd[r] - slots[r] * nh)] = s_coef[slots[r]] * acc[r];
            }
        }
    }
    __syncthreads();

    // ---- combine: nine slots in slot order, then the residual -------------------
    for (int hl = threadIdx.x; hl < nh; hl += kTokenThreads) {
        float sum = 0.0f;
#pragma unroll
        for (int slot = 0; slot < kSlots; ++slot) sum += y_s[slot * L.NH + hl];
        const int h = h0 + hl;
        if (a.residual) sum = bf16_bits_to_f32(static_cast<const uint16_t *>(a.residual)[h]) + sum;
        if (a.out_f32)
            static_cast<float *>(a.out)[h] = sum;
        else
            static_cast<uint16_t *>(a.out)[h] = f32_to_bf16_bits(sum);
    }

    // A failed wait: drain this CTA's copies (bounded) and publish the code.
    if (threadIdx.x == 0 && *reinterpret_cast<volatile int *>(err) != 0) {
        s_drain = 0;
        if (have_gu_shared) mbar_wait(&bars[0], 0, &s_drain, 1);
        if (have_gu_routed) mbar_wait(&bars[1], 0, &s_drain, 1);
        if (nh > 0) {
            mbar_wait(&bars[2], 0, &s_drain, 1);
            mbar_wait(&bars[3], 0, &s_drain, 1);
        }
        const int code = *reinterpret_cast<volatile int *>(err);
        if (a.s.host_error) *reinterpret_cast<volatile int *>(a.s.host_error) = code != 0 ? code : kErrWaitTimeout;
    }
}

constexpr size_t kTokenMaxSmem = 200 * 1024;
constexpr int kTokenMaxDevices = 64;

template <int XN>
cudaError_t launch_token_xn(const TokenArgs &a, int sms, size_t smem, cudaStream_t stream) {
    // The shared-memory opt-in is per device; set it once on each.
    static std::atomic<bool> configured[kTokenMaxDevices];
    auto *kernel = moe_token_kernel<XN>;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev < 0 || dev >= kTokenMaxDevices) return cudaErrorInvalidDevice;
    if (!configured[dev].load()) {
        err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTokenMaxSmem);
        if (err != cudaSuccess) return err;
        configured[dev].store(true);
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(kTokenThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

}  // namespace

size_t token_sync_bytes() { return kSyncWords * sizeof(unsigned); }

size_t token_smem_bytes(int sms, int H, int I, int gate_pitch, int down_pitch) {
    return token_layout(sms, H, I, gate_pitch, down_pitch).total;
}

bool token_supported(int sms, int E, int H, int I, int gate_pitch, int down_pitch) {
    if (sms < 1 || E < kTopK || E > 256) return false;
    // A CTA's gate/up pairs span at most two slots.
    if ((kSlots * I + sms - 1) / sms > I) return false;
    if (H % 256 != 0 || H > 2048 || I % 128 != 0 || I > 1024) return false;
    // Every warp of the grid routes at most one router row.
    if ((long long)sms * kTokenWarps < E + 1) return false;
    // Bulk-copy sizes and addresses are multiples of 16 bytes.
    if (gate_pitch % 16 != 0 || down_pitch % 16 != 0) return false;
    return token_smem_bytes(sms, H, I, gate_pitch, down_pitch) <= kTokenMaxSmem;
}

cudaError_t launch_token(const TokenArgs &a, int sms, cudaStream_t stream) {
    const size_t smem = token_smem_bytes(sms, a.H, a.I, a.scale_pitch[0], a.scale_pitch[2]);
    return a.H == 2048 ? launch_token_xn<64>(a, sms, smem, stream) : launch_token_xn<32>(a, sms, smem, stream);
}

}  // namespace nvfp4
