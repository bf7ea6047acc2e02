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

__device__ __forceinline__ void st_release_u32(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid-wide barrier over gridDim.x CTAs. Thread 0 reads the generation,
// arrives on the count, and either (last to arrive) resets the count and
// advances the generation, or waits -- bounded by kWaitLimitNs -- for the
// generation to advance. After a failure recorded in *err (by this wait or
// any other) the CTA still arrives but no longer waits. Returns false when
// the CTA passed without the barrier having opened.
__device__ bool grid_barrier(unsigned *count, unsigned *gen, int *err, int site, int *s_flag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned g0 = ld_acquire_u32(gen);
        __threadfence();
        const unsigned arrived = atomicAdd(count, 1u) + 1u;
        if (arrived == gridDim.x) {
            atomicExch(count, 0u);
            __threadfence();
            st_release_u32(gen, g0 + 1u);
        } else {
            unsigned long long t0 = 0;
            for (unsigned i = 0;; ++i) {
                if (ld_acquire_u32(gen) != g0) break;
                if ((i & 7u) == 7u) {
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
                __nanosleep(20);
            }
        }
        __threadfence();
        *s_flag = ok;
    }
    __syncthreads();
    return *s_flag != 0;
}

// Dot product of one 16-byte unit of a row (32 columns: two E4M3 blocks of
// 16) with 32 FP32 activations: per block the exact f16 codes times x in
// FP32, then times the block scale.
__device__ __forceinline__ float unit_dot(uint4 w, uint16_t sc, const float *x, float acc) {
    const uint32_t s2 = e4m3x2_to_f16x2(sc);
    const float2 s = __half22float2(*reinterpret_cast<const __half2 *>(&s2));
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    float p[2] = {0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t h[4];
        e2m1x8_to_f16x8(words[j], h);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h[m]));
            p[j >> 1] = fmaf(f.x, x[8 * j + 2 * m], p[j >> 1]);
            p[j >> 1] = fmaf(f.y, x[8 * j + 2 * m + 1], p[j >> 1]);
        }
    }
    acc = fmaf(p[0], s.x, acc);
    return fmaf(p[1], s.y, acc);
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
    L.act_s = o; o = align_up(o + sizeof(float) * kSlots * I, 128);
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

// XN: FP32 activations each lane keeps in registers for the gate/up rows
// (H / (lanes per row)); 64 for H = 2048, 32 for H <= 1024.
template <int XN>
__global__ void __launch_bounds__(kTokenThreads, 1) moe_token_kernel(TokenArgs a) {
    extern __shared__ __align__(128) uint8_t tsm[];
    __shared__ uint64_t bars[4];  // gate/up shared, gate/up routed, down shared, down routed
    __shared__ int s_ids[kSlots];
    __shared__ float s_w[kSlots];
    __shared__ float s_red[kTokenWarps];
    __shared__ float s_inv;
    __shared__ int s_flag;
    __shared__ int s_drain;

    const int H = a.H, I = a.I, E = a.E, R = E + 1;
    const int G = gridDim.x, c = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gpitch = a.scale_pitch[0], dpitch = a.scale_pitch[2];
    const TokenLayout L = token_layout(G, H, I, gpitch, dpitch);
    float *x_s = reinterpret_cast<float *>(tsm + L.x_s);
    float *act_s = reinterpret_cast<float *>(tsm + L.act_s);
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

    const size_t gp_row = H / 2, dp_row = I / 2;
    // Gate/up rows of pairs [v0, v1) (one slot) of expert e -> local pair index v0 - u0.
    auto issue_gate_up = [&](int v0, int v1, int e, uint64_t *bar) {
        const int r0 = v0 % I, n = v1 - v0, li = v0 - u0;
        const size_t row0 = (size_t)e * I + r0;
        const uint32_t pk = (uint32_t)(n * gp_row), sc = (uint32_t)(n * gpitch);
        bulk_g2s(gpk + li * gp_row, a.packed[0] + row0 * gp_row, pk, bar);
        bulk_g2s(upk + li * gp_row, a.packed[1] + row0 * gp_row, pk, bar);
        bulk_g2s(gsc + (size_t)li * gpitch, a.scales[0] + row0 * gpitch, sc, bar);
        bulk_g2s(usc + (size_t)li * gpitch, a.scales[1] + row0 * gpitch, sc, bar);
    };
    auto gate_up_bytes = [&](int v0, int v1) { return (uint32_t)((v1 - v0) * 2 * (gp_row + gpitch)); };
    auto issue_down = [&](int slot, int e, uint64_t *bar) {
        const size_t row0 = (size_t)e * H + h0;
        bulk_g2s(dpk + (size_t)slot * L.NH * dp_row, a.packed[2] + row0 * dp_row, (uint32_t)(nh * dp_row), bar);
        bulk_g2s(dsc + (size_t)slot * L.NH * dpitch, a.scales[2] + row0 * dpitch, (uint32_t)(nh * dpitch), bar);
    };
    const uint32_t down_slot_bytes = (uint32_t)(nh * (dp_row + dpitch));

    // ---- entry: barriers, the shared expert's rows, the router row --------
    bool have_gu_shared = shared_u0 < u1, have_gu_routed = u0 < (kSlots - 1) * I && u0 < u1;
    if (threadIdx.x == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) mbar_init(&bars[i], 1);
        fence_barrier_init();
        if (have_gu_shared) {
            mbar_arrive_expect_tx(&bars[0], gate_up_bytes(shared_u0, u1));
            issue_gate_up(shared_u0, u1, E, &bars[0]);
        }
        if (nh > 0) {
            mbar_arrive_expect_tx(&bars[2], down_slot_bytes);
            issue_down(kSlots - 1, E, &bars[2]);
        }
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

    // This lane's columns of x for the gate/up rows: LR lanes per row, lane
    // group q of RPW rows per warp pass, 16-byte units lr + LR*k.
    const int LR = H / XN, RPW = 32 / LR, q = lane / LR, lr = lane % LR;
    float xr[XN];
#pragma unroll
    for (int k = 0; k < XN / 32; ++k) {
        const int unit = lr + LR * k;
#pragma unroll
        for (int m = 0; m < 32; ++m) xr[32 * k + m] = x_s[unit * 32 + m];
    }

    grid_barrier(a.sync, a.sync + 32, err, kSiteTokenLogits, &s_flag);

    // ---- top-8 (every CTA) ---------------------------------------------------
    if (warp == 0) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = lane + 32 * i;
            v[i] = e < E ? __ldcg(a.s.logits + e) : -FLT_MAX;
        }
        const float sl = __ldcg(a.s.logits + E);
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
    __syncthreads();
    if (c == 0)
        for (int e = threadIdx.x; e < E; e += kTokenThreads) {
            int n = 0;
#pragma unroll
            for (int slot = 0; slot < kTopK; ++slot) n += s_ids[slot] == e;
            a.s.counts[e] = n;
        }

    // ---- routed rows: issue every copy at once ---------------------------------
    if (threadIdx.x == 0) {
        if (have_gu_routed) {
            const int end = min(u1, (kSlots - 1) * I);
            uint32_t bytes = 0;
            for (int v0 = u0; v0 < end;) {
                const int v1 = min(end, (v0 / I + 1) * I);
                bytes += gate_up_bytes(v0, v1);
                v0 = v1;
            }
            mbar_arrive_expect_tx(&bars[1], bytes);
            for (int v0 = u0; v0 < end;) {
                const int v1 = min(end, (v0 / I + 1) * I);
                issue_gate_up(v0, v1, s_ids[v0 / I], &bars[1]);
                v0 = v1;
            }
        }
        if (nh > 0) {
            mbar_arrive_expect_tx(&bars[3], down_slot_bytes * kTopK);
            for (int slot = 0; slot < kTopK; ++slot) issue_down(slot, s_ids[slot], &bars[3]);
        }
    }

    // ---- gate/up: shared-expert pairs first (already resident), then routed ----
    bool ok = true;
    auto gate_up_range = [&](int v0, int v1) {
        for (int base = v0 + warp * RPW; base < v1; base += kTokenWarps * RPW) {
            const int v = base + q;
            float g = 0.0f, u = 0.0f;
            int slot = 0;
            if (v < v1) {
                const int li = v - u0;
                slot = v / I;
                const uint8_t *gr = gpk + li * gp_row, *ur = upk + li * gp_row;
                const uint8_t *gs = gsc + (size_t)li * gpitch, *us = usc + (size_t)li * gpitch;
#pragma unroll
                for (int k = 0; k < XN / 32; ++k) {
                    const int unit = lr + LR * k;
                    const uint4 gw = *reinterpret_cast<const uint4 *>(gr + unit * 16);
                    const uint4 uw = *reinterpret_cast<const uint4 *>(ur + unit * 16);
                    const uint16_t gsv = *reinterpret_cast<const uint16_t *>(gs + unit * 2);
                    const uint16_t usv = *reinterpret_cast<const uint16_t *>(us + unit * 2);
                    g = unit_dot(gw, gsv, xr + 32 * k, g);
                    u = unit_dot(uw, usv, xr + 32 * k, u);
                }
            }
#pragma unroll
            for (int off = LR / 2; off >= 1; off >>= 1) {
                g += __shfl_xor_sync(0xffffffffu, g, off);
                u += __shfl_xor_sync(0xffffffffu, u, off);
            }
            if (v < v1 && lr == 0) {
                const int e = s_ids[slot];
                g *= __ldg(a.inv_scales + e);
                u *= __ldg(a.inv_scales + R + e);
                a.act[slot * I + v % I] = g / (1.0f + expf(-g)) * u;
            }
        }
    };
    if (have_gu_shared) {
        ok = mbar_wait(&bars[0], 0, err, kSiteTokenGateUp);
        if (ok) gate_up_range(shared_u0, u1);
    }
    if (have_gu_routed) {
        ok = mbar_wait(&bars[1], 0, err, kSiteTokenGateUp) && ok;
        if (ok) gate_up_range(u0, min(u1, (kSlots - 1) * I));
    }

    grid_barrier(a.sync + 64, a.sync + 96, err, kSiteTokenAct, &s_flag);

    // ---- down: the act vectors (rotated 16-byte groups, conflict-free) --------
    {
        const int per_slot = I / 4;  // float4 per slot
        const float4 *src = reinterpret_cast<const float4 *>(a.act);
        for (int idx = threadIdx.x; idx < kSlots * per_slot; idx += kTokenThreads) {
            const int slot = idx / per_slot, f = idx - slot * per_slot, unit = f >> 3, g4 = f & 7;
            reinterpret_cast<float4 *>(act_s + slot * I + unit * 32)[(g4 + unit) & 7] = __ldcg(src + idx);
        }
    }
    __syncthreads();
    if (nh > 0) {
        ok = mbar_wait(&bars[2], 0, err, kSiteTokenDown) && ok;
        ok = mbar_wait(&bars[3], 0, err, kSiteTokenDown) && ok;
    }
    if (ok && nh > 0) {
        // Rows d = slot * nh + (h - h0), slot-major; each warp a contiguous
        // range, LD lanes per row (one 16-byte unit each), RPD rows per pass.
        const int LD = I / 32 < 32 ? I / 32 : 32, RPD = 32 / LD, qd = lane / LD, ld = lane % LD;
        const int D = kSlots * nh;
        const int d0 = D * warp / kTokenWarps, d1 = D * (warp + 1) / kTokenWarps;
        float av[32];
        int cur = -1;
        for (int base = d0; base < d1; base += RPD) {
            const int d = base + qd;
            const int slot = d < d1 ? d / nh : cur;
            float acc = 0.0f;
            if (d < d1) {
                if (slot != cur) {
                    const float *src = act_s + slot * I + ld * 32;
#pragma unroll
                    for (int g4 = 0; g4 < 8; ++g4) {
                        const float4 t = reinterpret_cast<const float4 *>(src)[(g4 + ld) & 7];
                        av[4 * g4] = t.x;
                        av[4 * g4 + 1] = t.y;
                        av[4 * g4 + 2] = t.z;
                        av[4 * g4 + 3] = t.w;
                    }
                    cur = slot;
                }
                const int hl = d - slot * nh;
                const uint8_t *pr = dpk + ((size_t)slot * L.NH + hl) * dp_row;
                const uint8_t *sr = dsc + ((size_t)slot * L.NH + hl) * dpitch;
                acc = unit_dot(*reinterpret_cast<const uint4 *>(pr + ld * 16),
                               *reinterpret_cast<const uint16_t *>(sr + ld * 2), av, 0.0f);
            }
#pragma unroll
            for (int off = LD / 2; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
            if (d < d1 && ld == 0) {
                const int e = s_ids[slot];
                const float coef = s_w[slot] * __ldg(a.inv_scales + 2 * R + e);
                y_s[slot * L.NH + (d - slot * nh)] = coef * acc;
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
