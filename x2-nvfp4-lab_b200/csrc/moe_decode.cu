// Decode-path kernels; see moe_decode.cuh for the launch sequence.
#include "moe_decode.cuh"
#include "quant_terms.cuh"
#include "tma_util.cuh"

#include <atomic>
#include <cfloat>

namespace nvfp4 {

namespace {

constexpr int kRouteRowsPerCta = 4;   // one warp per router row, 128 threads
constexpr int kRouteTokens = 4;       // tokens per CTA column (independent accumulation chains)
constexpr int kRouteQuantCtas = 4;    // per token block, writing x's NVFP4 terms (tensor-core variant)

// Monotone map of a float to uint32 for redux.sync; -0 and +0 map alike so
// equal logits compare equal, as in the lab's selection loop.
__device__ __forceinline__ unsigned float_order_key(float v) {
    v = (v == 0.0f) ? 0.0f : v;
    const unsigned b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Inverse of float_order_key (zero comes back as +0).
__device__ __forceinline__ float float_from_order_key(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Shared-memory tables of the selection and dispatch step (E <= 256).
struct RouteSelectSmem {
    int ids[kDecodeMaxTokens * kTopK];
    float w[kDecodeMaxTokens * kTopK];
    float shared_w[kDecodeMaxTokens];
    int cnt[256];
    int off[257];
    int aidx[256];
    int aidx1[256];          // split by token half: the expert's half-1 group (after every half-0 group)
    int didx[256];           // split calls: the expert's first down group
    unsigned long long tokmask[256];
    float invd[257];
    int nrouted, nrouted1, ndown;
};

// Top-8 of token t by one warp from its logits in global memory: lane
// `slot` < 8 keeps the slot-th pick (largest logit first, the lowest id
// among equal logits, as the lab's selection loop), the softmax over the
// picks relative to the largest (denominator summed in slot order), and lane
// 8 the shared expert's sigmoid gate. Written to the scratch (ids, weights)
// and to the block's selection tables.
__device__ __forceinline__ void route_top8(const RouteArgs &a, int t, int lane, RouteSelectSmem &sm) {
    const DecodeScratch &s = a.s;
    const int E = a.E, R = E + 1;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = lane + 32 * i;
        v[i] = e < E ? __ldcg(s.logits + (size_t)t * R + e) : -FLT_MAX;
    }
    const float sl = __ldcg(s.logits + (size_t)t * R + E);
    // Lane `slot` keeps the slot-th pick.
    unsigned taken = 0;
    float my_v = 0.0f;
    int my_i = 0;
#pragma unroll 1
    for (int slot = 0; slot < kTopK; ++slot) {
        // Local best: strictly greater wins, so the lowest id survives ties.
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
        // Warp best: largest value, then the lowest id among equal values.
        const unsigned key = float_order_key(bv);
        const unsigned kmax = __reduce_max_sync(0xffffffffu, key);
        const unsigned imin = __reduce_min_sync(0xffffffffu, key == kmax ? (unsigned)bi : 0xffffffffu);
        bi = (int)imin;
        // The pick's value from its key (equal keys are equal values; a -0
        // comes back as +0, which leaves every later difference and exp
        // unchanged).
        bv = float_from_order_key(kmax);
        if (lane == slot) {
            my_v = bv;
            my_i = bi;
        }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    }
    // Softmax over the eight picks relative to the largest; the
    // denominator adds the picks in slot order.
    const float top0 = __shfl_sync(0xffffffffu, my_v, 0);
    const float my_e = lane < kTopK ? expf(my_v - top0) : 0.0f;
    float e8[kTopK];
#pragma unroll
    for (int slot = 0; slot < kTopK; ++slot) e8[slot] = __shfl_sync(0xffffffffu, my_e, slot);
    float den = 0.0f;
#pragma unroll
    for (int slot = 0; slot < kTopK; ++slot) den += e8[slot];
    if (lane < kTopK) {
        const float w = my_e / den;
        s.ids[t * kSlots + lane] = my_i;
        s.weights[t * kSlots + lane] = w;
        sm.ids[t * kTopK + lane] = my_i;
        sm.w[t * kTopK + lane] = w;
    } else if (lane == kTopK) {
        const float w = 1.0f / (1.0f + expf(-sl));
        s.ids[t * kSlots + kTopK] = E;
        s.weights[t * kSlots + kTopK] = w;
        sm.shared_w[t] = w;
    }
}

// Dispatch of the call's T tokens by the whole block, from the selection
// tables: per-expert counts and offsets, the stable permutation of (token,
// slot) pairs by expert, the compacted list of the experts computed here
// (routed ones in [e_first, e_first + e_count), then the shared expert when
// shared_here) with each one's token range, and the coefficient of every
// (group, token) pair (routing weight x inverse down global scale).
__device__ __forceinline__ void route_dispatch(const RouteArgs &a, RouteSelectSmem &sm) {
    const DecodeScratch &s = a.s;
    const int E = a.E, T = a.T;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Tensor-core calls above kDecodeTcMaxTokens tokens: an expert's tokens
    // 0-31 and 32-63 form separate groups (at most 32 tokens each, one
    // 128-row tile of terms), every half-0 group listed first.
    const bool split = a.quantize_x && T > kDecodeTcMaxTokens;
#pragma unroll 1
    for (int e = threadIdx.x; e < 256; e += blockDim.x) {
        sm.cnt[e] = 0;
        sm.tokmask[e] = 0ull;
    }
    __syncthreads();
#pragma unroll 1
    for (int i = threadIdx.x; i < T * kTopK; i += blockDim.x) {
        const int e = sm.ids[i];
        atomicAdd(&sm.cnt[e], 1);
        atomicOr(&sm.tokmask[e], 1ull << (i / kTopK));
    }
    __syncthreads();
    // Exclusive scans (counts -> offsets, local non-empty -> compact index).
    if (warp == 0) {
        // act: the expert has a group here (split: tokens of half 0); act1:
        // its half-1 group (split only); dact: its down groups (split only:
        // one, or one per half above kDecodeTcMaxTokens tokens).
        auto acts = [&](int e, int &c, int &act, int &act1, int &dact) {
            const bool own = e < E && e >= a.e_first && e < a.e_first + a.e_count;
            const unsigned long long m = e < E ? sm.tokmask[e] : 0ull;
            c = e < E ? sm.cnt[e] : 0;
            act = own && (split ? (m & 0xFFFFFFFFull) != 0ull : c > 0) ? 1 : 0;
            act1 = own && split && (m >> 32) != 0ull ? 1 : 0;
            dact = own && split && c > 0 ? (c > kDecodeTcMaxTokens ? 2 : 1) : 0;
        };
        // Lane l owns experts 8l .. 8l+7: their sums, an exclusive warp scan
        // of the sums, then the running offsets. The loops stay rolled: this
        // code runs once per call with cold instruction caches, where code
        // size is time (unrolled, the scan took 2 us).
        int sum = 0, asum = 0, asum1 = 0, dsum = 0;
#pragma unroll 1
        for (int i = 0; i < 8; ++i) {
            int c, act, act1, dact;
            acts(lane * 8 + i, c, act, act1, dact);
            sum += c;
            asum += act;
            asum1 += act1;
            dsum += dact;
        }
        int inc = sum, ainc = asum, ainc1 = asum1, dinc = dsum;
#pragma unroll 1
        for (int off = 1; off < 32; off <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, inc, off);
            const int ao = __shfl_up_sync(0xffffffffu, ainc, off);
            const int ao1 = __shfl_up_sync(0xffffffffu, ainc1, off);
            const int dof = __shfl_up_sync(0xffffffffu, dinc, off);
            if (lane >= off) {
                inc += o;
                ainc += ao;
                ainc1 += ao1;
                dinc += dof;
            }
        }
        int run = inc - sum, arun = ainc - asum, arun1 = ainc1 - asum1, drun = dinc - dsum;
#pragma unroll 1
        for (int i = 0; i < 8; ++i) {
            const int e = lane * 8 + i;
            int c, act, act1, dact;
            acts(e, c, act, act1, dact);
            if (e < E) {
                sm.off[e] = run;
                sm.aidx[e] = act ? arun : -1;
                sm.aidx1[e] = act1 ? arun1 : -1;
                sm.didx[e] = dact ? drun : -1;
            }
            run += c;
            arun += act;
            arun1 += act1;
            drun += dact;
        }
        if (lane == 31) {
            sm.off[E] = inc;
            sm.nrouted = ainc;
            sm.nrouted1 = ainc1;
            sm.ndown = dinc;
        }
    }
    __syncthreads();
    const int nrouted = sm.nrouted;
    // Group order: routed (half 0 when split), the shared expert's; then,
    // when split, the half-1 groups likewise.
    const int n0 = nrouted + (a.shared_here ? 1 : 0);
    const int nrouted1 = split ? sm.nrouted1 : 0;
    const int nact = split ? n0 + nrouted1 + (a.shared_here ? 1 : 0) : n0;
#pragma unroll 1
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        s.counts[e] = sm.cnt[e];
        s.offsets[e] = sm.off[e];
        const unsigned long long m = sm.tokmask[e];
        const int ai = sm.aidx[e];
        if (ai >= 0) {
            s.active_expert[ai] = e;
            s.tok_start[ai] = sm.off[e];
            s.tok_count[ai] = split ? __popcll(m & 0xFFFFFFFFull) : sm.cnt[e];
        }
        if (split && sm.aidx1[e] >= 0) {
            const int ai1 = n0 + sm.aidx1[e];
            s.active_expert[ai1] = e;
            s.tok_start[ai1] = sm.off[e] + __popcll(m & 0xFFFFFFFFull);
            s.tok_count[ai1] = __popcll(m >> 32);
        }
        const int dg = split ? sm.didx[e] : -1;
        if (dg >= 0) {
            const int c = sm.cnt[e], lo = __popcll(m & 0xFFFFFFFFull);
            const bool two = c > kDecodeTcMaxTokens;
            s.down_expert[dg] = e;
            s.down_start[dg] = sm.off[e];
            s.down_count[dg] = two ? lo : c;
            if (two) {
                s.down_expert[dg + 1] = e;
                s.down_start[dg + 1] = sm.off[e] + lo;
                s.down_count[dg + 1] = c - lo;
            }
        }
    }
    // Split calls: the down kernel's groups follow the routed ones with the
    // shared expert's two (tokens 32.., then 0-31).
    const int ndr = split ? sm.ndown : 0;
    if (threadIdx.x == 0) {
        s.offsets[E] = sm.off[E];
        *s.n_active = nact;
        *s.n_half0 = n0;
        if (split) *s.n_down = ndr + (a.shared_here ? 2 : 0);
    }
    // coef_tab is read only at the (group, token) pairs written below; the
    // groups of slot_group and coef_tab are the down kernel's (split calls:
    // the down groups).
#pragma unroll 1
    for (int i = threadIdx.x; i < T * kTopK; i += blockDim.x) {
        const int t = i / kTopK;
        const int e = sm.ids[i];
        const int rank = __popcll(sm.tokmask[e] & ((1ull << t) - 1ull));
        const int pos = sm.off[e] + rank;
        s.perm[pos] = i;
        s.tok_list[pos] = t;
        const int dg = sm.didx[e];
        const int ai = split ? (dg >= 0 ? dg + (sm.cnt[e] > kDecodeTcMaxTokens && t >= kDecodeTcMaxTokens ? 1 : 0) : -1)
                             : sm.aidx[e];
        s.inv_pos[i] = ai >= 0 ? pos : -1;
        s.slot_group[pos] = ai;
        if (ai >= 0) s.coef_tab[ai * kDecodeMaxTokens + t] = sm.w[i] * sm.invd[e];
    }
    if (a.shared_here) {
        const int ai0 = nrouted, ai1 = n0 + nrouted1;
#pragma unroll 1
        for (int t = threadIdx.x; t < T; t += blockDim.x) {
            const int pos = T * kTopK + t;
            const int ai = split ? ndr + (t >= kDecodeTcMaxTokens ? 0 : 1) : ai0;
            s.tok_list[pos] = t;
            s.slot_group[pos] = ai;
            s.coef_tab[ai * kDecodeMaxTokens + t] = sm.shared_w[t] * sm.invd[E];
        }
        if (threadIdx.x == 0) {
            s.active_expert[ai0] = E;
            s.tok_start[ai0] = T * kTopK;
            s.tok_count[ai0] = split ? kDecodeTcMaxTokens : T;
            if (split) {
                s.active_expert[ai1] = E;
                s.tok_start[ai1] = T * kTopK + kDecodeTcMaxTokens;
                s.tok_count[ai1] = T - kDecodeTcMaxTokens;
                // Its second half first: the down kernel spreads the last
                // group's tiles (here the full 32-token half) over its CTAs.
                for (int h = 0; h < 2; ++h) {
                    s.down_expert[ndr + 1 - h] = E;
                    s.down_start[ndr + 1 - h] = T * kTopK + kDecodeTcMaxTokens * h;
                    s.down_count[ndr + 1 - h] = h == 0 ? kDecodeTcMaxTokens : T - kDecodeTcMaxTokens;
                }
            }
        }
    }
}

// ---------------------------------------------------------------- routing
//
// Router logit of token t and row r (row E = shared gate), FP32 throughout
// as the lab's bf16_gemv_subgroup (nvfp4_gemv.cl:1223-1247) accumulates:
//   lane l owns columns j*128 + 4l + e (j ascending, then e = 0..3) and does
//   acc = acc + (bf16(W[r,k]) * x[t,k]) with the product and the sum each
//   rounded to FP32; the 32 lane sums combine by an xor butterfly (offsets
//   16, 8, 4, 2, 1). An optional per-expert bias is added last.
// The order is fixed, so the oracle reproduces every logit bit for bit.
//
// Grid: x = blocks of 4 router rows (one warp each), y = blocks of 4 tokens.
// Each CTA first copies its four router rows and its tokens (a contiguous
// [tt][H] range of x in the caller's format) into shared memory with 16-byte
// cp.async, so the dot products make no global round trip. The last CTA of a
// token block to finish runs top-8 for those tokens (one warp per token, so
// the selections of different blocks run on different SMs); the last token
// block to finish then dispatches.
__global__ void __launch_bounds__(128) moe_route_kernel(RouteArgs a) {
    extern __shared__ __align__(16) uint8_t route_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int R = a.E + 1;
    // CTAs past the router rows (tensor-core variant only) write the token
    // block's NVFP4 terms and take no ticket, so the chain logits -> top-8
    // -> dispatch never waits for the quantisation.
    const int nrow = (R + kRouteRowsPerCta - 1) / kRouteRowsPerCta;
    const bool quant_cta = (int)blockIdx.x >= nrow;
    const int row = blockIdx.x * kRouteRowsPerCta + warp;
    const int H = a.H;
    const int chunks = H / 128;
    const int t0 = blockIdx.y * kRouteTokens;
    const int tt = min(kRouteTokens, a.T - t0);
    DecodeScratch &s = a.s;
    const int esz = a.x_is_f32 ? 4 : 2;
    uint8_t *route_xs = route_smem;                                                     // [tt][H] of x
    uint16_t *route_w = reinterpret_cast<uint16_t *>(route_smem + (size_t)kRouteTokens * H * esz);  // [4][H]
    uint16_t *route_nw = route_w + (size_t)kRouteRowsPerCta * H;  // [H] RMSNorm weight (a.norm_w only)
    // Let the gate/up launch (programmatic dependent launch) get its CTAs
    // resident now; it waits for this grid's completion before reading.
    pdl_launch_dependents();

    // Every global input of the dot products is requested up front: the
    // warp's router row and the block's tokens go to shared memory by
    // cp.async, the row's bias to a register.
    const float bias = (a.bias && row < a.E) ? __ldg(a.bias + row) : 0.0f;
    {
        const uint8_t *wsrc = reinterpret_cast<const uint8_t *>(a.router + (size_t)min(row, R - 1) * H);
        uint8_t *wdst = reinterpret_cast<uint8_t *>(route_w + (size_t)warp * H);
        if (!quant_cta)
            for (int i = lane; i < H / 8; i += 32) cp_async16(wdst + 16 * i, wsrc + 16 * i);
        if (a.norm_w)  // bank data too
            for (int i = threadIdx.x; i < H / 8; i += blockDim.x)
                cp_async16(reinterpret_cast<uint8_t *>(route_nw) + 16 * i, reinterpret_cast<const uint8_t *>(a.norm_w) + 16 * i);
        // The router belongs to the bank; x and the scratch tables may be
        // written or still read by the preceding launch (this kernel is a
        // programmatic dependent launch): wait for it only now.
        pdl_wait();
        const uint8_t *src = static_cast<const uint8_t *>(a.x) + (size_t)t0 * H * esz;
        if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
            const int n16 = tt * H * esz / 16;
            for (int i = threadIdx.x; i < n16; i += blockDim.x) cp_async16(route_xs + 16 * i, src + 16 * i);
        } else if (a.x_is_f32) {
            for (int i = threadIdx.x; i < tt * H; i += blockDim.x)
                reinterpret_cast<float *>(route_xs)[i] = __ldg(reinterpret_cast<const float *>(src) + i);
        } else {
            for (int i = threadIdx.x; i < tt * H; i += blockDim.x)
                reinterpret_cast<uint16_t *>(route_xs)[i] = __ldg(reinterpret_cast<const uint16_t *>(src) + i);
        }
        cp_async_wait_all();
    }
    __syncthreads();

    // Optional RMSNorm of the staged tokens, with the bits of the standalone
    // RMSNorm kernel (runtime.cu): per token, 256 column-strided FP32 fmaf
    // partial sums (virtual thread v = tid and tid + 128), an xor butterfly
    // per warp of 32 partials, the eight warp sums added in order, rsqrtf,
    // then bf16(x * inv * w). Everything after reads the normalised copy.
    if (a.norm_w) {
        __shared__ float s_red[kRouteTokens][8];
        __shared__ float s_inv[kRouteTokens];
        uint16_t *xs = reinterpret_cast<uint16_t *>(route_xs);
#pragma unroll 1
        for (int j = 0; j < tt; ++j) {
            float ssa = 0.0f, ssb = 0.0f;
            for (int c = threadIdx.x; c < H; c += 256) {
                const float v = bf16_bits_to_f32(xs[(size_t)j * H + c]);
                ssa = fmaf(v, v, ssa);
            }
            for (int c = threadIdx.x + 128; c < H; c += 256) {
                const float v = bf16_bits_to_f32(xs[(size_t)j * H + c]);
                ssb = fmaf(v, v, ssb);
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) {
                ssa += __shfl_xor_sync(0xffffffffu, ssa, off);
                ssb += __shfl_xor_sync(0xffffffffu, ssb, off);
            }
            if (lane == 0) {
                s_red[j][warp] = ssa;
                s_red[j][warp + 4] = ssb;
            }
        }
        __syncthreads();
        if (threadIdx.x < tt) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < 8; ++w) tot += s_red[threadIdx.x][w];
            s_inv[threadIdx.x] = rsqrtf(tot / (float)H + a.norm_eps);
        }
        __syncthreads();
        // Two columns per step, the weight from its shared copy.
        uint32_t *xs2 = reinterpret_cast<uint32_t *>(xs);
        const uint32_t *nw2 = reinterpret_cast<const uint32_t *>(route_nw);
        for (int i = threadIdx.x; i < tt * H / 2; i += blockDim.x) {
            const int j = (2 * i) / H, c2 = i - j * (H / 2);
            const uint32_t xv = xs2[i], wv = nw2[c2];
            const float inv = s_inv[j];
            const uint32_t lo = f32_to_bf16_bits(bf16_bits_to_f32(xv & 0xFFFFu) * inv * bf16_bits_to_f32(wv & 0xFFFFu));
            const uint32_t hi = f32_to_bf16_bits(bf16_bits_to_f32(xv >> 16) * inv * bf16_bits_to_f32(wv >> 16));
            xs2[i] = lo | (hi << 16);
        }
        __syncthreads();
    }

    // FP16 copy of x for the in-register expert GEMVs (row block 0 converts
    // its tokens).
    if (blockIdx.x == 0 && !a.quantize_x) {
        for (int i = threadIdx.x; i < tt * H / 2; i += blockDim.x) {
            float2 v;
            if (a.x_is_f32) {
                v = reinterpret_cast<const float2 *>(route_xs)[i];
            } else {
                const uint32_t b = reinterpret_cast<const uint32_t *>(route_xs)[i];
                v = make_float2(bf16_bits_to_f32(b & 0xFFFFu), bf16_bits_to_f32(b >> 16));
            }
            reinterpret_cast<__half2 *>(s.x_f16 + (size_t)t0 * H)[i] = __floats2half2_rn(v.x, v.y);
        }
    }

    // The serial stretches of this kernel run once per layer call with cold
    // instruction caches, where code size is time: loops that need no
    // unrolling stay rolled (#pragma unroll 1).
    if (row < R && tt == 1) {
        // One token: a single accumulation chain, loads of four chunks in
        // flight (the same products and sums in the same order as below).
        float acc = 0.0f;
        const uint16_t *wr = route_w + (size_t)warp * H;
#pragma unroll 4
        for (int q = 0; q < chunks; ++q) {
            const int k = q * 128 + lane * 4;
            const uint2 wv = *reinterpret_cast<const uint2 *>(wr + k);
            float4 xv;
            if (a.x_is_f32) {
                xv = *reinterpret_cast<const float4 *>(route_xs + (size_t)k * 4);
            } else {
                const uint2 b = *reinterpret_cast<const uint2 *>(route_xs + (size_t)k * 2);
                xv = make_float4(bf16_bits_to_f32(b.x & 0xFFFFu), bf16_bits_to_f32(b.x >> 16),
                                 bf16_bits_to_f32(b.y & 0xFFFFu), bf16_bits_to_f32(b.y >> 16));
            }
            acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(wv.x & 0xFFFFu), xv.x));
            acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(wv.x >> 16), xv.y));
            acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(wv.y & 0xFFFFu), xv.z));
            acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(wv.y >> 16), xv.w));
        }
        float v = acc;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (lane == 0) {
            if (a.bias && row < a.E) v = __fadd_rn(v, bias);
            s.logits[(size_t)t0 * R + row] = v;
        }
    } else if (row < R) {
        // Several tokens: one FP32 chain per token in the fixed order above.
        // The loop body has no branches (missing tokens of a short block read
        // the block's last token and are not stored), so the four chains
        // interleave; the format branch sits outside the loop. Tokens go in
        // pairs through the packed f32x2 multiply and add (each element
        // rounded as the scalar instruction rounds it), half the instructions.
        static_assert(kRouteTokens % 2 == 0, "token pairs");
        unsigned long long acc2[kRouteTokens / 2];
#pragma unroll
        for (int j = 0; j < kRouteTokens / 2; ++j) acc2[j] = 0ull;  // (+0, +0)
        const uint16_t *wr = route_w + (size_t)warp * H;
        int xoff[kRouteTokens];
#pragma unroll
        for (int j = 0; j < kRouteTokens; ++j) xoff[j] = (j < tt ? j : tt - 1) * H;
        auto dots = [&](auto load_x) {
#pragma unroll 4
            for (int q = 0; q < chunks; ++q) {
                const int k = q * 128 + lane * 4;
                const uint2 wv = *reinterpret_cast<const uint2 *>(wr + k);
                const float w0 = bf16_bits_to_f32(wv.x & 0xFFFFu), w1 = bf16_bits_to_f32(wv.x >> 16);
                const float w2 = bf16_bits_to_f32(wv.y & 0xFFFFu), w3 = bf16_bits_to_f32(wv.y >> 16);
                float4 xv[kRouteTokens];
#pragma unroll
                for (int j = 0; j < kRouteTokens; ++j) xv[j] = load_x(xoff[j] + k);
                const unsigned long long ww0 = f32x2_pack(w0, w0), ww1 = f32x2_pack(w1, w1);
                const unsigned long long ww2 = f32x2_pack(w2, w2), ww3 = f32x2_pack(w3, w3);
#pragma unroll
                for (int j = 0; j < kRouteTokens / 2; ++j) {
                    const float4 xa = xv[2 * j], xb = xv[2 * j + 1];
                    acc2[j] = f32x2_add_rn(acc2[j], f32x2_mul_rn(ww0, f32x2_pack(xa.x, xb.x)));
                    acc2[j] = f32x2_add_rn(acc2[j], f32x2_mul_rn(ww1, f32x2_pack(xa.y, xb.y)));
                    acc2[j] = f32x2_add_rn(acc2[j], f32x2_mul_rn(ww2, f32x2_pack(xa.z, xb.z)));
                    acc2[j] = f32x2_add_rn(acc2[j], f32x2_mul_rn(ww3, f32x2_pack(xa.w, xb.w)));
                }
            }
        };
        if (a.x_is_f32) {
            dots([&](int idx) { return *reinterpret_cast<const float4 *>(route_xs + (size_t)idx * 4); });
        } else {
            dots([&](int idx) {
                const uint2 b = *reinterpret_cast<const uint2 *>(route_xs + (size_t)idx * 2);
                return make_float4(bf16_bits_to_f32(b.x & 0xFFFFu), bf16_bits_to_f32(b.x >> 16),
                                   bf16_bits_to_f32(b.y & 0xFFFFu), bf16_bits_to_f32(b.y >> 16));
            });
        }
        float acc[kRouteTokens];
#pragma unroll
        for (int j = 0; j < kRouteTokens / 2; ++j) f32x2_unpack(acc2[j], acc[2 * j], acc[2 * j + 1]);
#pragma unroll
        for (int j = 0; j < kRouteTokens; ++j) {
            float v = acc[j];
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
            if (lane == 0 && j < tt) {
                if (a.bias && row < a.E) v = __fadd_rn(v, bias);
                s.logits[(size_t)(t0 + j) * R + row] = v;
            }
        }
    }

    // Tensor-core variant: the block's tokens are also written as four NVFP4
    // terms (B rows 4t + j, scale atoms, global scale) by the block's
    // quantiser CTAs. The (token, 16-element block) pairs are spread over
    // them, one pair per thread; a CTA first reduces the amax of each token it
    // touches (from its shared-memory copy) so every CTA derives the same
    // global scale.
    if (quant_cta) {
        const int nb = H / 16;
        const int total = tt * nb;
        const int qc = (int)blockIdx.x - nrow, nq = (int)gridDim.x - nrow;
        const int p0 = (int)((long long)total * qc / nq);
        const int p1 = (int)((long long)total * (qc + 1) / nq);
        auto load_block = [&](int jt, int b, float (&v)[16]) {
            if (a.x_is_f32) {
                const float4 *p = reinterpret_cast<const float4 *>(route_xs + ((size_t)jt * H + 16 * b) * 4);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 f = p[q];
                    v[4 * q] = f.x;
                    v[4 * q + 1] = f.y;
                    v[4 * q + 2] = f.z;
                    v[4 * q + 3] = f.w;
                }
            } else {
                const uint4 *p = reinterpret_cast<const uint4 *>(route_xs + ((size_t)jt * H + 16 * b) * 2);
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const uint4 u = p[q];
                    const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        v[8 * q + 2 * h] = bf16_bits_to_f32(w4[h] & 0xFFFFu);
                        v[8 * q + 2 * h + 1] = bf16_bits_to_f32(w4[h] >> 16);
                    }
                }
            }
        };
        __shared__ float s_gq[kRouteTokens];
        __shared__ float s_amax[kRouteTokens][kRouteRowsPerCta];
        const int jt0 = p1 > p0 ? p0 / nb : 0, jt1 = p1 > p0 ? (p1 - 1) / nb : -1;
#pragma unroll 1
        for (int jt = jt0; jt <= jt1; ++jt) {
            float amax = 0.0f;
            for (int b = threadIdx.x; b < nb; b += blockDim.x) {
                float v[16];
                load_block(jt, b, v);
#pragma unroll
                for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            if (lane == 0) s_amax[jt][warp] = amax;
        }
        __syncthreads();
        if (threadIdx.x < kRouteTokens && (int)threadIdx.x >= jt0 && (int)threadIdx.x <= jt1) {
            const float (&m)[kRouteRowsPerCta] = s_amax[threadIdx.x];
            s_gq[threadIdx.x] = row_global_scale(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])));
        }
        __syncthreads();
        for (int pidx = p0 + threadIdx.x; pidx < p1; pidx += blockDim.x) {
            const int jt = pidx / nb, b = pidx - jt * nb;
            const int t = t0 + jt;
            const float g = s_gq[jt];
            if (b == 0) s.gx_tc[t] = g;
            float v[16];
            load_block(jt, b, v);
#pragma unroll 1
            for (int j = 0; j < kDecodeTcTerms; ++j) {
                uint32_t c0, c1;
                const uint32_t sc = quantize_block_term(v, g, c0, c1);
                const int n = kDecodeTcTerms * t + j;  // rows of token half n / 128 in its own tile
                *reinterpret_cast<uint2 *>(s.xq_tc + (size_t)n * (H / 2) + 8 * b) = make_uint2(c0, c1);
                s.xsf_tc[(size_t)(n >> 7) * (H / 64) * 512 + sf_atom_byte(n & 127, b)] = static_cast<uint8_t>(sc);
            }
        }
    }

    if (quant_cta) return;

    // The last row block of this token block runs top-8 for its tokens (one
    // warp per token); the last token block to finish then dispatches.
    __shared__ unsigned s_ticket;
    __shared__ RouteSelectSmem sm;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_ticket = atomicAdd(s.ticket + 1 + blockIdx.y, 1u);
    __syncthreads();
    if (s_ticket != (unsigned)nrow - 1u) return;
    __threadfence();
    // The coefficients need the inverse down scales: request them now,
    // store them after top-8.
    const float *inv_down = a.inv_scales + 2 * (size_t)R;
    float invd[3];
#pragma unroll
    for (int q = 0; q < 3; ++q) {
        const int e = threadIdx.x + 128 * q;
        invd[q] = e < R ? __ldg(inv_down + e) : 0.0f;
    }
    if (warp < tt) route_top8(a, t0 + warp, lane, sm);
#pragma unroll
    for (int q = 0; q < 3; ++q)
        if (threadIdx.x + 128 * q < R) sm.invd[threadIdx.x + 128 * q] = invd[q];
    if (threadIdx.x == 0) s.ticket[1 + blockIdx.y] = 0u;
    if (gridDim.y > 1) {
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) s_ticket = atomicAdd(s.ticket, 1u);
        __syncthreads();
        if (s_ticket != gridDim.y - 1) return;
        __threadfence();
        // Every token's picks, read back with all loads in flight at once.
        constexpr int kPer = (kDecodeMaxTokens * kSlots + 127) / 128;
        const int n = a.T * kSlots;
        int rid[kPer];
        float rw[kPer];
#pragma unroll
        for (int q = 0; q < kPer; ++q) {
            const int i = threadIdx.x + 128 * q;
            rid[q] = i < n ? __ldcg(s.ids + i) : 0;
            rw[q] = i < n ? __ldcg(s.weights + i) : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < kPer; ++q) {
            const int i = threadIdx.x + 128 * q;
            if (i < n) {
                const int t = i / kSlots, slot = i - t * kSlots;
                if (slot < kTopK) {
                    sm.ids[t * kTopK + slot] = rid[q];
                    sm.w[t * kTopK + slot] = rw[q];
                } else {
                    sm.shared_w[t] = rw[q];
                }
            }
        }
        if (threadIdx.x == 0) *s.ticket = 0u;
    }
    route_dispatch(a, sm);
}

}  // namespace

size_t decode_scratch_bytes(int E, int H, int I) {
    DecodeScratch s{};
    return decode_scratch_carve(s, nullptr, E, H, I);
}

size_t decode_route_scratch_bytes(int E, int H) {
    DecodeScratch s{};
    decode_scratch_carve(s, nullptr, E, H, 128);
    return reinterpret_cast<size_t>(s.act);
}

size_t decode_scratch_carve(DecodeScratch &s, void *base, int E, int H, int I) {
    const size_t T = kDecodeMaxTokens;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) & ~size_t(255);
        return static_cast<uint8_t *>(base) + o;
    };
    s.logits = reinterpret_cast<float *>(take(T * (E + 1) * 4));
    s.x_f16 = reinterpret_cast<__half *>(take(T * H * 2));
    s.ids = reinterpret_cast<int *>(take(T * kSlots * 4));
    s.weights = reinterpret_cast<float *>(take(T * kSlots * 4));
    s.counts = reinterpret_cast<int *>(take((size_t)E * 4));
    s.offsets = reinterpret_cast<int *>(take((size_t)(E + 1) * 4));
    s.perm = reinterpret_cast<int *>(take(T * kTopK * 4));
    s.inv_pos = reinterpret_cast<int *>(take(T * kTopK * 4));
    s.n_active = reinterpret_cast<int *>(take(4));
    s.n_half0 = reinterpret_cast<int *>(take(4));
    s.active_expert = reinterpret_cast<int *>(take((size_t)2 * (E + 1) * 4));
    s.tok_start = reinterpret_cast<int *>(take((size_t)2 * (E + 1) * 4));
    s.tok_count = reinterpret_cast<int *>(take((size_t)2 * (E + 1) * 4));
    s.n_down = reinterpret_cast<int *>(take(4));
    s.down_expert = reinterpret_cast<int *>(take((size_t)2 * (E + 1) * 4));
    s.down_start = reinterpret_cast<int *>(take((size_t)2 * (E + 1) * 4));
    s.down_count = reinterpret_cast<int *>(take((size_t)2 * (E + 1) * 4));
    s.tok_list = reinterpret_cast<int *>(take(T * kSlots * 4));
    s.coef_tab = reinterpret_cast<float *>(take((size_t)2 * (E + 1) * T * 4));
    s.ticket = reinterpret_cast<unsigned *>(take(kRouteTickets * 4));
    s.error = reinterpret_cast<int *>(take(4));
    s.slot_group = reinterpret_cast<int *>(take(T * kSlots * 4));
    s.act = reinterpret_cast<__half *>(take(T * kSlots * (size_t)I * 2));
    s.ypart = reinterpret_cast<float *>(take(T * kSlots * (size_t)H * 4));
    s.tile_count = reinterpret_cast<unsigned *>(take((size_t)(H / 64 + 1) * 4));
    s.xq_tc = take((size_t)kDecodeTcTerms * T * (H / 2));
    s.xsf_tc = take((size_t)2 * (H / 64) * 512);
    s.gx_tc = reinterpret_cast<float *>(take(T * 4));
    s.aq_tc = take((size_t)kDecodeTcTerms * T * kSlots * (I / 2));
    s.asf_tc = take((size_t)2 * (E + 1) * (I / 64) * 512);
    s.ga_tc = reinterpret_cast<float *>(take(T * kSlots * 4));
    return off;
}

namespace {

// Raise a routing kernel's dynamic shared-memory limit to all a CTA may hold,
// once per device (bit d of `done`).
template <typename K>
cudaError_t route_smem_limit(K kernel, std::atomic<uint64_t> &done) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
    if (bit && (done.load() & bit)) return cudaSuccess;
    cudaFuncAttributes fa{};
    err = cudaFuncGetAttributes(&fa, kernel);
    if (err != cudaSuccess) return err;
    int optin = 0;
    err = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (err != cudaSuccess) return err;
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
    if (err == cudaSuccess) done.fetch_or(bit);
    return err;
}

template <typename... KArgs>
cudaError_t launch_maybe_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                   bool dependent, const RouteArgs &a) {
    if (!dependent) {
        kernel<<<grid, block, smem, stream>>>(a);
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

}  // namespace

cudaError_t launch_route(const RouteArgs &a, cudaStream_t stream, bool dependent) {
    const int R = a.E + 1;
    const dim3 grid((R + kRouteRowsPerCta - 1) / kRouteRowsPerCta + (a.quantize_x ? kRouteQuantCtas : 0),
                    (a.T + kRouteTokens - 1) / kRouteTokens);
    const size_t smem = (size_t)kRouteTokens * a.H * (a.x_is_f32 ? 4 : 2) + (size_t)kRouteRowsPerCta * a.H * 2 +
                        (a.norm_w ? (size_t)a.H * 2 : 0);
    // The default dynamic limit is 48 KiB less the kernel's static shared
    // memory: raise it once per device.
    static std::atomic<uint64_t> done{0};
    const cudaError_t err = route_smem_limit(moe_route_kernel, done);
    if (err != cudaSuccess) return err;
    return launch_maybe_dependent(moe_route_kernel, grid, dim3(kRouteRowsPerCta * 32), smem, stream, dependent, a);
}

}  // namespace nvfp4
