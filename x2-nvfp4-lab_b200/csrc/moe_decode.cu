// Decode-path kernels; see moe_decode.cuh for the launch sequence.
#include "moe_decode.cuh"

#include <cfloat>
#include <map>
#include <mutex>

namespace nvfp4 {

namespace {

constexpr int kRouteRowsPerCta = 4;   // one warp per router row, 128 threads
constexpr int kRouteTokens = 8;       // tokens accumulated together (independent FP64 chains)

// Monotone map of a float to uint32 for redux.sync; -0 and +0 map alike so
// equal logits compare equal, as in the lab's selection loop.
__device__ __forceinline__ unsigned float_order_key(float v) {
    v = (v == 0.0f) ? 0.0f : v;
    const unsigned b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// ---------------------------------------------------------------- routing
//
// Router logit of token t and row r (row E = shared gate):
//   logit = fp32( sum_k bf16(W[r,k]) * x[t,k] )  accumulated in FP64.
// Lane l owns columns j*128 + 4l + e (j ascending, e = 0..3 ascending) and
// accumulates them with fma in that order; lanes combine with an xor
// butterfly (offsets 16, 8, 4, 2, 1). Every product of a BF16 and an FP32
// (or BF16) value is exact in FP64, so fma == mul+add and the oracle can
// reproduce the value bit for bit by following the same order. An optional
// per-expert FP32 bias is added to the rounded logit.
//
// Each warp owns one router row and accumulates up to kRouteTokens tokens
// at once (independent FMA chains); tokens are staged in shared memory as
// FP32 rows.
__global__ void __launch_bounds__(128) moe_route_kernel(RouteArgs a) {
    extern __shared__ __align__(16) float xs[];  // [kRouteTokens][H]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int R = a.E + 1;
    const int row = blockIdx.x * kRouteRowsPerCta + warp;
    const int H = a.H;
    const int chunks = H / 128;
    DecodeScratch &s = a.s;

    // FP16 copy of x for the expert GEMVs (tokens split across CTAs).
    for (int t = blockIdx.x; t < a.T; t += gridDim.x) {
        for (int k = threadIdx.x * 2; k < H; k += blockDim.x * 2) {
            float v0, v1;
            if (a.x_is_f32) {
                const float *xf = static_cast<const float *>(a.x) + (size_t)t * H + k;
                v0 = xf[0];
                v1 = xf[1];
            } else {
                const uint16_t *xb = static_cast<const uint16_t *>(a.x) + (size_t)t * H + k;
                v0 = bf16_bits_to_f32(xb[0]);
                v1 = bf16_bits_to_f32(xb[1]);
            }
            *reinterpret_cast<__half2 *>(s.x_f16 + (size_t)t * H + k) =
                __floats2half2_rn(v0, v1);
        }
    }

    for (int t0 = 0; t0 < a.T; t0 += kRouteTokens) {
        const int tt = min(kRouteTokens, a.T - t0);
        __syncthreads();
        for (int i = threadIdx.x; i < tt * (H / 4); i += blockDim.x) {
            const int j = i / (H / 4), k = (i - j * (H / 4)) * 4;
            float4 v;
            if (a.x_is_f32) {
                v = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(a.x) +
                                                           (size_t)(t0 + j) * H + k));
            } else {
                const uint2 b = __ldg(reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(a.x) +
                                                                      (size_t)(t0 + j) * H + k));
                v = make_float4(bf16_bits_to_f32(b.x & 0xFFFFu), bf16_bits_to_f32(b.x >> 16),
                                bf16_bits_to_f32(b.y & 0xFFFFu), bf16_bits_to_f32(b.y >> 16));
            }
            *reinterpret_cast<float4 *>(xs + j * H + k) = v;
        }
        __syncthreads();
        if (row < R) {
            const uint16_t *w = a.router + (size_t)row * H;
            double acc[kRouteTokens];
#pragma unroll
            for (int j = 0; j < kRouteTokens; ++j) acc[j] = 0.0;
            for (int q = 0; q < chunks; ++q) {
                const int k = q * 128 + lane * 4;
                const uint2 wv = __ldg(reinterpret_cast<const uint2 *>(w + k));
                const double w0 = bf16_bits_to_f32(wv.x & 0xFFFFu), w1 = bf16_bits_to_f32(wv.x >> 16);
                const double w2 = bf16_bits_to_f32(wv.y & 0xFFFFu), w3 = bf16_bits_to_f32(wv.y >> 16);
#pragma unroll
                for (int j = 0; j < kRouteTokens; ++j) {
                    if (j < tt) {
                        const float4 xv = *reinterpret_cast<const float4 *>(xs + j * H + k);
                        acc[j] = fma(w0, (double)xv.x, acc[j]);
                        acc[j] = fma(w1, (double)xv.y, acc[j]);
                        acc[j] = fma(w2, (double)xv.z, acc[j]);
                        acc[j] = fma(w3, (double)xv.w, acc[j]);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kRouteTokens; ++j) {
                if (j < tt) {
                    double v = acc[j];
#pragma unroll
                    for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                    if (lane == 0) {
                        float lv = (float)v;
                        if (a.bias && row < a.E) lv += a.bias[row];
                        s.logits[(size_t)(t0 + j) * R + row] = lv;
                    }
                }
            }
        }
    }

    // The last CTA to finish routes and dispatches every token.
    __shared__ unsigned s_ticket;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_ticket = atomicAdd(s.ticket, 1u);
    __syncthreads();
    if (s_ticket != gridDim.x - 1) return;
    __threadfence();

    __shared__ int s_ids[kDecodeMaxTokens * kTopK];
    __shared__ float s_w[kDecodeMaxTokens * kTopK];
    __shared__ float s_shared_w[kDecodeMaxTokens];
    __shared__ int s_cnt[256];
    __shared__ int s_off[257];
    __shared__ int s_aidx[256];
    __shared__ unsigned long long s_tokmask[256];
    __shared__ int s_nrouted;

    const int E = a.E, T = a.T;
    const float *inv_down = a.inv_scales + 2 * (size_t)R;

    // Top-8 per token: warp per token, lane l holds experts l + 32*i.
    for (int t = warp; t < T; t += blockDim.x / 32) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = lane + 32 * i;
            v[i] = e < E ? __ldcg(s.logits + (size_t)t * R + e) : -FLT_MAX;
        }
        unsigned taken = 0;
        float top_v[kTopK];
        int top_i[kTopK];
#pragma unroll
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
            bv = __shfl_sync(0xffffffffu, bv, bi & 31);
            top_v[slot] = bv;
            top_i[slot] = bi;
            if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        }
        if (lane == 0) {
            float den = 0.0f;
#pragma unroll
            for (int slot = 0; slot < kTopK; ++slot) den += expf(top_v[slot] - top_v[0]);
            for (int slot = 0; slot < kTopK; ++slot) {
                const float wgt = expf(top_v[slot] - top_v[0]) / den;
                s_ids[t * kTopK + slot] = top_i[slot];
                s_w[t * kTopK + slot] = wgt;
                s.ids[t * kSlots + slot] = top_i[slot];
                s.weights[t * kSlots + slot] = wgt;
            }
            const float sl = __ldcg(s.logits + (size_t)t * R + E);
            const float sw = 1.0f / (1.0f + expf(-sl));
            s_shared_w[t] = sw;
            s.ids[t * kSlots + kTopK] = E;
            s.weights[t * kSlots + kTopK] = sw;
        }
    }
    for (int e = threadIdx.x; e < 256; e += blockDim.x) {
        s_cnt[e] = 0;
        s_tokmask[e] = 0ull;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < T * kTopK; i += blockDim.x) {
        const int e = s_ids[i];
        atomicAdd(&s_cnt[e], 1);
        atomicOr(&s_tokmask[e], 1ull << (i / kTopK));
    }
    __syncthreads();
    // Exclusive scans (counts -> offsets, local non-empty -> compact index).
    if (warp == 0) {
        int loc[8], aloc[8];
        int sum = 0, asum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = lane * 8 + i;
            const int c = e < E ? s_cnt[e] : 0;
            const int act = (c > 0 && e >= a.e_first && e < a.e_first + a.e_count) ? 1 : 0;
            loc[i] = sum;
            aloc[i] = asum;
            sum += c;
            asum += act;
        }
        int inc = sum, ainc = asum;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, inc, off);
            const int ao = __shfl_up_sync(0xffffffffu, ainc, off);
            if (lane >= off) {
                inc += o;
                ainc += ao;
            }
        }
        const int excl = inc - sum, aexcl = ainc - asum;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = lane * 8 + i;
            if (e < E) {
                const int c = s_cnt[e];
                const int act = (c > 0 && e >= a.e_first && e < a.e_first + a.e_count) ? 1 : 0;
                s_off[e] = excl + loc[i];
                s_aidx[e] = act ? aexcl + aloc[i] : -1;
            }
        }
        if (lane == 31) {
            s_off[E] = inc;
            s_nrouted = ainc;
        }
    }
    __syncthreads();
    const int nrouted = s_nrouted;
    const int nact = nrouted + (a.shared_here ? 1 : 0);
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        s.counts[e] = s_cnt[e];
        s.offsets[e] = s_off[e];
        const int ai = s_aidx[e];
        if (ai >= 0) {
            s.active_expert[ai] = e;
            s.tok_start[ai] = s_off[e];
            s.tok_count[ai] = s_cnt[e];
            uint32_t m = 0;
            const unsigned long long tm = s_tokmask[e];
            for (int nt = 0; nt < kDecodeMaxTokens / 8; ++nt)
                if ((tm >> (nt * 8)) & 0xFFull) m |= 1u << nt;
            s.ntile_mask[ai] = m;
        }
    }
    if (threadIdx.x == 0) {
        s.offsets[E] = s_off[E];
        *s.n_active = nact;
    }
    for (int i = threadIdx.x; i < nact * kDecodeMaxTokens; i += blockDim.x) {
        s.pos_tab[i] = -1;
        s.coef_tab[i] = 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < T * kTopK; i += blockDim.x) {
        const int t = i / kTopK;
        const int e = s_ids[i];
        const int rank = __popcll(s_tokmask[e] & ((1ull << t) - 1ull));
        const int pos = s_off[e] + rank;
        s.perm[pos] = i;
        s.tok_list[pos] = t;
        const int ai = s_aidx[e];
        if (ai >= 0) {
            s.pos_tab[ai * kDecodeMaxTokens + t] = pos;
            s.coef_tab[ai * kDecodeMaxTokens + t] = s_w[i] * inv_down[e];
        }
    }
    if (a.shared_here) {
        const int ai = nrouted;
        for (int t = threadIdx.x; t < T; t += blockDim.x) {
            const int pos = T * kTopK + t;
            s.tok_list[pos] = t;
            s.pos_tab[ai * kDecodeMaxTokens + t] = pos;
            s.coef_tab[ai * kDecodeMaxTokens + t] = s_shared_w[t] * inv_down[E];
        }
        if (threadIdx.x == 0) {
            s.active_expert[ai] = E;
            s.tok_start[ai] = T * kTopK;
            s.tok_count[ai] = T;
            s.ntile_mask[ai] = (1u << ((T + 7) / 8)) - 1u;
        }
    }
    if (threadIdx.x == 0) *s.ticket = 0u;
}

// ------------------------------------------------------------ gate / up
//
// Work item = (active expert, 32-row tile of the intermediate dimension).
// Warp w computes rows (w&1)*16 .. +15 of the tile for gate and up over the
// K chunks q = w>>1, w>>1 + 4, ... (128 columns per chunk). Lane (g, c) reads
// 16 bytes (32 columns, two E4M3 blocks) of rows g and g+8; the 32 columns
// are decoded in registers to f16 (E2M1 * E4M3, exact) and fed to
// m16n8k16 MMAs whose B operand is the FP16 activation of up to eight of the
// expert's tokens. The k order inside an MMA is a permutation applied to A
// and B alike, so the dot product is unchanged. Partial sums of the four
// K-quarters are added in a fixed order, then SiLU(gate)*up is written FP16.
template <int NT>
__global__ void __launch_bounds__(256) moe_gate_up_kernel(GateUpArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int H = a.H, I = a.I, E = a.E;
    const int TS = act_tile_stride_bytes(H);
    uint8_t *xs = smem;
    float *red = reinterpret_cast<float *>(smem + NT * 8 * TS);  // [8][2][NT][4][32]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int mt = warp & 1, kq = warp >> 1;
    const int chunks = H / 128;
    const size_t row_bytes = H / 2, srow = H / 16;
    const DecodeScratch &s = a.s;
    const int nact = *s.n_active;
    const int mgroups = I / 32;
    const int items = nact * mgroups;

    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int ai = item / mgroups, mg = item - ai * mgroups;
        const int e = s.active_expert[ai];
        const int tstart = s.tok_start[ai], ntok = s.tok_count[ai];
        const int row = mg * 32 + mt * 16 + g;
        const size_t rbase = (size_t)e * I + row;
        const uint8_t *gp = a.gate_packed + rbase * row_bytes;
        const uint8_t *upp = a.up_packed + rbase * row_bytes;
        const uint8_t *gsc = a.gate_scales + rbase * srow;
        const uint8_t *usc = a.up_scales + rbase * srow;
        const float inv_gate = a.inv_scales[e];
        const float inv_up = a.inv_scales[(E + 1) + e];

        for (int tg = 0; tg < ntok; tg += NT * 8) {
            const int ncols = min(NT * 8, ntok - tg);
            __syncthreads();
            const int units_per_row = H / 8;
            for (int u = threadIdx.x; u < ncols * units_per_row; u += blockDim.x) {
                const int j = u / units_per_row, r = u - j * units_per_row;
                const int k = r * 8;
                const int q = k >> 7, cc = (k >> 5) & 3, v = (k >> 3) & 3;
                const int tok = s.tok_list[tstart + tg + j];
                const uint4 val = __ldg(reinterpret_cast<const uint4 *>(s.x_f16 + (size_t)tok * H + k));
                *reinterpret_cast<uint4 *>(xs + act_tile_offset(TS, j, q, cc, v)) = val;
            }
            __syncthreads();

            float cg[NT][4], cu[NT][4];
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int r = 0; r < 4; ++r) cg[n][r] = cu[n][r] = 0.0f;

            constexpr int QB = 4;
            for (int qb = kq; qb < chunks; qb += 4 * QB) {
                uint4 wg0[QB], wg8[QB], wu0[QB], wu8[QB];
                uint16_t sg0[QB], sg8[QB], su0[QB], su8[QB];
#pragma unroll
                for (int j = 0; j < QB; ++j) {
                    const int q = qb + 4 * j;
                    if (q < chunks) {
                        const size_t off = (size_t)q * 64 + c * 16;
                        wg0[j] = ldg_stream128(gp + off);
                        wg8[j] = ldg_stream128(gp + 8 * row_bytes + off);
                        wu0[j] = ldg_stream128(upp + off);
                        wu8[j] = ldg_stream128(upp + 8 * row_bytes + off);
                        const size_t soff = (size_t)q * 8 + 2 * c;
                        sg0[j] = ldg_u16(gsc + soff);
                        sg8[j] = ldg_u16(gsc + 8 * srow + soff);
                        su0[j] = ldg_u16(usc + soff);
                        su8[j] = ldg_u16(usc + 8 * srow + soff);
                    }
                }
#pragma unroll
                for (int j = 0; j < QB; ++j) {
                    const int q = qb + 4 * j;
                    if (q >= chunks) break;
                    const uint32_t scg0 = e4m3x2_to_f16x2(sg0[j]);
                    const uint32_t scg8 = e4m3x2_to_f16x2(sg8[j]);
                    const uint32_t scu0 = e4m3x2_to_f16x2(su0[j]);
                    const uint32_t scu8 = e4m3x2_to_f16x2(su8[j]);
                    const uint32_t *pg0 = &wg0[j].x, *pg8 = &wg8[j].x;
                    const uint32_t *pu0 = &wu0[j].x, *pu8 = &wu8[j].x;
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        uint32_t hg0[4], hg8[4], hu0[4], hu8[4];
                        e2m1x8_to_f16x8(pg0[v], hg0);
                        e2m1x8_to_f16x8(pg8[v], hg8);
                        e2m1x8_to_f16x8(pu0[v], hu0);
                        e2m1x8_to_f16x8(pu8[v], hu8);
                        const uint32_t mg0 = v < 2 ? f16x2_lo_lo(scg0) : f16x2_hi_hi(scg0);
                        const uint32_t mg8 = v < 2 ? f16x2_lo_lo(scg8) : f16x2_hi_hi(scg8);
                        const uint32_t mu0 = v < 2 ? f16x2_lo_lo(scu0) : f16x2_hi_hi(scu0);
                        const uint32_t mu8 = v < 2 ? f16x2_lo_lo(scu8) : f16x2_hi_hi(scu8);
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            hg0[b] = hmul2_u32(hg0[b], mg0);
                            hg8[b] = hmul2_u32(hg8[b], mg8);
                            hu0[b] = hmul2_u32(hu0[b], mu0);
                            hu8[b] = hmul2_u32(hu8[b], mu8);
                        }
#pragma unroll
                        for (int n = 0; n < NT; ++n) {
                            if (n * 8 >= ncols) break;
                            uint4 bv = make_uint4(0u, 0u, 0u, 0u);
                            if (n * 8 + g < ncols)
                                bv = *reinterpret_cast<const uint4 *>(xs + act_tile_offset(TS, n * 8 + g, q, c, v));
                            mma_16816(cg[n], hg0[0], hg8[0], hg0[1], hg8[1], bv.x, bv.y);
                            mma_16816(cg[n], hg0[2], hg8[2], hg0[3], hg8[3], bv.z, bv.w);
                            mma_16816(cu[n], hu0[0], hu8[0], hu0[1], hu8[1], bv.x, bv.y);
                            mma_16816(cu[n], hu0[2], hu8[2], hu0[3], hu8[3], bv.z, bv.w);
                        }
                    }
                }
            }
            // Fixed-order reduction of the four K-quarters.
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    red[((((kq * 2 + mt) * 2 + 0) * NT + n) * 4 + r) * 32 + lane] = cg[n][r];
                    red[((((kq * 2 + mt) * 2 + 1) * NT + n) * 4 + r) * 32 + lane] = cu[n][r];
                }
            __syncthreads();
            if (kq == 0) {
#pragma unroll
                for (int n = 0; n < NT; ++n) {
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        float gs = red[((((0 * 2 + mt) * 2 + 0) * NT + n) * 4 + r) * 32 + lane];
                        float us = red[((((0 * 2 + mt) * 2 + 1) * NT + n) * 4 + r) * 32 + lane];
#pragma unroll
                        for (int k2 = 1; k2 < 4; ++k2) {
                            gs += red[((((k2 * 2 + mt) * 2 + 0) * NT + n) * 4 + r) * 32 + lane];
                            us += red[((((k2 * 2 + mt) * 2 + 1) * NT + n) * 4 + r) * 32 + lane];
                        }
                        const int col = n * 8 + 2 * c + (r & 1);
                        if (col < ncols) {
                            const int rl = mt * 16 + g + (r >= 2 ? 8 : 0);
                            const float gate = gs * inv_gate;
                            const float up = us * inv_up;
                            const float act = gate / (1.0f + expf(-gate)) * up;
                            s.act[(size_t)(tstart + tg + col) * I + mg * 32 + rl] = __float2half_rn(act);
                        }
                    }
                }
            }
        }
    }
}

// -------------------------------------------------------- down + combine
//
// Work item = 16 output rows. The CTA's eight warps split the active experts
// (warp w takes experts w, w+8, ...). For one expert, lane (g, c) reads rows
// g and g+8 of W_down, the B operand column n of n-tile nt is the FP16
// activation of token nt*8+n for that expert (zero when the token is not
// routed there). Each expert's FP32 result is multiplied by
// routing_weight * inv_global_down and accumulated; warps are summed in a
// fixed order and the epilogue adds the residual.
template <int NT>
__global__ void __launch_bounds__(256) moe_down_kernel(DownArgs a) {
    extern __shared__ __align__(16) float red3[];  // [8][NT][4][32]
    const int H = a.H, I = a.I, T = a.T;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int chunks = I / 128;
    const size_t row_bytes = I / 2, srow = I / 16;
    const DecodeScratch &s = a.s;
    const int nact = *s.n_active;
    const int groups = H / 16;

    for (int hg = blockIdx.x; hg < groups; hg += gridDim.x) {
        float acc[NT][4];
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[n][r] = 0.0f;
        const int row = hg * 16 + g;

        for (int ai = warp; ai < nact; ai += 8) {
            const int e = s.active_expert[ai];
            const uint32_t mask = s.ntile_mask[ai];
            const uint8_t *wp = a.down_packed + ((size_t)e * H + row) * row_bytes;
            const uint8_t *sp = a.down_scales + ((size_t)e * H + row) * srow;
            int pos[NT];
            float coef0[NT], coef1[NT];
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const int tb = n * 8 + g;
                pos[n] = tb < T ? s.pos_tab[ai * kDecodeMaxTokens + tb] : -1;
                const int t0 = n * 8 + 2 * c;
                coef0[n] = t0 < T ? s.coef_tab[ai * kDecodeMaxTokens + t0] : 0.0f;
                coef1[n] = t0 + 1 < T ? s.coef_tab[ai * kDecodeMaxTokens + t0 + 1] : 0.0f;
            }
            float cacc[NT][4];
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int r = 0; r < 4; ++r) cacc[n][r] = 0.0f;

            constexpr int QB = 4;
            for (int qb = 0; qb < chunks; qb += QB) {
                uint4 w0[QB], w8[QB];
                uint16_t s0[QB], s8[QB];
#pragma unroll
                for (int j = 0; j < QB; ++j) {
                    const int q = qb + j;
                    if (q < chunks) {
                        const size_t off = (size_t)q * 64 + c * 16;
                        w0[j] = ldg_stream128(wp + off);
                        w8[j] = ldg_stream128(wp + 8 * row_bytes + off);
                        const size_t soff = (size_t)q * 8 + 2 * c;
                        s0[j] = ldg_u16(sp + soff);
                        s8[j] = ldg_u16(sp + 8 * srow + soff);
                    }
                }
#pragma unroll
                for (int j = 0; j < QB; ++j) {
                    const int q = qb + j;
                    if (q >= chunks) break;
                    const uint32_t sc0 = e4m3x2_to_f16x2(s0[j]);
                    const uint32_t sc8 = e4m3x2_to_f16x2(s8[j]);
                    uint4 bvs[NT][4];
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
#pragma unroll
                        for (int v = 0; v < 4; ++v) bvs[n][v] = make_uint4(0u, 0u, 0u, 0u);
                        if (((mask >> n) & 1u) && pos[n] >= 0) {
                            const __half *ap = s.act + (size_t)pos[n] * I + q * 128 + 32 * c;
#pragma unroll
                            for (int v = 0; v < 4; ++v) bvs[n][v] = ldcg128(ap + 8 * v);
                        }
                    }
                    const uint32_t *p0 = &w0[j].x, *p8 = &w8[j].x;
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        uint32_t h0[4], h8[4];
                        e2m1x8_to_f16x8(p0[v], h0);
                        e2m1x8_to_f16x8(p8[v], h8);
                        const uint32_t m0 = v < 2 ? f16x2_lo_lo(sc0) : f16x2_hi_hi(sc0);
                        const uint32_t m8 = v < 2 ? f16x2_lo_lo(sc8) : f16x2_hi_hi(sc8);
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            h0[b] = hmul2_u32(h0[b], m0);
                            h8[b] = hmul2_u32(h8[b], m8);
                        }
#pragma unroll
                        for (int n = 0; n < NT; ++n) {
                            if (!((mask >> n) & 1u)) continue;
                            const uint4 bv = bvs[n][v];
                            mma_16816(cacc[n], h0[0], h8[0], h0[1], h8[1], bv.x, bv.y);
                            mma_16816(cacc[n], h0[2], h8[2], h0[3], h8[3], bv.z, bv.w);
                        }
                    }
                }
            }
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                acc[n][0] = fmaf(coef0[n], cacc[n][0], acc[n][0]);
                acc[n][1] = fmaf(coef1[n], cacc[n][1], acc[n][1]);
                acc[n][2] = fmaf(coef0[n], cacc[n][2], acc[n][2]);
                acc[n][3] = fmaf(coef1[n], cacc[n][3], acc[n][3]);
            }
        }

#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int r = 0; r < 4; ++r) red3[((warp * NT + n) * 4 + r) * 32 + lane] = acc[n][r];
        __syncthreads();
        for (int i = threadIdx.x; i < 16 * T; i += blockDim.x) {
            const int t = i / 16, rl = i - t * 16;
            const int n = t >> 3, col = t & 7;
            const int gg = rl & 7;
            const int r = (rl >= 8 ? 2 : 0) + (col & 1);
            const int ln = gg * 4 + (col >> 1);
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < 8; ++w) v += red3[((w * NT + n) * 4 + r) * 32 + ln];
            const size_t o = (size_t)t * H + hg * 16 + rl;
            if (a.out_f32) {
                static_cast<float *>(a.out)[o] = v;
            } else {
                if (a.residual)
                    v += bf16_bits_to_f32(static_cast<const uint16_t *>(a.residual)[o]);
                static_cast<uint16_t *>(a.out)[o] = f32_to_bf16_bits(v);
            }
        }
        __syncthreads();
    }
}

// Raise a kernel's dynamic shared-memory limit once per device (the
// attribute call costs microseconds of host time, so it is not repeated on
// every launch).
template <typename K>
cudaError_t set_smem(K kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    static std::mutex m;
    static std::map<std::pair<int, const void *>, size_t> done;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    std::lock_guard<std::mutex> lock(m);
    auto key = std::make_pair(dev, reinterpret_cast<const void *>(kernel));
    auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return cudaSuccess;
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (err == cudaSuccess) done[key] = bytes;
    return err;
}

constexpr size_t kSmemLimit = 227 * 1024;

}  // namespace

size_t decode_scratch_bytes(int E, int H, int I) {
    DecodeScratch s{};
    return decode_scratch_carve(s, nullptr, E, H, I);
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
    s.n_active = reinterpret_cast<int *>(take(4));
    s.active_expert = reinterpret_cast<int *>(take((size_t)(E + 1) * 4));
    s.tok_start = reinterpret_cast<int *>(take((size_t)(E + 1) * 4));
    s.tok_count = reinterpret_cast<int *>(take((size_t)(E + 1) * 4));
    s.tok_list = reinterpret_cast<int *>(take(T * kSlots * 4));
    s.pos_tab = reinterpret_cast<int *>(take((size_t)(E + 1) * T * 4));
    s.coef_tab = reinterpret_cast<float *>(take((size_t)(E + 1) * T * 4));
    s.ntile_mask = reinterpret_cast<uint32_t *>(take((size_t)(E + 1) * 4));
    s.act = reinterpret_cast<__half *>(take(T * kSlots * (size_t)I * 2));
    s.ticket = reinterpret_cast<unsigned *>(take(4));
    return off;
}

cudaError_t launch_route(const RouteArgs &a, cudaStream_t stream) {
    const int R = a.E + 1;
    const int grid = (R + kRouteRowsPerCta - 1) / kRouteRowsPerCta;
    const size_t smem = (size_t)kRouteTokens * a.H * sizeof(float);
    if (smem > kSmemLimit) return cudaErrorInvalidValue;
    cudaError_t err = set_smem(moe_route_kernel, smem);
    if (err != cudaSuccess) return err;
    moe_route_kernel<<<grid, kRouteRowsPerCta * 32, smem, stream>>>(a);
    return cudaGetLastError();
}

template <int NT>
static size_t gate_up_smem(int H) {
    return (size_t)NT * 8 * act_tile_stride_bytes(H) + (size_t)8 * 2 * NT * 4 * 32 * 4;
}

template <int NT>
static cudaError_t launch_gate_up_nt(const GateUpArgs &a, int items_ub, int grid_cap, cudaStream_t stream) {
    const size_t smem = gate_up_smem<NT>(a.H);
    cudaError_t err = set_smem(moe_gate_up_kernel<NT>, smem);
    if (err != cudaSuccess) return err;
    const int grid = items_ub < grid_cap ? items_ub : grid_cap;
    moe_gate_up_kernel<NT><<<grid, 256, smem, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_gate_up(const GateUpArgs &a, int T, int grid_cap, cudaStream_t stream) {
    const int routed_ub = a.E < T * kTopK ? a.E : T * kTopK;
    const int items_ub = (routed_ub + 1) * (a.I / 32);
    if (T <= 8 || gate_up_smem<2>(a.H) > kSmemLimit)
        return launch_gate_up_nt<1>(a, items_ub, grid_cap, stream);
    if (T <= 16 || gate_up_smem<4>(a.H) > kSmemLimit)
        return launch_gate_up_nt<2>(a, items_ub, grid_cap, stream);
    return launch_gate_up_nt<4>(a, items_ub, grid_cap, stream);
}

template <int NT>
static cudaError_t launch_down_nt(const DownArgs &a, int grid_cap, cudaStream_t stream) {
    const size_t smem = (size_t)8 * NT * 4 * 32 * 4;
    cudaError_t err = set_smem(moe_down_kernel<NT>, smem);
    if (err != cudaSuccess) return err;
    const int groups = a.H / 16;
    const int grid = groups < grid_cap ? groups : grid_cap;
    moe_down_kernel<NT><<<grid, 256, smem, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_down(const DownArgs &a, int grid_cap, cudaStream_t stream) {
    if (a.T <= 8) return launch_down_nt<1>(a, grid_cap, stream);
    if (a.T <= 16) return launch_down_nt<2>(a, grid_cap, stream);
    if (a.T <= 32) return launch_down_nt<4>(a, grid_cap, stream);
    return launch_down_nt<8>(a, grid_cap, stream);
}

}  // namespace nvfp4
