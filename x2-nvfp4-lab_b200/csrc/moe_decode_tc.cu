// Tensor-core expert GEMVs of the decode path (calls of up to 32 tokens on
// banks whose H and I are multiples of 256).
//
// The weights stream through tcgen05 block-scaled NVFP4 MMAs
// (kind::mxf4nvf4, M 128, N 128, K 64, FP32 accumulators in tensor memory),
// so no instruction of the CTA touches a weight byte: the hardware applies
// the E4M3 block scales. The activations enter as four NVFP4 terms per row
// sharing the row's FP32 global scale (term j+1 quantises what terms 1..j
// left over; quant_terms.cuh: the routing kernel writes x's terms,
// quantize_act_tc_kernel those of SiLU(gate)*up). The four terms of a row
// are four B rows (the N dimension) rather than extra K, so every weight tile
// is read from shared memory by one MMA and the epilogue adds the four
// accumulator columns of a row. A B tile of 128 rows holds 32 rows x 4 terms:
//   gate/up  B = the terms of every token of the call (one tile, resident in
//            L2, re-read per stage); column 4t + j is term j of token t.
//   down     B = the terms of the group's slot rows (they are consecutive in
//            dispatch order): rows 4*tok_start .. of the activation terms.
//
// One persistent CTA per SM walks (active expert group, 128-row weight tile)
// items. Warp roles: warp 0 producer (TMA tiles of the weights and of B,
// bulk copies of the scale-factor atoms, all on the stage's mbarrier), warp 1
// MMA issuer and tensor-memory owner, warps 2-5 epilogue, warps 6-9 weight
// scale factors: each stage's atoms go from shared memory into tensor memory
// by tcgen05.st, one 32-lane quarter per warp, so the MMA thread issues only
// MMAs and commits (a tcgen05.cp per atom costs the issuing thread about as
// much as an MMA). Every mbarrier wait is bounded; on a timeout the CTA
// records the error, drains its copies and MMAs in flight, frees its tensor
// memory and exits.
#include "moe_decode.cuh"
#include "quant_terms.cuh"
#include "tcgen05_util.cuh"
#include "tma_util.cuh"

#include <atomic>

namespace nvfp4 {

namespace {

constexpr int kTcThreads = 320;
constexpr int kSfWarp0 = 6;  // first scale-factor warp
constexpr int kTile = 128;                     // weight rows per item, B rows per tile
constexpr int kTileBytes = kTile * 128;        // 128 rows x 128 bytes (256 FP4 columns)
constexpr int kSfStage = 4 * 512;              // four 64-column scale atoms
constexpr int kStageK = 256;

__device__ __forceinline__ uint8_t *align1024(uint8_t *p) {
    return reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ __half f32_to_f16_sat(float v) {
    uint16_t h;
    asm("cvt.rn.satfinite.f16.f32 %0, %1;" : "=h"(h) : "f"(v));
    return __ushort_as_half(h);
}

// Bounded wait that ignores the shared error word (used to drain copies in
// flight after a failure).
__device__ __forceinline__ bool mbar_wait_drain(uint64_t *bar, uint32_t parity) {
    const unsigned long long t0 = global_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u && global_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ void report(const DecodeScratch &s) {
    const int code = *reinterpret_cast<volatile int *>(s.error);
    if (s.host_error) *reinterpret_cast<volatile int *>(s.host_error) = code != 0 ? code : kErrWaitTimeout;
}

struct Item {
    int ai, e, mt, tstart, ntok;
};

__device__ __forceinline__ Item load_item(const DecodeScratch &s, int item, int mtiles) {
    Item it;
    it.ai = item / mtiles;
    it.mt = item - it.ai * mtiles;
    it.e = s.active_expert[it.ai];
    it.tstart = s.tok_start[it.ai];
    it.ntok = min(s.tok_count[it.ai], kDecodeTcMaxTokens);
    return it;
}

// ------------------------------------------------------------- gate / up
//
// Items (active group, 128 rows of I) in a strided order; every item reads
// the same B tile (the terms of every token), so x's scale factors are
// copied into tensor memory once per CTA. Per 256-column stage: TMA of the
// gate and up tiles and of the B slice, bulk copies of the gate and up scale
// atoms; the MMA thread copies the eight weight atoms and issues eight MMAs.
constexpr int kGuS = 4;
constexpr int kGuStage = 3 * kTileBytes + 2 * kSfStage;   // A gate, A up, B, SFA gate, SFA up
constexpr int kSfbMax = 32 * 512;                         // x scale atoms for H <= 2048
constexpr int kGuColSfa = 256;                             // + st * 32 (gate 16, up 16)
constexpr int kGuColSfb = kGuColSfa + kGuS * 32;           // + 4 per 64 columns of H
constexpr size_t kGuSmem = 1024 + (size_t)kGuS * kGuStage + kSfbMax + 1024;
static_assert(kGuColSfb + 128 <= 512, "tensor memory overflow");
static_assert(kGuSmem <= 232448, "shared memory overflow");

__global__ void __launch_bounds__(kTcThreads, 1)
    moe_gate_up_tc_kernel(const __grid_constant__ CUtensorMap tm_g, const __grid_constant__ CUtensorMap tm_u,
                          const __grid_constant__ CUtensorMap tm_b, DecodeTcArgs a) {
    constexpr int S = kGuS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align1024(smem_raw);
    uint8_t *sfb_stage = smem + (size_t)S * kGuStage;
    uint64_t *full = reinterpret_cast<uint64_t *>(sfb_stage + kSfbMax);
    uint64_t *empty = full + S;
    uint64_t *acc_full = empty + S;
    uint64_t *acc_empty = acc_full + 1;
    uint64_t *sfb_full = acc_empty + 1;
    uint64_t *drain = sfb_full + 1;
    uint64_t *sfa_full = drain + 1;  // [S] the stage's weight scale factors are in tensor memory
    uint64_t *sfb_ready = sfa_full + S;  // x's scale factors are in tensor memory
    uint64_t *sfa_in = sfb_ready + 1;    // [S] the stage's weight scale atoms are in shared memory
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sfa_in + S);
    int *acc_ok = reinterpret_cast<int *>(tmem_slot + 1);
    int *col_tok = reinterpret_cast<int *>(tmem_slot + 4);       // [2][32] token of each group row
    float *col_scale = reinterpret_cast<float *>(col_tok + 64);  // [2][32] its global scale
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const DecodeScratch &s = a.s;
    int *err = s.error;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 1);
        mbar_init(sfb_full, 1);
        mbar_init(drain, 1);
        for (int i = 0; i < S; ++i) {
            mbar_init(sfa_full + i, 4);
            mbar_init(sfa_in + i, 1);
        }
        mbar_init(sfb_ready, 4);
        fence_barrier_init();
        prefetch_tensormap(&tm_g);
        prefetch_tensormap(&tm_u);
        prefetch_tensormap(&tm_b);
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, 512);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // routing tables and x's terms are read from here on
    pdl_launch_dependents();

    const int mtiles = a.I / kTile;
    const int total = *s.n_active * mtiles;
    // Calls above kDecodeTcMaxTokens tokens: the items of the half-0 groups
    // ([0, hi)) and of the half-1 groups ([lo, total)) go to two sets of CTAs
    // in proportion to their counts (the launch gives at least two CTAs);
    // each set reads its half's 128-row tile of x's terms.
    int lo = 0, hi = total, nctas = (int)gridDim.x, rank = (int)blockIdx.x, half = 0;
    if (a.T > kDecodeTcMaxTokens) {
        const int t0 = *s.n_half0 * mtiles;
        int g0 = total > 0 ? (int)(((long long)gridDim.x * t0 + total / 2) / total) : 0;
        if (t0 > 0 && g0 < 1) g0 = 1;
        if (t0 < total && g0 > (int)gridDim.x - 1) g0 = (int)gridDim.x - 1;
        if (rank < g0) {
            hi = t0;
            nctas = g0;
        } else {
            half = 1;
            lo = t0;
            rank -= g0;
            nctas = (int)gridDim.x - g0;
        }
    }
    // Within a set, strided items over the fewest CTAs that need no more
    // waves than the set: every working CTA then walks the same number of
    // items (or one fewer), and the weight stream of the SMs left idle goes
    // to them instead of to a last partial wave.
    const int span = hi - lo;
    const int waves = nctas > 0 ? (span + nctas - 1) / nctas : 0;
    const int ctas = waves > 0 ? (span + waves - 1) / waves : 0;
    const bool works = rank < ctas;
    const int first = works ? lo + rank : hi;  // this CTA's first item
    const int kstages = a.H / kStageK;
    const int kw = a.H / 64;

    if (warp == 0) {
        // ------------------------------------------------------ producer
        uint32_t it = 0;
        bool ok = true;
        if (lane == 0 && works) {
            mbar_arrive_expect_tx(sfb_full, kw * 512);
            bulk_g2s(sfb_stage, a.sfb + (size_t)half * kw * 512, kw * 512, sfb_full);
        }
        for (int item = first; item < hi && ok; item += ctas) {
            const Item ti = load_item(s, item, mtiles);
            const int arow = ti.e * a.I + ti.mt * kTile;
            const size_t sfa_off = (size_t)(arow / kTile) * kw * 512;
            for (int ks = 0; ks < kstages; ++ks, ++it) {
                const int st = it % S;
                const uint32_t ph = (it / S) & 1u;
                int okw = 1;
                if (lane == 0) okw = mbar_wait(empty + st, ph ^ 1u, err, kSiteGemmEmpty) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, okw, 0)) {
                    ok = false;
                    break;
                }
                uint8_t *stage = smem + (size_t)st * kGuStage;
                if (lane == 0) {
                    // The scale atoms first and on their own barrier: the
                    // store warps need only them, and they land first.
                    mbar_arrive_expect_tx(sfa_in + st, 2 * kSfStage);
                    bulk_g2s(stage + 3 * kTileBytes, a.sfa[0] + sfa_off + (size_t)ks * kSfStage, kSfStage, sfa_in + st);
                    bulk_g2s(stage + 3 * kTileBytes + kSfStage, a.sfa[1] + sfa_off + (size_t)ks * kSfStage, kSfStage,
                             sfa_in + st);
                    mbar_arrive_expect_tx(full + st, 3 * kTileBytes);
                    tma_load_2d(stage, &tm_g, full + st, ks * 128, arow);
                    tma_load_2d(stage + kTileBytes, &tm_u, full + st, ks * 128, arow);
                    tma_load_2d(stage + 2 * kTileBytes, &tm_b, full + st, ks * 128, kTile * half);
                }
            }
        }
        if (!ok || *reinterpret_cast<volatile int *>(err) != 0) {
            // Drain the copies still in flight before the CTA exits.
            if (lane == 0) {
                if (works) mbar_wait_drain(sfb_full, 0);
                const uint32_t first = it > (uint32_t)S ? it - S : 0u;
                for (uint32_t k = first; k < it; ++k) {
                    mbar_wait_drain(full + (k % S), (k / S) & 1u);
                    mbar_wait_drain(sfa_in + (k % S), (k / S) & 1u);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_mxf4nvf4(kTile);
            const uint32_t smem_base = smem_u32(smem);
            uint32_t it = 0, tcount = 0;
            bool ok = true;
            if (works) {
                ok = mbar_wait(sfb_ready, 0, err, kSiteGemmFull);
                tc::fence_after_sync();
            }
            for (int item = first; item < hi && ok; item += ctas, ++tcount) {
                if (tcount > 0 && !mbar_wait(acc_empty, (tcount - 1) & 1u, err, kSiteGemmAccEmpty)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                for (int ks = 0; ks < kstages; ++ks, ++it) {
                    const int st = it % S;
                    const uint32_t ph = (it / S) & 1u;
                    if (!mbar_wait(full + st, ph, err, kSiteGemmFull) ||
                        !mbar_wait(sfa_full + st, ph, err, kSiteGemmFull)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t sb = smem_base + (uint32_t)st * kGuStage;
                    const uint32_t tsfa = tmem + kGuColSfa + (uint32_t)st * 32;
#pragma unroll
                    for (int at = 0; at < 4; ++at) {
                        const uint32_t acc = (ks | at) != 0 ? 1u : 0u;
                        const uint64_t bdesc = tc::smem_desc_sw128(sb + 2 * kTileBytes + 32 * at);
                        const uint32_t tsfb = tmem + kGuColSfb + 4 * (ks * 4 + at);
                        tc::mma_mxf4nvf4(tmem, tc::smem_desc_sw128(sb + 32 * at), bdesc, idesc, tsfa + 4 * at, tsfb,
                                         acc);
                        tc::mma_mxf4nvf4(tmem + 128, tc::smem_desc_sw128(sb + kTileBytes + 32 * at), bdesc, idesc,
                                         tsfa + 16 + 4 * at, tsfb, acc);
                    }
                    tc::commit(empty + st);
                }
                if (!ok) break;
                tc::commit(acc_full);
            }
            tc::commit(drain);
            mbar_wait_drain(drain, 0);
        }
        __syncwarp();
    } else if (warp >= kSfWarp0) {
        // ------------------------------------------------- scale factors
        // Stage st's eight weight atoms (gate 0-3, up 0-3, 512 bytes apart)
        // into columns tsfa + 4a of this warp's lane quarter. The slot is
        // free: the stage was refilled only after the MMAs that read the
        // slot's previous atoms completed.
        const uint32_t quarter = (uint32_t)(32 * (warp & 3)) << 16;
        uint32_t it = 0;
        bool ok = true;
        // First x's kw scale atoms (every item's B, kw a multiple of 4),
        // four per store.
        if (works) {
            ok = __all_sync(0xffffffffu, mbar_wait(sfb_full, 0, err, kSiteGemmFull));
            if (ok) {
#pragma unroll 1
                for (int at = 0; at < kw; at += 4)
                    tc::st_sf_atoms<4>(tmem + quarter + kGuColSfb + 4 * at, sfb_stage + at * 512, 512, lane);
                tc::wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(sfb_ready);
            }
        }
        for (int item = first; item < hi && ok; item += ctas) {
            for (int ks = 0; ks < kstages; ++ks, ++it) {
                const int st = it % S;
                if (!__all_sync(0xffffffffu, mbar_wait(sfa_in + st, (it / S) & 1u, err, kSiteGemmFull))) {
                    ok = false;
                    break;
                }
                tc::st_sf_atoms<8>(tmem + quarter + kGuColSfa + (uint32_t)st * 32,
                                   smem + (size_t)st * kGuStage + 3 * kTileBytes, 512, lane);
                tc::wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(sfa_full + st);
            }
        }
    } else {
        // ----------------------------------------------------- epilogue
        const int sub = warp & 3;
        const int et = threadIdx.x - 64;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * sub) << 16);
        uint32_t tcount = 0;
        for (int item = first; item < hi; item += ctas, ++tcount) {
            const Item ti = load_item(s, item, mtiles);
            int *ctok = col_tok + 32 * (tcount & 1);
            float *cscale = col_scale + 32 * (tcount & 1);
            if (et < ti.ntok) {
                const int t = s.tok_list[ti.tstart + et];
                ctok[et] = t - kDecodeTcMaxTokens * half;  // its column block in this half's tile
                cscale[et] = s.gx_tc[t];
            }
            const float ig = a.inv_scales[ti.e], iu = a.inv_scales[(a.E + 1) + ti.e];
            if (et == 0) *acc_ok = mbar_wait(acc_full, tcount & 1u, err, kSiteGemmAccFull) ? 1 : 0;
            named_barrier(1, 128);
            if (!*reinterpret_cast<volatile int *>(acc_ok)) break;
            tc::fence_after_sync();
            const int m = ti.mt * kTile + 32 * sub + lane;
            // Column 4t + j of the accumulators is term j of token t. The
            // accumulator is handed back as soon as its last columns are in
            // registers (one batch of four tokens in the common case).
            for (int i0 = 0; i0 < ti.ntok; i0 += 4) {
                uint32_t rg[4][4], ru[4][4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int t = ctok[i0 + q < ti.ntok ? i0 + q : i0];
                    tc::ld_32x32b_x4(lane_base + 4 * t, rg[q]);
                    tc::ld_32x32b_x4(lane_base + 128 + 4 * t, ru[q]);
                }
                tc::wait_ld();
                if (i0 + 4 >= ti.ntok) {
                    tc::fence_before_sync();
                    named_barrier(1, 128);
                    if (et == 0) mbar_arrive(acc_empty);
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int i = i0 + q;
                    if (i < ti.ntok) {
                        const float gs = ((__uint_as_float(rg[q][0]) + __uint_as_float(rg[q][1])) +
                                          __uint_as_float(rg[q][2])) + __uint_as_float(rg[q][3]);
                        const float us = ((__uint_as_float(ru[q][0]) + __uint_as_float(ru[q][1])) +
                                          __uint_as_float(ru[q][2])) + __uint_as_float(ru[q][3]);
                        const float cs = cscale[i];
                        const float gate = gs * (ig * cs);
                        const float up = us * (iu * cs);
                        s.act[(size_t)(ti.tstart + i) * a.I + m] = f32_to_f16_sat(gate / (1.0f + expf(-gate)) * up);
                    }
                }
            }
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
    }
    if (threadIdx.x == 0 && *reinterpret_cast<volatile int *>(err) != 0) report(s);
}

// ------------------------------------------------------------------ down
//
// Each CTA walks a contiguous range of (active group, 128 rows of H) items
// (after at most one tile of the shared expert's group, whose tiles are
// spread over the grid), so consecutive items mostly share their group:
// the group's B tile (its
// slot rows' terms over all of K = I) and scale atoms are loaded into one of
// two B buffers and copied into tensor memory once per group. A stage is one
// item's weight tile over all of K (KB 256-column boxes) and its scale atoms.
template <int KB>
struct DnCfg {
    static constexpr int kStage = KB * kTileBytes + KB * kSfStage;
    static constexpr int kS = KB == 1 ? 8 : 4;
    static constexpr int kAtoms = KB * 4;                   // 64-column scale atoms over K
    static constexpr int kColSfa = 256;                     // + st * kAtoms * 4
    static constexpr int kColSfb = kColSfa + kS * kAtoms * 4;  // + bb * kAtoms * 4
    static constexpr size_t kSmem = 1024 + (size_t)(kS + 2) * kStage + 1024;
    static_assert(kColSfb + 2 * kAtoms * 4 <= 512, "tensor memory overflow");
    static_assert(kSmem <= 232448, "shared memory overflow");
    static_assert(kStage % 1024 == 0, "stage must keep 1024-byte tile alignment");
};

template <int KB>
__global__ void __launch_bounds__(kTcThreads, 1)
    moe_down_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                       DecodeTcArgs a) {
    using Cfg = DnCfg<KB>;
    constexpr int S = Cfg::kS;
    constexpr int kw = Cfg::kAtoms;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align1024(smem_raw);
    uint8_t *bbuf = smem + (size_t)S * Cfg::kStage;  // [2] B tile + scale atoms
    uint64_t *full = reinterpret_cast<uint64_t *>(bbuf + 2 * Cfg::kStage);
    uint64_t *empty = full + S;
    uint64_t *bfull = empty + S;       // [2]
    uint64_t *bempty = bfull + 2;      // [2]
    uint64_t *acc_full = bempty + 2;   // [2]
    uint64_t *acc_empty = acc_full + 2;  // [2]
    uint64_t *drain = acc_empty + 2;
    uint64_t *sfa_full = drain + 1;      // [S] the stage's weight scale factors are in tensor memory
    uint64_t *sfa_in = sfa_full + S;     // [S] the stage's weight scale atoms are in shared memory
    uint64_t *sfb_ready = sfa_in + S;    // [2] the B buffer's scale factors are in tensor memory
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sfb_ready + 2);
    int *acc_ok = reinterpret_cast<int *>(tmem_slot + 1);
    float *col_scale = reinterpret_cast<float *>(tmem_slot + 4);  // [2][32]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const DecodeScratch &s = a.s;
    int *err = s.error;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bfull + b, 1);
            mbar_init(bempty + b, 1);
            mbar_init(acc_full + b, 1);
            mbar_init(acc_empty + b, 1);
        }
        mbar_init(drain, 1);
        for (int i = 0; i < S; ++i) {
            mbar_init(sfa_full + i, 4);
            mbar_init(sfa_in + i, 1);
        }
        mbar_init(sfb_ready, 4);
        mbar_init(sfb_ready + 1, 4);
        fence_barrier_init();
        prefetch_tensormap(&tm_a);
        prefetch_tensormap(&tm_b);
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, 512);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    // This grid starts only after the gate/up grid has completed (the
    // launches between, with programmatic serialisation, trigger their
    // dependents only after waiting for it), so the routing tables are
    // complete here; the activation terms and their scales are read only
    // after each role's griddepcontrol.wait.
    const int mtiles = a.H / kTile;
    const int total = *s.n_active * mtiles;
    // Items over the fewest CTAs that need no more waves than the grid, each
    // CTA taking the same count (or one fewer). The shared expert's groups
    // (the last one, or above kDecodeTcMaxTokens tokens the last two: a row
    // for every token) have the costliest items: their tiles go one each to
    // evenly spaced CTAs, first in their lists, and the other items split
    // into contiguous runs around them, so consecutive items of a CTA mostly
    // share their group.
    const int waves = (total + (int)gridDim.x - 1) / (int)gridDim.x;
    const int ctas = waves > 0 ? (total + waves - 1) / waves : 0;
    const int shg = a.T > kDecodeTcMaxTokens && 2 * mtiles <= ctas ? 2 : 1;
    const int sh = a.shared_last && total > 0 && shg * mtiles <= ctas ? shg * mtiles : 0;
    const int routed = total - sh;
    int sh_lo = 0, sh_hi = 0, r_lo = 0, r_hi = 0;
    if ((int)blockIdx.x < ctas) {
        const long long b = blockIdx.x;
        sh_lo = (int)((b * sh + ctas - 1) / ctas);
        sh_hi = (int)(((b + 1) * sh + ctas - 1) / ctas);
        r_lo = (int)((b * total) / ctas) - sh_lo;
        r_hi = (int)(((b + 1) * total) / ctas) - sh_hi;
    }
    const int nsh = sh_hi - sh_lo;
    const int count = nsh + (r_hi - r_lo);
    auto item_at = [&](int j) { return j < nsh ? routed + sh_lo + j : r_lo + (j - nsh); };

    if (warp == 0) {
        // ------------------------------------------------------ producer
        uint32_t it = 0, nb = 0;
        int prev_ai = -1;
        bool ok = true;
        // A weight stage (one item's tile and scale atoms) depends on no
        // earlier kernel of the call: the first S are requested before the
        // wait for the activations, so they stream while that completes.
        const int pre = count < S ? count : S;
        auto load_weights = [&](const Item &w, int st) {
            uint8_t *stage = smem + (size_t)st * Cfg::kStage;
            const int arow = w.e * a.H + w.mt * kTile;
            mbar_arrive_expect_tx(sfa_in + st, kw * 512);
            bulk_g2s(stage + KB * kTileBytes, a.sfa[0] + (size_t)(arow / kTile) * kw * 512, kw * 512, sfa_in + st);
            mbar_arrive_expect_tx(full + st, KB * kTileBytes);
#pragma unroll
            for (int box = 0; box < KB; ++box) tma_load_2d(stage + box * kTileBytes, &tm_a, full + st, box * 128, arow);
        };
        // Lane j requests item j's stage (the items' table reads in flight
        // together).
        if (lane < pre) load_weights(load_item(s, item_at(lane), mtiles), lane);
        it = (uint32_t)pre;
        pdl_wait();
        pdl_launch_dependents();
        if (lane == 0) {
            Item ti{};
            for (int j = 0; j < count && ok; ++j) {
                const int item = item_at(j);
                // Consecutive items mostly share their group: its metadata is
                // loaded once per group.
                if (item / mtiles != prev_ai) {
                    ti = load_item(s, item, mtiles);
                } else {
                    ti.mt = item - ti.ai * mtiles;
                }
                if (ti.ai != prev_ai) {
                    const uint32_t bb = nb & 1u, use = nb >> 1;
                    if (use > 0 && !mbar_wait(bempty + bb, (use - 1) & 1u, err, kSiteGemmEmpty)) {
                        ok = false;
                        break;
                    }
                    uint8_t *b = bbuf + (size_t)bb * Cfg::kStage;
                    mbar_arrive_expect_tx(bfull + bb, Cfg::kStage);
#pragma unroll
                    for (int box = 0; box < KB; ++box)
                        tma_load_2d(b + box * kTileBytes, &tm_b, bfull + bb, box * 128, kDecodeTcTerms * ti.tstart);
                    bulk_g2s(b + KB * kTileBytes, a.sfb + (size_t)ti.ai * kw * 512, kw * 512, bfull + bb);
                    ++nb;
                    prev_ai = ti.ai;
                }
                if (j < pre) continue;  // its weights were requested before the wait
                const int st = it % S;
                const uint32_t ph = (it / S) & 1u;
                if (!mbar_wait(empty + st, ph ^ 1u, err, kSiteGemmEmpty)) {
                    ok = false;
                    break;
                }
                load_weights(ti, st);
                ++it;
            }
            if (!ok || *reinterpret_cast<volatile int *>(err) != 0) {
                // Drain the copies still in flight before the CTA exits.
                const uint32_t first = it > (uint32_t)S ? it - S : 0u;
                for (uint32_t k = first; k < it; ++k) {
                    mbar_wait_drain(full + (k % S), (k / S) & 1u);
                    mbar_wait_drain(sfa_in + (k % S), (k / S) & 1u);
                }
                const uint32_t bfirst = nb > 2u ? nb - 2 : 0u;
                for (uint32_t k = bfirst; k < nb; ++k) mbar_wait_drain(bfull + (k & 1u), (k >> 1) & 1u);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA
        pdl_wait();
        pdl_launch_dependents();
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_mxf4nvf4(kTile);
            const uint32_t smem_base = smem_u32(smem);
            const uint32_t bbuf_base = smem_u32(bbuf);
            uint32_t it = 0, tcount = 0, nb = 0;
            int prev_ai = -1;
            bool ok = true;
            for (int j = 0; j < count && ok; ++j, ++tcount) {
                const int item = item_at(j);
                const int ai = item / mtiles;  // items are ordered group-major
                if (ai != prev_ai) {
                    if (nb > 0) tc::commit(bempty + ((nb - 1) & 1u));
                    const uint32_t bb = nb & 1u;
                    if (!mbar_wait(bfull + bb, (nb >> 1) & 1u, err, kSiteGemmFull) ||
                        !mbar_wait(sfb_ready + bb, (nb >> 1) & 1u, err, kSiteGemmFull)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    ++nb;
                    prev_ai = ai;
                }
                const uint32_t bb = (nb - 1) & 1u;
                const uint32_t buf = tcount & 1u, use = tcount >> 1;
                if (use > 0 && !mbar_wait(acc_empty + buf, (use - 1) & 1u, err, kSiteGemmAccEmpty)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const int st = it % S;
                if (!mbar_wait(full + st, (it / S) & 1u, err, kSiteGemmFull) ||
                    !mbar_wait(sfa_full + st, (it / S) & 1u, err, kSiteGemmFull)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                tc::fence_proxy_async_smem();
                const uint32_t sb = smem_base + (uint32_t)st * Cfg::kStage;
                const uint32_t tsfa = tmem + Cfg::kColSfa + (uint32_t)st * kw * 4;
                const uint32_t tsfb = tmem + Cfg::kColSfb + bb * kw * 4;
                const uint32_t bsm = bbuf_base + bb * Cfg::kStage;
#pragma unroll
                for (int k = 0; k < kw; ++k) {
                    const uint32_t off = (k >> 2) * kTileBytes + 32 * (k & 3);
                    tc::mma_mxf4nvf4(tmem + buf * 128, tc::smem_desc_sw128(sb + off), tc::smem_desc_sw128(bsm + off),
                                     idesc, tsfa + 4 * k, tsfb + 4 * k, k != 0 ? 1u : 0u);
                }
                tc::commit(empty + st);
                tc::commit(acc_full + buf);
                ++it;
            }
            tc::commit(drain);
            mbar_wait_drain(drain, 0);
        }
        __syncwarp();
    } else if (warp >= kSfWarp0) {
        // ------------------------------------------------- scale factors
        // At a group change the group's kw B atoms (after its B tile) into
        // columns kColSfb + bb * kw * 4 + 4a, then per item its kw weight
        // atoms (512 bytes apart after its tile) into columns tsfa + 4a, of
        // this warp's lane quarter. A B buffer's columns are free once the
        // buffer has been refilled, a stage's once the stage has (see gate /
        // up).
        pdl_wait();
        pdl_launch_dependents();
        const uint32_t quarter = (uint32_t)(32 * (warp & 3)) << 16;
        uint32_t it = 0, nb = 0;
        int prev_ai = -1;
        for (int j = 0; j < count; ++j, ++it) {
            const int ai = item_at(j) / mtiles;
            if (ai != prev_ai) {
                const uint32_t bb = nb & 1u;
                if (!__all_sync(0xffffffffu, mbar_wait(bfull + bb, (nb >> 1) & 1u, err, kSiteGemmFull))) break;
                tc::st_sf_atoms<kw>(tmem + quarter + Cfg::kColSfb + bb * kw * 4,
                                    bbuf + (size_t)bb * Cfg::kStage + KB * kTileBytes, 512, lane);
                tc::wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(sfb_ready + bb);
                ++nb;
                prev_ai = ai;
            }
            const int st = it % S;
            if (!__all_sync(0xffffffffu, mbar_wait(sfa_in + st, (it / S) & 1u, err, kSiteGemmFull))) break;
            tc::st_sf_atoms<kw>(tmem + quarter + Cfg::kColSfa + (uint32_t)st * kw * 4,
                                smem + (size_t)st * Cfg::kStage + KB * kTileBytes, 512, lane);
            tc::wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(sfa_full + st);
        }
    } else {
        // ----------------------------------------------------- epilogue
        pdl_wait();
        pdl_launch_dependents();
        const int sub = warp & 3;
        const int et = threadIdx.x - 64;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * sub) << 16);
        uint32_t tcount = 0, gcount = 0;
        Item ti{};
        ti.ai = -1;
        for (int j = 0; j < count; ++j, ++tcount) {
            const int item = item_at(j);
            // Group metadata and the per-row scales change only with the group
            // (double-buffered by group count: a warp still computing the
            // previous item reads the other buffer).
            if (item / mtiles != ti.ai) {
                ti = load_item(s, item, mtiles);
                ++gcount;
                if (et < ti.ntok) {
                    const int p = ti.tstart + et;
                    const int t = s.tok_list[p];
                    col_scale[32 * (gcount & 1) + et] = s.ga_tc[p] * s.coef_tab[ti.ai * kDecodeMaxTokens + t];
                }
            } else {
                ti.mt = item - ti.ai * mtiles;
            }
            const float *cscale = col_scale + 32 * (gcount & 1);
            const uint32_t buf = tcount & 1u;
            if (et == 0) *acc_ok = mbar_wait(acc_full + buf, (tcount >> 1) & 1u, err, kSiteGemmAccFull) ? 1 : 0;
            named_barrier(1, 128);
            if (!*reinterpret_cast<volatile int *>(acc_ok)) break;
            tc::fence_after_sync();
            const int m = ti.mt * kTile + 32 * sub + lane;
            // Column 4i + j is term j of the group's i-th slot row.
            for (int c0 = 0; c0 < 4 * ti.ntok; c0 += 32) {
                uint32_t r[32];
                tc::ld_32x32b_x32(lane_base + buf * 128 + c0, r);
                tc::wait_ld();
                if (c0 + 32 >= 4 * ti.ntok) {
                    tc::fence_before_sync();
                    named_barrier(1, 128);
                    if (et == 0) mbar_arrive(acc_empty + buf);
                }
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int i = c0 / 4 + q;
                    if (i < ti.ntok) {
                        const float y = ((__uint_as_float(r[4 * q]) + __uint_as_float(r[4 * q + 1])) +
                                         __uint_as_float(r[4 * q + 2])) + __uint_as_float(r[4 * q + 3]);
                        s.ypart[(size_t)(ti.tstart + i) * a.H + m] = y * cscale[i];
                    }
                }
            }
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
    }
    if (threadIdx.x == 0 && *reinterpret_cast<volatile int *>(err) != 0) report(s);
}

// Activation rows -> four NVFP4 terms per dispatch position p, one warp per
// row and one 16-element block per lane: codes to row 4p + j, scale bytes to
// the atoms of p's active group at B row 4(p - tok_start) + j, the row's
// global scale to ga_tc[p]. Positions of groups computed elsewhere (-1) are
// skipped.
__global__ void __launch_bounds__(256) quantize_act_tc_kernel(DecodeScratch s, int rows, int I) {
    pdl_wait();  // the gate/up activations are read from here on
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int p = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (p >= rows) return;
    const int nb = I / 16;
    const __half *row = s.act + (size_t)p * I;
    auto load_block = [&](int b, float (&v)[16]) {
        const uint4 *q = reinterpret_cast<const uint4 *>(row + 16 * b);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint4 u = q[k];
            const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w4[h]));
                v[8 * k + 2 * h] = f.x;
                v[8 * k + 2 * h + 1] = f.y;
            }
        }
    };
    // Up to 512 columns (a block per lane) the row stays in registers from
    // the amax pass to the term pass, and its load is issued together with
    // the group lookup.
    float v0[16];
    const bool one = nb <= 32;
    if (one) {
        if (lane < nb) {
            load_block(lane, v0);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v0[i] = 0.0f;
        }
    }
    const int ai = s.slot_group[p];
    if (ai < 0) return;
    const int n0 = kDecodeTcTerms * (p - s.tok_start[ai]);
    if (n0 < 0 || n0 + kDecodeTcTerms > kTile) return;
    float amax = 0.0f;
    if (one) {
#pragma unroll
        for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v0[i]));
    } else {
        for (int b = lane; b < nb; b += 32) {
            float v[16];
            load_block(b, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float g = row_global_scale(amax);
    if (lane == 0) s.ga_tc[p] = g;
    uint8_t *atoms = s.asf_tc + (size_t)ai * (I / 64) * 512;
    auto write_terms = [&](int b, float (&v)[16]) {
        // Terms in a loop that is not unrolled: this kernel runs once per
        // layer call with cold instruction caches, where code size is time.
#pragma unroll 1
        for (int j = 0; j < kDecodeTcTerms; ++j) {
            uint32_t c0, c1;
            const uint32_t sc = quantize_block_term(v, g, c0, c1);
            *reinterpret_cast<uint2 *>(s.aq_tc + ((size_t)kDecodeTcTerms * p + j) * (I / 2) + 8 * b) =
                make_uint2(c0, c1);
            atoms[sf_atom_byte(n0 + j, b)] = static_cast<uint8_t>(sc);
        }
    };
    if (one) {
        if (lane < nb) write_terms(lane, v0);
    } else {
        for (int b = lane; b < nb; b += 32) {
            float v[16];
            load_block(b, v);
            write_terms(b, v);
        }
    }
}

template <typename K>
cudaError_t set_smem_once(K kernel, size_t bytes, std::atomic<uint64_t> &done) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
    if (bit && (done.load() & bit)) return cudaSuccess;
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (err == cudaSuccess) done.fetch_or(bit);
    return err;
}

template <typename Kern, typename... Args>
cudaError_t launch_tc(Kern kernel, size_t smem, std::atomic<uint64_t> &done, int grid, cudaStream_t stream,
                      Args... args) {
    cudaError_t err = set_smem_once(kernel, smem, done);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

int tc_grid(int T, int E, int mtiles, int sms) {
    // Upper bound on the active groups: routed experts plus the shared one,
    // per token half above kDecodeTcMaxTokens tokens.
    auto groups = [&](int t) { return (E < t * kTopK ? E : t * kTopK) + 1; };
    const int groups_ub = T > kDecodeTcMaxTokens ? groups(kDecodeTcMaxTokens) + groups(T - kDecodeTcMaxTokens)
                                                 : groups(T);
    const int items_ub = groups_ub * mtiles;
    const int grid = items_ub < sms ? items_ub : sms;
    // The gate/up kernel gives each token half at least one CTA.
    return T > kDecodeTcMaxTokens && grid < 2 ? 2 : grid;
}

}  // namespace

bool decode_tc_supported(int H, int I) {
    return H % 256 == 0 && I % 256 == 0 && H <= 32 * 64 && (I == 256 || I == 512);
}

cudaError_t make_decode_tc_maps(DecodeTcMaps &m, const DecodeScratch &s, int H, int I) {
    if (H % 256 != 0 || I % 256 != 0) return cudaErrorInvalidValue;
    cudaError_t err = make_tensor_map_u8(&m.xq, s.xq_tc, H / 2, H / 2, (uint64_t)kDecodeTcTerms * kDecodeMaxTokens,
                                         128, kTile, CU_TENSOR_MAP_SWIZZLE_128B);
    if (err != cudaSuccess) return err;
    return make_tensor_map_u8(&m.aq, s.aq_tc, I / 2, I / 2,
                              (uint64_t)kDecodeTcTerms * kDecodeMaxTokens * kSlots, 128, kTile,
                              CU_TENSOR_MAP_SWIZZLE_128B);
}

cudaError_t launch_quantize_act_tc(const DecodeScratch &s, int T, int I, cudaStream_t stream) {
    if (T < 1 || T > kDecodeMaxTokens || I % 256 != 0) return cudaErrorInvalidValue;
    const int rows = T * kSlots;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((rows + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, quantize_act_tc_kernel, s, rows, I);
}

cudaError_t launch_gate_up_tc(const CUtensorMap &w_gate, const CUtensorMap &w_up, const DecodeTcMaps &m,
                              const DecodeTcArgs &a, int T, int sms, cudaStream_t stream) {
    if (T < 1 || T > kDecodeMaxTokens || T != a.T || !decode_tc_supported(a.H, a.I)) return cudaErrorInvalidValue;
    static std::atomic<uint64_t> done{0};
    return launch_tc(moe_gate_up_tc_kernel, kGuSmem, done, tc_grid(T, a.E, a.I / kTile, sms), stream, w_gate, w_up,
                     m.xq, a);
}

cudaError_t launch_down_tc(const CUtensorMap &w_down, const DecodeTcMaps &m, const DecodeTcArgs &a, int T, int sms,
                           cudaStream_t stream) {
    if (T < 1 || T > kDecodeMaxTokens || T != a.T || !decode_tc_supported(a.H, a.I)) return cudaErrorInvalidValue;
    const int grid = tc_grid(T, a.E, a.H / kTile, sms);
    if (a.I == 256) {
        static std::atomic<uint64_t> done{0};
        return launch_tc(moe_down_tc_kernel<1>, DnCfg<1>::kSmem, done, grid, stream, w_down, m.aq, a);
    }
    static std::atomic<uint64_t> done{0};
    return launch_tc(moe_down_tc_kernel<2>, DnCfg<2>::kSmem, done, grid, stream, w_down, m.aq, a);
}

}  // namespace nvfp4
