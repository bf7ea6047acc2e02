// Grouped expert GEMMs of the prefill path on tcgen05 block-scaled NVFP4 MMA.
//
// One persistent CTA per SM walks (column tile, weight-row tile) pairs. A
// column tile is up to 128 consecutive slot rows of one expert group (the
// dispatch order keeps an expert's rows together); a weight-row tile is 128
// rows of that expert's projection(s). Warp roles:
//   warp 0     producer: per 256-column K stage, TMA tile loads of the weight
//              rows and of the J activation-term tiles (128 padded slot rows
//              each; 128-byte swizzle) and bulk copies of the weight and
//              activation scale-factor atoms (stored in tcgen05 atom layout);
//              all complete on the stage's mbarrier.
//   warp 1     MMA issuer: one thread issues kind::mxf4nvf4 MMAs (M 128
//              slot rows of an activation term as A, N 128 weight rows as B
//              -- 256 for gate/up, whose gate and up rows form one operand --
//              K 64) into FP32 accumulators in tensor memory once the
//              stage's tiles have landed and its scale factors are in tensor
//              memory, then commits the stage back to the producer and,
//              after the last stage, the accumulator to the epilogue. Warp 1
//              also owns the tensor-memory allocation.
//   warps 6-9  scale factors: each stage's weight and activation scale atoms
//              go from shared memory into that stage's tensor-memory columns
//              by tcgen05.st, one 32-lane quarter per warp (the layout
//              tcgen05.cp 32x128b.warpx4 would give), so the MMA thread
//              issues no copies (a tcgen05.cp per atom costs the issuing
//              thread about as much as an MMA).
//   warps 2-5  epilogue: tcgen05.ld of the accumulator rows of their
//              sub-partition (one slot row per thread; the down GEMM
//              double-buffers its accumulator so this overlaps the next
//              tile's MMAs), the slot row's scale, then
//              gate/up: act = SiLU(gate) * up as FP16 [slot row][I];
//              down:    y = coef * acc as FP16 [slot row][H],
//              in 16-byte stores of consecutive outputs.
// Every mbarrier wait is bounded; on a timeout the CTA records the error,
// drains its copies and MMAs in flight, frees its tensor memory and exits.
#include "moe_prefill.cuh"
#include "tcgen05_util.cuh"
#include "tma_util.cuh"

#include <atomic>

namespace nvfp4 {

namespace {

constexpr int kGemmThreads = 320;
constexpr int kSfWarp0 = 6;  // first scale-factor warp
constexpr int kTileBytes = kPrefillTileM * 128;  // 128 rows x 128 bytes (256 FP4 columns)
constexpr int kSfStage = 4 * 512;                // four 64-column scale atoms
constexpr int kStageK = 256;

template <int NA, int J, int S>
struct GemmCfg {
    static constexpr int kA = NA * kTileBytes;
    static constexpr int kB = J * kTileBytes;
    static constexpr int kSfa = NA * kSfStage;
    static constexpr int kSfb = J * kSfStage;
    static constexpr int kStage = kA + kB + kSfa + kSfb;
    static constexpr uint32_t kTxTiles = kA + kB;   // the stage's code tiles (TMA), on `full`
    static constexpr uint32_t kTxSf = kSfa + kSfb;    // its scale atoms (bulk copies), on `sfa_in`
    // Down (one projection) double-buffers its accumulator so the epilogue
    // of one tile overlaps the MMAs of the next; gate/up holds two
    // accumulators (gate, up) in one buffer.
    static constexpr int kNumAcc = NA == 1 ? 2 : 1;
    static constexpr int kColAcc1 = 128;
    // Scale factors get one tensor-memory region per pipeline stage: PTX
    // orders tcgen05.cp before later MMAs but not MMAs before a later
    // tcgen05.cp, so a region is rewritten only after the MMAs that read it
    // have committed (the producer refills a stage after that commit).
    static constexpr int kSfCols = NA * 16 + J * 16;        // per stage: SFA then SFB
    // Stage blocks start on 32-column boundaries (the store warps write up
    // to 32 columns per tcgen05.st).
    static constexpr int kSfStride = (kSfCols + 31) & ~31;
    static constexpr int kColSf = 256;
    static constexpr int kColsUsed = kColSf + S * kSfStride;
    static constexpr uint32_t kTmemCols = kColsUsed <= 256 ? 256u : 512u;
    // Alignment slack, the stages, then barriers, the tensor-memory slot and
    // the accumulator-ready flag.
    static constexpr size_t kSmem = 1024 + (size_t)S * kStage + 2048;
    static_assert(kStage % 1024 == 0, "stage must keep 1024-byte tile alignment");
    static_assert(kColsUsed <= 512, "tensor memory overflow");
};

__device__ __forceinline__ uint8_t *align1024(uint8_t *p) {
    return reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Two FP32 values rounded to FP16 (round to nearest even, finite values
// saturated to +-65504): `lo` in the low half (the lower address).
__device__ __forceinline__ uint32_t pack_f16x2_sat(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

// Bounded wait that ignores the shared error word (used to drain copies in
// flight after a failure). Returns false if the phase never completed.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t *bar, uint32_t parity) {
    const unsigned long long t0 = global_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u && global_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ void report(const PrefillScratch &s) {
    const int code = *reinterpret_cast<volatile int *>(s.error);
    if (s.host_error) *reinterpret_cast<volatile int *>(s.host_error) = code != 0 ? code : kErrWaitTimeout;
}

struct TileInfo {
    int ai, e, n0, nvalid, mt;
};

__device__ __forceinline__ TileInfo tile_info(const PrefillScratch &s, int tile, int mtiles) {
    TileInfo t;
    const int ct = tile / mtiles;
    t.mt = tile - ct * mtiles;
    t.ai = s.tile_group[ct];
    t.n0 = s.tile_n0[ct];
    t.e = s.active_expert[t.ai];
    t.nvalid = min(kPrefillTileN, s.tok_start[t.ai] + s.tok_count[t.ai] - t.n0);
    return t;
}

// A warp walks this CTA's tiles with the descriptions of the next 32 held
// one per lane: lane l loads tile `first + l * stride` (all lanes' dependent
// table loads in flight at once) and `lane_tile` hands tile k to every lane.
__device__ __forceinline__ TileInfo batch_tiles(const PrefillScratch &s, int first, int stride, int total,
                                                int mtiles, int lane) {
    TileInfo t{};
    const int tile = first + lane * stride;
    if (tile < total) t = tile_info(s, tile, mtiles);
    return t;
}

__device__ __forceinline__ TileInfo lane_tile(const TileInfo &mine, int k) {
    TileInfo t;
    t.ai = __shfl_sync(0xffffffffu, mine.ai, k);
    t.e = __shfl_sync(0xffffffffu, mine.e, k);
    t.n0 = __shfl_sync(0xffffffffu, mine.n0, k);
    t.nvalid = __shfl_sync(0xffffffffu, mine.nvalid, k);
    t.mt = __shfl_sync(0xffffffffu, mine.mt, k);
    return t;
}

template <int MODE, int J, int S>
__global__ void __launch_bounds__(kGemmThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tm_a0, const __grid_constant__ CUtensorMap tm_a1,
                    const __grid_constant__ CUtensorMap tm_b, GemmArgs a) {
    constexpr int NA = MODE == 0 ? 2 : 1;
    using Cfg = GemmCfg<NA, J, S>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align1024(smem_raw);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * Cfg::kStage);
    uint64_t *empty = full + S;
    uint64_t *acc_full = empty + S;      // [kNumAcc]
    uint64_t *acc_empty = acc_full + 2;  // [kNumAcc]
    uint64_t *drain = acc_empty + 2;
    uint64_t *sf_in = drain + 1;     // [S] the stage's scale atoms are in shared memory
    uint64_t *sf_full = sf_in + S;   // [S] the stage's scale factors are in tensor memory (4 store warps)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sf_full + S);
    int *acc_ok = reinterpret_cast<int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const PrefillScratch &s = a.s;
    int *err = s.error;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(full + i, 1);  // producer lane 0 (arrive + transaction bytes)
            mbar_init(empty + i, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full + b, 1);
            mbar_init(acc_empty + b, 1);
        }
        mbar_init(drain, 1);
        for (int i = 0; i < S; ++i) {
            mbar_init(sf_in + i, 1);
            mbar_init(sf_full + i, 4);
        }
        fence_barrier_init();
        prefetch_tensormap(&tm_a0);
        if (NA == 2) prefetch_tensormap(&tm_a1);
        prefetch_tensormap(&tm_b);
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // routing tables and activation terms are read from here on
    pdl_launch_dependents();

    const int mtiles = a.M / kPrefillTileM;
    const int total = *s.n_tiles * mtiles;
    const int kstages = a.K / kStageK;
    const int kw = a.K / 64;

    if (warp == 0) {
        // ------------------------------------------------------ producer
        uint32_t it = 0;
        bool ok = true;
        TileInfo mine{};
        for (int tile = blockIdx.x, k = 0; tile < total && ok; tile += gridDim.x, k = (k + 1) & 31) {
            if (k == 0) mine = batch_tiles(s, tile, gridDim.x, total, mtiles, lane);
            const TileInfo ti = lane_tile(mine, k);
            const int arow = ti.e * a.M + ti.mt * kPrefillTileM;
            const size_t sfa_off = (size_t)(arow / kPrefillTileM) * kw * 512;
            const int sf_blocks = s.max_rows / kPrefillTileN;
            for (int ks = 0; ks < kstages; ++ks, ++it) {
                const int st = it % S;
                const uint32_t ph = (it / S) & 1u;
                int okw = 1;
                if (lane == 0) okw = mbar_wait(empty + st, ph ^ 1u, err, kSiteGemmEmpty) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, okw, 0)) {
                    ok = false;
                    break;
                }
                uint8_t *stage = smem + (size_t)st * Cfg::kStage;
                uint8_t *sfb = stage + Cfg::kA + Cfg::kB + Cfg::kSfa;
                if (lane == 0) {
                    // The scale atoms first and on their own barrier: the
                    // store warps need only them, and they land first.
                    mbar_arrive_expect_tx(sf_in + st, Cfg::kTxSf);
                    bulk_g2s(stage + Cfg::kA + Cfg::kB, a.sfa[0] + sfa_off + (size_t)ks * kSfStage, kSfStage,
                             sf_in + st);
                    if (NA == 2)
                        bulk_g2s(stage + Cfg::kA + Cfg::kB + kSfStage, a.sfa[1] + sfa_off + (size_t)ks * kSfStage,
                                 kSfStage, sf_in + st);
#pragma unroll
                    for (int j = 0; j < J; ++j)
                        bulk_g2s(sfb + j * kSfStage,
                                 a.sfb + ((size_t)(j * sf_blocks + ti.n0 / kPrefillTileN) * kw + ks * 4) * 512,
                                 kSfStage, sf_in + st);
                    mbar_arrive_expect_tx(full + st, Cfg::kTxTiles);
                    tma_load_2d(stage, &tm_a0, full + st, ks * 128, arow);
                    if (NA == 2) tma_load_2d(stage + kTileBytes, &tm_a1, full + st, ks * 128, arow);
                    // The column tile is one 128-row block of slot rows: one
                    // TMA box of codes per activation term.
#pragma unroll
                    for (int j = 0; j < J; ++j)
                        tma_load_2d(stage + Cfg::kA + j * kTileBytes, &tm_b, full + st, ks * 128, j * a.Rb + ti.n0);
                }
            }
        }
        if (!ok || *reinterpret_cast<volatile int *>(err) != 0) {
            // Drain: wait for the copies of the last stages issued.
            if (lane == 0) {
                const uint32_t first = it > (uint32_t)S ? it - S : 0u;
                for (uint32_t k = first; k < it; ++k) {
                    mbar_wait_drain(full + (k % S), (k / S) & 1u);
                    mbar_wait_drain(sf_in + (k % S), (k / S) & 1u);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_mxf4nvf4(NA * kPrefillTileM);
            const uint32_t smem_base = smem_u32(smem);
            uint32_t it = 0, tcount = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++tcount) {
                const uint32_t buf = tcount % Cfg::kNumAcc;
                const uint32_t use = tcount / Cfg::kNumAcc;  // uses of this buffer before this tile
                if (use > 0 && !mbar_wait(acc_empty + buf, (use - 1) & 1u, err, kSiteGemmAccEmpty)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t dacc = tmem + buf * 128;
                for (int ks = 0; ks < kstages; ++ks, ++it) {
                    const int st = it % S;
                    const uint32_t ph = (it / S) & 1u;
                    if (!mbar_wait(full + st, ph, err, kSiteGemmFull) ||
                        !mbar_wait(sf_full + st, ph, err, kSiteGemmFull)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    tc::fence_proxy_async_smem();
                    const uint32_t sb = smem_base + (uint32_t)st * Cfg::kStage;
                    const uint32_t tsfa = tmem + Cfg::kColSf + (uint32_t)st * Cfg::kSfStride;
                    const uint32_t tsfb = tsfa + NA * 16;
                    // The activation term is the A operand (accumulator lane =
                    // slot row) and the weight rows are B (column = weight
                    // row). Gate/up issues one N = 256 MMA per step: the
                    // gate tile and the up tile are consecutive in the stage,
                    // so together they are one 256-row K-major operand, whose
                    // accumulator columns 0-127 are gate and 128-255 up, and
                    // whose scale factors the store warps interleave
                    // accordingly (8 columns per 64-wide K step).
#pragma unroll
                    for (int at = 0; at < 4; ++at) {
#pragma unroll
                        for (int j = 0; j < J; ++j) {
                            const uint32_t acc = (ks | at | j) != 0 ? 1u : 0u;
                            const uint64_t xdesc = tc::smem_desc_sw128(sb + Cfg::kA + j * kTileBytes + 32 * at);
                            tc::mma_mxf4nvf4(dacc, xdesc, tc::smem_desc_sw128(sb + 32 * at), idesc,
                                             tsfb + 16 * j + 4 * at, tsfa + 4 * NA * at, acc);
                        }
                    }
                    tc::commit(empty + st);
                }
                if (!ok) break;
                tc::commit(acc_full + buf);
            }
            // Every MMA of this CTA has completed before tensor memory is freed.
            tc::commit(drain);
            mbar_wait_drain(drain, 0);
        }
        __syncwarp();
    } else if (warp >= kSfWarp0) {
        // ------------------------------------------------- scale factors
        // Stage st's atoms are contiguous in shared memory (the weights' NA x
        // 4, then the activation terms' J x 4, 512 bytes apart) and go to the
        // stage's contiguous columns tsfa.. (4 per atom) of this warp's lane
        // quarter. The columns are free: the producer refills a stage (and
        // so its sf_in) only after the MMAs that read its previous atoms
        // have committed.
        constexpr int kAtoms = (NA + J) * 4;
        const uint32_t quarter = (uint32_t)(32 * (warp & 3)) << 16;
        uint32_t it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
            for (int ks = 0; ks < kstages; ++ks, ++it) {
                const int st = it % S;
                if (!__all_sync(0xffffffffu, mbar_wait(sf_in + st, (it / S) & 1u, err, kSiteGemmFull))) {
                    ok = false;
                    break;
                }
                const uint32_t cols = tmem + quarter + Cfg::kColSf + (uint32_t)st * Cfg::kSfStride;
                const uint8_t *atoms = smem + (size_t)st * Cfg::kStage + Cfg::kA + Cfg::kB;
                // Gate/up: the first eight atoms are the gate and up weights'
                // (four each), interleaved per K step for the N = 256 MMA.
                if constexpr (NA == 2) tc::st_sf_atoms<8, true>(cols, atoms, 512, lane);
#pragma unroll
                for (int a8 = NA == 2 ? 8 : 0; a8 + 8 <= kAtoms; a8 += 8)
                    tc::st_sf_atoms<8>(cols + 4 * a8, atoms + a8 * 512, 512, lane);
                if constexpr (kAtoms % 8 == 4) tc::st_sf_atoms<4>(cols + 4 * (kAtoms - 4), atoms + (kAtoms - 4) * 512,
                                                                  512, lane);
                tc::wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(sf_full + st);
            }
        }
    } else {
        // ----------------------------------------------------- epilogue
        // Accumulator lane = slot row of the column tile, column = weight
        // row: each thread owns one slot row and writes its outputs as runs
        // of 32 consecutive FP16 values (four 16-byte stores), so a tile's
        // results leave in 16-byte pieces with no per-element branches.
        const int sub = warp & 3;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * sub) << 16);
        const bool leader = threadIdx.x == 64;
        uint32_t tcount = 0;
        TileInfo mine{};
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++tcount) {
            if ((tcount & 31u) == 0) mine = batch_tiles(s, tile, gridDim.x, total, mtiles, lane);
            const TileInfo ti = lane_tile(mine, tcount & 31u);
            const int r = 32 * sub + lane;  // slot row within the column tile
            const bool valid = r < ti.nvalid;
            const int p = ti.n0 + r;
            // The row's scale is fetched before the accumulator wait.
            float cs = 0.0f;
            if (valid) cs = MODE == 0 ? s.gx[s.tok_list[p]] : s.coef[p] * s.ga[p];
            // One thread waits for the accumulator and the decision is
            // shared, so every epilogue warp leaves the loop together.
            const uint32_t buf = tcount % Cfg::kNumAcc;
            if (leader)
                *acc_ok = mbar_wait(acc_full + buf, (tcount / Cfg::kNumAcc) & 1u, err, kSiteGemmAccFull) ? 1 : 0;
            named_barrier(1, 128);
            if (!*reinterpret_cast<volatile int *>(acc_ok)) break;
            tc::fence_after_sync();
            const int m0 = ti.mt * kPrefillTileM;
            if (MODE == 0) {
                // SiLU(gate) * up is rounded to FP16 right away, so the fast
                // exponential and division (a few ulp of FP32) suffice; the
                // accumulator is handed back once its last columns are in
                // registers, so the next tile's MMAs overlap this arithmetic.
                const float gs = a.inv_scales[ti.e] * cs, us = a.inv_scales[(a.E + 1) + ti.e] * cs;
                uint4 *dst = reinterpret_cast<uint4 *>(s.act + (size_t)p * a.M + m0);
                // Two 64-column halves: the accumulator is released once the
                // second half is in registers.
#pragma unroll 1
                for (int c0 = 0; c0 < kPrefillTileM; c0 += 64) {
                    uint32_t rg[64], ru[64];
                    tc::ld_32x32b_x32(lane_base + c0, *reinterpret_cast<uint32_t(*)[32]>(rg));
                    tc::ld_32x32b_x32(lane_base + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(rg + 32));
                    tc::ld_32x32b_x32(lane_base + Cfg::kColAcc1 + c0, *reinterpret_cast<uint32_t(*)[32]>(ru));
                    tc::ld_32x32b_x32(lane_base + Cfg::kColAcc1 + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(ru + 32));
                    tc::wait_ld();
                    if (c0 + 64 == kPrefillTileM) {
                        tc::fence_before_sync();
                        named_barrier(1, 128);
                        if (leader) mbar_arrive(acc_empty + buf);
                    }
                    if (valid) {
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            uint32_t h[4];
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const int n = 8 * k + 2 * q;
                                const float g0 = __uint_as_float(rg[n]) * gs, g1 = __uint_as_float(rg[n + 1]) * gs;
                                const float u0 = __uint_as_float(ru[n]) * us, u1 = __uint_as_float(ru[n + 1]) * us;
                                h[q] = pack_f16x2_sat(__fdividef(g0, 1.0f + __expf(-g0)) * u0,
                                                      __fdividef(g1, 1.0f + __expf(-g1)) * u1);
                            }
                            dst[c0 / 8 + k] = make_uint4(h[0], h[1], h[2], h[3]);
                        }
                    }
                }
            } else {
                // All 128 columns come into registers first, so the
                // accumulator is released before any arithmetic.
                uint32_t acc[kPrefillTileM];
#pragma unroll
                for (int q = 0; q < kPrefillTileM / 32; ++q)
                    tc::ld_32x32b_x32(lane_base + buf * 128 + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(acc + 32 * q));
                tc::wait_ld();
                tc::fence_before_sync();
                named_barrier(1, 128);
                if (leader) mbar_arrive(acc_empty + buf);
                if (valid) {
                    uint4 *dst = reinterpret_cast<uint4 *>(s.ypart + (size_t)p * a.M + m0);
#pragma unroll
                    for (int k = 0; k < kPrefillTileM / 8; ++k)
                        dst[k] = make_uint4(
                            pack_f16x2_sat(__uint_as_float(acc[8 * k + 0]) * cs, __uint_as_float(acc[8 * k + 1]) * cs),
                            pack_f16x2_sat(__uint_as_float(acc[8 * k + 2]) * cs, __uint_as_float(acc[8 * k + 3]) * cs),
                            pack_f16x2_sat(__uint_as_float(acc[8 * k + 4]) * cs, __uint_as_float(acc[8 * k + 5]) * cs),
                            pack_f16x2_sat(__uint_as_float(acc[8 * k + 6]) * cs, __uint_as_float(acc[8 * k + 7]) * cs));
                }
            }
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, Cfg::kTmemCols);
    }
    if (threadIdx.x == 0 && *reinterpret_cast<volatile int *>(err) != 0) report(s);
}

// ------------------------------------------- down GEMM, activations resident
//
// The down GEMM's reduction is short (K = I = 512), so a column tile's whole
// activation operand -- J terms x 128 slot rows x K codes, with its scale
// factors -- fits in shared memory and tensor memory. Each CTA takes a
// contiguous range of (column tile, weight-row tile) pairs in column-tile-
// major order, loads each of its two or three column tiles once, and streams
// only the weight tiles (128 rows x K codes and their atoms) through an
// S-stage ring; moe_gemm_kernel<1> reloads the activation tiles for every
// weight-row tile. Roles as in moe_gemm_kernel; the MMAs of a tile run in
// its order (K step, then term), so the outputs are the same bits.
//   shared memory: A [J][KB] 16 KB boxes | A atoms [J][4 KB] | S x (W [KB]
//                  16 KB boxes | W atoms [KB*4][512 B]) | barriers
//   tensor memory: accumulators 2 x 128 columns | A scale factors J x 16 KB
//                  columns | W scale factors S x 16 KB columns
template <int J, int KB, int S>
struct DownResCfg {
    static constexpr int kAtomsA = 4 * KB;                   // per term (K / 64)
    static constexpr int kA = J * KB * kTileBytes;
    static constexpr int kASf = J * kAtomsA * 512;
    static constexpr int kW = KB * kTileBytes;
    static constexpr int kWSf = kAtomsA * 512;
    static constexpr int kStage = kW + kWSf;
    static constexpr int kColA = 256;
    static constexpr int kColW = kColA + J * KB * 16;
    static constexpr int kColsUsed = kColW + S * KB * 16;
    static constexpr size_t kBarOff = (size_t)kA + kASf + (size_t)S * kStage;
    static constexpr size_t kSmem = 1024 + kBarOff + 1024;
    static_assert(kA % 1024 == 0 && kASf % 1024 == 0 && kStage % 1024 == 0, "1024-byte tile alignment");
    static_assert(kColsUsed <= 512, "tensor memory overflow");
    static_assert(kSmem <= 232448, "shared memory overflow");
    static_assert(KB == 2, "the scale-factor stores write eight atoms (32 columns) at a time");
};

template <int J, int KB, int S>
__global__ void __launch_bounds__(kGemmThreads, 1)
    moe_down_resident_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_act,
                             GemmArgs a) {
    using Cfg = DownResCfg<J, KB, S>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align1024(smem_raw);
    uint8_t *a_tiles = smem;
    uint8_t *a_atoms = smem + Cfg::kA;
    uint8_t *w_stages = a_atoms + Cfg::kASf;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::kBarOff);
    uint64_t *w_full = bars;              // [S] weight tiles landed (producer arrive + bytes)
    uint64_t *w_empty = w_full + S;       // [S] MMAs of the stage committed
    uint64_t *w_sf_in = w_empty + S;      // [S] weight atoms landed
    uint64_t *w_sf_full = w_sf_in + S;    // [S] weight atoms in tensor memory (4 store warps)
    uint64_t *a_full = w_sf_full + S;     // activation tiles landed
    uint64_t *a_empty = a_full + 1;       // MMAs of the column tile committed
    uint64_t *a_sf_in = a_empty + 1;      // activation atoms landed
    uint64_t *a_sf_full = a_sf_in + 1;    // activation atoms in tensor memory
    uint64_t *acc_full = a_sf_full + 1;   // [2]
    uint64_t *acc_empty = acc_full + 2;   // [2]
    uint64_t *drain = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    int *acc_ok = reinterpret_cast<int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const PrefillScratch &s = a.s;
    int *err = s.error;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(w_full + i, 1);
            mbar_init(w_empty + i, 1);
            mbar_init(w_sf_in + i, 1);
            mbar_init(w_sf_full + i, 4);
        }
        mbar_init(a_full, 1);
        mbar_init(a_empty, 1);
        mbar_init(a_sf_in, 1);
        mbar_init(a_sf_full, 4);
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full + b, 1);
            mbar_init(acc_empty + b, 1);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        prefetch_tensormap(&tm_w);
        prefetch_tensormap(&tm_act);
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, 512);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // routing tables and activation terms are read from here on
    pdl_launch_dependents();

    const int mtiles = a.M / kPrefillTileM;
    const int total = *s.n_tiles * mtiles;
    // This CTA's contiguous range of tiles (column-tile major).
    const int lo = (int)(((long long)blockIdx.x * total) / gridDim.x);
    const int hi = (int)(((long long)(blockIdx.x + 1) * total) / gridDim.x);
    constexpr int kw = 4 * KB;  // 64-column K steps

    if (warp == 0) {
        // ------------------------------------------------------ producer
        uint32_t wit = 0, an = 0;
        int cur_ct = -1;
        bool ok = true;
        TileInfo mine{};
        const int sf_blocks = s.max_rows / kPrefillTileN;
        for (int tile = lo; tile < hi && ok; ++tile) {
            const int k = (tile - lo) & 31;
            if (k == 0) mine = batch_tiles(s, tile, 1, total, mtiles, lane);
            const TileInfo ti = lane_tile(mine, k);
            const int ct = tile / mtiles;
            // The tile's weight stage first: the ring runs ahead into a new
            // column tile while the previous one's MMAs finish.
            const int st = wit % S;
            const uint32_t ph = (wit / S) & 1u;
            int okw = 1;
            if (lane == 0) okw = mbar_wait(w_empty + st, ph ^ 1u, err, kSiteGemmEmpty) ? 1 : 0;
            if (!__shfl_sync(0xffffffffu, okw, 0)) {
                ok = false;
                break;
            }
            if (lane == 0) {
                uint8_t *stage = w_stages + (size_t)st * Cfg::kStage;
                const int wrow = ti.e * a.M + ti.mt * kPrefillTileM;
                mbar_arrive_expect_tx(w_sf_in + st, Cfg::kWSf);
                bulk_g2s(stage + Cfg::kW, a.sfa[0] + (size_t)(wrow / kPrefillTileM) * kw * 512, Cfg::kWSf,
                         w_sf_in + st);
                mbar_arrive_expect_tx(w_full + st, Cfg::kW);
#pragma unroll
                for (int kb = 0; kb < KB; ++kb)
                    tma_load_2d(stage + kb * kTileBytes, &tm_w, w_full + st, kb * 128, wrow);
            }
            ++wit;
            if (ct != cur_ct) {
                // The activation buffer (and its tensor-memory scale
                // factors) is refilled once the previous column tile's MMAs
                // have committed.
                if (lane == 0 && an > 0) okw = mbar_wait(a_empty, (an - 1) & 1u, err, kSiteGemmEmpty) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, okw, 0)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(a_sf_in, Cfg::kASf);
#pragma unroll
                    for (int j = 0; j < J; ++j)
                        bulk_g2s(a_atoms + j * (kw * 512),
                                 a.sfb + (size_t)(j * sf_blocks + ti.n0 / kPrefillTileN) * kw * 512, kw * 512, a_sf_in);
                    mbar_arrive_expect_tx(a_full, Cfg::kA);
#pragma unroll
                    for (int j = 0; j < J; ++j)
#pragma unroll
                        for (int kb = 0; kb < KB; ++kb)
                            tma_load_2d(a_tiles + (j * KB + kb) * kTileBytes, &tm_act, a_full, kb * 128,
                                        j * a.Rb + ti.n0);
                }
                cur_ct = ct;
                ++an;
            }
        }
        if (!ok || *reinterpret_cast<volatile int *>(err) != 0) {
            // Drain: wait for the copies of the last stages issued and of the
            // last activation load.
            if (lane == 0) {
                const uint32_t first = wit > (uint32_t)S ? wit - S : 0u;
                for (uint32_t q = first; q < wit; ++q) {
                    mbar_wait_drain(w_full + (q % S), (q / S) & 1u);
                    mbar_wait_drain(w_sf_in + (q % S), (q / S) & 1u);
                }
                if (an > 0) {
                    mbar_wait_drain(a_full, (an - 1) & 1u);
                    mbar_wait_drain(a_sf_in, (an - 1) & 1u);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_mxf4nvf4(kPrefillTileM);
            const uint32_t a_base = smem_u32(a_tiles);
            const uint32_t w_base = smem_u32(w_stages);
            uint32_t wit = 0, tcount = 0, an = 0;
            int cur_ct = -1;
            bool ok = true;
            for (int tile = lo; tile < hi && ok; ++tile, ++tcount) {
                const int ct = tile / mtiles;
                if (ct != cur_ct) {
                    if (cur_ct >= 0) tc::commit(a_empty);
                    if (!mbar_wait(a_full, an & 1u, err, kSiteGemmFull) ||
                        !mbar_wait(a_sf_full, an & 1u, err, kSiteGemmFull)) {
                        ok = false;
                        break;
                    }
                    cur_ct = ct;
                    ++an;
                }
                const uint32_t buf = tcount & 1u;
                const uint32_t use = tcount >> 1;
                if (use > 0 && !mbar_wait(acc_empty + buf, (use - 1) & 1u, err, kSiteGemmAccEmpty)) {
                    ok = false;
                    break;
                }
                const int st = wit % S;
                const uint32_t ph = (wit / S) & 1u;
                if (!mbar_wait(w_full + st, ph, err, kSiteGemmFull) ||
                    !mbar_wait(w_sf_full + st, ph, err, kSiteGemmFull)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                tc::fence_proxy_async_smem();
                const uint32_t dacc = tmem + buf * 128;
                const uint32_t wb = w_base + (uint32_t)st * Cfg::kStage;
                const uint32_t tsfw = tmem + Cfg::kColW + (uint32_t)st * (KB * 16);
#pragma unroll
                for (int kb = 0; kb < KB; ++kb) {
#pragma unroll
                    for (int at = 0; at < 4; ++at) {
#pragma unroll
                        for (int j = 0; j < J; ++j) {
                            const uint32_t acc = (kb | at | j) != 0 ? 1u : 0u;
                            const uint64_t adesc =
                                tc::smem_desc_sw128(a_base + (uint32_t)(j * KB + kb) * kTileBytes + 32 * at);
                            const uint64_t wdesc = tc::smem_desc_sw128(wb + (uint32_t)kb * kTileBytes + 32 * at);
                            tc::mma_mxf4nvf4(dacc, adesc, wdesc, idesc,
                                             tmem + Cfg::kColA + (uint32_t)(j * kw + 4 * kb + at) * 4,
                                             tsfw + (uint32_t)(4 * kb + at) * 4, acc);
                        }
                    }
                }
                tc::commit(w_empty + st);
                tc::commit(acc_full + buf);
                ++wit;
            }
            // Every MMA of this CTA has completed before tensor memory is freed.
            tc::commit(drain);
            mbar_wait_drain(drain, 0);
        }
        __syncwarp();
    } else if (warp >= kSfWarp0) {
        // ------------------------------------------------- scale factors
        const uint32_t quarter = (uint32_t)(32 * (warp & 3)) << 16;
        uint32_t wit = 0, an = 0;
        int cur_ct = -1;
        bool ok = true;
        for (int tile = lo; tile < hi && ok; ++tile) {
            const int ct = tile / mtiles;
            if (ct != cur_ct) {
                if (!__all_sync(0xffffffffu, mbar_wait(a_sf_in, an & 1u, err, kSiteGemmFull))) {
                    ok = false;
                    break;
                }
#pragma unroll
                for (int j = 0; j < J; ++j)
                    tc::st_sf_atoms<8>(tmem + quarter + Cfg::kColA + (uint32_t)j * (kw * 4), a_atoms + j * (kw * 512),
                                       512, lane);
                tc::wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(a_sf_full);
                cur_ct = ct;
                ++an;
            }
            const int st = wit % S;
            if (!__all_sync(0xffffffffu, mbar_wait(w_sf_in + st, (wit / S) & 1u, err, kSiteGemmFull))) {
                ok = false;
                break;
            }
            tc::st_sf_atoms<8>(tmem + quarter + Cfg::kColW + (uint32_t)st * (KB * 16),
                               w_stages + (size_t)st * Cfg::kStage + Cfg::kW, 512, lane);
            tc::wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(w_sf_full + st);
            ++wit;
        }
    } else {
        // ----------------------------------------------------- epilogue
        // As moe_gemm_kernel<1>: one slot row per thread, all 128 columns in
        // registers before the accumulator is released, FP16 partials.
        const int sub = warp & 3;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * sub) << 16);
        const bool leader = threadIdx.x == 64;
        uint32_t tcount = 0;
        TileInfo mine{};
        for (int tile = lo; tile < hi; ++tile, ++tcount) {
            const int k = (tile - lo) & 31;
            if (k == 0) mine = batch_tiles(s, tile, 1, total, mtiles, lane);
            const TileInfo ti = lane_tile(mine, k);
            const int r = 32 * sub + lane;
            const bool valid = r < ti.nvalid;
            const int p = ti.n0 + r;
            float cs = 0.0f;
            if (valid) cs = s.coef[p] * s.ga[p];
            const uint32_t buf = tcount & 1u;
            if (leader) *acc_ok = mbar_wait(acc_full + buf, (tcount >> 1) & 1u, err, kSiteGemmAccFull) ? 1 : 0;
            named_barrier(1, 128);
            if (!*reinterpret_cast<volatile int *>(acc_ok)) break;
            tc::fence_after_sync();
            uint32_t acc[kPrefillTileM];
#pragma unroll
            for (int q = 0; q < kPrefillTileM / 32; ++q)
                tc::ld_32x32b_x32(lane_base + buf * 128 + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(acc + 32 * q));
            tc::wait_ld();
            tc::fence_before_sync();
            named_barrier(1, 128);
            if (leader) mbar_arrive(acc_empty + buf);
            if (valid) {
                uint4 *dst = reinterpret_cast<uint4 *>(s.ypart + (size_t)p * a.M + ti.mt * kPrefillTileM);
#pragma unroll
                for (int q = 0; q < kPrefillTileM / 8; ++q)
                    dst[q] = make_uint4(
                        pack_f16x2_sat(__uint_as_float(acc[8 * q + 0]) * cs, __uint_as_float(acc[8 * q + 1]) * cs),
                        pack_f16x2_sat(__uint_as_float(acc[8 * q + 2]) * cs, __uint_as_float(acc[8 * q + 3]) * cs),
                        pack_f16x2_sat(__uint_as_float(acc[8 * q + 4]) * cs, __uint_as_float(acc[8 * q + 5]) * cs),
                        pack_f16x2_sat(__uint_as_float(acc[8 * q + 6]) * cs, __uint_as_float(acc[8 * q + 7]) * cs));
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

template <int MODE, int J, int S>
cudaError_t launch_cfg(const CUtensorMap &a0, const CUtensorMap &a1, const CUtensorMap &b, const GemmArgs &a,
                       int grid, cudaStream_t stream) {
    constexpr int NA = MODE == 0 ? 2 : 1;
    using Cfg = GemmCfg<NA, J, S>;
    static std::atomic<uint64_t> done{0};
    cudaError_t err = set_smem_once(moe_gemm_kernel<MODE, J, S>, Cfg::kSmem, done);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = Cfg::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, moe_gemm_kernel<MODE, J, S>, a0, a1, b, a);
}

template <int J, int KB, int S>
cudaError_t launch_down_res(const CUtensorMap &w, const CUtensorMap &act, const GemmArgs &a, int grid,
                            cudaStream_t stream) {
    using Cfg = DownResCfg<J, KB, S>;
    static std::atomic<uint64_t> done{0};
    cudaError_t err = set_smem_once(moe_down_resident_kernel<J, KB, S>, Cfg::kSmem, done);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = Cfg::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, moe_down_resident_kernel<J, KB, S>, w, act, a);
}

int gemm_grid(const GemmArgs &a, int sms) {
    const long long coltiles = (long long)a.s.max_tiles;
    const long long tiles = coltiles * (a.M / kPrefillTileM);
    return (int)(tiles < sms ? tiles : sms);
}

}  // namespace

cudaError_t launch_gemm_gate_up(const PrefillMaps &m, const GemmArgs &a, int sms, cudaStream_t stream) {
    if (a.K % kStageK != 0 || a.M % kPrefillTileM != 0) return cudaErrorInvalidValue;
    const int grid = gemm_grid(a, sms);
    switch (a.J) {
        case 1: return launch_cfg<0, 1, 4>(m.w[0], m.w[1], m.xq, a, grid, stream);
        case 2: return launch_cfg<0, 2, 3>(m.w[0], m.w[1], m.xq, a, grid, stream);
        case 3: return launch_cfg<0, 3, 2>(m.w[0], m.w[1], m.xq, a, grid, stream);
        case 4: return launch_cfg<0, 4, 2>(m.w[0], m.w[1], m.xq, a, grid, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemm_down(const PrefillMaps &m, const GemmArgs &a, int sms, cudaStream_t stream) {
    if (a.K % kStageK != 0 || a.M % kPrefillTileM != 0) return cudaErrorInvalidValue;
    const int grid = gemm_grid(a, sms);
    // K = 512 (the shape's intermediate size): the column tile's activation
    // terms stay resident for all of its weight-row tiles.
    if (a.K == 2 * kStageK) {
        switch (a.J) {
            case 1: return launch_down_res<1, 2, 5>(m.w[2], m.aq, a, grid, stream);
            case 2: return launch_down_res<2, 2, 4>(m.w[2], m.aq, a, grid, stream);
            case 3: return launch_down_res<3, 2, 3>(m.w[2], m.aq, a, grid, stream);
            case 4: return launch_down_res<4, 2, 2>(m.w[2], m.aq, a, grid, stream);
            default: return cudaErrorInvalidValue;
        }
    }
    switch (a.J) {
        case 1: return launch_cfg<1, 1, 6>(m.w[2], m.w[2], m.aq, a, grid, stream);
        case 2: return launch_cfg<1, 2, 4>(m.w[2], m.w[2], m.aq, a, grid, stream);
        case 3: return launch_cfg<1, 3, 3>(m.w[2], m.w[2], m.aq, a, grid, stream);
        case 4: return launch_cfg<1, 4, 2>(m.w[2], m.w[2], m.aq, a, grid, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace nvfp4
