// Dense NVFP4 linear on tcgen05 block-scaled MMA.
//
// The same arithmetic as the decode path's expert GEMVs: the weights stream
// through `tcgen05.mma.kind::mxf4nvf4.block_scale.block16` (M 128 weight
// rows, N 128, K 64, FP32 accumulators in tensor memory), so no instruction
// of the CTA touches a weight byte and the hardware applies the E4M3 block
// scales. The FP32 activations enter as six NVFP4 terms per vector sharing
// the vector's FP32 global scale (quant_terms.cuh); the six terms of vector v
// are B rows 6v .. 6v + 5, so one B tile carries 21 vectors and the epilogue
// adds each vector's six accumulator columns in term order.
//
//   linear_terms_kernel  (vector, 128 blocks of 16 columns) per CTA: the
//                        vector's absolute maximum, then one block per thread
//                        -> six terms (codes at B row 6v + j, scale bytes in
//                        tcgen05 atom layout); blocks past `cols` are zero.
//   linear_tc_kernel     one persistent CTA per SM walks 128-row tiles in a
//                        strided order over the fewest CTAs that need no
//                        more waves than the grid. Warp 0 producer (per
//                        256-column stage: TMA of the weight tile and of the
//                        activation-term tile, bulk copies of both sets of
//                        scale atoms; the first stages' weight parts are
//                        requested before the wait for the terms), warp 1
//                        MMA issuer and tensor-memory owner, warps 6-9 store
//                        each stage's scale atoms into tensor memory
//                        (tcgen05.st, one lane quarter each), warps 2-5
//                        epilogue (double-buffered accumulator: one weight row
//                        per thread, each vector's six terms summed, scaled
//                        and stored as FP32).
// Every mbarrier wait is bounded; on a timeout the CTA records the error,
// drains its copies and MMAs in flight, frees its tensor memory and exits.
#include "linear_tc.cuh"
#include "quant_terms.cuh"
#include "tcgen05_util.cuh"
#include "tma_util.cuh"

#include <atomic>

namespace nvfp4 {

namespace {

constexpr int kLtThreads = 320;
constexpr int kLtSfWarp0 = 6;
constexpr int kLtTile = 128;
constexpr int kLtTileBytes = kLtTile * 128;       // 128 rows x 128 bytes (256 FP4 columns)
constexpr int kLtSfStage = 4 * 512;               // four 64-column scale atoms
constexpr int kLtStage = 2 * kLtTileBytes + 2 * kLtSfStage;  // W tile, X tile, W atoms, X atoms
constexpr int kLtS = 6;
constexpr int kLtColSf = 256;                     // after the two 128-column accumulators
constexpr int kLtSfCols = 32;                     // per stage: W atoms 16 columns, X atoms 16
constexpr size_t kLtSmem = 1024 + (size_t)kLtS * kLtStage + 1024;
static_assert(kLtColSf + kLtS * kLtSfCols <= 512, "tensor memory overflow");
static_assert(kLtSmem <= 232448, "shared memory overflow");
static_assert(kLtStage % 1024 == 0, "stage must keep 1024-byte tile alignment");

enum LinearWaitSite : int {
    kSiteLinearEmpty = 61,
    kSiteLinearFull = 62,
    kSiteLinearAccEmpty = 63,
    kSiteLinearAccFull = 64,
};

struct LinearTcArgs {
    const uint8_t *w_atoms;
    const uint8_t *x_atoms;
    const float *gx;
    float *dst;        // this pass's first vector: dst[v][r] at dst + v * rows + r
    int rows;
    int kstages;
    int tiles;
    int nv;            // vectors of this pass (<= kLinTcVectors)
    float inv_global;
    int *err;
    int *host_err;
};

__device__ __forceinline__ uint8_t *align1024(uint8_t *p) {
    return reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ bool mbar_wait_drain(uint64_t *bar, uint32_t parity) {
    const unsigned long long t0 = global_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u && global_ns() - t0 > kWaitLimitNs) return false;
    }
}

// Weight scale bytes [rows][scale_pitch] -> atoms [tiles][kb64][512 B]:
// byte (r % 32) * 16 + ((r % 128) / 32) * 4 + (k % 4) of atom (r / 128, k / 4).
__global__ void linear_atoms_kernel(uint8_t *atoms, const uint8_t *scales, int scale_pitch, int rows, int k16,
                                    int kb64) {
    const size_t n = (size_t)rows * k16;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / k16), k = (int)(i - (size_t)r * k16);
        const size_t dst = ((size_t)(r / 128) * kb64 + k / 4) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (k % 4);
        atoms[dst] = scales[(size_t)r * scale_pitch + k];
    }
}

// Six terms of vector v's 16-column block b (one thread each); blocks at or
// past `nb` (the padding up to the last stage) are written as zero codes and
// zero scales. Every CTA of a vector first reduces the vector's absolute
// maximum (the same value in each), so all derive the same global scale.
__global__ void __launch_bounds__(128) linear_terms_kernel(const float *x, int cols, int nbp, uint8_t *xq,
                                                           uint8_t *x_atoms, float *gx) {
    // The linear kernel's weight stream does not read these terms until it
    // waits on this grid: let it start now.
    pdl_launch_dependents();
    __shared__ float s_max[4];
    const int v = blockIdx.y;
    const float *row = x + (size_t)v * cols;
    const int nb = cols / 16;
    float amax = 0.0f;
    for (int i = threadIdx.x; i < cols / 4; i += blockDim.x) {
        const float4 f = __ldg(reinterpret_cast<const float4 *>(row) + i);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(s_max[0], s_max[1]), fmaxf(s_max[2], s_max[3]));
    const float g = row_global_scale(amax);
    if (blockIdx.x == 0 && threadIdx.x == 0) gx[v] = g;
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nbp) return;
    const size_t row_bytes = (size_t)nbp * 8;
    if (b >= nb) {
#pragma unroll 1
        for (int j = 0; j < kLinTcTerms; ++j) {
            const int n = kLinTcTerms * v + j;
            *reinterpret_cast<uint2 *>(xq + (size_t)n * row_bytes + 8 * b) = make_uint2(0u, 0u);
            x_atoms[sf_atom_byte(n, b)] = 0;
        }
        return;
    }
    float vals[16];
    const float4 *p = reinterpret_cast<const float4 *>(row + 16 * b);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float4 f = __ldg(p + q);
        vals[4 * q] = f.x;
        vals[4 * q + 1] = f.y;
        vals[4 * q + 2] = f.z;
        vals[4 * q + 3] = f.w;
    }
    // Terms in a loop that is not unrolled: the kernel runs once per call
    // with cold instruction caches, where code size is time.
#pragma unroll 1
    for (int j = 0; j < kLinTcTerms; ++j) {
        uint32_t c0, c1;
        const uint32_t sc = quantize_block_term(vals, g, c0, c1);
        const int n = kLinTcTerms * v + j;
        *reinterpret_cast<uint2 *>(xq + (size_t)n * row_bytes + 8 * b) = make_uint2(c0, c1);
        x_atoms[sf_atom_byte(n, b)] = static_cast<uint8_t>(sc);
    }
}

__global__ void __launch_bounds__(kLtThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                     LinearTcArgs a) {
    constexpr int S = kLtS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align1024(smem_raw);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * kLtStage);
    uint64_t *empty = full + S;
    uint64_t *sf_in = empty + S;      // [S] the stage's scale atoms are in shared memory
    uint64_t *sf_full = sf_in + S;    // [S] ... and in tensor memory (four store warps)
    uint64_t *acc_full = sf_full + S; // [2]
    uint64_t *acc_empty = acc_full + 2;  // [2]
    uint64_t *drain = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    int *acc_ok = reinterpret_cast<int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int *err = a.err;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, 1);
            mbar_init(sf_in + i, 1);
            mbar_init(sf_full + i, 4);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full + b, 1);
            mbar_init(acc_empty + b, 1);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        prefetch_tensormap(&tm_w);
        prefetch_tensormap(&tm_x);
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, 512);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    // Tiles strided over the fewest CTAs that need no more waves than the
    // grid (every working CTA then takes the same count, or one fewer).
    const int waves = (a.tiles + (int)gridDim.x - 1) / (int)gridDim.x;
    const int ctas = (a.tiles + waves - 1) / waves;
    const int first = (int)blockIdx.x < ctas ? (int)blockIdx.x : a.tiles;
    const int ntile = first < a.tiles ? (a.tiles - first + ctas - 1) / ctas : 0;
    const int nstage = ntile * a.kstages;
    const int kw = 4 * a.kstages;  // 64-column atoms over K

    if (warp == 0) {
        // ------------------------------------------------------ producer
        // Stage `it` is (tile first + (it / kstages) * ctas, ks = it % kstages).
        auto tile_of = [&](uint32_t it) { return first + (int)(it / a.kstages) * ctas; };
        auto issue_w = [&](uint32_t it) {
            const int st = it % S, ks = it % a.kstages, tile = tile_of(it);
            uint8_t *stage = smem + (size_t)st * kLtStage;
            mbar_arrive_expect_tx(sf_in + st, 2 * kLtSfStage);
            bulk_g2s(stage + 2 * kLtTileBytes, a.w_atoms + ((size_t)tile * kw + ks * 4) * 512, kLtSfStage, sf_in + st);
            mbar_arrive_expect_tx(full + st, 2 * kLtTileBytes);
            tma_load_2d(stage, &tm_w, full + st, ks * 128, tile * kLtTile);
        };
        auto issue_x = [&](uint32_t it) {
            const int st = it % S, ks = it % a.kstages;
            uint8_t *stage = smem + (size_t)st * kLtStage;
            bulk_g2s(stage + 2 * kLtTileBytes + kLtSfStage, a.x_atoms + (size_t)ks * 4 * 512, kLtSfStage, sf_in + st);
            tma_load_2d(stage + kLtTileBytes, &tm_x, full + st, ks * 128, 0);
        };
        // The weights depend on no earlier launch: the first S stages' weight
        // parts are requested before the wait for the activation terms.
        const uint32_t pre = (uint32_t)(nstage < S ? nstage : S);
        if (lane == 0)
            for (uint32_t it = 0; it < pre; ++it) issue_w(it);
        pdl_wait();
        pdl_launch_dependents();
        uint32_t it = 0;
        bool ok = true;
        if (lane == 0) {
            for (; it < pre; ++it) issue_x(it);
            for (; it < (uint32_t)nstage; ++it) {
                const int st = it % S;
                if (!mbar_wait(empty + st, ((it / S) & 1u) ^ 1u, err, kSiteLinearEmpty)) {
                    ok = false;
                    break;
                }
                issue_w(it);
                issue_x(it);
            }
            if (!ok || *reinterpret_cast<volatile int *>(err) != 0) {
                // Drain the copies of the last stages issued.
                const uint32_t lo = it > (uint32_t)S ? it - S : 0u;
                for (uint32_t k = lo; k < it; ++k) {
                    mbar_wait_drain(full + (k % S), (k / S) & 1u);
                    mbar_wait_drain(sf_in + (k % S), (k / S) & 1u);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA
        pdl_wait();
        pdl_launch_dependents();
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_mxf4nvf4(kLtTile);
            const uint32_t smem_base = smem_u32(smem);
            uint32_t it = 0;
            bool ok = true;
            for (int t = 0; t < ntile && ok; ++t) {
                const uint32_t buf = (uint32_t)t & 1u, use = (uint32_t)t >> 1;
                if (use > 0 && !mbar_wait(acc_empty + buf, (use - 1) & 1u, err, kSiteLinearAccEmpty)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                for (int ks = 0; ks < a.kstages; ++ks, ++it) {
                    const int st = it % S;
                    const uint32_t ph = (it / S) & 1u;
                    if (!mbar_wait(full + st, ph, err, kSiteLinearFull) ||
                        !mbar_wait(sf_full + st, ph, err, kSiteLinearFull)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    tc::fence_proxy_async_smem();
                    const uint32_t sb = smem_base + (uint32_t)st * kLtStage;
                    const uint32_t tsf = tmem + kLtColSf + (uint32_t)st * kLtSfCols;
#pragma unroll
                    for (int at = 0; at < 4; ++at)
                        tc::mma_mxf4nvf4(tmem + buf * 128, tc::smem_desc_sw128(sb + 32 * at),
                                         tc::smem_desc_sw128(sb + kLtTileBytes + 32 * at), idesc, tsf + 4 * at,
                                         tsf + 16 + 4 * at, (ks | at) != 0 ? 1u : 0u);
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
    } else if (warp >= kLtSfWarp0) {
        // ------------------------------------------------- scale factors
        // A stage's eight atoms (weights 0-3, activation terms 0-3, 512 bytes
        // apart) into its 32 columns of this warp's lane quarter; the columns
        // are free once the producer has refilled the stage.
        pdl_wait();
        pdl_launch_dependents();
        const uint32_t quarter = (uint32_t)(32 * (warp & 3)) << 16;
        for (uint32_t it = 0; it < (uint32_t)nstage; ++it) {
            const int st = it % S;
            if (!__all_sync(0xffffffffu, mbar_wait(sf_in + st, (it / S) & 1u, err, kSiteLinearFull))) break;
            tc::st_sf_atoms<8>(tmem + quarter + kLtColSf + (uint32_t)st * kLtSfCols,
                               smem + (size_t)st * kLtStage + 2 * kLtTileBytes, 512, lane);
            tc::wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(sf_full + st);
        }
    } else {
        // ----------------------------------------------------- epilogue
        pdl_wait();
        pdl_launch_dependents();
        const int sub = warp & 3;
        const bool leader = threadIdx.x == 64;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * sub) << 16);
        const int ncols = kLinTcTerms * a.nv;
        float gs[kLinTcVectors];
#pragma unroll
        for (int v = 0; v < kLinTcVectors; ++v) gs[v] = v < a.nv ? a.gx[v] * a.inv_global : 0.0f;
        for (int t = 0; t < ntile; ++t) {
            const uint32_t buf = (uint32_t)t & 1u;
            if (leader) *acc_ok = mbar_wait(acc_full + buf, ((uint32_t)t >> 1) & 1u, err, kSiteLinearAccFull) ? 1 : 0;
            named_barrier(1, 128);
            if (!*reinterpret_cast<volatile int *>(acc_ok)) break;
            tc::fence_after_sync();
            // All columns in use come into registers (up to 128), then the
            // accumulator goes back to the MMA thread.
            uint32_t acc[128];
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (32 * q < ncols)
                    tc::ld_32x32b_x32(lane_base + buf * 128 + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(acc + 32 * q));
            tc::wait_ld();
            tc::fence_before_sync();
            named_barrier(1, 128);
            if (leader) mbar_arrive(acc_empty + buf);
            const int r = (first + t * ctas) * kLtTile + 32 * sub + lane;
            if (r < a.rows) {
#pragma unroll
                for (int v = 0; v < kLinTcVectors; ++v) {
                    if (v < a.nv) {
                        float y = __uint_as_float(acc[kLinTcTerms * v]);
#pragma unroll
                        for (int j = 1; j < kLinTcTerms; ++j) y += __uint_as_float(acc[kLinTcTerms * v + j]);
                        a.dst[(size_t)v * a.rows + r] = y * gs[v];
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
    if (threadIdx.x == 0 && *reinterpret_cast<volatile int *>(err) != 0 && a.host_err) {
        const int code = *reinterpret_cast<volatile int *>(err);
        *reinterpret_cast<volatile int *>(a.host_err) = code != 0 ? code : kErrWaitTimeout;
    }
}

}  // namespace

cudaError_t init_linear_tc(LinearTcState &st, const uint8_t *packed, int packed_pitch, const uint8_t *scales,
                           int scale_pitch, int rows, int cols, cudaStream_t stream) {
    st.kstages = (cols + kLinTcStageK - 1) / kLinTcStageK;
    st.tiles = (rows + kLtTile - 1) / kLtTile;
    const int kb64 = 4 * st.kstages;
    const size_t w_atoms = (size_t)st.tiles * kb64 * 512;
    const size_t xq = (size_t)kLtTile * st.kstages * 128;
    const size_t x_atoms = (size_t)kb64 * 512;
    cudaError_t e;
    if ((e = cudaMalloc(&st.w_atoms, w_atoms)) != cudaSuccess) return e;
    if ((e = cudaMalloc(&st.xq, xq)) != cudaSuccess) return e;
    if ((e = cudaMalloc(&st.x_atoms, x_atoms)) != cudaSuccess) return e;
    if ((e = cudaMalloc(&st.gx, kLinTcVectors * sizeof(float))) != cudaSuccess) return e;
    if ((e = cudaMalloc(&st.err, sizeof(int))) != cudaSuccess) return e;
    if ((e = cudaMemsetAsync(st.w_atoms, 0, w_atoms, stream)) != cudaSuccess) return e;
    if ((e = cudaMemsetAsync(st.xq, 0, xq, stream)) != cudaSuccess) return e;
    if ((e = cudaMemsetAsync(st.x_atoms, 0, x_atoms, stream)) != cudaSuccess) return e;
    if ((e = cudaMemsetAsync(st.err, 0, sizeof(int), stream)) != cudaSuccess) return e;
    const size_t n = (size_t)rows * (cols / 16);
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    linear_atoms_kernel<<<grid, 256, 0, stream>>>(st.w_atoms, scales, scale_pitch, rows, cols / 16, kb64);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = make_tensor_map_u8(&st.map_w, packed, (uint64_t)packed_pitch, (uint64_t)packed_pitch, (uint64_t)rows,
                                128, kLtTile, CU_TENSOR_MAP_SWIZZLE_128B)) != cudaSuccess)
        return e;
    return make_tensor_map_u8(&st.map_x, st.xq, (uint64_t)st.kstages * 128, (uint64_t)st.kstages * 128, kLtTile, 128,
                              kLtTile, CU_TENSOR_MAP_SWIZZLE_128B);
}

void free_linear_tc(LinearTcState &st) {
    if (st.w_atoms) cudaFree(st.w_atoms);
    if (st.xq) cudaFree(st.xq);
    if (st.x_atoms) cudaFree(st.x_atoms);
    if (st.gx) cudaFree(st.gx);
    if (st.err) cudaFree(st.err);
    st = LinearTcState{};
}

cudaError_t launch_linear_tc(const LinearTcState &st, const float *x, int vectors, int rows, int cols,
                             float inv_global, float *dst, int sm_count, cudaStream_t stream) {
    if (vectors <= 0 || cols % 16 != 0 || (reinterpret_cast<uintptr_t>(x) & 15u) != 0) return cudaErrorInvalidValue;
    static std::atomic<uint64_t> configured{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
    if (!bit || !(configured.load() & bit)) {
        e = cudaFuncSetAttribute(linear_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kLtSmem);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    const int nbp = st.kstages * (kLinTcStageK / 16);
    const int grid = st.tiles < sm_count ? st.tiles : sm_count;
    for (int v0 = 0; v0 < vectors; v0 += kLinTcVectors) {
        const int nv = vectors - v0 < kLinTcVectors ? vectors - v0 : kLinTcVectors;
        linear_terms_kernel<<<dim3((nbp + 127) / 128, nv), 128, 0, stream>>>(x + (size_t)v0 * cols, cols, nbp,
                                                                             st.xq, st.x_atoms, st.gx);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        LinearTcArgs a{};
        a.w_atoms = st.w_atoms;
        a.x_atoms = st.x_atoms;
        a.gx = st.gx;
        a.dst = dst + (size_t)v0 * rows;
        a.rows = rows;
        a.kstages = st.kstages;
        a.tiles = st.tiles;
        a.nv = nv;
        a.inv_global = inv_global;
        a.err = st.err;
        a.host_err = st.host_err_dev;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kLtThreads);
        cfg.dynamicSmemBytes = kLtSmem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if ((e = cudaLaunchKernelEx(&cfg, linear_tc_kernel, st.map_w, st.map_x, a)) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace nvfp4
