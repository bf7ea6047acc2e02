// TMA-fed expert GEMVs and the combine kernel of the decode path.
//
// Both GEMV kernels are persistent: one producer warp streams weight tiles
// into a ring of shared-memory stages with 2D TMA loads into its own CTA, four
// consumer warps decode E2M1 x E4M3 to f16 in registers and run m16n8k16
// MMAs against FP16 token rows held in shared memory, and mbarriers hand
// stages back and forth. Every mbarrier wait is bounded (tma_util.cuh) and
// reports a timeout through the scratch error word.
//
// moe_gate_up_tma_kernel  item = (active expert, 32 rows of the intermediate
//                          dimension); gate and up tiles stream together;
//                          SiLU(gate) * up is written as FP16.
// moe_down_tma_kernel     item = (active expert, 64 rows of hidden); each
//                          expert's output, scaled by routing weight and
//                          inverse global scale, is written per (token, slot).
// moe_combine_kernel      out = sum of the nine slots in slot order (the lab's
//                          reduce, nvfp4_gemv.cl:1443-1457) + residual.
// In both GEMVs the producer warp also copies the item's FP16 token rows for
// the stage's K range into the stage (cp.async, completing on the same
// mbarrier as the TMA bytes), so consumers read both operands from shared
// memory. A token group holds up to NT*8 tokens; an expert with more tokens
// streams its tiles once per group.
//
// Weight tiles land in shared memory with the 128-byte TMA swizzle: 16-byte
// unit u of row r sits at r*128 + ((u ^ (r & 7)) << 4). Lane (g, c) reads
// units 2c and 2c+1 of rows g and g+8, i.e. columns [64c, 64c+64) of each
// 256-column box, so the eight lanes of an LDS.128 phase hit eight distinct
// bank groups. Token rows use the same column split: a row stores 64-column
// segments at a 144-byte stride and rows at a pitch of 4 mod 8 sixteen-byte
// units, so the four lanes of a row and the eight rows of a phase land on
// distinct bank groups.
//
// A 256-column box may extend past the end of K (K is a multiple of 128):
// TMA fills the weight side with zeros and the token side is not read there,
// so no stale value can enter a product.
#include "moe_decode.cuh"
#include "tma_util.cuh"

#include <atomic>

namespace nvfp4 {

namespace {

constexpr int kBoxK = 256;            // K elements per TMA box (128 bytes)
constexpr int kBoxBytes = 128;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kGuRows = 32;
constexpr int kDnRows = 64;

__host__ __device__ constexpr int tok_pitch(int k) {
    return (k / 64) * 144 + 16 * ((4 - ((k / 64) * 9) % 8 + 8) % 8);
}

__device__ __forceinline__ int tok_offset(int pitch, int j, int k) {
    return j * pitch + (k >> 6) * 144 + (k & 63) * 2;
}

__device__ __forceinline__ uint8_t *align1024(uint8_t *p) {
    return reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Publish the recorded wait failure (its site code) to the bank's
// host-visible word (a plain store: no atomics on host memory).
__device__ __forceinline__ void publish_timeout(const DecodeScratch &s) {
    const int code = *reinterpret_cast<volatile int *>(s.error);
    if (s.host_error) *reinterpret_cast<volatile int *>(s.host_error) = code != 0 ? code : kErrWaitTimeout;
}

__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }

// Decode one 16-byte unit (32 columns, two E4M3 blocks) of a row into 16
// f16x2 words multiplied by their block scales; `sc` holds the two scale
// bytes (low byte = first block).
__device__ __forceinline__ void decode_unit(const uint4 &u, uint16_t sc, uint32_t (&h)[16]) {
    const uint32_t s2 = e4m3x2_to_f16x2(sc);
    const uint32_t m0 = f16x2_lo_lo(s2), m1 = f16x2_hi_hi(s2);
    const uint32_t *w = &u.x;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        uint32_t t[4];
        e2m1x8_to_f16x8(w[v], t);
        const uint32_t m = v < 2 ? m0 : m1;
#pragma unroll
        for (int j = 0; j < 4; ++j) h[4 * v + j] = hmul2_u32(t[j], m);
    }
}

// Routing metadata of one work item (active expert ai, row tile mt).
struct ItemMeta {
    int ai, mt, e, tstart, ntok;
};

__device__ __forceinline__ ItemMeta load_item(const DecodeScratch &s, int item, int mtiles) {
    ItemMeta m;
    m.ai = item / mtiles;
    m.mt = item - m.ai * mtiles;
    m.e = s.active_expert[m.ai];
    m.tstart = s.tok_start[m.ai];
    m.ntok = s.tok_count[m.ai];
    return m;
}

// ------------------------------------------------------------ gate / up

template <int NT, int BOXES, int S>
struct GuCfg {
    static constexpr int kPacked = BOXES * kGuRows * kBoxBytes;   // per projection
    static constexpr int kScales = kGuRows * BOXES * 16;          // per projection
    static constexpr int kTokPitch = tok_pitch(BOXES * kBoxK);
    static constexpr int kTok = NT * 8 * kTokPitch;
    static constexpr int kStage = (2 * kPacked + 2 * kScales + kTok + 1023) & ~1023;
    static constexpr int kRed = 2 * 2 * NT * 4 * 32 * 4;
};

template <int NT, int BOXES, int S>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gate_up_tma_kernel(const __grid_constant__ CUtensorMap tm_gp, const __grid_constant__ CUtensorMap tm_gs,
                           const __grid_constant__ CUtensorMap tm_up, const __grid_constant__ CUtensorMap tm_us,
                           GateUpArgs a) {
    using Cfg = GuCfg<NT, BOXES, S>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align1024(smem_raw);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + S * Cfg::kStage);
    uint64_t *empty = full + S;
    float *red = reinterpret_cast<float *>(empty + S);        // [2 mtile][2 proj][NT][4][32]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const DecodeScratch &s = a.s;
    int *err = s.error;
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(full + i, 1 + 32);  // TMA transaction arrive + one cp.async arrive per producer lane
            mbar_init(empty + i, kConsumerWarps);
        }
        fence_barrier_init();
        prefetch_tensormap(&tm_gp);
        prefetch_tensormap(&tm_up);
        prefetch_tensormap(&tm_gs);
        prefetch_tensormap(&tm_us);
    }
    __syncthreads();
    const int H = a.H, I = a.I, E = a.E;
    const int mtiles = I / kGuRows;
    const int kboxes = (H + kBoxK - 1) / kBoxK;
    const int slices = (kboxes + BOXES - 1) / BOXES;
    constexpr int kSK = BOXES * kBoxK;
    constexpr uint32_t kTx = 2 * Cfg::kPacked + 2 * Cfg::kScales;

    if (warp == kConsumerWarps) {
        pdl_wait();  // the routing kernel's outputs are read from here on
        pdl_launch_dependents();
        // Output-tile tickets of the down kernel that follows (which reads
        // them only after this grid completes).
        if (blockIdx.x == 0)
            for (int i = lane; i < H / kDnRows; i += 32) s.tile_count[i] = 0u;
        // Metadata is prefetched one item ahead and the token ids of a
        // group are held in registers, so no global load sits between two
        // stage refills. The first item's table entries are requested
        // together with the item count (an entry past the count is never
        // used).
        ItemMeta nxt{};
        if ((int)blockIdx.x < (E + 1) * mtiles) nxt = load_item(s, blockIdx.x, mtiles);
        const int items = *s.n_active * mtiles;
        uint32_t it = 0;
        for (int item = blockIdx.x; item < items; item += gridDim.x) {
            const ItemMeta cur = nxt;
            if (item + (int)gridDim.x < items) nxt = load_item(s, item + gridDim.x, mtiles);
            const int y = cur.e * I + cur.mt * kGuRows;
            const int tstart = cur.tstart, ntok = cur.ntok;
            for (int tg = 0; tg < ntok; tg += NT * 8) {
                const int ncols = min(NT * 8, ntok - tg);
                const int my_tok = lane < ncols ? s.tok_list[tstart + tg + lane] : 0;
                for (int sl = 0; sl < slices; ++sl, ++it) {
                    const int st = it % S;
                    const uint32_t ph = (it / S) & 1u;
                    int ok = 1;
                    if (lane == 0) ok = mbar_wait(empty + st, ph ^ 1u, err, kSiteGateUpEmpty) ? 1 : 0;
                    if (!__shfl_sync(0xffffffffu, ok, 0)) {
                        if (lane == 0) publish_timeout(s);
                        return;
                    }
                    uint8_t *stage = smem + st * Cfg::kStage;
                    if (lane == 0) {
                        mbar_arrive_expect_tx(full + st, kTx);
#pragma unroll
                        for (int b = 0; b < BOXES; ++b) {
                            const int x = (sl * BOXES + b) * kBoxBytes;
                            tma_load_2d(stage + b * kGuRows * kBoxBytes, &tm_gp, full + st, x, y);
                            tma_load_2d(stage + Cfg::kPacked + b * kGuRows * kBoxBytes, &tm_up, full + st, x, y);
                        }
                        tma_load_2d(stage + 2 * Cfg::kPacked, &tm_gs, full + st, sl * BOXES * 16, y);
                        tma_load_2d(stage + 2 * Cfg::kPacked + Cfg::kScales, &tm_us, full + st, sl * BOXES * 16, y);
                    }
                    uint8_t *tok = stage + 2 * Cfg::kPacked + 2 * Cfg::kScales;
                    constexpr int per_row = kSK / 8;  // a multiple of 32: every lane runs the same trips
                    for (int i = lane; i < ncols * per_row; i += 32) {
                        const int j = i / per_row, kk = (i - j * per_row) * 8;
                        const int k = sl * kSK + kk;
                        const int t = __shfl_sync(0xffffffffu, my_tok, j);
                        if (k < H) cp_async16(tok + tok_offset(Cfg::kTokPitch, j, kk), s.x_f16 + (size_t)t * H + k);
                    }
                    cp_async_arrive_noinc(full + st);
                }
            }
        }
        return;
    }

    constexpr int kBoxesPerWarp = BOXES / 2;
    bool failed = false;
    const int mtile = warp & 1, kh = warp >> 1;
    const int g = lane >> 2, c = lane & 3;
    const int r0 = mtile * 16 + g, r1 = r0 + 8;
    uint32_t it = 0;
    ItemMeta nxt{};
    float nx_gate = 0.0f, nx_up = 0.0f;
    int items = 0;
    // Round item = -1 runs before the wait on the routing kernel: one slice
    // of the product code below over stage 0's uninitialised bytes, waiting
    // for no barrier and storing nothing, its sums dropped. The code then
    // sits in the SM's instruction cache when the first real slice lands
    // (fetching it cold from DRAM cost ~3 us of a one-token call).
    for (int item = -1; item < items; item = item < 0 ? (int)blockIdx.x : item + (int)gridDim.x) {
        const bool warm = item < 0;
        ItemMeta cur{};
        float inv_gate = 0.0f, inv_up = 0.0f;
        if (!warm) {
            cur = nxt;
            inv_gate = nx_gate;
            inv_up = nx_up;
            if (item + (int)gridDim.x < items) {
                nxt = load_item(s, item + gridDim.x, mtiles);
                nx_gate = a.inv_scales[nxt.e];
                nx_up = a.inv_scales[(E + 1) + nxt.e];
            }
        }
        const int mt = cur.mt;
        const int tstart = cur.tstart, ntok = warm ? 1 : cur.ntok;
        const int nsl = warm ? 1 : slices;
        for (int tg = 0; tg < ntok; tg += NT * 8) {
            const int ncols = warm ? NT * 8 : min(NT * 8, ntok - tg);
            // Two accumulators per projection (k-slot halves) halve the
            // dependent MMA chains; they are added once per token group.
            float cg[NT][4], cu[NT][4], cg2[NT][4], cu2[NT][4];
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int r = 0; r < 4; ++r) cg[n][r] = cu[n][r] = cg2[n][r] = cu2[n][r] = 0.0f;

            for (int sl = 0; sl < nsl; ++sl, ++it) {
                const int st = it % S;
                const uint32_t ph = (it / S) & 1u;
                // After a failed wait the warp keeps walking the loops (without
                // waiting or computing) so the named barriers below still see
                // all four consumer warps.
                if (failed) continue;
                if (!warm && !mbar_wait(full + st, ph, err, kSiteGateUpFull)) {
                    publish_timeout(s);
                    failed = true;
                    continue;
                }
                const uint8_t *stage = smem + st * Cfg::kStage;
                const uint8_t *gsc = stage + 2 * Cfg::kPacked;
                const uint8_t *usc = gsc + Cfg::kScales;
                const uint8_t *tok = usc + Cfg::kScales;
#pragma unroll
                for (int bb = 0; bb < kBoxesPerWarp; ++bb) {
                    const int b = kh * kBoxesPerWarp + bb;
                    const int kb = sl * BOXES + b;
                    if (kb >= kboxes) break;
                    const uint8_t *gbox = stage + b * kGuRows * kBoxBytes;
                    const uint8_t *ubox = stage + Cfg::kPacked + b * kGuRows * kBoxBytes;
                    const uint32_t sg0 = lds32(gsc + r0 * (BOXES * 16) + b * 16 + 4 * c);
                    const uint32_t sg1 = lds32(gsc + r1 * (BOXES * 16) + b * 16 + 4 * c);
                    const uint32_t su0 = lds32(usc + r0 * (BOXES * 16) + b * 16 + 4 * c);
                    const uint32_t su1 = lds32(usc + r1 * (BOXES * 16) + b * 16 + 4 * c);
#pragma unroll
                    for (int uu = 0; uu < 2; ++uu) {
                        const int kloc = b * kBoxK + 64 * c + 32 * uu;
                        // Lanes past the end of K keep issuing the warp-wide
                        // MMAs with zero token operands (the weight side is
                        // zero-filled by TMA there).
                        const bool kin = sl * kSK + kloc < H;
                        const int unit = ((2 * c + uu) ^ g) << 4;
                        uint32_t hg0[16], hg1[16], hu0[16], hu1[16];
                        decode_unit(lds128(gbox + r0 * kBoxBytes + unit), (uint16_t)(sg0 >> (16 * uu)), hg0);
                        decode_unit(lds128(gbox + r1 * kBoxBytes + unit), (uint16_t)(sg1 >> (16 * uu)), hg1);
                        decode_unit(lds128(ubox + r0 * kBoxBytes + unit), (uint16_t)(su0 >> (16 * uu)), hu0);
                        decode_unit(lds128(ubox + r1 * kBoxBytes + unit), (uint16_t)(su1 >> (16 * uu)), hu1);
#pragma unroll
                        for (int n = 0; n < NT; ++n) {
                            if (n * 8 >= ncols) break;
                            const bool have = n * 8 + g < ncols;
#pragma unroll
                            for (int w = 0; w < 4; ++w) {
                                uint4 bv = make_uint4(0u, 0u, 0u, 0u);
                                if (have && kin) bv = lds128(tok + tok_offset(Cfg::kTokPitch, n * 8 + g, kloc + 8 * w));
                                mma_16816(cg[n], hg0[4 * w], hg1[4 * w], hg0[4 * w + 1], hg1[4 * w + 1], bv.x, bv.y);
                                mma_16816(cg2[n], hg0[4 * w + 2], hg1[4 * w + 2], hg0[4 * w + 3], hg1[4 * w + 3], bv.z,
                                          bv.w);
                                mma_16816(cu[n], hu0[4 * w], hu1[4 * w], hu0[4 * w + 1], hu1[4 * w + 1], bv.x, bv.y);
                                mma_16816(cu2[n], hu0[4 * w + 2], hu1[4 * w + 2], hu0[4 * w + 3], hu1[4 * w + 3], bv.z,
                                          bv.w);
                            }
                        }
                    }
                }
                __syncwarp();
                if (!warm && lane == 0) mbar_arrive(empty + st);
            }
            if (warm) break;
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    cg[n][r] += cg2[n][r];
                    cu[n][r] += cu2[n][r];
                }
            // Fixed-order reduction of the two K halves, then SiLU(gate)*up.
            if (kh == 1) {
#pragma unroll
                for (int n = 0; n < NT; ++n)
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        red[(((mtile * 2 + 0) * NT + n) * 4 + r) * 32 + lane] = cg[n][r];
                        red[(((mtile * 2 + 1) * NT + n) * 4 + r) * 32 + lane] = cu[n][r];
                    }
            }
            named_barrier(1, kConsumerWarps * 32);
            if (kh == 0) {
#pragma unroll
                for (int n = 0; n < NT; ++n) {
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const int col = n * 8 + 2 * c + (r & 1);
                        if (col < ncols) {
                            const float gs = cg[n][r] + red[(((mtile * 2 + 0) * NT + n) * 4 + r) * 32 + lane];
                            const float us = cu[n][r] + red[(((mtile * 2 + 1) * NT + n) * 4 + r) * 32 + lane];
                            const float gate = gs * inv_gate;
                            const float up = us * inv_up;
                            const int rl = (r >= 2) ? r1 : r0;
                            s.act[(size_t)(tstart + tg + col) * I + mt * kGuRows + rl] =
                                __float2half_rn(gate / (1.0f + expf(-gate)) * up);
                        }
                    }
                }
            }
            named_barrier(1, kConsumerWarps * 32);
        }
        if (warm) {
            pdl_wait();  // the routing kernel's outputs are read from here on
            pdl_launch_dependents();
            items = *s.n_active * mtiles;
            it = 0;
            if (blockIdx.x < items) {
                nxt = load_item(s, blockIdx.x, mtiles);
                nx_gate = a.inv_scales[nxt.e];
                nx_up = a.inv_scales[(E + 1) + nxt.e];
            }
        }
    }
}

// ------------------------------------------------------------------ down

// Output rows h..h+3 of token t (combine_quad over the down arguments).
__device__ __forceinline__ void combine_quad(const DownArgs &a, int t, int h) {
    const CombineOut c{a.residual, a.out, a.out_f32, a.shared_here, a.T, a.H};
    combine_quad(c, a.s, t, h);
}

template <int NT, int BOXES, int S>
struct DnCfg {
    static constexpr int kPacked = BOXES * kDnRows * kBoxBytes;
    static constexpr int kScales = kDnRows * BOXES * 16;
    static constexpr int kTokPitch = tok_pitch(BOXES * kBoxK);
    static constexpr int kTok = NT * 8 * kTokPitch;
    static constexpr int kStage = (kPacked + kScales + kTok + 1023) & ~1023;
};

template <int NT, int BOXES, int S>
__global__ void __launch_bounds__(kThreads, 1)
    moe_down_tma_kernel(const __grid_constant__ CUtensorMap tm_dp, const __grid_constant__ CUtensorMap tm_ds,
                        DownArgs a) {
    using Cfg = DnCfg<NT, BOXES, S>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align1024(smem_raw);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + S * Cfg::kStage);
    uint64_t *empty = full + S;
    __shared__ int s_flag[2];  // [0] a consumer warp gave up waiting; [1] this CTA combines the current tile
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const DecodeScratch &s = a.s;
    int *err = s.error;
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(full + i, 1 + 32);  // TMA transaction arrive + one cp.async arrive per producer lane
            mbar_init(empty + i, kConsumerWarps);
        }
        fence_barrier_init();
        prefetch_tensormap(&tm_dp);
        prefetch_tensormap(&tm_ds);
        s_flag[0] = 0;
    }
    __syncthreads();
    const int H = a.H, I = a.I;
    const int rtiles = H / kDnRows;
    const int kboxes = (I + kBoxK - 1) / kBoxK;
    const int slices = (kboxes + BOXES - 1) / BOXES;
    constexpr int kSK = BOXES * kBoxK;
    constexpr uint32_t kTx = Cfg::kPacked + Cfg::kScales;

    if (warp == kConsumerWarps) {
        // The routing tables are complete when this grid starts: the gate/up
        // grid triggers its dependents only after its own wait on the
        // routing kernel. So the weight tiles of the first S stages (which no
        // kernel of the call writes) are requested before the wait on the
        // gate/up grid; the activation rows it writes are copied after it.
        const int items = *s.n_active * rtiles;
        auto load_weights = [&](int st, int y, int sl) {
            uint8_t *stage = smem + st * Cfg::kStage;
            mbar_arrive_expect_tx(full + st, kTx);
            for (int b = 0; b < BOXES; ++b)
                tma_load_2d(stage + b * kDnRows * kBoxBytes, &tm_dp, full + st, (sl * BOXES + b) * kBoxBytes, y);
            tma_load_2d(stage + Cfg::kPacked, &tm_ds, full + st, sl * BOXES * 16, y);
        };
        uint32_t pre = 0;  // stages whose weights are already requested (all start empty)
        if (lane == 0)
            for (int item = blockIdx.x; item < items && pre < (uint32_t)S; item += gridDim.x) {
                const ItemMeta m = load_item(s, item, rtiles);
                for (int tg = 0; tg < m.ntok && pre < (uint32_t)S; tg += NT * 8)
                    for (int sl = 0; sl < slices && pre < (uint32_t)S; ++sl, ++pre)
                        load_weights((int)pre, m.e * H + m.mt * kDnRows, sl);
            }
        pre = __shfl_sync(0xffffffffu, pre, 0);
        pdl_wait();  // the gate/up activations are read from here on
        pdl_launch_dependents();
        uint32_t it = 0;
        ItemMeta nxt{};
        if (blockIdx.x < items) nxt = load_item(s, blockIdx.x, rtiles);
        for (int item = blockIdx.x; item < items; item += gridDim.x) {
            const ItemMeta cur = nxt;
            if (item + (int)gridDim.x < items) nxt = load_item(s, item + gridDim.x, rtiles);
            const int y = cur.e * H + cur.mt * kDnRows;
            const int tstart = cur.tstart, ntok = cur.ntok;
            for (int tg = 0; tg < ntok; tg += NT * 8) {
                const int ncols = min(NT * 8, ntok - tg);
                for (int sl = 0; sl < slices; ++sl, ++it) {
                    const int st = it % S;
                    const uint32_t ph = (it / S) & 1u;
                    uint8_t *stage = smem + st * Cfg::kStage;
                    if (it >= pre) {
                        int ok = 1;
                        if (lane == 0) ok = mbar_wait(empty + st, ph ^ 1u, err, kSiteDownEmpty) ? 1 : 0;
                        if (!__shfl_sync(0xffffffffu, ok, 0)) {
                            if (lane == 0) publish_timeout(s);
                            return;
                        }
                        if (lane == 0) load_weights(st, y, sl);
                    }
                    uint8_t *tok = stage + Cfg::kPacked + Cfg::kScales;
                    const int per_row = kSK / 8;
                    for (int i = lane; i < ncols * per_row; i += 32) {
                        const int j = i / per_row, kk = (i - j * per_row) * 8;
                        const int k = sl * kSK + kk;
                        if (k < I)
                            cp_async16(tok + tok_offset(Cfg::kTokPitch, j, kk),
                                       s.act + (size_t)(tstart + tg + j) * I + k);
                    }
                    cp_async_arrive_noinc(full + st);
                }
            }
        }
        return;
    }

    pdl_wait();  // routing tables and gate/up activations are read from here on
    pdl_launch_dependents();
    const int nact = *s.n_active;
    const int items = nact * rtiles;
    const int g = lane >> 2, c = lane & 3;
    const int r0 = warp * 16 + g, r1 = r0 + 8;
    uint32_t it = 0;
    ItemMeta nxt{};
    if (blockIdx.x < items) nxt = load_item(s, blockIdx.x, rtiles);
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const ItemMeta cur = nxt;
        if (item + (int)gridDim.x < items) nxt = load_item(s, item + gridDim.x, rtiles);
        const int ai = cur.ai, rt = cur.mt;
        const int tstart = cur.tstart, ntok = cur.ntok;
        bool failed = false;
        for (int tg = 0; tg < ntok; tg += NT * 8) {
            const int ncols = min(NT * 8, ntok - tg);
            // Output scales of this lane's columns, loaded before the K loop
            // so their latency overlaps it.
            float coefs[NT][2];
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int col = n * 8 + 2 * c + h;
                    coefs[n][h] = col < ncols
                                      ? s.coef_tab[ai * kDecodeMaxTokens + s.tok_list[tstart + tg + col]]
                                      : 0.0f;
                }
            float cd[NT][4], cd2[NT][4];  // two chains, added once per token group
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int r = 0; r < 4; ++r) cd[n][r] = cd2[n][r] = 0.0f;
            for (int sl = 0; sl < slices; ++sl, ++it) {
                const int st = it % S;
                const uint32_t ph = (it / S) & 1u;
                if (!__all_sync(0xffffffffu, mbar_wait(full + st, ph, err, kSiteDownFull))) {
                    failed = true;
                    break;
                }
                const uint8_t *stage = smem + st * Cfg::kStage;
                const uint8_t *sc = stage + Cfg::kPacked;
                const uint8_t *tok = sc + Cfg::kScales;
#pragma unroll
                for (int b = 0; b < BOXES; ++b) {
                    const int kb = sl * BOXES + b;
                    if (kb >= kboxes) break;
                    const uint8_t *box = stage + b * kDnRows * kBoxBytes;
                    const uint32_t s0 = lds32(sc + r0 * (BOXES * 16) + b * 16 + 4 * c);
                    const uint32_t s1 = lds32(sc + r1 * (BOXES * 16) + b * 16 + 4 * c);
#pragma unroll
                    for (int uu = 0; uu < 2; ++uu) {
                        const int kloc = b * kBoxK + 64 * c + 32 * uu;
                        const bool kin = sl * kSK + kloc < I;  // see gate/up
                        const int unit = ((2 * c + uu) ^ g) << 4;
                        uint32_t h0[16], h1[16];
                        decode_unit(lds128(box + r0 * kBoxBytes + unit), (uint16_t)(s0 >> (16 * uu)), h0);
                        decode_unit(lds128(box + r1 * kBoxBytes + unit), (uint16_t)(s1 >> (16 * uu)), h1);
#pragma unroll
                        for (int n = 0; n < NT; ++n) {
                            if (n * 8 >= ncols) break;
                            const bool have = n * 8 + g < ncols;
#pragma unroll
                            for (int w = 0; w < 4; ++w) {
                                uint4 bv = make_uint4(0u, 0u, 0u, 0u);
                                if (have && kin) bv = lds128(tok + tok_offset(Cfg::kTokPitch, n * 8 + g, kloc + 8 * w));
                                mma_16816(cd[n], h0[4 * w], h1[4 * w], h0[4 * w + 1], h1[4 * w + 1], bv.x, bv.y);
                                mma_16816(cd2[n], h0[4 * w + 2], h1[4 * w + 2], h0[4 * w + 3], h1[4 * w + 3], bv.z,
                                          bv.w);
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty + st);
            }
            if (failed) break;
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int r = 0; r < 4; ++r) cd[n][r] += cd2[n][r];
            // Scaled partial output of this expert for each of its tokens.
#pragma unroll
            for (int n = 0; n < NT; ++n) {
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int col = n * 8 + 2 * c + (r & 1);
                    if (col < ncols) {
                        const int j = tg + col;
                        const int row = rt * kDnRows + ((r >= 2) ? r1 : r0);
                        s.ypart[(size_t)(tstart + j) * H + row] = coefs[n][r & 1] * cd[n][r];
                    }
                }
            }
        }
        if (failed) publish_timeout(s);
        if (!a.fuse_combine) {
            if (failed) return;
            continue;
        }
        // Fused combine: publish this group's partial tile and take a ticket
        // for output tile rt; the CTA holding the tile's last ticket (every
        // other active group's partial is then written) sums the tile. All
        // four consumer warps reach both barriers, a warp that gave up
        // waiting included, and leave together.
        if (failed && lane == 0) s_flag[0] = 1;
        __threadfence();
        named_barrier(1, kConsumerWarps * 32);
        if (threadIdx.x == 0 && !s_flag[0])
            s_flag[1] = atomicAdd(s.tile_count + rt, 1u) == (unsigned)(nact - 1) ? 1 : 0;
        named_barrier(1, kConsumerWarps * 32);
        if (s_flag[0]) return;
        if (s_flag[1]) {
            __threadfence();
            constexpr int kQuads = kDnRows / 4;
#pragma unroll 1
            for (int i = threadIdx.x; i < a.T * kQuads; i += kConsumerWarps * 32)
                combine_quad(a, i / kQuads, rt * kDnRows + (i % kQuads) * 4);
        }
    }
    // No active group (an expert range that no token routes to): the output
    // is the residual alone, one tile per CTA.
    if (a.fuse_combine && items == 0) {
        constexpr int kQuads = kDnRows / 4;
#pragma unroll 1
        for (int t0 = blockIdx.x; t0 < rtiles; t0 += gridDim.x)
#pragma unroll 1
            for (int i = threadIdx.x; i < a.T * kQuads; i += kConsumerWarps * 32)
                combine_quad(a, i / kQuads, t0 * kDnRows + (i % kQuads) * 4);
    }
}

// ------------------------------------------------------------- combine

__global__ void __launch_bounds__(256) moe_combine_kernel(DownArgs a) {
    const DecodeScratch &s = a.s;
    const int H = a.H, T = a.T;
    const int t = blockIdx.y;
    const int h = blockIdx.x * blockDim.x + threadIdx.x;  // the grid covers H: one column per thread
    const size_t o = (size_t)t * H + h;
    const uint16_t *res = static_cast<const uint16_t *>(a.residual);
    float r = 0.0f;
    if (res && a.residual_early && h < H) r = bf16_bits_to_f32(res[o]);
    pdl_wait();
    pdl_launch_dependents();
    if (h >= H) return;
    if (res && !a.residual_early) r = bf16_bits_to_f32(res[o]);
    float v = 0.0f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        const int p = s.inv_pos[t * kTopK + k];
        if (p >= 0) v += s.ypart[(size_t)p * H + h];
    }
    if (a.shared_here) v += s.ypart[(size_t)(T * kTopK + t) * H + h];
    if (res) v += r;
    if (a.out_f32)
        static_cast<float *>(a.out)[o] = v;
    else
        static_cast<uint16_t *>(a.out)[o] = f32_to_bf16_bits(v);
}

// --------------------------------------------------------------- launches

// Raise a kernel's dynamic shared-memory limit once per device. `done` is a
// per-kernel bitmask of devices already configured.
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

// Resident CTAs per SM of a kernel at `smem` bytes of dynamic shared memory
// (at least 1), so persistent grids fill every SM slot.
template <typename K>
int ctas_per_sm(K kernel, size_t smem) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kThreads, smem) != cudaSuccess || n < 1) return 1;
    return n;
}

// Launch with programmatic stream serialisation: the kernel may start while
// its predecessor drains and calls griddepcontrol.wait before reading it.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args &&...args) {
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
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <int NT, int BOXES, int S>
cudaError_t launch_gate_up_cfg(const StreamMaps &m, const GateUpArgs &a, int items_ub, int sms,
                               cudaStream_t stream) {
    using Cfg = GuCfg<NT, BOXES, S>;
    const size_t smem = 1024 + S * Cfg::kStage + 2 * S * 8 + Cfg::kRed;
    static std::atomic<uint64_t> done{0};
    cudaError_t err = set_smem_once(moe_gate_up_tma_kernel<NT, BOXES, S>, smem, done);
    if (err != cudaSuccess) return err;
    static const int per_sm = ctas_per_sm(moe_gate_up_tma_kernel<NT, BOXES, S>, smem);
    const int grid = items_ub < sms * per_sm ? items_ub : sms * per_sm;
    const CUtensorMap &gs = BOXES == 4 ? m.scales[0] : m.scales_half[0];
    const CUtensorMap &us = BOXES == 4 ? m.scales[1] : m.scales_half[1];
    return launch_pdl(moe_gate_up_tma_kernel<NT, BOXES, S>, dim3(grid), dim3(kThreads), smem, stream, m.packed[0], gs,
                      m.packed[1], us, a);
}

template <int NT, int BOXES, int S>
cudaError_t launch_down_cfg(const StreamMaps &m, const DownArgs &a, int items_ub, int sms, cudaStream_t stream) {
    using Cfg = DnCfg<NT, BOXES, S>;
    const size_t smem = 1024 + S * Cfg::kStage + 2 * S * 8;
    static std::atomic<uint64_t> done{0};
    cudaError_t err = set_smem_once(moe_down_tma_kernel<NT, BOXES, S>, smem, done);
    if (err != cudaSuccess) return err;
    static const int per_sm = ctas_per_sm(moe_down_tma_kernel<NT, BOXES, S>, smem);
    const int grid = items_ub < sms * per_sm ? items_ub : sms * per_sm;
    return launch_pdl(moe_down_tma_kernel<NT, BOXES, S>, dim3(grid), dim3(kThreads), smem, stream, m.packed[2],
                      m.scales_half[2], a);
}

}  // namespace

cudaError_t make_tensor_map_u8(CUtensorMap *map, const void *base, uint64_t row_bytes, uint64_t pitch,
                               uint64_t rows, uint32_t box_bytes, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
    using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static EncodeFn encode = nullptr;
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (err != cudaSuccess) return err;
        if (q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
        encode = reinterpret_cast<EncodeFn>(fn);
    }
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {pitch};
    const cuuint32_t box[2] = {box_bytes, box_rows};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box,
                              elem, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_stream_maps(StreamMaps &m, uint8_t *const packed[3], uint8_t *const scales[3], int E, int H,
                             int I) {
    const uint64_t slots = static_cast<uint64_t>(E) + 1;
    for (int p = 0; p < 3; ++p) {
        const uint64_t rows = slots * (p < 2 ? I : H);
        const uint64_t k = p < 2 ? H : I;
        const uint64_t pitch = (k / 16 + 15) & ~uint64_t(15);
        const uint32_t box_rows = p < 2 ? kGuRows : kDnRows;
        cudaError_t err = make_tensor_map_u8(&m.packed[p], packed[p], k / 2, k / 2, rows, kBoxBytes, box_rows,
                                             CU_TENSOR_MAP_SWIZZLE_128B);
        if (err != cudaSuccess) return err;
        // Scale boxes cover four (scales) or two (scales_half) 256-column boxes.
        err = make_tensor_map_u8(&m.scales[p], scales[p], k / 16, pitch, rows, 64, box_rows,
                                 CU_TENSOR_MAP_SWIZZLE_NONE);
        if (err != cudaSuccess) return err;
        err = make_tensor_map_u8(&m.scales_half[p], scales[p], k / 16, pitch, rows, 32, box_rows,
                                 CU_TENSOR_MAP_SWIZZLE_NONE);
        if (err != cudaSuccess) return err;
    }
    return cudaSuccess;
}

// Token-group width by the expected tokens per routed expert (T*8 slots over
// min(E, T*8) experts): one group of 8 columns covers the typical decode
// batch, and a narrow token area leaves room for more pipeline stages. An
// expert with more tokens (the shared expert, skewed routing) re-streams its
// tile once per group, mostly from L2.
static int tokens_per_expert(int T, int E) {
    const int slots = T * kTopK;
    const int experts = E < slots ? E : slots;
    return (slots + experts - 1) / experts;
}

cudaError_t launch_gate_up_tma(const StreamMaps &m, const GateUpArgs &a, int T, int sms, cudaStream_t stream) {
    const int routed_ub = a.E < T * kTopK ? a.E : T * kTopK;
    const int items_ub = (routed_ub + 1) * (a.I / kGuRows);
    const int tpe = tokens_per_expert(T, a.E);
    // With at most one item per SM (small calls) a 4-stage ring keeps a whole
    // item's weights in flight; otherwise 2-stage rings let three CTAs share
    // an SM.
    if (tpe <= 8 && items_ub <= sms) return launch_gate_up_cfg<1, 2, 4>(m, a, items_ub, sms, stream);
    if (tpe <= 8) return launch_gate_up_cfg<1, 2, 2>(m, a, items_ub, sms, stream);
    if (tpe <= 16) return launch_gate_up_cfg<2, 2, 5>(m, a, items_ub, sms, stream);
    return launch_gate_up_cfg<4, 2, 3>(m, a, items_ub, sms, stream);
}

cudaError_t launch_down_tma(const StreamMaps &m, const DownArgs &a, int sms, cudaStream_t stream, bool with_combine) {
    const int T = a.T;
    const int routed_ub = a.E < T * kTopK ? a.E : T * kTopK;
    const int items_ub = (routed_ub + 1) * (a.H / kDnRows);
    cudaError_t err;
    const int tpe = tokens_per_expert(T, a.E);
    DownArgs da = a;
    da.fuse_combine = with_combine && T <= kFusedCombineMaxTokens ? 1 : 0;
    if (tpe <= 8)
        err = launch_down_cfg<1, 2, 2>(m, da, items_ub, sms, stream);
    else if (tpe <= 16)
        err = launch_down_cfg<2, 2, 4>(m, da, items_ub, sms, stream);
    else
        err = launch_down_cfg<4, 2, 3>(m, da, items_ub, sms, stream);
    if (err != cudaSuccess) return err;
    return with_combine && !da.fuse_combine ? launch_combine(a, stream) : cudaSuccess;
}

cudaError_t launch_combine(const DownArgs &a, cudaStream_t stream) {
    const dim3 grid((a.H + 255) / 256, a.T);
    return launch_pdl(moe_combine_kernel, grid, dim3(256), 0, stream, a);
}

}  // namespace nvfp4
