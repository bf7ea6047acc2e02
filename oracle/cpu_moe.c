/*
 * cpu_moe.c -- CPU restatement of the lab's NVFP4 MoE layer.
 * TEST INFRASTRUCTURE / CPU BASELINE ONLY: loaded by tests and by the
 * cpu_baseline leg of bench.py; the product library never links it.
 *
 * Row kernel: portable restatement of the lab's ARM NEON GEMV
 * (native_nvfp4/runtime/nvfp4_cpu.cpp:19-34 E4M3 decode, :36-87 neon_row):
 *   - doubled-value E2M1 table {0,1,2,3,4,6,8,12,0,-1,...,-12};
 *   - per 16-column block, scale = E4M3(s) * inverse_global * 0.5;
 *   - four FP32 lane accumulators, lane i taking columns i, 4+i, 8+i, 12+i
 *     of each block as acc += (q2 * x) * scale (multiply then add, as the
 *     non-fused vmlaq_n_f32);
 *   - final pairwise horizontal add (l0 + l1) + (l2 + l3).
 * Threading follows nvfp4_cpu_gemv_impl (nvfp4_cpu.cpp:163-204): rows are
 * split into contiguous ranges, one std::thread-equivalent per range.
 *
 * Layer: router and shared-gate logits in FP32 in the CUDA routing kernel's
 * lane order (bit-identical to it and to nvfp4_oracle.router_logits), top-8
 * with the lowest id on ties and renormalised weights (nvfp4_gemv.cl:
 * 1249-1295), gate/up/SiLU*up/down per selected expert
 * (bench_moe_routed_layer.py:97-103), weighted combine over the nine slots
 * in slot order (nvfp4_gemv.cl:1443-1457) and the residual add.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define TOPK 8
#define SLOTS 9

typedef struct nvfp4_oracle_bank {
    int experts;
    int hidden;
    int intermediate;
    const uint8_t *packed[3]; /* [(E+1)][rows][cols/2], rows x cols = I x H (0,1) or H x I (2) */
    const uint8_t *scales[3]; /* [(E+1)][rows][cols/16] */
    const float *inv_scales;  /* [3][E+1], 1 / weight_global_scale */
    const uint16_t *router;   /* [(E+1)][H] BF16, row E = shared gate */
    const float *router_bias; /* [E] or NULL */
} nvfp4_oracle_bank;

static float e4m3_to_float(uint8_t value) {
    value &= 0x7f;
    if (value == 0 || value == 0x7f) return 0.0f;
    const uint32_t exponent = (value >> 3) & 0xf;
    const uint32_t mantissa = value & 0x7;
    if (exponent == 0) return (float)mantissa * (1.0f / 512.0f);
    union {
        uint32_t bits;
        float value;
    } converted;
    converted.bits = (exponent + 120u) << 23 | mantissa << 20;
    return converted.value;
}

static const int8_t kQ2[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

static float row_dot(const uint8_t *packed, const uint8_t *scales, const float *x, int cols,
                     float inverse_global_scale) {
    float lane[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int blocks = cols / 16;
    for (int block = 0; block < blocks; ++block) {
        const uint8_t *bytes = packed + block * 8;
        float q[16];
        for (int j = 0; j < 8; ++j) {
            q[2 * j] = (float)kQ2[bytes[j] & 0x0f];
            q[2 * j + 1] = (float)kQ2[bytes[j] >> 4];
        }
        const float scale = e4m3_to_float(scales[block]) * inverse_global_scale * 0.5f;
        const float *xb = x + block * 16;
        for (int g = 0; g < 4; ++g) {
            for (int i = 0; i < 4; ++i) {
                const float prod = q[4 * g + i] * xb[4 * g + i];
                const float scaled = prod * scale;
                lane[i] = lane[i] + scaled;
            }
        }
    }
    return (lane[0] + lane[1]) + (lane[2] + lane[3]);
}

static float bf16_to_float(uint16_t bits) {
    union {
        uint32_t u;
        float f;
    } v;
    v.u = (uint32_t)bits << 16;
    return v.f;
}

/* ----------------------------------------------------------- thread pool */

typedef struct {
    void (*fn)(void *, int, int);
    void *ctx;
    int begin;
    int end;
} range_job;

static void *range_main(void *arg) {
    range_job *job = (range_job *)arg;
    job->fn(job->ctx, job->begin, job->end);
    return NULL;
}

/* Split [0, n) into `threads` contiguous ranges; the caller runs range 0. */
static void parallel_for(int n, int threads, void (*fn)(void *, int, int), void *ctx) {
    if (threads < 1) threads = 1;
    if (threads > n) threads = n;
    if (threads <= 1) {
        if (n > 0) fn(ctx, 0, n);
        return;
    }
    pthread_t *tids = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
    range_job *jobs = (range_job *)malloc(sizeof(range_job) * (size_t)threads);
    for (int w = 0; w < threads; ++w) {
        jobs[w].fn = fn;
        jobs[w].ctx = ctx;
        jobs[w].begin = (int)((long long)n * w / threads);
        jobs[w].end = (int)((long long)n * (w + 1) / threads);
    }
    for (int w = 1; w < threads; ++w) pthread_create(&tids[w], NULL, range_main, &jobs[w]);
    fn(ctx, jobs[0].begin, jobs[0].end);
    for (int w = 1; w < threads; ++w) pthread_join(tids[w], NULL);
    free(jobs);
    free(tids);
}

/* ------------------------------------------------------------------ GEMV */

typedef struct {
    const uint8_t *packed;
    const uint8_t *scales;
    int cols;
    float inv;
    const float *x;
    float *dst;
} gemv_ctx;

static void gemv_rows(void *p, int begin, int end) {
    gemv_ctx *c = (gemv_ctx *)p;
    for (int r = begin; r < end; ++r)
        c->dst[r] = row_dot(c->packed + (size_t)r * (c->cols / 2), c->scales + (size_t)r * (c->cols / 16),
                            c->x, c->cols, c->inv);
}

/* Same contract as nvfp4_cpu_gemv_f32 (nvfp4_runtime.cpp:1388-1416):
 * weight_global_scale is a divisor. Returns 0 on success. */
int nvfp4_oracle_cpu_gemv(const uint8_t *packed, const uint8_t *scales, int rows, int cols,
                          float weight_global_scale, const float *x, float *dst, int threads) {
    if (!packed || !scales || rows <= 0 || cols <= 0 || cols % 16 != 0 || weight_global_scale == 0.0f ||
        !x || !dst || threads < 0)
        return 1;
    gemv_ctx c = {packed, scales, cols, 1.0f / weight_global_scale, x, dst};
    parallel_for(rows, threads, gemv_rows, &c);
    return 0;
}

/* --------------------------------------------------------------- routing */

/* FP32 dot in the CUDA routing kernel's lane order (see file header). */
static float router_dot(const uint16_t *w, const float *x, int H) {
    float lane[32];
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int j = 0; j < H / 128; ++j)
            for (int e = 0; e < 4; ++e) {
                const int k = j * 128 + 4 * l + e;
                const float prod = bf16_to_float(w[k]) * x[k];
                acc = acc + prod;
            }
        lane[l] = acc;
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float next[32];
        for (int l = 0; l < 32; ++l) next[l] = lane[l] + lane[l ^ off];
        memcpy(lane, next, sizeof(lane));
    }
    return lane[0];
}

/* ------------------------------------------------------------------ layer */

typedef struct {
    const nvfp4_oracle_bank *bank;
    const float *x;   /* [T][H] */
    int T;
    int *ids;         /* [T][9] */
    float *weights;   /* [T][9] */
    float *logits;    /* [T][E+1] */
    float *act;       /* [T][9][I] */
    float *y;         /* [T][9][H] */
} layer_ctx;

static void route_tokens(void *p, int begin, int end) {
    layer_ctx *c = (layer_ctx *)p;
    const nvfp4_oracle_bank *b = c->bank;
    const int E = b->experts, H = b->hidden;
    for (int t = begin; t < end; ++t) {
        float *lg = c->logits + (size_t)t * (E + 1);
        for (int r = 0; r <= E; ++r) lg[r] = router_dot(b->router + (size_t)r * H, c->x + (size_t)t * H, H);
        if (b->router_bias)
            for (int e = 0; e < E; ++e) lg[e] = lg[e] + b->router_bias[e];
        unsigned char taken[256];
        memset(taken, 0, sizeof(taken));
        float top_v[TOPK];
        int top_i[TOPK];
        for (int s = 0; s < TOPK; ++s) {
            float best = -3.402823466e+38f;
            int best_id = 0;
            for (int e = 0; e < E; ++e) {
                if (!taken[e] && lg[e] > best) {
                    best = lg[e];
                    best_id = e;
                }
            }
            top_v[s] = best;
            top_i[s] = best_id;
            taken[best_id] = 1;
        }
        float den = 0.0f;
        for (int s = 0; s < TOPK; ++s) den += expf(top_v[s] - top_v[0]);
        for (int s = 0; s < TOPK; ++s) {
            c->ids[t * SLOTS + s] = top_i[s];
            c->weights[t * SLOTS + s] = expf(top_v[s] - top_v[0]) / den;
        }
        c->ids[t * SLOTS + TOPK] = E;
        c->weights[t * SLOTS + TOPK] = 1.0f / (1.0f + expf(-lg[E]));
    }
}

/* Work item = (token, slot, row) of the gate/up projections. */
static void gate_up_items(void *p, int begin, int end) {
    layer_ctx *c = (layer_ctx *)p;
    const nvfp4_oracle_bank *b = c->bank;
    const int E = b->experts, H = b->hidden, I = b->intermediate;
    const size_t mp = (size_t)I * H / 2, ms = (size_t)I * H / 16;
    for (int it = begin; it < end; ++it) {
        const int row = it % I;
        const int ts = it / I;
        const int t = ts / SLOTS, slot = ts % SLOTS;
        const int e = c->ids[t * SLOTS + slot];
        const float *x = c->x + (size_t)t * H;
        const float g = row_dot(b->packed[0] + e * mp + (size_t)row * (H / 2),
                                b->scales[0] + e * ms + (size_t)row * (H / 16), x, H,
                                b->inv_scales[e]);
        const float u = row_dot(b->packed[1] + e * mp + (size_t)row * (H / 2),
                                b->scales[1] + e * ms + (size_t)row * (H / 16), x, H,
                                b->inv_scales[(E + 1) + e]);
        c->act[((size_t)t * SLOTS + slot) * I + row] = g / (1.0f + expf(-g)) * u;
    }
}

static void down_items(void *p, int begin, int end) {
    layer_ctx *c = (layer_ctx *)p;
    const nvfp4_oracle_bank *b = c->bank;
    const int E = b->experts, H = b->hidden, I = b->intermediate;
    const size_t mp = (size_t)I * H / 2, ms = (size_t)I * H / 16;
    for (int it = begin; it < end; ++it) {
        const int row = it % H;
        const int ts = it / H;
        const int t = ts / SLOTS, slot = ts % SLOTS;
        const int e = c->ids[t * SLOTS + slot];
        c->y[((size_t)t * SLOTS + slot) * H + row] =
            row_dot(b->packed[2] + e * mp + (size_t)row * (I / 2), b->scales[2] + e * ms + (size_t)row * (I / 16),
                    c->act + ((size_t)t * SLOTS + slot) * I, I, b->inv_scales[2 * (E + 1) + e]);
    }
}

/* Routing only (router and shared-gate logits, top-8, weights, slot 8) for T
 * tokens -- the checker of full-size prefill calls, whose expert products
 * would take the scalar row kernel minutes. Only bank->experts, hidden,
 * router and router_bias are read. ids/weights [T][9], logits [T][E+1].
 * Returns 0 on success. */
int nvfp4_oracle_route(const nvfp4_oracle_bank *bank, const float *x, int T, int32_t *ids_out,
                       float *weights_out, float *logits_out, int threads) {
    if (!bank || !x || !ids_out || !weights_out || !logits_out || T <= 0 || bank->experts < 8 ||
        bank->experts > 256 || bank->hidden % 128 || !bank->router)
        return 1;
    layer_ctx c;
    memset(&c, 0, sizeof(c));
    c.bank = bank;
    c.x = x;
    c.T = T;
    c.ids = ids_out;
    c.weights = weights_out;
    c.logits = logits_out;
    parallel_for(T, threads, route_tokens, &c);
    return 0;
}

/* Full layer for T tokens. x [T][H] FP32; residual [T][H] or NULL; out
 * [T][H]. ids/weights [T][9] and logits [T][E+1] are optional outputs.
 * Returns 0 on success. */
int nvfp4_oracle_moe_forward(const nvfp4_oracle_bank *bank, const float *x, int T, const float *residual,
                             float *out, int32_t *ids_out, float *weights_out, float *logits_out,
                             int threads) {
    if (!bank || !x || !out || T <= 0 || bank->experts < 8 || bank->experts > 256 || bank->hidden % 128 ||
        bank->intermediate % 16)
        return 1;
    const int E = bank->experts, H = bank->hidden, I = bank->intermediate;
    layer_ctx c;
    c.bank = bank;
    c.x = x;
    c.T = T;
    c.ids = (int *)malloc(sizeof(int) * (size_t)T * SLOTS);
    c.weights = (float *)malloc(sizeof(float) * (size_t)T * SLOTS);
    c.logits = (float *)malloc(sizeof(float) * (size_t)T * (E + 1));
    c.act = (float *)malloc(sizeof(float) * (size_t)T * SLOTS * I);
    c.y = (float *)malloc(sizeof(float) * (size_t)T * SLOTS * H);
    if (!c.ids || !c.weights || !c.logits || !c.act || !c.y) {
        free(c.ids);
        free(c.weights);
        free(c.logits);
        free(c.act);
        free(c.y);
        return 2;
    }
    parallel_for(T, threads, route_tokens, &c);
    parallel_for(T * SLOTS * I, threads, gate_up_items, &c);
    parallel_for(T * SLOTS * H, threads, down_items, &c);
    for (int t = 0; t < T; ++t) {
        for (int h = 0; h < H; ++h) {
            float sum = 0.0f;
            for (int s = 0; s < SLOTS; ++s)
                sum += c.weights[t * SLOTS + s] * c.y[((size_t)t * SLOTS + s) * H + h];
            out[(size_t)t * H + h] = residual ? residual[(size_t)t * H + h] + sum : sum;
        }
    }
    if (ids_out) memcpy(ids_out, c.ids, sizeof(int) * (size_t)T * SLOTS);
    if (weights_out) memcpy(weights_out, c.weights, sizeof(float) * (size_t)T * SLOTS);
    if (logits_out) memcpy(logits_out, c.logits, sizeof(float) * (size_t)T * (E + 1));
    free(c.ids);
    free(c.weights);
    free(c.logits);
    free(c.act);
    free(c.y);
    return 0;
}
