/*
 * CPU restatement of the reference MoE feed-forward path (TEST INFRASTRUCTURE:
 * the parity oracle and the timed CPU baseline; the product never links it).
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off). Contraction is
 * off because the reference's scalar paths multiply and add separately; where
 * the reference (or this restatement) fuses, fmaf() is called explicitly.
 *
 * Reference paths below are relative to the happyme531/open_rknpu2_lm_infer root.
 */
#include "moe_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int oracle_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE binary16 <-> binary32 (exact widening; round-to-nearest-even narrowing). */
float oracle_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        float v = ldexpf((float)man, -24);
        return sign ? -v : v;
    }
    if (exp == 31) return u2f(sign | 0x7f800000u | (man << 13));
    return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

uint16_t oracle_float_to_half(float f) {
    uint32_t u = f2u(f), sign = (u >> 16) & 0x8000u;
    float a = fabsf(f);
    if (a != a) return (uint16_t)(sign | 0x7e00u);
    if (a >= 65520.0f) return (uint16_t)(sign | 0x7c00u);
    if (a < 6.103515625e-05f) { /* subnormal half: multiple of 2^-24 */
        float q = rintf(ldexpf(a, 24));
        return (uint16_t)(sign | (uint16_t)q);
    }
    int e;
    float m = frexpf(a, &e);            /* a = m * 2^e, m in [0.5,1) */
    float q = rintf(ldexpf(m, 11));     /* 11 significant bits, RNE */
    if (q >= 2048.0f) { q = 1024.0f; e += 1; }
    int exp = e - 1 + 15;
    if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | ((uint32_t)exp << 10) | ((uint32_t)q - 1024u));
}

/* Rust f32::total_cmp key (src/model/qwen35/moe.rs:58 sorts with total_cmp). */
int32_t oracle_total_key(float v) {
    int32_t b = (int32_t)f2u(v);
    return b ^ (int32_t)((uint32_t)(b >> 31) >> 1);
}

/* dense_dot (src/model/cpu.rs:96-153). NEON16 restates the aarch64 F32 branch
 * (:127-144): four 4-lane FMA accumulators over 16-element steps, reduced as
 * (a+b)+(c+d) lane-wise then vaddvq = (v0+v1)+(v2+v3), then the scalar tail
 * (:148-151). SEQUENTIAL restates the x86 build, where only the scalar tail
 * loop runs: sum += w*x with a separately rounded product. */
static float router_dot(const float *w, const float *x, int H, int order) {
    float sum = 0.0f;
    int i = 0;
    if (order == ORACLE_ROUTER_NEON16) {
        float l[16];
        for (int j = 0; j < 16; ++j) l[j] = 0.0f;
        for (; i + 16 <= H; i += 16)
            for (int j = 0; j < 16; ++j) l[j] = fmaf(w[i + j], x[i + j], l[j]);
        float v[4];
        for (int j = 0; j < 4; ++j) {
            float ab = l[j] + l[4 + j];
            float cd = l[8 + j] + l[12 + j];
            v[j] = ab + cd;
        }
        sum = (v[0] + v[1]) + (v[2] + v[3]);
    }
    if (order == ORACLE_ROUTER_TF32) {
        /* Tf32Linear (src/npu/tf32.rs:142-170): both operands narrowed to TF32
         * by dropping the low 13 mantissa bits; the reference's own check
         * (src/npu/tf32.rs:212-224) is the f64 sum of those products within
         * 5e-5, which is what this computes (rounded once to f32). */
        double acc = 0.0;
        for (; i < H; ++i)
            acc += (double)u2f(f2u(w[i]) & ~0x1fffu) * (double)u2f(f2u(x[i]) & ~0x1fffu);
        return (float)acc;
    }
    for (; i < H; ++i) {
        float p = w[i] * x[i];
        sum = sum + p;
    }
    return sum;
}

/* sigmoid (src/ops/activation.rs:7-14): the two branches keep exp's argument
 * non-positive. */
float oracle_sigmoid(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
    float e = expf(x);
    return e / (1.0f + e);
}

/* Cpu::dense_head_batch (src/model/cpu.rs:302-316): every output keeps the
 * single-row dot's order. */
void oracle_router_logits(const float *x, const float *router, const float *bias, int T,
                          int H, int E, int order, float *logits) {
#pragma omp parallel for schedule(static)
    for (long idx = 0; idx < (long)T * E; ++idx) {
        long t = idx / E, e = idx % E;
        float l = router_dot(router + e * (long)H, x + t * (long)H, H, order);
        if (bias) l = l + bias[e];
        logits[idx] = l;
    }
}

/* routes() (src/model/qwen35/moe.rs:51-67) + pruning::apply
 * (src/model/experts/pruning.rs:32-41). Returns 0, or -1 on invalid top-k. */
int oracle_routes(const float *logits, int T, int E, int k, float min_weight,
                  int32_t *ids, float *weights) {
    if (k <= 0 || k > E) return -1;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        const float *l = logits + (long)t * E;
        int32_t *id = ids + (long)t * k;
        float *w = weights + (long)t * k;
        /* k selection passes = the first k of the sort by (key desc, id asc). */
        for (int r = 0; r < k; ++r) {
            int best = -1;
            int32_t bk = 0;
            for (int e = 0; e < E; ++e) {
                int taken = 0;
                for (int q = 0; q < r; ++q) taken |= (id[q] == e);
                if (taken) continue;
                int32_t key = oracle_total_key(l[e]);
                if (best < 0 || key > bk) { best = e; bk = key; }
            }
            id[r] = best;
        }
        float max = l[id[0]];
        for (int r = 0; r < k; ++r) w[r] = expf(l[id[r]] - max);
        float sum = -0.0f;
        for (int r = 0; r < k; ++r) sum = sum + w[r];
        for (int r = 0; r < k; ++r) w[r] = w[r] / sum;
        if (min_weight != 0.0f)
            for (int r = 1; r < k; ++r)
                if (w[r] < min_weight) w[r] = 0.0f;
    }
    return 0;
}

/* Ling's grouped sigmoid routing, RoutingScratch::routes
 * (src/model/ling3tiny/moe.rs:146-223): score = sigmoid(logit), selected =
 * score + bias; a group's score is the sum of its two largest selected values
 * (total_cmp); the top_groups groups by (score desc, index asc) are enabled;
 * the k largest selected values among their experts, (selected desc, id asc),
 * in that order, are chosen; weight = score / (sum of chosen scores in chosen
 * order + 1e-20) for k > 1, else score, times routing_scale. Returns 0, or -1
 * for a geometry the reference's config check rejects
 * (src/model/ling3tiny/config.rs:113-124). */
int oracle_ling_routes(const float *logits, const float *bias, int T, int E, int groups,
                       int top_groups, int k, float routing_scale, int32_t *ids,
                       float *weights) {
    if (groups <= 0 || E % groups != 0 || E / groups < 2 || top_groups <= 0 ||
        top_groups > groups || k <= 0 || k > top_groups * (E / groups) || !(routing_scale > 0.0f))
        return -1;
    const int width = E / groups;
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (int t = 0; t < T; ++t) {
        const float *l = logits + (long)t * E;
        int32_t *id = ids + (long)t * k;
        float *w = weights + (long)t * k;
        float *score = (float *)malloc(sizeof(float) * (size_t)E);
        float *sel = (float *)malloc(sizeof(float) * (size_t)E);
        float *gscore = (float *)malloc(sizeof(float) * (size_t)groups);
        char *enabled = (char *)calloc((size_t)groups, 1);
        if (!score || !sel || !gscore || !enabled) { bad = 1; }
        else {
            for (int e = 0; e < E; ++e) {
                score[e] = oracle_sigmoid(l[e]);
                sel[e] = score[e] + bias[e];
            }
            for (int g = 0; g < groups; ++g) {
                const float *v = sel + (long)g * width;
                float first = v[0], second = v[1];
                if (oracle_total_key(second) > oracle_total_key(first)) {
                    float tmp = first; first = second; second = tmp;
                }
                for (int j = 2; j < width; ++j) {
                    if (oracle_total_key(v[j]) > oracle_total_key(first)) {
                        second = first;
                        first = v[j];
                    } else if (oracle_total_key(v[j]) > oracle_total_key(second)) {
                        second = v[j];
                    }
                }
                gscore[g] = first + second;
            }
            /* the top_groups groups of the order (score desc, index asc) */
            for (int r = 0; r < top_groups; ++r) {
                int best = -1;
                for (int g = 0; g < groups; ++g) {
                    if (enabled[g]) continue;
                    if (best < 0 || oracle_total_key(gscore[g]) > oracle_total_key(gscore[best]))
                        best = g;
                }
                enabled[best] = 1;
            }
            /* the first k of the order (selected desc, id asc) among enabled experts */
            for (int r = 0; r < k; ++r) {
                int best = -1;
                for (int e = 0; e < E; ++e) {
                    if (!enabled[e / width]) continue;
                    int taken = 0;
                    for (int q = 0; q < r; ++q) taken |= (id[q] == e);
                    if (taken) continue;
                    if (best < 0 || oracle_total_key(sel[e]) > oracle_total_key(sel[best]))
                        best = e;
                }
                id[r] = best;
            }
            float sum = -0.0f;
            for (int r = 0; r < k; ++r) sum = sum + score[id[r]];
            sum = sum + 1e-20f;
            for (int r = 0; r < k; ++r)
                w[r] = (k > 1 ? score[id[r]] / sum : score[id[r]]) * routing_scale;
        }
        free(score); free(sel); free(gscore); free(enabled);
    }
    return bad ? -1 : 0;
}

/* Grouping of assignments a = t*k + r by expert, ascending a inside a group;
 * assignments whose weight is not > 0 are skipped (src/model/experts/paged.rs:
 * 586-600 builds the jobs in assignment order and skips zero routes;
 * :495-506 combines only routes > 0). Returns the kept count, or -1 for an
 * expert id out of range. */
int oracle_permute(const int32_t *ids, const float *weights, int T, int k, int E,
                   int32_t *perm, int32_t *offsets) {
    long n = (long)T * k;
    int32_t *count = (int32_t *)calloc((size_t)E + 1, sizeof(int32_t));
    for (long a = 0; a < n; ++a) {
        if (!(weights[a] > 0.0f)) continue;
        if (ids[a] < 0 || ids[a] >= E) { free(count); return -1; }
        count[ids[a]]++;
    }
    offsets[0] = 0;
    for (int e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + count[e];
    for (int e = 0; e < E; ++e) count[e] = offsets[e];
    for (long a = 0; a < n; ++a)
        if (weights[a] > 0.0f) perm[count[ids[a]]++] = (int32_t)a;
    int kept = offsets[E];
    free(count);
    return kept;
}

/* Dynamic per-row symmetric int8 quantisation.
 * MOE rule (native MoE input and middle; llm_generated_docs/
 * MOE_CPU_FUSION_20261023.md:13): s = maxabs/127, q = round-half-even(x/s),
 * clamp +-127, all-zero row -> s = 1.
 * DENSE rule (dense W8A8/W4A8 Linear; llm_generated_docs/MODELS.md:26 and
 * QWEN3_W4A8_SWIGLU_MAXABS_FUSION_20261022.md): s = max(maxabs/127, FLT_MIN),
 * q = round-half-away(x * (1/s)), clamp +-127, all-zero row -> s = 1. */
void oracle_quantize(const float *x, int rows, int cols, int rule, int8_t *q, float *s) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const float *xr = x + (long)r * cols;
        float m = 0.0f;
        for (int c = 0; c < cols; ++c) {
            float a = fabsf(xr[c]);
            if (a > m) m = a;
        }
        float sc;
        if (m == 0.0f) {
            sc = 1.0f;
        } else {
            sc = m / 127.0f;
            if (rule == ORACLE_QUANT_DENSE && !(sc >= FLT_MIN)) sc = FLT_MIN;
        }
        s[r] = sc;
        float inv = 1.0f / sc;
        int8_t *qr = q + (long)r * cols;
        for (int c = 0; c < cols; ++c) {
            float v = rule == ORACLE_QUANT_MOE ? rintf(xr[c] / sc) : roundf(xr[c] * inv);
            if (v > 127.0f) v = 127.0f;
            if (v < -127.0f) v = -127.0f;
            qr[c] = (int8_t)v;
        }
    }
}

/* Integer accumulators of q[rows][K] x codes[K][N]. Per-channel: acc[rows][N]
 * over the full K (exact INT32, as the native library reconstructs its K
 * slices exactly: llm_generated_docs/MINICPMV47_35A3_FUSED_MOE_20261019.md:77).
 * Grouped: acc[rows][K/group][N], one INT32 sum per group. */
#define ROWB 8
void oracle_gemm_acc(const int8_t *q, int rows, const oracle_qmat *w, int32_t *acc) {
    const int K = w->k, N = w->n;
    const int G = w->group > 0 ? K / w->group : 1;
    const int gs = w->group > 0 ? w->group : K;
#pragma omp parallel for schedule(dynamic, 1)
    for (int r0 = 0; r0 < rows; r0 += ROWB) {
        int nr = rows - r0 < ROWB ? rows - r0 : ROWB;
        int32_t *tmp = (int32_t *)malloc(sizeof(int32_t) * (size_t)ROWB * N);
        for (int g = 0; g < G; ++g) {
            memset(tmp, 0, sizeof(int32_t) * (size_t)ROWB * N);
            for (int kk = g * gs; kk < (g + 1) * gs; ++kk) {
                const int8_t *wk = w->codes + (long)kk * N;
                for (int i = 0; i < nr; ++i) {
                    int32_t qv = q[(long)(r0 + i) * K + kk];
                    int32_t *t = tmp + (long)i * N;
                    for (int n = 0; n < N; ++n) t[n] += qv * (int32_t)wk[n];
                }
            }
            for (int i = 0; i < nr; ++i)
                memcpy(acc + ((long)(r0 + i) * G + g) * N, tmp + (long)i * N,
                       sizeof(int32_t) * (size_t)N);
        }
        free(tmp);
    }
}

/* Dequantised GEMM, out[rows][N] f32.
 * Per-channel: ((float)acc * s_x) * s_w[n]  (dequant order fixed here).
 * Grouped:     f = sum_g fmaf((float)acc_g, s_w[g][n], f) over ascending g,
 *              then f * s_x. */
static void gemm_dequant_rows(const int8_t *q, const float *s, int nr, int K,
                              const oracle_qmat *w, float *out, int32_t *tmp, float *facc) {
    const int N = w->n;
    if (w->group <= 0) {
        memset(tmp, 0, sizeof(int32_t) * (size_t)nr * N);
        for (int kk = 0; kk < K; ++kk) {
            const int8_t *wk = w->codes + (long)kk * N;
            for (int i = 0; i < nr; ++i) {
                int32_t qv = q[(long)i * K + kk];
                int32_t *t = tmp + (long)i * N;
                for (int n = 0; n < N; ++n) t[n] += qv * (int32_t)wk[n];
            }
        }
        for (int i = 0; i < nr; ++i)
            for (int n = 0; n < N; ++n) {
                float a = (float)tmp[(long)i * N + n] * s[i];
                out[(long)i * N + n] = a * w->scales[n];
            }
        return;
    }
    const int gs = w->group, G = K / gs;
    memset(facc, 0, sizeof(float) * (size_t)nr * N);
    for (int g = 0; g < G; ++g) {
        memset(tmp, 0, sizeof(int32_t) * (size_t)nr * N);
        for (int kk = g * gs; kk < (g + 1) * gs; ++kk) {
            const int8_t *wk = w->codes + (long)kk * N;
            for (int i = 0; i < nr; ++i) {
                int32_t qv = q[(long)i * K + kk];
                int32_t *t = tmp + (long)i * N;
                for (int n = 0; n < N; ++n) t[n] += qv * (int32_t)wk[n];
            }
        }
        const uint16_t *sg = w->gscales + (long)g * N;
        for (int i = 0; i < nr; ++i)
            for (int n = 0; n < N; ++n)
                facc[(long)i * N + n] = fmaf((float)tmp[(long)i * N + n],
                                             oracle_half_to_float(sg[n]), facc[(long)i * N + n]);
    }
    for (int i = 0; i < nr; ++i)
        for (int n = 0; n < N; ++n) out[(long)i * N + n] = facc[(long)i * N + n] * s[i];
}

void oracle_gemm_dequant(const int8_t *q, const float *s, int rows, const oracle_qmat *w,
                         float *out) {
    const int K = w->k, N = w->n;
#pragma omp parallel for schedule(dynamic, 1)
    for (int r0 = 0; r0 < rows; r0 += ROWB) {
        int nr = rows - r0 < ROWB ? rows - r0 : ROWB;
        int32_t *tmp = (int32_t *)malloc(sizeof(int32_t) * (size_t)ROWB * N);
        float *facc = (float *)malloc(sizeof(float) * (size_t)ROWB * N);
        gemm_dequant_rows(q + (long)r0 * K, s + r0, nr, K, w, out + (long)r0 * N, tmp, facc);
        free(tmp);
        free(facc);
    }
}

/* x86 SwiGLU of native/cpu_kernels/swiglu.cpp:23-25, with the gate/up split of
 * Cpu::swiglu (src/model/cpu.rs:269-294): gate = row[i], up = row[width+i]. */
void oracle_swiglu(const float *gu, int rows, int width, float *out) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r)
        for (int i = 0; i < width; ++i) {
            float g = gu[(long)r * 2 * width + i];
            float u = gu[(long)r * 2 * width + width + i];
            float d = 1.0f + expf(-g);
            out[(long)r * width + i] = (g / d) * u;
        }
}

/* rms_norm (src/ops/norm.rs:81-106): sequential sum of squares, then
 * 1/sqrt(mean + eps), y = (x*scale)*w (w or 1+w when zero-centred). */
void oracle_rms_norm(const float *x, const float *weight, int rows, int width, float eps,
                     int zero_centered, float *out) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const float *xr = x + (long)r * width;
        float sum = -0.0f;
        for (int i = 0; i < width; ++i) {
            float p = xr[i] * xr[i];
            sum = sum + p;
        }
        float scale = 1.0f / sqrtf(sum / (float)width + eps);
        for (int i = 0; i < width; ++i) {
            float wv = zero_centered ? 1.0f + weight[i] : weight[i];
            out[(long)r * width + i] = (xr[i] * scale) * wv;
        }
    }
}

/* One expert SwiGLU FFN over rows already quantised: gate/up -> SwiGLU ->
 * requantise (rule) -> down. */
static void expert_ffn(const int8_t *qx, const float *sx, int nr, const oracle_qmat *gu,
                       const oracle_qmat *dn, int rule, float *mid, int8_t *qm, float *sm,
                       float *y) {
    const int H = gu->k, I = dn->k;
    float *gub = (float *)malloc(sizeof(float) * (size_t)nr * 2 * I);
    int32_t *tmp = (int32_t *)malloc(sizeof(int32_t) * (size_t)nr * (2 * I > H ? 2 * I : H));
    float *facc = (float *)malloc(sizeof(float) * (size_t)nr * (2 * I > H ? 2 * I : H));
    gemm_dequant_rows(qx, sx, nr, H, gu, gub, tmp, facc);
    for (int r = 0; r < nr; ++r)
        for (int i = 0; i < I; ++i) {
            float g = gub[(long)r * 2 * I + i];
            float u = gub[(long)r * 2 * I + I + i];
            float d = 1.0f + expf(-g);
            mid[(long)r * I + i] = (g / d) * u;
        }
    /* row quantisation, serial here: the caller parallelises over row blocks */
    for (int r = 0; r < nr; ++r) {
        const float *xr = mid + (long)r * I;
        float m = 0.0f;
        for (int c = 0; c < I; ++c) { float a = fabsf(xr[c]); if (a > m) m = a; }
        float sc;
        if (m == 0.0f) sc = 1.0f;
        else { sc = m / 127.0f; if (rule == ORACLE_QUANT_DENSE && !(sc >= FLT_MIN)) sc = FLT_MIN; }
        sm[r] = sc;
        float inv = 1.0f / sc;
        for (int c = 0; c < I; ++c) {
            float v = rule == ORACLE_QUANT_MOE ? rintf(xr[c] / sc) : roundf(xr[c] * inv);
            if (v > 127.0f) v = 127.0f;
            if (v < -127.0f) v = -127.0f;
            qm[(long)r * I + c] = (int8_t)v;
        }
    }
    gemm_dequant_rows(qm, sm, nr, I, dn, y, tmp, facc);
    free(gub);
    free(tmp);
    free(facc);
}

typedef struct { int e, row0, nr; } job_t;

/* Moe::run semantics (src/npu/moe.rs:324-387 over the native call): caller
 * supplies ids/routes; output = weighted routed combine (+ shared expert). */
int oracle_moe_run(const oracle_layer *L, int T, const float *x, const int32_t *ids,
                   const float *weights, float *out, oracle_dump *dump) {
    const int H = L->hidden, I = L->inter, E = L->experts, k = L->top;
    long n = (long)T * k;
    int32_t *perm = (int32_t *)malloc(sizeof(int32_t) * (size_t)(n > 0 ? n : 1));
    int32_t *offsets = (int32_t *)malloc(sizeof(int32_t) * (size_t)(E + 1));
    int A = oracle_permute(ids, weights, T, k, E, perm, offsets);
    if (A < 0) { free(perm); free(offsets); return -1; }
    int8_t *qx = (int8_t *)malloc((size_t)T * H + 1);
    float *sx = (float *)malloc(sizeof(float) * (size_t)T + 4);
    oracle_quantize(x, T, H, ORACLE_QUANT_MOE, qx, sx);

    /* gather the quantised rows of every kept assignment in permuted order */
    int8_t *qa = (int8_t *)malloc((size_t)A * H + 1);
    float *sa = (float *)malloc(sizeof(float) * (size_t)A + 4);
    for (int p = 0; p < A; ++p) {
        int t = perm[p] / k;
        memcpy(qa + (long)p * H, qx + (long)t * H, (size_t)H);
        sa[p] = sx[t];
    }
    float *mid = (float *)malloc(sizeof(float) * (size_t)A * I + 4);
    int8_t *qm = (int8_t *)malloc((size_t)A * I + 1);
    float *sm = (float *)malloc(sizeof(float) * (size_t)A + 4);
    float *y = (float *)malloc(sizeof(float) * (size_t)A * H + 4);

    int njobs = 0;
    for (int e = 0; e < E; ++e) njobs += (offsets[e + 1] - offsets[e] + ROWB - 1) / ROWB;
    job_t *jobs = (job_t *)malloc(sizeof(job_t) * (size_t)(njobs + 1));
    njobs = 0;
    for (int e = 0; e < E; ++e)
        for (int r = offsets[e]; r < offsets[e + 1]; r += ROWB) {
            jobs[njobs].e = e;
            jobs[njobs].row0 = r;
            jobs[njobs].nr = offsets[e + 1] - r < ROWB ? offsets[e + 1] - r : ROWB;
            ++njobs;
        }
#pragma omp parallel for schedule(dynamic, 1)
    for (int j = 0; j < njobs; ++j) {
        job_t jb = jobs[j];
        expert_ffn(qa + (long)jb.row0 * H, sa + jb.row0, jb.nr, &L->gate_up[jb.e],
                   &L->down[jb.e], ORACLE_QUANT_MOE, mid + (long)jb.row0 * I,
                   qm + (long)jb.row0 * I, sm + jb.row0, y + (long)jb.row0 * H);
    }
    free(jobs);

    /* position of each assignment in the permuted order (-1 if skipped) */
    int32_t *pos = (int32_t *)malloc(sizeof(int32_t) * (size_t)(n > 0 ? n : 1));
    for (long a = 0; a < n; ++a) pos[a] = -1;
    for (int p = 0; p < A; ++p) pos[perm[p]] = p;

    /* combine in rank order (src/model/experts/paged.rs:495-506) */
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t)
        for (int c = 0; c < H; ++c) {
            float sum = 0.0f;
            for (int r = 0; r < k; ++r) {
                long a = (long)t * k + r;
                if (weights[a] > 0.0f) sum = fmaf(y[(long)pos[a] * H + c], weights[a], sum);
            }
            out[(long)t * H + c] = sum;
        }
    if (dump && dump->routed) memcpy(dump->routed, out, sizeof(float) * (size_t)T * H);

    /* shared expert: joint (MoE rules on the shared input quantisation,
     * llm_generated_docs/MOE_ROUTED_SHARED_JOINT_20261023.md:19) or a separate
     * dense FFN (src/model/ling3tiny/moe.rs:378-388 -> cpu.add). */
    if (L->shared_inter > 0 && L->shared_gate_up && L->shared_down) {
        const int Is = L->shared_inter;
        float *sh = (float *)malloc(sizeof(float) * (size_t)T * H + 4);
        int8_t *qs = qx;
        float *ss = sx;
        int rule = ORACLE_QUANT_MOE;
        if (L->shared_mode == ORACLE_SHARED_DENSE) {
            rule = ORACLE_QUANT_DENSE;
            qs = (int8_t *)malloc((size_t)T * H + 1);
            ss = (float *)malloc(sizeof(float) * (size_t)T + 4);
            oracle_quantize(x, T, H, ORACLE_QUANT_DENSE, qs, ss);
        }
        float *smid = (float *)malloc(sizeof(float) * (size_t)T * Is + 4);
        int8_t *sqm = (int8_t *)malloc((size_t)T * Is + 1);
        float *ssm = (float *)malloc(sizeof(float) * (size_t)T + 4);
#pragma omp parallel for schedule(dynamic, 1)
        for (int r0 = 0; r0 < T; r0 += ROWB) {
            int nr = T - r0 < ROWB ? T - r0 : ROWB;
            expert_ffn(qs + (long)r0 * H, ss + r0, nr, L->shared_gate_up, L->shared_down, rule,
                       smid + (long)r0 * Is, sqm + (long)r0 * Is, ssm + r0, sh + (long)r0 * H);
        }
        if (L->shared_gate) {
            /* the gate merge of src/model/qwen35/moe.rs:334-347: gate = dense_head
             * of the [1][hidden] gate row (the router's dot order), scale =
             * 1 / (1 + exp(-gate)), projected += scale * attended */
#pragma omp parallel for schedule(static)
            for (int t = 0; t < T; ++t) {
                float g = router_dot(L->shared_gate, x + (long)t * H, H, L->router_order);
                float scale = 1.0f / (1.0f + expf(-g));
                if (dump && dump->shared_scale) dump->shared_scale[t] = scale;
                for (int c = 0; c < H; ++c) {
                    long i = (long)t * H + c;
                    float p = scale * sh[i];
                    out[i] = out[i] + p;
                }
            }
        } else {
            for (long i = 0; i < (long)T * H; ++i) out[i] = out[i] + sh[i];
        }
        if (dump && dump->shared) memcpy(dump->shared, sh, sizeof(float) * (size_t)T * H);
        if (qs != qx) { free(qs); free(ss); }
        free(smid); free(sqm); free(ssm); free(sh);
    }

    if (dump) {
        dump->n_assign = A;
        if (dump->perm) memcpy(dump->perm, perm, sizeof(int32_t) * (size_t)A);
        if (dump->offsets) memcpy(dump->offsets, offsets, sizeof(int32_t) * (size_t)(E + 1));
        if (dump->qx) memcpy(dump->qx, qx, (size_t)T * H);
        if (dump->sx) memcpy(dump->sx, sx, sizeof(float) * (size_t)T);
        if (dump->middle) memcpy(dump->middle, mid, sizeof(float) * (size_t)A * I);
        if (dump->qm) memcpy(dump->qm, qm, (size_t)A * I);
        if (dump->sm) memcpy(dump->sm, sm, sizeof(float) * (size_t)A);
        if (dump->y) memcpy(dump->y, y, sizeof(float) * (size_t)A * H);
    }
    free(pos); free(perm); free(offsets); free(qx); free(sx); free(qa); free(sa);
    free(mid); free(qm); free(sm); free(y);
    return 0;
}

/* Routed::forward + the decoder residual (src/model/qwen35/moe.rs:188-226,
 * src/model/qwen35/decoder.rs:215-217): router -> routes -> run ->
 * out = residual + projected (residual may be NULL). With the grouped sigmoid
 * rule the routes are Ling's (FeedForward::run, src/model/ling3tiny/
 * moe.rs:354-394: router projection, routes per row, bank run, + shared). */
int oracle_moe_forward(const oracle_layer *L, int T, const float *x, const float *residual,
                       float *out, oracle_dump *dump) {
    const int E = L->experts, k = L->top, H = L->hidden;
    float *logits = (float *)malloc(sizeof(float) * (size_t)T * E + 4);
    int32_t *ids = (int32_t *)malloc(sizeof(int32_t) * (size_t)T * k + 4);
    float *w = (float *)malloc(sizeof(float) * (size_t)T * k + 4);
    oracle_router_logits(x, L->router, L->router_bias, T, H, E, L->router_order, logits);
    int rc = L->route_rule == ORACLE_ROUTE_GROUPED_SIGMOID
                 ? oracle_ling_routes(logits, L->expert_bias, T, E, L->groups, L->top_groups, k,
                                      L->routing_scale, ids, w)
                 : oracle_routes(logits, T, E, k, L->min_weight, ids, w);
    if (rc == 0) rc = oracle_moe_run(L, T, x, ids, w, out, dump);
    if (rc == 0 && residual)
        for (long i = 0; i < (long)T * H; ++i) out[i] = residual[i] + out[i];
    if (dump) {
        if (dump->logits) memcpy(dump->logits, logits, sizeof(float) * (size_t)T * E);
        if (dump->ids) memcpy(dump->ids, ids, sizeof(int32_t) * (size_t)T * k);
        if (dump->weights) memcpy(dump->weights, w, sizeof(float) * (size_t)T * k);
    }
    free(logits); free(ids); free(w);
    return rc;
}
