/*
 * laya_oracle.c -- CPU restatement of the reference forward pass.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the oracle the CUDA path is checked
 * against, and the timed CPU baseline beside the GPU numbers. Nothing in the
 * product (the CUDA library, its C ABI or the host package) links, loads or
 * calls it; only tests/, the smoke check and bench.py's CPU-baseline leg do.
 *
 * It restates laya-zig's `forward()` (src/main.zig:2641-2817) in C, keeping
 * the reference's order of operations and arithmetic:
 *   - f32 everywhere, F16/BF16 weights widened exactly to f32;
 *   - the packed 16-column GEMM: per 384-deep k-chunk one sequential FMA
 *     chain per output, chunk results added into `out`
 *     (src/main.zig:910-1018, linear16 1088-1099, bias 1073-1079);
 *   - two-pass LayerNorm (83-95); scalar erf/gelu by Abramowitz-Stegun 7.1.26
 *     (60-70); softmax (72-81);
 *   - expv (range reduction + 7th-order Taylor) and geluv (595-630), used by
 *     the encoder GLU and the attention softmax;
 *   - attention (2419-2489): dot64 summation shape, expv over 8-key blocks
 *     and exp on the tail, weights below 1e-20 skipped, normalised after PV;
 *   - RoPE with rotate-half pairing and f32 cos/sin of inv_freq*pos
 *     (2491-2521; inv_freq 2399-2401), theta 160000 on every encoder layer;
 *   - head layers, scorer and act/escalate head (2714-2814).
 * Compile with -ffp-contract=off: the Zig build evaluates a*b+c as two
 * roundings unless it says @mulAdd, and so does this file (fmaf / FMA
 * intrinsics appear exactly where the reference has @mulAdd).
 *
 * Vector reductions (`@reduce(.Add, v)`) are summed lane 0..7 in order.
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#define LO_AVX2 1
#endif

#define D 768
#define H 12
#define HD 64
#define NL 22
#define INTER 1152
#define HEAD_LAYERS 2
#define HEAD_FF (4 * D)
#define WINDOW 64
#define VOCAB 256000
#define PN 16
#define PKC 384
static const float EPS = 1e-5f;
static const float ROPE_THETA = 160000.0f;

enum { LO_F32 = 0, LO_F16 = 1, LO_BF16 = 2 };

typedef struct {
    const char* name;
    int dtype;
    const void* data;
    uint64_t numel;
} lo_tensor;

/* A weight matrix as the file holds it: raw 16-bit elements plus their tag. */
typedef struct {
    const uint16_t* p;
    int dtype;
} mat16;

typedef struct {
    mat16 wqkv, wo, wi, wo2;
    float* attn_norm; /* NULL at layer 0 */
    float* mlp_norm;
    int sliding;
} enc_layer;

typedef struct {
    float *norm1_w, *norm1_b, *norm2_w, *norm2_b;
    mat16 in_w;
    float* in_b;
    mat16 out_w;
    float* out_b;
    mat16 l1_w;
    float* l1_b;
    mat16 l2_w;
    float* l2_b;
} head_layer;

typedef struct {
    mat16 emb;
    float *emb_norm, *final_norm, *type_emb;
    enc_layer layers[NL];
    head_layer head[HEAD_LAYERS];
    float *s0w, *s0b, *s1w, *s1b, *s3w, *s3b, *a0w, *a0b, *a2w, *a2b;
    float inv_freq[32];
    float* owned[128];
    int n_owned;
} lo_model;

/* ------------------------------------------------------------------ widening */
static inline float f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ff, u;
    if (e == 0) {
        if (m == 0) {
            u = s;
        } else { /* subnormal */
            int sh = 0;
            while (!(m & 0x400)) { m <<= 1; sh++; }
            m &= 0x3ff;
            u = s | ((uint32_t)(113 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        u = s | 0x7f800000u | (m << 13);
    } else {
        u = s | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline float w16(const mat16* m, size_t i) {
    return m->dtype == LO_F16 ? f16_to_f32(m->p[i]) : bf16_to_f32(m->p[i]);
}

/* ------------------------------------------------------------------ scalar math
 * src/main.zig:60-95 */
static float lo_erf(float x) {
    const float s = x < 0 ? -1.0f : 1.0f;
    const float a = fabsf(x);
    const float t = 1.0f / (1.0f + 0.3275911f * a);
    const float poly = ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
    return s * (1.0f - poly * expf(-a * a));
}

float lo_gelu(float x) { return 0.5f * x * (1.0f + lo_erf(x * 0.70710678118654752440f)); }

static void softmax(float* x, int n) {
    float mx = -INFINITY;
    for (int i = 0; i < n; i++) mx = fmaxf(mx, x[i]);
    float sum = 0;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

static void layer_norm(float* x, const float* w, const float* b) {
    const float n = (float)D;
    float mean = 0;
    for (int i = 0; i < D; i++) mean += x[i];
    mean /= n;
    float varr = 0;
    for (int i = 0; i < D; i++) {
        const float d = x[i] - mean;
        varr += d * d;
    }
    varr = 1.0f / sqrtf(varr / n + EPS);
    for (int i = 0; i < D; i++) x[i] = (x[i] - mean) * varr * w[i] + (b ? b[i] : 0.0f);
}

/* ------------------------------------------------------------------ vector math
 * src/main.zig:595-630, one lane at a time. */
static inline float expv1(float x) {
    const float c = fmaxf(fminf(x, 88.0f), -87.0f);
    const float n = roundf(c * 1.4426950408889634f);
    const int32_t ni = (int32_t)n;
    const uint32_t sb = (uint32_t)(ni + 127) * 0x800000u;
    float scale;
    memcpy(&scale, &sb, 4);
    const float r = c - n * 0.6931471805599453f;
    float p = (float)(1.0 / 5040.0);
    p = fmaf(p, r, (float)(1.0 / 720.0));
    p = fmaf(p, r, (float)(1.0 / 120.0));
    p = fmaf(p, r, (float)(1.0 / 24.0));
    p = fmaf(p, r, (float)(1.0 / 6.0));
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return p * scale;
}

static inline float geluv1(float x) {
    const float ax = fabsf(x);
    const float a = ax * 0.7071067811865476f;
    const float t = 1.0f / (1.0f + a * 0.3275911f);
    float p = 1.061405429f;
    p = fmaf(p, t, -1.453152027f);
    p = fmaf(p, t, 1.421413741f);
    p = fmaf(p, t, -0.284496736f);
    p = fmaf(p, t, 0.254829592f);
    const float e = 1.0f - (p * t) * expv1(0.0f - a * a);
    return 0.5f * (x + ax * e);
}

void lo_expv(const float* x, float* out, int n) {
    for (int i = 0; i < n; i++) out[i] = expv1(x[i]);
}

void lo_geluv(const float* x, float* out, int n) {
    for (int i = 0; i < n; i++) out[i] = geluv1(x[i]);
}

void lo_gelu_n(const float* x, float* out, int n) {
    for (int i = 0; i < n; i++) out[i] = lo_gelu(x[i]);
}

static inline float hsum8(const float* v) {
    float s = v[0];
    for (int i = 1; i < 8; i++) s += v[i];
    return s;
}

/* dotv / dotvw (src/main.zig:382-400, 585-593): two 8-lane accumulators over
 * 16-wide steps, one more 8-wide step, scalar tail, tail + reduce(a0 + a1). */
static float dotv(const float* a, const float* b, int n) {
    float a0[8] = {0}, a1[8] = {0};
    int i = 0;
    for (; i + 16 <= n; i += 16)
        for (int l = 0; l < 8; l++) {
            a0[l] = fmaf(a[i + l], b[i + l], a0[l]);
            a1[l] = fmaf(a[i + 8 + l], b[i + 8 + l], a1[l]);
        }
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) a0[l] = fmaf(a[i + l], b[i + l], a0[l]);
    float s = 0;
    for (; i < n; i++) s += a[i] * b[i];
    float t[8];
    for (int l = 0; l < 8; l++) t[l] = a0[l] + a1[l];
    return s + hsum8(t);
}

/* ------------------------------------------------------------------ packed GEMM
 * out[i][j] = sum_k x[i][k] * w[j][k]; src/main.zig:910-1018. */
/* panel[t*PN + c] = w[(jg+c)*k + kb + t]: 16 weight rows widened to f32 and
 * stored k-major (packPanel, src/main.zig:910-927). Widening is exact, so the
 * loop order here does not affect any value. */
static void pack_panel(float* panel, const mat16* w, int k, int jg, int kb, int kc) {
    for (int c = 0; c < PN; c++) {
        const uint16_t* row = w->p + (size_t)(jg + c) * k + kb;
        if (w->dtype == LO_BF16) {
            for (int t = 0; t < kc; t++) {
                const uint32_t u = (uint32_t)row[t] << 16;
                memcpy(&panel[t * PN + c], &u, 4);
            }
        } else {
            for (int t = 0; t < kc; t++) panel[t * PN + c] = f16_to_f32(row[t]);
        }
    }
}

static void micro_kernel(int mr, const float* panel, const float* x, float* out, int n, int k, int ib, int jg, int kb,
                         int kc, int accumulate) {
#ifdef LO_AVX2
    __m256 acc[6][2];
    for (int i = 0; i < mr; i++) acc[i][0] = acc[i][1] = _mm256_setzero_ps();
    for (int t = 0; t < kc; t++) {
        const __m256 b0 = _mm256_loadu_ps(panel + t * PN), b1 = _mm256_loadu_ps(panel + t * PN + 8);
        for (int i = 0; i < mr; i++) {
            const __m256 a = _mm256_set1_ps(x[(size_t)(ib + i) * k + kb + t]);
            acc[i][0] = _mm256_fmadd_ps(a, b0, acc[i][0]);
            acc[i][1] = _mm256_fmadd_ps(a, b1, acc[i][1]);
        }
    }
    for (int i = 0; i < mr; i++) {
        float* o = out + (size_t)(ib + i) * n + jg;
        if (accumulate) {
            _mm256_storeu_ps(o, _mm256_add_ps(_mm256_loadu_ps(o), acc[i][0]));
            _mm256_storeu_ps(o + 8, _mm256_add_ps(_mm256_loadu_ps(o + 8), acc[i][1]));
        } else {
            _mm256_storeu_ps(o, acc[i][0]);
            _mm256_storeu_ps(o + 8, acc[i][1]);
        }
    }
#else
    float acc[6][PN];
    for (int i = 0; i < mr; i++)
        for (int c = 0; c < PN; c++) acc[i][c] = 0.0f;
    for (int t = 0; t < kc; t++)
        for (int i = 0; i < mr; i++) {
            const float a = x[(size_t)(ib + i) * k + kb + t];
            for (int c = 0; c < PN; c++) acc[i][c] = fmaf(a, panel[t * PN + c], acc[i][c]);
        }
    for (int i = 0; i < mr; i++) {
        float* o = out + (size_t)(ib + i) * n + jg;
        for (int c = 0; c < PN; c++) o[c] = accumulate ? o[c] + acc[i][c] : acc[i][c];
    }
#endif
}

static void linear16(float* out, const float* x, const mat16* w, const float* bias, int rows, int n, int k, int nt) {
    const int nblk = n / PN;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
    for (int b = 0; b < nblk; b++) {
        float panel[PN * PKC];
        const int jg = b * PN;
        for (int kb = 0; kb < k; kb += PKC) {
            const int kc = k - kb < PKC ? k - kb : PKC;
            pack_panel(panel, w, k, jg, kb, kc);
            const int acc = kb != 0;
            int i = 0;
            for (; i + 6 <= rows; i += 6) micro_kernel(6, panel, x, out, n, k, i, jg, kb, kc, acc);
            for (; i + 4 <= rows; i += 4) micro_kernel(4, panel, x, out, n, k, i, jg, kb, kc, acc);
            for (; i + 2 <= rows; i += 2) micro_kernel(2, panel, x, out, n, k, i, jg, kb, kc, acc);
            for (; i < rows; i++) micro_kernel(1, panel, x, out, n, k, i, jg, kb, kc, acc);
        }
    }
    if (n % PN) { /* packTail (src/main.zig:1002-1012): per-column dotvw */
        const int jlo = n / PN * PN;
        float* wr = (float*)malloc(sizeof(float) * k);
        for (int jj = jlo; jj < n; jj++) {
            for (int t = 0; t < k; t++) wr[t] = w16(w, (size_t)jj * k + t);
            for (int i = 0; i < rows; i++) out[(size_t)i * n + jj] = dotv(x + (size_t)i * k, wr, k);
        }
        free(wr);
    }
    if (bias) {
#pragma omp parallel for num_threads(nt)
        for (int i = 0; i < rows; i++)
            for (int j = 0; j < n; j++) out[(size_t)i * n + j] += bias[j];
    }
}

/* The packed GEMM on its own, for the --selftest known-answer checks
 * (src/main.zig:420-536). w is F16/BF16 [n][k]. */
void lo_linear16(float* out, const float* x, const uint16_t* w, int wdtype, const float* bias, int rows, int n, int k,
                 int nt) {
    mat16 m = {w, wdtype};
    linear16(out, x, &m, bias, rows, n, k, nt);
}

/* ------------------------------------------------------------------ attention
 * src/main.zig:2419-2489 */
static float dot64(const float* a, const float* b) {
    float a0[8], a1[8], a2[8], a3[8], t[8];
    for (int l = 0; l < 8; l++) {
        a0[l] = a[l] * b[l];
        a1[l] = a[8 + l] * b[8 + l];
        a2[l] = a[16 + l] * b[16 + l];
        a3[l] = a[24 + l] * b[24 + l];
    }
    for (int l = 0; l < 8; l++) {
        a0[l] = fmaf(a[32 + l], b[32 + l], a0[l]);
        a1[l] = fmaf(a[40 + l], b[40 + l], a1[l]);
        a2[l] = fmaf(a[48 + l], b[48 + l], a2[l]);
        a3[l] = fmaf(a[56 + l], b[56 + l], a3[l]);
    }
    for (int l = 0; l < 8; l++) t[l] = (a0[l] + a1[l]) + (a2[l] + a3[l]);
    return hsum8(t);
}

static void attention(const float* q, const float* k, const float* v, float* out, int L, int win, int nt) {
    const float scale = 1.0f / sqrtf((float)HD);
#pragma omp parallel num_threads(nt)
    {
        float* rowp = (float*)malloc(sizeof(float) * (L > 2 * WINDOW + 1 ? L : 2 * WINDOW + 1));
#pragma omp for schedule(dynamic, 4)
        for (int i = 0; i < L; i++) {
            float* row = out + (size_t)i * D;
            int klo = 0, khi = L;
            if (win >= 0) {
                klo = i >= win ? i - win : 0;
                khi = i + win + 1 < L ? i + win + 1 : L;
            }
            const int cnt = khi - klo;
            for (int h = 0; h < H; h++) {
                const float* qi = q + (size_t)i * D + h * HD;
                float mx = -INFINITY;
                for (int j = klo; j < khi; j++) {
                    const float s = dot64(qi, k + (size_t)j * D + h * HD) * scale;
                    rowp[j - klo] = s;
                    mx = fmaxf(mx, s);
                }
                float sv[8] = {0};
                int tv = 0;
                for (; tv + 8 <= cnt; tv += 8)
                    for (int l = 0; l < 8; l++) {
                        const float e = expv1(rowp[tv + l] - mx);
                        rowp[tv + l] = e;
                        sv[l] += e;
                    }
                float sum = hsum8(sv);
                for (; tv < cnt; tv++) {
                    const float e = expf(rowp[tv] - mx);
                    rowp[tv] = e;
                    sum += e;
                }
                const float inv = 1.0f / sum;
                float r[HD];
                for (int c = 0; c < HD; c++) r[c] = 0.0f;
                for (int t = 0; t < cnt; t++) {
                    const float p = rowp[t];
                    if (p < 1e-20f) continue;
                    const float* vr = v + (size_t)(klo + t) * D + h * HD;
                    for (int c = 0; c < HD; c++) r[c] = fmaf(p, vr[c], r[c]);
                }
                for (int c = 0; c < HD; c++) row[h * HD + c] = r[c] * inv;
            }
        }
        free(rowp);
    }
}

/* src/main.zig:2496-2521 */
static void rope(float* x, int L, const float* inv, int nt) {
#pragma omp parallel for num_threads(nt)
    for (int p = 0; p < L; p++) {
        const float pos = (float)p;
        float cs[64], sn[64];
        for (int j = 0; j < 32; j++) {
            const float f = inv[j] * pos;
            cs[j] = cosf(f);
            sn[j] = sinf(f);
            cs[j + 32] = cs[j];
            sn[j + 32] = sn[j];
        }
        for (int h = 0; h < H; h++) {
            float* b = x + (size_t)p * D + h * HD;
            for (int d = 0; d < 32; d++) {
                const float x0 = b[d], x1 = b[d + 32];
                b[d] = x0 * cs[d] - x1 * sn[d];
                b[d + 32] = x1 * cs[d + 32] + x0 * sn[d + 32];
            }
        }
    }
}

/* ------------------------------------------------------------------ model */
static const lo_tensor* find(const lo_tensor* t, int n, const char* name) {
    for (int i = 0; i < n; i++)
        if (strcmp(t[i].name, name) == 0) return &t[i];
    return NULL;
}

static int get_mat(lo_model* m, const lo_tensor* t, int n, const char* name, uint64_t numel, mat16* out, char* err,
                   int errlen) {
    (void)m;
    const lo_tensor* e = find(t, n, name);
    if (!e) return snprintf(err, errlen, "missing tensor: %s", name), -1;
    if (e->dtype != LO_F16 && e->dtype != LO_BF16) return snprintf(err, errlen, "tensor %s: dtype %d", name, e->dtype), -2;
    if (e->numel != numel) return snprintf(err, errlen, "tensor %s: %llu elements", name, (unsigned long long)e->numel), -3;
    out->p = (const uint16_t*)e->data;
    out->dtype = e->dtype;
    return 0;
}

static float* get_f32(lo_model* m, const lo_tensor* t, int n, const char* name, uint64_t numel, char* err, int errlen) {
    const lo_tensor* e = find(t, n, name);
    if (!e) return snprintf(err, errlen, "missing tensor: %s", name), (float*)NULL;
    if (e->numel != numel) return snprintf(err, errlen, "tensor %s: %llu elements", name, (unsigned long long)e->numel), (float*)NULL;
    float* o = (float*)malloc(sizeof(float) * numel);
    for (uint64_t i = 0; i < numel; i++) {
        if (e->dtype == LO_F32) o[i] = ((const float*)e->data)[i];
        else if (e->dtype == LO_F16) o[i] = f16_to_f32(((const uint16_t*)e->data)[i]);
        else o[i] = bf16_to_f32(((const uint16_t*)e->data)[i]);
    }
    m->owned[m->n_owned++] = o;
    return o;
}

void lo_destroy(void* h) {
    lo_model* m = (lo_model*)h;
    if (!m) return;
    for (int i = 0; i < m->n_owned; i++) free(m->owned[i]);
    free(m);
}

/* loadModel (src/main.zig:2311-2404): matrices stay views, small tensors
 * become f32 copies. Returns NULL and fills err on a missing or mistyped
 * tensor. */
void* lo_create(const lo_tensor* t, int n, char* err, int errlen) {
    lo_model* m = (lo_model*)calloc(1, sizeof(lo_model));
    char nm[160];
#define MAT(dst, name, numel) \
    if (get_mat(m, t, n, name, numel, &(dst), err, errlen)) goto fail
#define VEC(dst, name, numel) \
    if (!((dst) = get_f32(m, t, n, name, numel, err, errlen))) goto fail
    MAT(m->emb, "encoder.embeddings.tok_embeddings.weight", (uint64_t)VOCAB * D);
    VEC(m->emb_norm, "encoder.embeddings.norm.weight", D);
    VEC(m->final_norm, "encoder.final_norm.weight", D);
    VEC(m->type_emb, "type_emb.weight", 3 * D);
    for (int l = 0; l < NL; l++) {
        enc_layer* e = &m->layers[l];
        if (l > 0) {
            snprintf(nm, sizeof nm, "encoder.layers.%d.attn_norm.weight", l);
            VEC(e->attn_norm, nm, D);
        }
        snprintf(nm, sizeof nm, "encoder.layers.%d.attn.Wqkv.weight", l);
        MAT(e->wqkv, nm, 3 * D * D);
        snprintf(nm, sizeof nm, "encoder.layers.%d.attn.Wo.weight", l);
        MAT(e->wo, nm, D * D);
        snprintf(nm, sizeof nm, "encoder.layers.%d.mlp.Wi.weight", l);
        MAT(e->wi, nm, 2 * INTER * D);
        snprintf(nm, sizeof nm, "encoder.layers.%d.mlp.Wo.weight", l);
        MAT(e->wo2, nm, D * INTER);
        snprintf(nm, sizeof nm, "encoder.layers.%d.mlp_norm.weight", l);
        VEC(e->mlp_norm, nm, D);
        e->sliding = (l % 3) != 0; /* src/main.zig:2366 */
    }
    for (int l = 0; l < HEAD_LAYERS; l++) {
        head_layer* h = &m->head[l];
#define HN(s) (snprintf(nm, sizeof nm, "head.layers.%d." s, l), nm)
        VEC(h->norm1_w, HN("norm1.weight"), D);
        VEC(h->norm1_b, HN("norm1.bias"), D);
        VEC(h->norm2_w, HN("norm2.weight"), D);
        VEC(h->norm2_b, HN("norm2.bias"), D);
        MAT(h->in_w, HN("self_attn.in_proj_weight"), 3 * D * D);
        VEC(h->in_b, HN("self_attn.in_proj_bias"), 3 * D);
        MAT(h->out_w, HN("self_attn.out_proj.weight"), D * D);
        VEC(h->out_b, HN("self_attn.out_proj.bias"), D);
        MAT(h->l1_w, HN("linear1.weight"), HEAD_FF * D);
        VEC(h->l1_b, HN("linear1.bias"), HEAD_FF);
        MAT(h->l2_w, HN("linear2.weight"), D * HEAD_FF);
        VEC(h->l2_b, HN("linear2.bias"), D);
#undef HN
    }
    VEC(m->s0w, "scorer.0.weight", D);
    VEC(m->s0b, "scorer.0.bias", D);
    VEC(m->s1w, "scorer.1.weight", D * D);
    VEC(m->s1b, "scorer.1.bias", D);
    VEC(m->s3w, "scorer.3.weight", D);
    VEC(m->s3b, "scorer.3.bias", 1);
    VEC(m->a0w, "act_head.0.weight", 256 * (D + 4));
    VEC(m->a0b, "act_head.0.bias", 256);
    VEC(m->a2w, "act_head.2.weight", 2 * 256);
    VEC(m->a2b, "act_head.2.bias", 2);
    for (int j = 0; j < 32; j++) m->inv_freq[j] = 1.0f / powf(ROPE_THETA, (float)j / 32.0f);
    return m;
fail:
    lo_destroy(m);
    return NULL;
#undef MAT
#undef VEC
}

/* ------------------------------------------------------------------ forward */
static void norm_into(const float* x, float* xn, int L, const float* w, const float* b, int nt) {
#pragma omp parallel for num_threads(nt)
    for (int i = 0; i < L; i++) {
        memcpy(xn + (size_t)i * D, x + (size_t)i * D, sizeof(float) * D);
        layer_norm(xn + (size_t)i * D, w, b);
    }
}

static void add_res(float* x, const float* xn, int L, int nt) {
#pragma omp parallel for num_threads(nt)
    for (int i = 0; i < L * D; i++) x[i] += xn[i];
}

static void split_qkv(float* q, float* k, float* v, const float* qkv, int L) {
    for (int i = 0; i < L; i++) {
        memcpy(q + (size_t)i * D, qkv + (size_t)i * 3 * D, sizeof(float) * D);
        memcpy(k + (size_t)i * D, qkv + (size_t)i * 3 * D + D, sizeof(float) * D);
        memcpy(v + (size_t)i * D, qkv + (size_t)i * 3 * D + 2 * D, sizeof(float) * D);
    }
}

static void stats(double* st, int tag, const float* x, int L, float* trace) {
    if (st) {
        double s = 0, a = 0;
        for (size_t i = 0; i < (size_t)L * D; i++) {
            s += x[i];
            a += fabs((double)x[i]);
        }
        double* o = st + tag * 5;
        o[0] = x[0];
        o[1] = L * D > 1 ? x[1] : 0;
        o[2] = L * D > 2 ? x[2] : 0;
        o[3] = s;
        o[4] = a;
    }
    if (trace) memcpy(trace + (size_t)tag * L * D, x, sizeof(float) * L * D);
}

/* Tags in `stats`/`trace` order: 0 emb, 1..22 l0..l21, 23 final, 24 temb,
 * 25 h0, 26 h1 (the reference's --dumpstats tags, src/main.zig:2651-2753). */
int lo_forward(void* h, const uint32_t* ids, int L, int qtype, const uint32_t* markers, int K, float* logits,
               float* act, float* pooled, float* hidden, double* st, float* trace, int nt) {
    const lo_model* m = (const lo_model*)h;
    if (!m || L <= 0 || qtype < 0 || qtype > 2) return -1;
    for (int i = 0; i < L; i++)
        if (ids[i] >= VOCAB) return -2;
    for (int r = 0; r < K; r++)
        if ((int)markers[r] >= L) return -3;
    if (nt <= 0) nt = 1;
    const size_t LD = (size_t)L * D;
    float* x = (float*)malloc(sizeof(float) * LD);
    float* xn = (float*)malloc(sizeof(float) * LD);
    float* q = (float*)malloc(sizeof(float) * LD);
    float* k = (float*)malloc(sizeof(float) * LD);
    float* v = (float*)malloc(sizeof(float) * LD);
    float* ctx = (float*)malloc(sizeof(float) * LD);
    float* qkv = (float*)malloc(sizeof(float) * LD * 3);
    float* mlp = (float*)malloc(sizeof(float) * (size_t)L * 2 * INTER);
    float* mlp2 = (float*)malloc(sizeof(float) * (size_t)L * INTER);
    float* ff = (float*)malloc(sizeof(float) * (size_t)L * HEAD_FF);

    /* embeddings + norm (embedJob 2543-2550, normJob 2552-2555) */
#pragma omp parallel for num_threads(nt)
    for (int i = 0; i < L; i++) {
        for (int d = 0; d < D; d++) x[(size_t)i * D + d] = w16(&m->emb, (size_t)ids[i] * D + d);
        layer_norm(x + (size_t)i * D, m->emb_norm, NULL);
    }
    stats(st, 0, x, L, trace);

    for (int l = 0; l < NL; l++) {
        const enc_layer* e = &m->layers[l];
        const float* attn_in = x;
        if (e->attn_norm) {
            norm_into(x, xn, L, e->attn_norm, NULL, nt);
            attn_in = xn;
        }
        linear16(qkv, attn_in, &e->wqkv, NULL, L, 3 * D, D, nt);
        split_qkv(q, k, v, qkv, L);
        rope(q, L, m->inv_freq, nt);
        rope(k, L, m->inv_freq, nt);
        attention(q, k, v, ctx, L, e->sliding ? WINDOW : -1, nt);
        linear16(xn, ctx, &e->wo, NULL, L, D, D, nt);
        add_res(x, xn, L, nt);
        norm_into(x, xn, L, e->mlp_norm, NULL, nt);
        linear16(mlp, xn, &e->wi, NULL, L, 2 * INTER, D, nt);
        /* mlpJob (2557-2569): INTER is a multiple of 8, so geluv covers it */
#pragma omp parallel for num_threads(nt)
        for (int i = 0; i < L; i++) {
            const float* mi = mlp + (size_t)i * 2 * INTER;
            float* o = mlp2 + (size_t)i * INTER;
            for (int j = 0; j < INTER; j++) o[j] = geluv1(mi[j]) * mi[j + INTER];
        }
        linear16(xn, mlp2, &e->wo2, NULL, L, D, INTER, nt);
        add_res(x, xn, L, nt);
        stats(st, 1 + l, x, L, trace);
    }

    for (int i = 0; i < L; i++) layer_norm(x + (size_t)i * D, m->final_norm, NULL);
    stats(st, 23, x, L, trace);
    {
        const float* te = m->type_emb + (size_t)qtype * D; /* typeEmbJob 2610-2617 */
        for (int i = 0; i < L; i++)
            for (int d = 0; d < D; d++) x[(size_t)i * D + d] += te[d];
    }
    stats(st, 24, x, L, trace);

    for (int l = 0; l < HEAD_LAYERS; l++) {
        const head_layer* hl = &m->head[l];
        norm_into(x, xn, L, hl->norm1_w, hl->norm1_b, nt);
        linear16(qkv, xn, &hl->in_w, hl->in_b, L, 3 * D, D, nt);
        split_qkv(q, k, v, qkv, L);
        attention(q, k, v, ctx, L, -1, nt);
        linear16(xn, ctx, &hl->out_w, hl->out_b, L, D, D, nt);
        add_res(x, xn, L, nt);
        norm_into(x, xn, L, hl->norm2_w, hl->norm2_b, nt);
        linear16(ff, xn, &hl->l1_w, hl->l1_b, L, HEAD_FF, D, nt);
        for (size_t i = 0; i < (size_t)L * HEAD_FF; i++) ff[i] = ff[i] > 0 ? ff[i] : 0; /* reluJob */
        linear16(xn, ff, &hl->l2_w, hl->l2_b, L, D, HEAD_FF, nt);
        add_res(x, xn, L, nt);
        stats(st, 25 + l, x, L, trace);
    }

    memcpy(pooled, x, sizeof(float) * D);

    /* scorer (2759-2769) */
    for (int r = 0; r < K; r++) {
        float mv[D], h1[D];
        memcpy(mv, x + (size_t)markers[r] * D, sizeof mv);
        layer_norm(mv, m->s0w, m->s0b);
        for (int j = 0; j < D; j++) h1[j] = dotv(mv, m->s1w + (size_t)j * D, D);
        for (int d = 0; d < D; d++) h1[d] = lo_gelu(h1[d] + m->s1b[d]);
        logits[r] = dotv(h1, m->s3w, D) + m->s3b[0];
    }

    /* act / escalate head (2787-2814) */
    {
        float* p = (float*)malloc(sizeof(float) * (K > 0 ? K : 1));
        memcpy(p, logits, sizeof(float) * K);
        softmax(p, K);
        const float kk = (float)(K > 2 ? K : 2);
        float ent = 0;
        for (int r = 0; r < K; r++)
            if (p[r] > 1e-12f) ent -= p[r] * logf(p[r]);
        ent /= logf(kk);
        float t0 = 0, t1 = 0;
        for (int r = 0; r < K; r++) {
            if (p[r] > t0) {
                t1 = t0;
                t0 = p[r];
            } else if (p[r] > t1) {
                t1 = p[r];
            }
        }
        free(p);
        float act_in[D + 4], h256[256], a2[2];
        memcpy(act_in, pooled, sizeof(float) * D);
        act_in[D] = t0;
        act_in[D + 1] = t0 - t1;
        act_in[D + 2] = ent;
        act_in[D + 3] = kk / 255.0f;
        for (int i = 0; i < 256; i++) h256[i] = dotv(act_in, m->a0w + (size_t)i * (D + 4), D + 4);
        for (int i = 0; i < 256; i++) h256[i] = lo_gelu(h256[i] + m->a0b[i]);
        for (int i = 0; i < 2; i++) a2[i] = dotv(h256, m->a2w + i * 256, 256) + m->a2b[i];
        softmax(a2, 2);
        act[0] = a2[0];
        act[1] = a2[1];
    }
    if (hidden) memcpy(hidden, x, sizeof(float) * LD);
    free(x); free(xn); free(q); free(k); free(v); free(ctx); free(qkv); free(mlp); free(mlp2); free(ff);
    return 0;
}

int lo_max_threads(void) { return omp_get_max_threads(); }
