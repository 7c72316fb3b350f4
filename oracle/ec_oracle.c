/*
 * ec_oracle.c -- TEST INFRASTRUCTURE ONLY.  A CPU restatement of EdgeCore's
 * inference numerics (reference src/kernels.c and src/gpt2.c), used by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker for
 * the CUDA library.  Nothing in edgecore_b200/ links or calls this file.
 *
 * Parity pin: this restatement is checked bit-for-bit against the reference
 * compiled from its own sources (oracle/_ref, recipe in oracle/Makefile) and
 * against the golden vectors committed under tests/golden/.
 *
 * Every function follows the reference's evaluation order so that, compiled
 * with -std=c11 (which disables floating-point contraction in GCC), results
 * are bit-identical to the reference on the same host libm:
 *   - gemm_fp16/bf16: 8 independent FMA lanes over k, the AVX2 horizontal-sum
 *     order, then a scalar tail (reference src/kernels.c:29-64, :5-15)
 *   - gemm_int8: exact int32 dot, epilogue bias + ((float)dot*as)*bs
 *     (reference src/kernels.c:153-168)
 *   - activation quantisation: fp32 fabsf max, maxa/127.0f, lrintf(x/s),
 *     clamp (reference src/gpt2.c:446-461)
 */
#include "edgecore.h"   /* the repo's drop-in header: fp16 helpers, ARCH_*, ROPE_* */

#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define ECO_MAX_TENSORS 4096

#define ECO_API __attribute__((visibility("default")))

/* Transcendentals.  The default build calls the host libm exactly as the
 * reference does (its results are libm-specific: glibc's expf and tanhf are
 * not correctly rounded).  The CUDA library computes exactly these host
 * functions (its device expf / tanhf restate glibc's algorithms, checked
 * against the host library by oracle/libm_check.c and the GPU tests), so the
 * restatement is the GPU path's bit-level oracle as well as the
 * reference's. */
#define eco_expf expf
#define eco_tanhf tanhf

/* The host libm's expf / tanhf on n values (the GPU's device restatements
 * are checked against these). */
ECO_API void eco_libm(const float *x, float *e, float *t, int n)
{
    for (int i = 0; i < n; i++) {
        if (e) e[i] = expf(x[i]);
        if (t) t[i] = tanhf(x[i]);
    }
}

/* ------------------------------------------------------------------ */
/* GEMM restatements                                                    */
/* ------------------------------------------------------------------ */

/* AVX2 hsum_ps order (reference src/kernels.c:5-15): fold the high 128-bit
 * half onto the low one, then (l0+l1) + (l2+l3). */
static float eco_hsum8(const float l[8])
{
    float a0 = l[0] + l[4], a1 = l[1] + l[5], a2 = l[2] + l[6], a3 = l[3] + l[7];
    float s01 = a0 + a1;
    float s23 = a2 + a3;
    return s01 + s23;
}

typedef float (*eco_cvt16)(uint16_t);

static float eco_dot16(const float *a, const uint16_t *b, int K, eco_cvt16 cvt)
{
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int k = 0;
    for (; k + 8 <= K; k += 8)
        for (int j = 0; j < 8; j++)
            lane[j] = fmaf(a[k + j], cvt(b[k + j]), lane[j]);
    float r = eco_hsum8(lane);
    for (; k < K; k++) r += a[k] * cvt(b[k]);
    return r;
}

/* reference src/kernels.c:129-139 */
ECO_API void eco_gemm_fp16(float *C, const float *A, const uint16_t *B, int M, int K, int N)
{
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++)
        for (int m = 0; m < M; m++)
            C[(size_t)m * N + n] = eco_dot16(A + (size_t)m * K, B + (size_t)n * K, K, fp16_to_f32);
}

/* reference src/kernels.c:141-151 */
ECO_API void eco_gemm_bf16(float *C, const float *A, const uint16_t *B, int M, int K, int N)
{
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++)
        for (int m = 0; m < M; m++)
            C[(size_t)m * N + n] = eco_dot16(A + (size_t)m * K, B + (size_t)n * K, K, bf16_to_f32);
}

/* reference src/kernels.c:153-168 (the int32 dot is exact, so any order is) */
ECO_API void eco_gemm_int8(float *C, const int8_t *A, const float *a_scale,
                           const int8_t *B, const float *b_scale, const float *bias,
                           int M, int K, int N)
{
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++) {
        const int8_t *w = B + (size_t)n * K;
        float bs = b_scale ? b_scale[n] : 1.0f;
        float bv = bias ? bias[n] : 0.0f;
        for (int m = 0; m < M; m++) {
            const int8_t *x = A + (size_t)m * K;
            int32_t acc = 0;
            for (int k = 0; k < K; k++) acc += (int32_t)x[k] * (int32_t)w[k];
            float t = (float)acc * a_scale[m];
            t = t * bs;
            C[(size_t)m * N + n] = bv + t;
        }
    }
}

/* reference src/gpt2.c:446-461 */
ECO_API void eco_quantize_rows(int8_t *q, float *scale, const float *x, int M, int K)
{
    for (int m = 0; m < M; m++) {
        const float *r = x + (size_t)m * K;
        float mx = 0.0f;
        for (int k = 0; k < K; k++) {
            float v = fabsf(r[k]);
            if (v > mx) mx = v;
        }
        float s = mx > 0.0f ? mx / 127.0f : 1.0f;
        scale[m] = s;
        for (int k = 0; k < K; k++) {
            long v = lrintf(r[k] / s);
            if (v > 127) v = 127;
            if (v < -128) v = -128;
            q[(size_t)m * K + k] = (int8_t)v;
        }
    }
}

/* ------------------------------------------------------------------ */
/* Elementwise restatements                                             */
/* ------------------------------------------------------------------ */

/* reference src/gpt2.c:398-414 */
ECO_API void eco_layernorm(float *out, const float *in, const float *g, const float *b,
                           int M, int N, double eps)
{
    for (int m = 0; m < M; m++) {
        const float *r = in + (size_t)m * N;
        double mean = 0.0, var = 0.0;
        for (int i = 0; i < N; i++) mean += r[i];
        mean /= N;
        for (int i = 0; i < N; i++) { double d = r[i] - mean; var += d * d; }
        var /= N;
        double rstd = 1.0 / sqrt(var + eps);
        for (int i = 0; i < N; i++) {
            float t = (float)(((double)r[i] - mean) * rstd);
            out[(size_t)m * N + i] = t * g[i] + b[i];
        }
    }
}

/* reference src/gpt2.c:592-604 */
ECO_API void eco_rmsnorm(float *out, const float *in, const float *g, int M, int N, double eps)
{
    for (int m = 0; m < M; m++) {
        const float *r = in + (size_t)m * N;
        double ss = 0.0;
        for (int i = 0; i < N; i++) ss += (double)r[i] * r[i];
        double rstd = 1.0 / sqrt(ss / N + eps);
        for (int i = 0; i < N; i++) {
            float t = (float)((double)r[i] * rstd);
            out[(size_t)m * N + i] = t * g[i];
        }
    }
}

/* reference src/gpt2.c:393-396 */
static float eco_gelu(float x)
{
    float c = 0.044715f * x;
    c = c * x;
    c = c * x;
    float t = eco_tanhf(0.7978845608028654f * (x + c));
    return (0.5f * x) * (1.0f + t);
}

/* reference src/gpt2.c:587-590 */
static float eco_silu(float x) { return x / (1.0f + eco_expf(-x)); }

/* RoPE inverse frequencies incl. the YaRN ramp (reference src/gpt2.c:608-644). */
ECO_API void eco_rope_inv_freq(double *inv, int half, double theta, int rope_type,
                               double yarn_factor, double yarn_orig_max)
{
    int dim = 2 * half;
    for (int i = 0; i < half; i++) inv[i] = pow(1.0 / theta, (double)(2 * i) / (double)dim);
    if (rope_type != ROPE_YARN) return;
    const double two_pi = 6.28318530717958647692;
    double lb = log(theta);
    double lo = floor((double)dim * log(yarn_orig_max / (32.0 * two_pi)) / (2.0 * lb));
    double hi = ceil((double)dim * log(yarn_orig_max / (1.0 * two_pi)) / (2.0 * lb));
    if (lo < 0.0) lo = 0.0;
    if (hi > (double)(dim - 1)) hi = (double)(dim - 1);
    double span = hi - lo;
    if (span < 1.0) span = 1.0;
    for (int i = 0; i < half; i++) {
        double ramp = ((double)i - lo) / span;
        if (ramp < 0.0) ramp = 0.0;
        if (ramp > 1.0) ramp = 1.0;
        double e = inv[i];
        inv[i] = (e / yarn_factor) * ramp + e * (1.0 - ramp);
    }
}

/* cos/sin of one position, scaled (reference src/gpt2.c:646-654). */
ECO_API void eco_rope_cos_sin(double *c, double *s, const double *inv, int half, int pos, double scale)
{
    for (int i = 0; i < half; i++) {
        double f = (double)pos * inv[i];
        c[i] = cos(f) * scale;
        s[i] = sin(f) * scale;
    }
}

/* NeoX half-split rotation of one head (reference src/gpt2.c:656-665). */
static void eco_rotate(float *v, int half, const double *c, const double *s)
{
    for (int i = 0; i < half; i++) {
        float a = v[i], b = v[i + half];
        double lo = (double)a * c[i];
        lo = lo - (double)b * s[i];
        double hi = (double)a * s[i];
        hi = hi + (double)b * c[i];
        v[i] = (float)lo;
        v[i + half] = (float)hi;
    }
}

/* ------------------------------------------------------------------ */
/* Model                                                                */
/* ------------------------------------------------------------------ */

enum { ECO_F32 = 0, ECO_F16 = 1, ECO_I8 = 2, ECO_TXT = 3, ECO_BF16 = 4 };

typedef struct {
    const void *w; const float *s, *b;   /* b is only used where the reference uses it */
} eco_lin;

typedef struct {
    const float *n1g, *n1b, *n2g, *n2b;
    eco_lin qkv, proj, fc, fc2;                  /* gpt2 */
    eco_lin q, k, v, o, gate, up, down;          /* qwen2 */
} eco_layer;

typedef struct eco_model {
    /* meta */
    int arch, L, H, KVH, E, hd, kv, I, V, ctx, C, B, prec, rope_type, sw, tie;
    double eps, theta, yf, yom, yaf;
    /* tensors (point into the file buffer) */
    unsigned char *file; size_t fsize;
    const uint16_t *wte, *wpe, *lm;
    const float *nfg, *nfb;
    eco_layer *lw;
    /* state */
    uint16_t *kc, *vc;                           /* [L][B][C][kv] */
    /* taps: residual after embedding and after each layer, [L+1][M][E] */
    float *taps; int taps_cap;
} eco_model;

static size_t eco_dsize(int dt) { return dt == ECO_F32 ? 4 : dt == ECO_I8 ? 1 : dt == ECO_TXT ? 1 : 2; }

typedef struct { char name[128]; int dt; size_t off, bytes; } eco_t;

static int eco_line(const unsigned char **p, const unsigned char *end, char *buf, size_t cap)
{
    size_t n = 0;
    if (*p >= end) return -1;
    while (*p < end && **p != '\n') { if (**p != '\r' && n + 1 < cap) buf[n++] = (char)**p; (*p)++; }
    if (*p < end) (*p)++;
    buf[n] = 0;
    return 0;
}

static const eco_t *eco_find(const eco_t *t, int n, const char *name)
{
    for (int i = 0; i < n; i++) if (!strcmp(t[i].name, name)) return &t[i];
    return NULL;
}

ECO_API void eco_close(eco_model *m)
{
    if (!m) return;
    free(m->file); free(m->lw); free(m->kc); free(m->vc); free(m->taps);
    free(m);
}

/* Load an .ecm file the way reference gpt2_load does (src/gpt2.c:161-366):
 * meta defaults, precision from the first linear, qwen2 defaults, binding. */
ECO_API eco_model *eco_open(const char *path, int batch_cap, int max_ctx)
{
    FILE *f = fopen(path, "rb");
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    eco_model *m = calloc(1, sizeof *m);
    m->file = malloc((size_t)sz);
    m->fsize = (size_t)sz;
    if (fread(m->file, 1, (size_t)sz, f) != (size_t)sz) { fclose(f); eco_close(m); return NULL; }
    fclose(f);
    if (sz < 5 || memcmp(m->file, "ECM1\n", 5)) { eco_close(m); return NULL; }

    m->eps = 1e-5;
    m->B = batch_cap < 1 ? 1 : batch_cap;
    const unsigned char *p = m->file + 5, *end = m->file + sz;
    char ln[1024];
    while (1) {
        if (eco_line(&p, end, ln, sizeof ln)) { eco_close(m); return NULL; }
        if (!strcmp(ln, "END_META")) break;
        char *eq = strchr(ln, '=');
        if (!eq) continue;
        *eq = 0;
        const char *k = ln, *v = eq + 1;
        if (!strcmp(k, "n_layer")) m->L = atoi(v);
        else if (!strcmp(k, "n_head")) m->H = atoi(v);
        else if (!strcmp(k, "n_kv_head")) m->KVH = atoi(v);
        else if (!strcmp(k, "intermediate")) m->I = atoi(v);
        else if (!strcmp(k, "n_embd")) m->E = atoi(v);
        else if (!strcmp(k, "n_ctx")) m->ctx = atoi(v);
        else if (!strcmp(k, "vocab")) m->V = atoi(v);
        else if (!strcmp(k, "eps")) m->eps = atof(v);
        else if (!strcmp(k, "rope_theta")) m->theta = atof(v);
        else if (!strcmp(k, "rope_type")) m->rope_type = !strcmp(v, "yarn") ? ROPE_YARN : ROPE_DEFAULT;
        else if (!strcmp(k, "yarn_factor")) m->yf = atof(v);
        else if (!strcmp(k, "yarn_attention_factor")) m->yaf = atof(v);
        else if (!strcmp(k, "yarn_orig_max")) m->yom = atof(v);
        else if (!strcmp(k, "sliding_window")) m->sw = atoi(v);
        else if (!strcmp(k, "tie_word_embeddings")) m->tie = atoi(v);
        else if (!strcmp(k, "arch")) m->arch = (!strcmp(v, "qwen2") || !strcmp(v, "olmo3")) ? ARCH_QWEN2 : ARCH_GPT2;
    }
    /* 512 entries in the reference (src/gpt2.c:180-181); more here so that the
     * 28-layer config-4 model (534 tensors) can serve as a CPU baseline */
    eco_t *t = calloc(ECO_MAX_TENSORS, sizeof *t);
    int nt = 0;
    while (1) {
        if (eco_line(&p, end, ln, sizeof ln)) { free(t); eco_close(m); return NULL; }
        if (!strcmp(ln, "END_TENSORS")) break;
        char name[128], ds[16];
        if (sscanf(ln, "%127s %15s", name, ds) < 2) continue;
        int dt;
        if (!strcmp(ds, "fp32")) dt = ECO_F32;
        else if (!strcmp(ds, "fp16")) dt = ECO_F16;
        else if (!strcmp(ds, "int8")) dt = ECO_I8;
        else if (!strcmp(ds, "text")) dt = ECO_TXT;
        else if (!strcmp(ds, "bf16")) dt = ECO_BF16;
        else continue;
        /* dims follow the first two words */
        const char *q = ln;
        for (int w = 0; w < 2; w++) { while (*q == ' ') q++; while (*q && *q != ' ') q++; }
        size_t ne = 1;
        if (dt == ECO_TXT) ne = strtoull(q, NULL, 10);
        else {
            while (*q) {
                while (*q == ' ') q++;
                if (!*q) break;
                char *e2;
                ne *= strtoull(q, &e2, 10);
                q = e2;
            }
        }
        snprintf(t[nt].name, sizeof t[nt].name, "%s", name);
        t[nt].dt = dt;
        t[nt].bytes = ne * eco_dsize(dt);
        if (++nt >= ECO_MAX_TENSORS) { free(t); eco_close(m); return NULL; }
    }
    size_t off = (size_t)(p - m->file);
    for (int i = 0; i < nt; i++) { t[i].off = off; off += t[i].bytes; }
    const unsigned char *base = m->file;
#define ECO_PTR(ty, tn) ((tn) ? (const ty *)(base + (tn)->off) : NULL)

    const eco_t *twte = eco_find(t, nt, "wte"), *tnf = eco_find(t, nt, "ln_f.g");
    const eco_t *tl0 = eco_find(t, nt, m->arch == ARCH_QWEN2 ? "blocks.0.q.w" : "blocks.0.attn.w");
    if (!twte || !tnf || !tl0) { free(t); eco_close(m); return NULL; }
    m->prec = tl0->dt == ECO_F16 ? 1 : tl0->dt == ECO_I8 ? 0 : tl0->dt == ECO_BF16 ? 2 : -1;
    if (m->prec < 0) { free(t); eco_close(m); return NULL; }
    m->wte = ECO_PTR(uint16_t, twte);
    m->nfg = ECO_PTR(float, tnf);
    if (m->arch == ARCH_QWEN2) {
        if (m->KVH <= 0) m->KVH = m->H;
        m->hd = m->E / (m->H > 0 ? m->H : 1);
        m->kv = m->KVH * m->hd;
        if (m->I <= 0) m->I = 4 * m->E;
        if (m->theta <= 0) m->theta = 10000.0;
        if (m->yom <= 0) m->yom = m->ctx;
        if (m->yf <= 0) m->yf = 1.0;
        if (m->yaf <= 0) m->yaf = 1.0;
        const eco_t *tlm = eco_find(t, nt, "lm_head.w");
        m->lm = (tlm && !m->tie) ? ECO_PTR(uint16_t, tlm) : m->wte;
    } else {
        m->wpe = ECO_PTR(uint16_t, eco_find(t, nt, "wpe"));
        m->nfb = ECO_PTR(float, eco_find(t, nt, "ln_f.b"));
        if (!m->wpe || !m->nfb) { free(t); eco_close(m); return NULL; }
        m->KVH = m->H; m->hd = m->E / m->H; m->kv = m->E; m->I = 4 * m->E;
        m->lm = m->wte;
    }
    m->lw = calloc((size_t)m->L, sizeof *m->lw);
    char nm[192];
    for (int l = 0; l < m->L; l++) {
        eco_layer *W = &m->lw[l];
#define ECO_GET(ty, fmt) (snprintf(nm, sizeof nm, fmt, l), ECO_PTR(ty, eco_find(t, nt, nm)))
        W->n1g = ECO_GET(float, "blocks.%d.ln_1.g");
        W->n1b = ECO_GET(float, "blocks.%d.ln_1.b");
        W->n2g = ECO_GET(float, "blocks.%d.ln_2.g");
        W->n2b = ECO_GET(float, "blocks.%d.ln_2.b");
        const char *qn[7] = {"q", "k", "v", "o", "gate", "up", "down"};
        const char *gn[4] = {"attn", "proj", "fc", "fc2"};
        eco_lin *ql[7] = {&W->q, &W->k, &W->v, &W->o, &W->gate, &W->up, &W->down};
        eco_lin *gl[4] = {&W->qkv, &W->proj, &W->fc, &W->fc2};
        int cnt = m->arch == ARCH_QWEN2 ? 7 : 4;
        for (int s = 0; s < cnt; s++) {
            const char *sf = m->arch == ARCH_QWEN2 ? qn[s] : gn[s];
            eco_lin *L = m->arch == ARCH_QWEN2 ? ql[s] : gl[s];
            snprintf(nm, sizeof nm, "blocks.%d.%s.w", l, sf);
            const eco_t *tw = eco_find(t, nt, nm);
            snprintf(nm, sizeof nm, "blocks.%d.%s.s", l, sf);
            const eco_t *ts = eco_find(t, nt, nm);
            snprintf(nm, sizeof nm, "blocks.%d.%s.b", l, sf);
            const eco_t *tb = eco_find(t, nt, nm);
            if (!tw || (m->arch == ARCH_GPT2 && (!tb || (m->prec == 0 && !ts)))) {
                free(t); eco_close(m); return NULL;
            }
            L->w = base + tw->off;
            L->s = (m->prec == 0) ? ECO_PTR(float, ts) : NULL;
            L->b = ECO_PTR(float, tb);
        }
#undef ECO_GET
    }
#undef ECO_PTR
    free(t);
    m->C = (max_ctx > 0 && max_ctx < m->ctx) ? max_ctx : m->ctx;
    size_t kvn = (size_t)m->L * m->B * m->C * m->kv;
    m->kc = calloc(kvn, 2);
    m->vc = calloc(kvn, 2);
    if (!m->kc || !m->vc) { eco_close(m); return NULL; }
    return m;
}

ECO_API void eco_info(const eco_model *m, int *o)
{
    int v[16] = {m->arch, m->prec, m->L, m->H, m->KVH, m->E, m->hd, m->I, m->V,
                 m->ctx, m->C, m->B, m->kv, m->tie, 0, 0};
    memcpy(o, v, sizeof v);
}

ECO_API void eco_reset_kv(eco_model *m)
{
    size_t kvn = (size_t)m->L * m->B * m->C * m->kv;
    memset(m->kc, 0, kvn * 2);
    memset(m->vc, 0, kvn * 2);
}

/* linear() (reference src/gpt2.c:420-464); use_bias mirrors which call sites
 * pass a bias (gpt2 passes the stored bias, qwen2 passes NULL). */
static void eco_linear(const eco_model *m, const eco_lin *L, int use_bias,
                       const float *in, float *out, int M, int K, int N)
{
    const float *bias = use_bias ? L->b : NULL;
    if (m->prec == 0) {
        int8_t *q = malloc((size_t)M * K);
        float *qs = malloc((size_t)M * sizeof(float));
        eco_quantize_rows(q, qs, in, M, K);
        eco_gemm_int8(out, q, qs, (const int8_t *)L->w, L->s, bias, M, K, N);
        free(q); free(qs);
        return;
    }
    if (m->prec == 1) eco_gemm_fp16(out, in, (const uint16_t *)L->w, M, K, N);
    else eco_gemm_bf16(out, in, (const uint16_t *)L->w, M, K, N);
    if (bias)
        for (int i = 0; i < M; i++)
            for (int n = 0; n < N; n++) out[(size_t)i * N + n] += bias[n];
}

/* One attention row: token at `pos` of slot cache kb/vb (stride kv) against
 * positions [lo, pos] (reference src/gpt2.c:527-557 and :743-777). */
static void eco_attend(const float *q, const uint16_t *kb, const uint16_t *vb, int kvs,
                       int lo, int pos, int hd, double inv_hd, float *sc, float *o)
{
    float mx = -FLT_MAX;
    for (int p = lo; p <= pos; p++) {
        const uint16_t *kp = kb + (size_t)p * kvs;
        float s = 0.0f;
        for (int d = 0; d < hd; d++) s += q[d] * fp16_to_f32(kp[d]);
        s = (float)(s * inv_hd);
        sc[p] = s;
        if (s > mx) mx = s;
    }
    double sum = 0.0;
    for (int p = lo; p <= pos; p++) { sc[p] = eco_expf(sc[p] - mx); sum += sc[p]; }
    double inv = 1.0 / sum;
    for (int p = lo; p <= pos; p++) sc[p] = (float)(sc[p] * inv);
    for (int d = 0; d < hd; d++) o[d] = 0.0f;
    for (int p = lo; p <= pos; p++) {
        const uint16_t *vp = vb + (size_t)p * kvs;
        float w = sc[p];
        for (int d = 0; d < hd; d++) o[d] += w * fp16_to_f32(vp[d]);
    }
}

static float eco_h(const eco_model *m, uint16_t v) { return m->prec == 2 ? bf16_to_f32(v) : fp16_to_f32(v); }

/* Enable per-layer taps for forwards of up to max_m rows (0 disables). */
ECO_API void eco_set_taps(eco_model *m, int max_m)
{
    free(m->taps);
    m->taps = max_m > 0 ? calloc((size_t)(m->L + 1) * max_m * m->E, sizeof(float)) : NULL;
    m->taps_cap = max_m;
}

ECO_API const float *eco_get_taps(const eco_model *m) { return m->taps; }

/* gpt2_forward / qwen2_forward (reference src/gpt2.c:470-581, :667-805). */
ECO_API void eco_forward(eco_model *m, const int *tok, const int *pos, const int *seqs,
                         int M, float *logits)
{
    const int E = m->E, H = m->H, hd = m->hd, kv = m->kv, C = m->C, V = m->V;
    const double inv_hd = 1.0 / sqrt((double)hd);
    const int wide = m->arch == ARCH_QWEN2 ? (E + 2 * kv > 2 * m->I ? E + 2 * kv : 2 * m->I) : 4 * E;
    float *x = malloc((size_t)M * E * sizeof(float));
    float *h = malloc((size_t)M * 4 * E * sizeof(float) + (size_t)M * E * sizeof(float));
    float *big = malloc((size_t)M * wide * sizeof(float));
    float *at = malloc((size_t)M * E * sizeof(float));
    float *sc = malloc((size_t)C * sizeof(float));
    double inv[512], cs[512], sn[512];
    int half = hd / 2;
    if (half > 512) half = 512;
    if (m->arch == ARCH_QWEN2) eco_rope_inv_freq(inv, half, m->theta, m->rope_type, m->yf, m->yom);
    const int tap = m->taps && M <= m->taps_cap;

    for (int i = 0; i < M; i++)
        for (int d = 0; d < E; d++) {
            float e = eco_h(m, m->wte[(size_t)tok[i] * E + d]);
            if (m->arch == ARCH_GPT2) e = e + eco_h(m, m->wpe[(size_t)pos[i] * E + d]);
            x[(size_t)i * E + d] = e;
        }
    if (tap) memcpy(m->taps, x, (size_t)M * E * sizeof(float));

    const size_t lstride = (size_t)m->B * C * kv;
    for (int l = 0; l < m->L; l++) {
        const eco_layer *W = &m->lw[l];
        uint16_t *kc = m->kc + lstride * l, *vc = m->vc + lstride * l;
        float *q, *kk, *vv;
        int qs, ks;          /* row strides of q and k/v in `big` */
        if (m->arch == ARCH_GPT2) {
            eco_layernorm(h, x, W->n1g, W->n1b, M, E, m->eps);
            eco_linear(m, &W->qkv, 1, h, big, M, E, 3 * E);
            q = big; kk = big + E; vv = big + 2 * E; qs = ks = 3 * E;
        } else {
            eco_rmsnorm(h, x, W->n1g, M, E, m->eps);
            eco_linear(m, &W->q, 0, h, big, M, E, E);
            eco_linear(m, &W->k, 0, h, big + (size_t)M * E, M, E, kv);
            eco_linear(m, &W->v, 0, h, big + (size_t)M * (E + kv), M, E, kv);
            q = big; kk = big + (size_t)M * E; vv = big + (size_t)M * (E + kv); qs = E; ks = kv;
            for (int i = 0; i < M; i++) {
                eco_rope_cos_sin(cs, sn, inv, half, pos[i], m->yaf);
                for (int hh = 0; hh < H; hh++) eco_rotate(q + (size_t)i * qs + (size_t)hh * hd, half, cs, sn);
                for (int g = 0; g < m->KVH; g++) eco_rotate(kk + (size_t)i * ks + (size_t)g * hd, half, cs, sn);
            }
        }
        for (int i = 0; i < M; i++) {
            int slot = seqs ? seqs[i] : i;
            if (slot >= m->B) slot = m->B - 1;
            uint16_t *kr = kc + (size_t)slot * C * kv + (size_t)pos[i] * kv;
            uint16_t *vr = vc + (size_t)slot * C * kv + (size_t)pos[i] * kv;
            for (int d = 0; d < kv; d++) {
                kr[d] = f32_to_fp16(kk[(size_t)i * ks + d]);
                vr[d] = f32_to_fp16(vv[(size_t)i * ks + d]);
            }
        }
        for (int hh = 0; hh < H; hh++) {
            int g = m->arch == ARCH_QWEN2 ? hh * m->KVH / H : hh;
            for (int i = 0; i < M; i++) {
                int slot = seqs ? seqs[i] : i;
                if (slot >= m->B) slot = m->B - 1;
                int lo = 0;
                if (m->arch == ARCH_QWEN2 && m->sw > 0) { lo = pos[i] - m->sw + 1; if (lo < 0) lo = 0; }
                eco_attend(q + (size_t)i * qs + (size_t)hh * hd,
                           kc + (size_t)slot * C * kv + (size_t)g * hd,
                           vc + (size_t)slot * C * kv + (size_t)g * hd,
                           kv, lo, pos[i], hd, inv_hd, sc, at + (size_t)i * E + (size_t)hh * hd);
            }
        }
        if (m->arch == ARCH_GPT2) {
            eco_linear(m, &W->proj, 1, at, h, M, E, E);
            for (size_t i = 0; i < (size_t)M * E; i++) x[i] += h[i];
            eco_layernorm(h, x, W->n2g, W->n2b, M, E, m->eps);
            eco_linear(m, &W->fc, 1, h, big, M, E, 4 * E);
            for (size_t i = 0; i < (size_t)M * 4 * E; i++) big[i] = eco_gelu(big[i]);
            eco_linear(m, &W->fc2, 1, big, h, M, 4 * E, E);
            for (size_t i = 0; i < (size_t)M * E; i++) x[i] += h[i];
        } else {
            const int I = m->I;
            eco_linear(m, &W->o, 0, at, h, M, E, E);
            for (size_t i = 0; i < (size_t)M * E; i++) x[i] += h[i];
            eco_rmsnorm(h, x, W->n2g, M, E, m->eps);
            eco_linear(m, &W->gate, 0, h, big, M, E, I);
            eco_linear(m, &W->up, 0, h, big + (size_t)M * I, M, E, I);
            for (size_t i = 0; i < (size_t)M * I; i++) big[i] = eco_silu(big[i]) * big[(size_t)M * I + i];
            eco_linear(m, &W->down, 0, big, h, M, I, E);
            for (size_t i = 0; i < (size_t)M * E; i++) x[i] += h[i];
        }
        if (tap) memcpy(m->taps + (size_t)(l + 1) * M * E, x, (size_t)M * E * sizeof(float));
    }
    if (m->arch == ARCH_GPT2) eco_layernorm(h, x, m->nfg, m->nfb, M, E, m->eps);
    else eco_rmsnorm(h, x, m->nfg, M, E, m->eps);
    if (m->prec == 2) eco_gemm_bf16(logits, h, m->lm, M, E, V);
    else eco_gemm_fp16(logits, h, m->lm, M, E, V);
    free(x); free(h); free(big); free(at); free(sc);
}

/* The half-precision helpers of include/edgecore.h, exported for tests. */
ECO_API uint16_t eco_f2h(float f) { return f32_to_fp16(f); }
ECO_API float eco_h2f(uint16_t h) { return fp16_to_f32(h); }
ECO_API float eco_gelu_x(float x) { return eco_gelu(x); }
ECO_API float eco_silu_x(float x) { return eco_silu(x); }
