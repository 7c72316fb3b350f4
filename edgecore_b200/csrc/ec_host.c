/*
 * ec_host.c -- host side of the drop-in replacement for EdgeCore's
 * src/gpt2.c: .ecm parsing, gpt2_load / gpt2_free / gpt2_forward /
 * qwen2_forward, and the edgecore_b200.h extensions built on them.
 *
 * A loaded model keeps the reference's host-visible state (the mmap'd file,
 * the bound host weight pointers, full-size host KV buffers, the tokenizer)
 * and adds device state, found through a registry keyed by the GPT2 address:
 *   - every linear uploaded once in the packed layout of ec_decode.h (rows
 *     padded to a multiple of 16 elements; Qwen2 q|k|v fused with RoPE
 *     partners adjacent, gate|up fused and interleaved; fusing is exact since
 *     the reference quantises the same input once per projection);
 *   - a device KV arena [n_layer][batch_cap][eff_ctx][n_kv_embd] fp16, the
 *     reference cache layout (src/gpt2.c:312-317);
 *   - RoPE cos/sin tables in fp64 from the host libm with the reference
 *     formula (src/gpt2.c:608-654), so the rotation is bit-exact;
 *   - workspaces.
 * Forward calls of up to 8 token rows and batched decode of up to 7 streams
 * run the persistent decode kernel (ec_decode.cu); larger calls (prefill,
 * batched decode from 8 streams) run per-layer kernels.
 */
#define _GNU_SOURCE
#include "edgecore.h"
#include "edgecore_b200.h"
#include "ec_launch.h"
#include "ec_decode.h"

#include <cuda_runtime_api.h>
#include <fcntl.h>
#include <pthread.h>
#include <stdarg.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* The tokenizer is the reference's src/tokenizer.c, present when this library
 * is linked into the reference runtime; absent (NULL) in other processes. */
#pragma weak tokenizer_load
#pragma weak tokenizer_free

#define EC_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------ */
/* errors                                                              */
/* ------------------------------------------------------------------ */

static __thread char g_err[512];

static void ec_seterr(const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

EC_EXPORT const char *ec_last_error(void) { return g_err; }

/* For the other translation units of the library (not exported). */
void ec_set_error_text(const char *msg) { ec_seterr("%s", msg); }
EC_EXPORT const char *ec_version(void) { return "edgecore_b200 0.2 sm_100a"; }

#define CK(call)                                                                               \
    do {                                                                                       \
        cudaError_t e_ = (cudaError_t)(call);                                                  \
        if (e_ != cudaSuccess) {                                                               \
            ec_seterr("%s:%d: %s: %s", __FILE__, __LINE__, #call, cudaGetErrorString(e_));     \
            return -1;                                                                         \
        }                                                                                      \
    } while (0)

/* For the void reference entry points: report and abort, as the reference
 * exits on an unrecoverable forward error (src/gpt2.c:442-445). */
static void ec_fatal(const char *where)
{
    fprintf(stderr, "edgecore_b200: %s: %s\n", where, g_err[0] ? g_err : "error");
    abort();
}

/* ------------------------------------------------------------------ */
/* .ecm parsing (the format read by reference src/gpt2.c:34-136)        */
/* ------------------------------------------------------------------ */

static const char *ec_readline(const char *p, const char *end, char *line, size_t cap)
{
    size_t n = 0;
    if (p >= end) return NULL;
    while (p < end && *p != '\n') {
        if (*p != '\r' && n + 1 < cap) line[n++] = *p;
        p++;
    }
    line[n] = '\0';
    if (p < end) p++;
    return p;
}

static size_t ec_dtype_bytes(int dt)
{
    return dt == 0 ? 4 : dt == 1 ? 2 : dt == 2 ? 1 : dt == 4 ? 2 : 0;
}

EC_EXPORT int ecm_parse(const void *data, size_t size, EcmTensor *out, int max, GPT2 *meta)
{
    const char *p = (const char *)data, *end = p + size;
    char line[1024];
    if (size < 5 || memcmp(p, ECM_MAGIC, 5) != 0) {
        fprintf(stderr, "ecm: bad magic\n");
        return -1;
    }
    p += 5;
    for (;;) {
        p = ec_readline(p, end, line, sizeof line);
        if (!p) return -1;
        if (!strcmp(line, "END_META")) break;
        char *eq = strchr(line, '=');
        if (!eq) continue;
        *eq = '\0';
        const char *k = line, *v = eq + 1;
        if (!strcmp(k, "model_name")) snprintf(meta->model_name, sizeof meta->model_name, "%s", v);
        else if (!strcmp(k, "n_layer")) meta->n_layer = atoi(v);
        else if (!strcmp(k, "n_head")) meta->n_head = atoi(v);
        else if (!strcmp(k, "n_kv_head")) meta->n_kv_head = atoi(v);
        else if (!strcmp(k, "intermediate")) meta->intermediate = atoi(v);
        else if (!strcmp(k, "n_embd")) meta->n_embd = atoi(v);
        else if (!strcmp(k, "n_ctx")) meta->n_ctx = atoi(v);
        else if (!strcmp(k, "vocab")) meta->vocab = atoi(v);
        else if (!strcmp(k, "n_params")) meta->n_params = (size_t)strtoull(v, NULL, 10);
        else if (!strcmp(k, "eps")) meta->eps = atof(v);
        else if (!strcmp(k, "rope_theta")) meta->rope_theta = atof(v);
        else if (!strcmp(k, "rope_type")) meta->rope_type = !strcmp(v, "yarn") ? ROPE_YARN : ROPE_DEFAULT;
        else if (!strcmp(k, "yarn_factor")) meta->yarn_factor = atof(v);
        else if (!strcmp(k, "yarn_attention_factor")) meta->yarn_attention_factor = atof(v);
        else if (!strcmp(k, "yarn_orig_max")) meta->yarn_orig_max = atof(v);
        else if (!strcmp(k, "sliding_window")) meta->sliding_window = atoi(v);
        else if (!strcmp(k, "tie_word_embeddings")) meta->tie_word_embeddings = atoi(v);
        else if (!strcmp(k, "eos_token_id")) meta->eos_token_id = atoi(v);
        else if (!strcmp(k, "arch"))
            meta->arch = (!strcmp(v, "qwen2") || !strcmp(v, "olmo3")) ? ARCH_QWEN2 : ARCH_GPT2;
    }
    int nt = 0;
    for (;;) {
        p = ec_readline(p, end, line, sizeof line);
        if (!p) return -1;
        if (!strcmp(line, "END_TENSORS")) break;
        EcmTensor *t = &out[nt];
        memset(t, 0, sizeof *t);
        char name[128], ds[16];
        if (sscanf(line, "%127s %15s", name, ds) < 2) continue;
        if (!strcmp(ds, "fp32")) t->dtype = 0;
        else if (!strcmp(ds, "fp16")) t->dtype = 1;
        else if (!strcmp(ds, "int8")) t->dtype = 2;
        else if (!strcmp(ds, "text")) t->dtype = 3;
        else if (!strcmp(ds, "bf16")) t->dtype = 4;
        else continue;
        snprintf(t->name, sizeof t->name, "%s", name);
        const char *q = line;
        for (int w = 0; w < 2; w++) {
            while (*q == ' ') q++;
            while (*q && *q != ' ') q++;
        }
        if (t->dtype == 3) {
            t->ndims = 1;
            t->dims[0] = (size_t)strtoull(q, NULL, 10);
            t->nelems = t->bytes = t->dims[0];
        } else {
            t->nelems = 1;
            while (*q) {
                while (*q == ' ') q++;
                if (!*q) break;
                char *e2;
                size_t d = (size_t)strtoull(q, &e2, 10);
                if (e2 == q) break;
                if (t->ndims < 4) t->dims[t->ndims++] = d;
                t->nelems *= d;
                q = e2;
            }
            t->bytes = t->nelems * ec_dtype_bytes(t->dtype);
        }
        if (++nt >= max) return -1;
    }
    size_t off = (size_t)(p - (const char *)data);
    for (int i = 0; i < nt; i++) {
        out[i].offset = off;
        off += out[i].bytes;
    }
    return nt;
}

static const EcmTensor *ec_find(const EcmTensor *t, int n, const char *name)
{
    for (int i = 0; i < n; i++)
        if (!strcmp(t[i].name, name)) return &t[i];
    return NULL;
}

/* ------------------------------------------------------------------ */
/* device state                                                         */
/* ------------------------------------------------------------------ */

typedef struct {
    void *w;            /* packed [N][ldw]: Kp weights + {scale, bias, 0, 0} fp32 tail */
    float *s, *b;       /* [N] scales (int8), bias, or NULL (copies for the GEMM path) */
    int N, K, Kp, ldw, wt, unit;
} ec_lin;

typedef struct {
    float *n1g, *n1b, *n2g, *n2b;
    ec_lin qkv, o, up, down;   /* up = gate|up (qwen2) or fc (gpt2); down = down / fc2 */
} ec_dlayer;

/* Kernel classes reported by ec_decode_profile. */
enum { EC_PC_STEP = 0, EC_PC_GEMM = 1, EC_PC_ATTN = 2, EC_PC_NORM = 3, EC_PC_OTHER = 4, EC_PC_N = 5 };
#define EC_PROF_MAX 1024

typedef struct ec_dev {
    GPT2 *owner;
    int device, num_sms;
    cudaStream_t stream, own_stream;
    int arch, prec, wt, hwt, L, E, Ep, H, KVH, hd, kv, I, V, C, B, window;
    double eps;
    /* weights */
    uint16_t *wte, *wpe, *lm;
    float *nfg, *nfb;
    ec_dlayer *lw;
    int v0, v1;                /* vocab shard [v0, v1) */
    /* KV arena: per layer [kv_pages][EC_KV_PAGE][kv] fp16 for K and for V;
     * slot s holds positions [64 j, 64 j + 64) in page pt[s][j] */
    uint16_t *kc, *vc;
    size_t layer_kv;           /* elements per layer: kv_pages * EC_KV_PAGE * kv */
    int kv_pages, mp;          /* pages per layer, pages per slot (ceil(C / 64)) */
    int *h_pt, *d_pt;          /* page table [B][mp], -1 = unmapped (h_pt pinned) */
    int *free_pages, nfree;    /* stack of unmapped pages */
    int *kv_undo, nundo;       /* entries mapped by the current call (rolled back if it fails) */
    int pt_dirty;
    double *rope_cos, *rope_sin;
    /* persistent decode kernel */
    ec_mk_layer *d_mk_layers;
    int mk_grid;
    unsigned *d_bar;           /* two barrier counters (128 B apart) and the abort flag */
    int *d_abort, *d_mk_err;
    int bar_par, bar_reset;    /* counter of the next launch; 1: clear all three first */
    int *h_blk, *d_blk;        /* attention block table of the staged rows (ec_attn_args.blocks) */
    int nblk;                  /* 0: no table for the current call */
    int *h_res, *h_res_dev;    /* pinned, mapped: completion word | ids [8] | max [8] */
    int res_seq;
    float *amax_v;
    int *amax_i;
    /* workspaces */
    int cap;                   /* rows */
    float *x, *h, *qkv, *q, *att, *act, *big;
    int8_t *aq;
    float *as;
    void *split;          /* 16-bit activation parts for the tensor-core GEMMs */
    size_t split_bytes;
    int *acc32;           /* split-K int8 GEMMs: int32 tile sums and tile counters, kept zero */
    size_t acc32_elems;
    unsigned *tile_cnt;
    float *attn_part;
    size_t attn_part_floats;
    float *logits;
    int logit_rows;
    void *amax_part;
    int amax_chunks;
    void *lm_part;             /* argmax partials of the fused lm_head (EC_EPI_ARGMAX) */
    size_t lm_part_bytes;
    int *d_tok, *d_pos, *d_slot, *d_ids;
    float *d_max;
    int *d_hist;
    int hist_cap;
    int *h_in;                 /* pinned: tok | pos | slot */
    int *h_ids;
    float *h_max;
    float *h_logits;
    size_t h_logits_cap;
    /* batched decode: one captured CUDA graph per step shape (0: full greedy
     * step, 1: hidden rows only); ws_gen counts workspace reallocations and
     * vocab-shard changes, which invalidate the graphs */
    struct { cudaGraphExec_t exec; int M, maxlen, chunk, hist, kernels; unsigned gen; } bg[2];
    unsigned ws_gen;
    int *d_counter;
    /* taps */
    int taps_on;
    float *taps;
    int taps_rows;
    /* per-launch event profiling */
    int prof_on, prof_n, prof_ready;
    cudaEvent_t prof_ev[2 * EC_PROF_MAX];
    int prof_cls[EC_PROF_MAX];
    double prof_bytes[EC_PROF_MAX];
} ec_dev;

/* ---- registry: GPT2 address -> device state ---- */

static pthread_mutex_t g_reg_mu = PTHREAD_MUTEX_INITIALIZER;
static struct { GPT2 *g; ec_dev *d; } g_reg[256];

static ec_dev *ec_lookup(const GPT2 *g)
{
    ec_dev *d = NULL;
    pthread_mutex_lock(&g_reg_mu);
    for (int i = 0; i < 256; i++)
        if (g_reg[i].g == g) { d = g_reg[i].d; break; }
    pthread_mutex_unlock(&g_reg_mu);
    return d;
}

static int ec_register(GPT2 *g, ec_dev *d)
{
    int ok = -1;
    pthread_mutex_lock(&g_reg_mu);
    for (int i = 0; i < 256; i++)
        if (!g_reg[i].g) { g_reg[i].g = g; g_reg[i].d = d; ok = 0; break; }
    pthread_mutex_unlock(&g_reg_mu);
    if (ok) ec_seterr("too many loaded models (256)");
    return ok;
}

static void ec_unregister(GPT2 *g)
{
    pthread_mutex_lock(&g_reg_mu);
    for (int i = 0; i < 256; i++)
        if (g_reg[i].g == g) { g_reg[i].g = NULL; g_reg[i].d = NULL; }
    pthread_mutex_unlock(&g_reg_mu);
}

static int round16(int k) { return (k + 15) & ~15; }

#define EC_MAX_TENSORS 4096   /* tensor entries of one .ecm file */

/* ---- uploads ---- */

static int ec_upload(void **dst, const void *src, size_t bytes)
{
    CK(cudaMalloc(dst, bytes ? bytes : 16));
    if (bytes) CK(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice));
    return 0;
}

static int ec_upload_f32(float **dst, const float *src, int n)
{
    if (!src) { *dst = NULL; return 0; }
    return ec_upload((void **)dst, src, (size_t)n * sizeof(float));
}

/* Build a packed linear: row r of the device matrix is host row rows_w[r]
 * (K elements), its scale *rows_s[r] and bias *rows_b[r] (either table or
 * entry may be NULL: scale 1 / no bias).  Host tensors may be unaligned. */
static int ec_make_lin(ec_lin *l, int wt, int K, int N, int unit, const void *const *rows_w,
                       const float *const *rows_s, const float *const *rows_b)
{
    memset(l, 0, sizeof *l);
    const int elt = wt == EC_W_I8 ? 1 : 2;
    l->N = N;
    l->K = K;
    l->Kp = round16(K);
    l->ldw = l->Kp + 16 / elt;
    l->wt = wt;
    l->unit = unit;
    const size_t rb = (size_t)l->ldw * elt;
    unsigned char *hw = calloc((size_t)N, rb);
    if (!hw) { ec_seterr("out of host memory"); return -1; }
    for (int r = 0; r < N; r++) {
        unsigned char *row = hw + (size_t)r * rb;
        memcpy(row, rows_w[r], (size_t)K * elt);
        float tail[4] = {1.0f, 0.0f, 0.0f, 0.0f};
        if (rows_s && rows_s[r]) memcpy(&tail[0], rows_s[r], 4);
        if (rows_b && rows_b[r]) memcpy(&tail[1], rows_b[r], 4);
        memcpy(row + (size_t)l->Kp * elt, tail, sizeof tail);
    }
    int rc = ec_upload(&l->w, hw, (size_t)N * rb);
    free(hw);
    if (rc) return -1;
    int have_s = 0, have_b = 0;
    for (int r = 0; r < N; r++) {
        have_s |= rows_s && rows_s[r] != NULL;
        have_b |= rows_b && rows_b[r] != NULL;
    }
    float *tmp = malloc((size_t)N * sizeof(float));
    for (int pass = 0; pass < 2 && !rc; pass++) {
        if (!(pass == 0 ? have_s : have_b)) continue;
        const float *const *src = pass == 0 ? rows_s : rows_b;
        for (int r = 0; r < N; r++) {
            float v = pass == 0 ? 1.0f : 0.0f;
            if (src[r]) memcpy(&v, src[r], 4);
            tmp[r] = v;
        }
        rc = ec_upload((void **)(pass == 0 ? &l->s : &l->b), tmp, (size_t)N * sizeof(float));
    }
    free(tmp);
    return rc;
}

static void ec_free_lin(ec_lin *l)
{
    cudaFree(l->w);
    cudaFree(l->s);
    cudaFree(l->b);
    memset(l, 0, sizeof *l);
}

#define ROWP(base, r, K, elt) ((const void *)((const char *)(base) + (size_t)(r) * (K) * (elt)))
#define SCP(base, r) ((base) ? (const float *)((const char *)(base) + (size_t)(r) * 4) : NULL)

/* A plain linear (file order). */
static int ec_plain_lin(ec_lin *l, int wt, const void *w, const float *s, const float *b, int N, int K)
{
    const int elt = wt == EC_W_I8 ? 1 : 2;
    const void **rw = malloc((size_t)N * sizeof *rw);
    const float **rs = malloc((size_t)N * sizeof *rs), **rbias = malloc((size_t)N * sizeof *rbias);
    for (int r = 0; r < N; r++) {
        rw[r] = ROWP(w, r, K, elt);
        rs[r] = SCP(s, r);
        rbias[r] = SCP(b, r);
    }
    int rc = ec_make_lin(l, wt, K, N, 1, rw, rs, rbias);
    free(rw); free(rs); free(rbias);
    return rc;
}

/* Qwen2 q|k|v packed: in every q and k head the RoPE partners i and
 * i + head_dim/2 become rows 2i and 2i+1; then the v rows in file order.
 * The reference passes no bias to these projections (src/gpt2.c:709-711). */
static int ec_qkv_lin(ec_lin *l, int wt, const struct LayerW *S, int E, int kv, int hd, int H, int KVH)
{
    const int elt = wt == EC_W_I8 ? 1 : 2, half = hd / 2, N = E + 2 * kv;
    const void **rw = malloc((size_t)N * sizeof *rw);
    const float **rs = malloc((size_t)N * sizeof *rs);
    int r = 0;
    for (int h = 0; h < H + KVH; h++) {
        const void *w = h < H ? S->q_w : S->k_w;
        const float *s = h < H ? S->q_s : S->k_s;
        const int base = (h < H ? h : h - H) * hd;
        for (int i = 0; i < half; i++)
            for (int t = 0; t < 2; t++, r++) {
                rw[r] = ROWP(w, base + i + t * half, E, elt);
                rs[r] = SCP(s, base + i + t * half);
            }
    }
    for (int d = 0; d < kv; d++, r++) {
        rw[r] = ROWP(S->v_w, d, E, elt);
        rs[r] = SCP(S->v_s, d);
    }
    int rc = ec_make_lin(l, wt, E, N, 2, rw, rs, NULL);
    free(rw); free(rs);
    return rc;
}

/* Qwen2 gate|up interleaved: row 2j = gate j, row 2j+1 = up j. */
static int ec_gateup_lin(ec_lin *l, int wt, const struct LayerW *S, int E, int I)
{
    const int elt = wt == EC_W_I8 ? 1 : 2;
    const void **rw = malloc((size_t)2 * I * sizeof *rw);
    const float **rs = malloc((size_t)2 * I * sizeof *rs);
    for (int j = 0; j < I; j++) {
        rw[2 * j] = ROWP(S->gate_w, j, E, elt);
        rs[2 * j] = SCP(S->gate_s, j);
        rw[2 * j + 1] = ROWP(S->up_w, j, E, elt);
        rs[2 * j + 1] = SCP(S->up_s, j);
    }
    int rc = ec_make_lin(l, wt, E, 2 * I, 2, rw, rs, NULL);
    free(rw); free(rs);
    return rc;
}

/* RoPE tables: inverse frequencies with the YaRN ramp and cos/sin per position
 * scaled by the attention factor, in fp64 (reference src/gpt2.c:608-654). */
static int ec_rope_tables(ec_dev *d, const GPT2 *g)
{
    const int half = d->hd / 2, dim = 2 * half;
    double *inv = malloc((size_t)half * sizeof(double));
    for (int i = 0; i < half; i++) inv[i] = pow(1.0 / g->rope_theta, (double)(2 * i) / (double)dim);
    if (g->rope_type == ROPE_YARN) {
        const double two_pi = 6.28318530717958647692;
        const double lb = log(g->rope_theta);
        double lo = floor((double)dim * log(g->yarn_orig_max / (32.0 * two_pi)) / (2.0 * lb));
        double hi = ceil((double)dim * log(g->yarn_orig_max / (1.0 * two_pi)) / (2.0 * lb));
        if (lo < 0.0) lo = 0.0;
        if (hi > (double)(dim - 1)) hi = (double)(dim - 1);
        const double span = hi - lo < 1.0 ? 1.0 : hi - lo;
        for (int i = 0; i < half; i++) {
            double ramp = ((double)i - lo) / span;
            ramp = ramp < 0.0 ? 0.0 : (ramp > 1.0 ? 1.0 : ramp);
            const double e = inv[i];
            inv[i] = (e / g->yarn_factor) * ramp + e * (1.0 - ramp);
        }
    }
    const size_t n = (size_t)d->C * half;
    double *c = malloc(n * sizeof(double)), *s = malloc(n * sizeof(double));
    const double scale = g->yarn_attention_factor;
    for (int p = 0; p < d->C; p++)
        for (int i = 0; i < half; i++) {
            const double f = (double)p * inv[i];
            c[(size_t)p * half + i] = cos(f) * scale;
            s[(size_t)p * half + i] = sin(f) * scale;
        }
    int rc = ec_upload((void **)&d->rope_cos, c, n * sizeof(double));
    if (!rc) rc = ec_upload((void **)&d->rope_sin, s, n * sizeof(double));
    free(inv); free(c); free(s);
    return rc;
}

/* 16-bit [rows][E] table -> device with row stride Ep. */
static int ec_upload_table(uint16_t **dst, const uint16_t *src, int rows, int E, int Ep)
{
    CK(cudaMalloc((void **)dst, (size_t)rows * Ep * 2));
    if (Ep != E) CK(cudaMemset(*dst, 0, (size_t)rows * Ep * 2));
    CK(cudaMemcpy2D(*dst, (size_t)Ep * 2, src, (size_t)E * 2, (size_t)E * 2, (size_t)rows, cudaMemcpyHostToDevice));
    return 0;
}

/* ---- persistent-kernel descriptors ---- */

static ec_mk_mat ec_mk_of(const ec_lin *l)
{
    ec_mk_mat m;
    memset(&m, 0, sizeof m);
    m.w = l->w;
    m.N = l->N;
    m.K = l->K;
    m.Kp = l->Kp;
    m.ldw = l->ldw;
    m.meta = l->ldw > l->Kp ? ((l->s ? 1 : 0) | (l->b ? 2 : 0)) : 0;
    m.unit = l->unit;
    const int rb = l->ldw * (l->wt == EC_W_I8 ? 1 : 2);
    int tr = EC_MK_TILE / rb;
    if (tr > EC_MK_MAX_TILE_ROWS) tr = EC_MK_MAX_TILE_ROWS;
    tr -= tr % l->unit;   /* as many whole units as a ring slot holds: fewest tiles per CTA */
    m.tile_rows = tr;   /* 0 if a unit of rows does not fit a ring slot */
    return m;
}

static int ec_mk_build(ec_dev *d)
{
    ec_mk_layer *h = calloc((size_t)d->L, sizeof *h);
    int ok = 1;
    for (int l = 0; l < d->L; l++) {
        const ec_dlayer *W = &d->lw[l];
        h[l].qkv = ec_mk_of(&W->qkv);
        h[l].o = ec_mk_of(&W->o);
        h[l].up = ec_mk_of(&W->up);
        h[l].down = ec_mk_of(&W->down);
        ok &= h[l].qkv.tile_rows > 0 && h[l].o.tile_rows > 0 && h[l].up.tile_rows > 0 && h[l].down.tile_rows > 0;
        h[l].n1g = W->n1g; h[l].n1b = W->n1b; h[l].n2g = W->n2g; h[l].n2b = W->n2b;
        h[l].kc = d->kc + d->layer_kv * l;
        h[l].vc = d->vc + d->layer_kv * l;
    }
    int rc = ec_upload((void **)&d->d_mk_layers, h, (size_t)d->L * sizeof *h);
    free(h);
    if (rc) return -1;
    d->mk_grid = ok ? d->num_sms : 0;   /* 0: the persistent kernel is not usable */
    /* a pair of barrier counters used alternately (each launch zeroes the
     * other one for its successor) and the abort flag, on separate lines */
    CK(cudaMalloc((void **)&d->d_bar, 512));
    d->d_abort = (int *)(d->d_bar + 64);
    d->bar_par = 0;
    d->bar_reset = 1;
    /* small results of host-array decode calls, written by the kernel
     * straight into pinned host memory */
    CK(cudaHostAlloc((void **)&d->h_res, 256, cudaHostAllocMapped));
    memset(d->h_res, 0, 256);
    if (cudaHostGetDevicePointer((void **)&d->h_res_dev, d->h_res, 0) != cudaSuccess) {
        cudaGetLastError();
        d->h_res_dev = NULL;
    }
    CK(cudaMalloc((void **)&d->d_mk_err, 16));
    CK(cudaMemset(d->d_mk_err, 0, 16));
    CK(cudaMalloc((void **)&d->amax_v, (size_t)d->num_sms * EC_MK_MT * 4));
    CK(cudaMalloc((void **)&d->amax_i, (size_t)d->num_sms * EC_MK_MT * 4));
    return 0;
}

#define EC_TILE_CNT 256

/* ---- workspaces ---- */

static void ec_free_work(ec_dev *d)
{
    cudaFree(d->x); cudaFree(d->h); cudaFree(d->qkv); cudaFree(d->q); cudaFree(d->att); cudaFree(d->act);
    cudaFree(d->big); cudaFree(d->aq); cudaFree(d->as); cudaFree(d->d_tok); cudaFree(d->d_pos); cudaFree(d->d_slot);
    cudaFree(d->d_ids); cudaFree(d->d_max);
    cudaFreeHost(d->h_in); cudaFreeHost(d->h_ids); cudaFreeHost(d->h_max);
    cudaFreeHost(d->h_blk); cudaFree(d->d_blk);
    d->h_blk = NULL;
    d->d_blk = NULL;
    d->x = d->h = d->qkv = d->q = d->att = d->act = d->big = NULL;
    d->aq = NULL;
    cudaFree(d->split);
    d->split = NULL;
    d->split_bytes = 0;
    d->as = NULL;
    d->d_tok = d->d_pos = d->d_slot = d->d_ids = NULL;
    d->d_max = NULL;
    d->h_in = d->h_ids = NULL;
    d->h_max = NULL;
    d->cap = 0;
}

/* Grow the row-indexed workspaces to at least M rows. */
static int ec_ensure(ec_dev *d, int M)
{
    if (M <= d->cap) return 0;
    int cap = d->cap ? d->cap : 8;
    while (cap < M) cap *= 2;
    CK(cudaStreamSynchronize(d->stream));
    ec_free_work(d);
    const int act = d->arch == ARCH_QWEN2 ? d->I : 4 * d->E;
    const int big = d->arch == ARCH_QWEN2 ? 2 * d->I : 1;
    const int qkvw = d->E + 2 * d->kv;
    int kmax = d->arch == ARCH_QWEN2 ? (d->E > d->I ? d->E : d->I) : 4 * d->E;
    kmax = round16(kmax);
    CK(cudaMalloc((void **)&d->x, (size_t)cap * d->E * 4));
    CK(cudaMalloc((void **)&d->h, (size_t)cap * d->E * 4));
    CK(cudaMalloc((void **)&d->qkv, (size_t)cap * qkvw * 4));
    CK(cudaMalloc((void **)&d->q, (size_t)cap * d->E * 4));
    CK(cudaMalloc((void **)&d->att, (size_t)cap * d->E * 4));
    CK(cudaMalloc((void **)&d->act, (size_t)cap * act * 4));
    CK(cudaMalloc((void **)&d->big, (size_t)cap * big * 4));
    CK(cudaMalloc((void **)&d->aq, (size_t)cap * kmax));
    CK(cudaMalloc((void **)&d->as, (size_t)cap * 4));
    if (cap >= EC_TC_MIN_M) {   /* the lm_head is always 16-bit; bf16 needs three parts */
        d->split_bytes = ec_gemm_tc_split_bytes(d->prec == 2 ? EC_W_BF16 : EC_W_F16, cap, kmax);
        CK(cudaMalloc(&d->split, d->split_bytes));
    }
    if (cap >= EC_TC_MIN_M && !d->acc32) {
        /* split-K happens for outputs of at most num_sms/2 tiles of 128 x 256 */
        d->acc32_elems = (size_t)(d->num_sms / 2) * 128 * 256;
        CK(cudaMalloc((void **)&d->acc32, d->acc32_elems * 4));
        CK(cudaMemset(d->acc32, 0, d->acc32_elems * 4));
        CK(cudaMalloc((void **)&d->tile_cnt, EC_TILE_CNT * 4));
        CK(cudaMemset(d->tile_cnt, 0, EC_TILE_CNT * 4));
    }
    CK(cudaMalloc((void **)&d->d_tok, (size_t)cap * 4));
    CK(cudaMalloc((void **)&d->d_pos, (size_t)cap * 4));
    CK(cudaMalloc((void **)&d->d_slot, (size_t)cap * 4));
    CK(cudaMalloc((void **)&d->d_ids, (size_t)cap * 4));
    CK(cudaMalloc((void **)&d->d_max, (size_t)cap * 4));
    CK(cudaMallocHost((void **)&d->h_in, (size_t)cap * 3 * 4));
    CK(cudaMallocHost((void **)&d->h_blk, (size_t)cap * 2 * 4));
    CK(cudaMalloc((void **)&d->d_blk, (size_t)cap * 2 * 4));
    CK(cudaMallocHost((void **)&d->h_ids, (size_t)cap * 4));
    CK(cudaMallocHost((void **)&d->h_max, (size_t)cap * 4));
    d->cap = cap;
    d->ws_gen++;
    return 0;
}

static int ec_pick_nsplit(int max_len)
{
    /* ~64 positions per split, power of two, each split <= 1024 positions */
    const int need = (max_len + 63) / 64;
    int ns = 1;
    while (ns < need && ns < 64) ns *= 2;
    while ((max_len + ns - 1) / ns > 1024) ns *= 2;
    return ns;
}

/* Attended-length bound for a call whose rows attend at most max_len
 * positions: a power of two >= 64, capped at eff_ctx. */
static int ec_len_bucket(const ec_dev *d, int max_len)
{
    int b = 64;
    while (b < max_len) b *= 2;
    return b < d->C ? b : d->C;
}

static int ec_ensure_attn(ec_dev *d, int M, int maxlen)
{
    const size_t need = ec_attention_scratch_floats(M, d->H, d->hd, ec_pick_nsplit(maxlen));
    if (need <= d->attn_part_floats) return 0;
    CK(cudaStreamSynchronize(d->stream));
    cudaFree(d->attn_part);
    d->attn_part = NULL;
    CK(cudaMalloc((void **)&d->attn_part, need * 4));
    d->attn_part_floats = need;
    d->ws_gen++;
    return 0;
}

static int ec_ensure_logits(ec_dev *d, int rows)
{
    if (rows <= d->logit_rows) return 0;
    CK(cudaStreamSynchronize(d->stream));
    cudaFree(d->logits);
    d->logits = NULL;
    CK(cudaMalloc((void **)&d->logits, (size_t)rows * (d->v1 - d->v0) * 4));
    d->logit_rows = rows;
    d->ws_gen++;
    return 0;
}

static int ec_ensure_amax(ec_dev *d, int M)
{
    const int chunks = 2 * d->num_sms;
    const int rows = d->cap > M ? d->cap : M;
    if (d->amax_part && d->amax_chunks >= chunks && d->cap >= M) return 0;
    CK(cudaStreamSynchronize(d->stream));
    cudaFree(d->amax_part);
    d->amax_part = NULL;
    CK(cudaMalloc(&d->amax_part, (size_t)rows * chunks * 8));
    d->amax_chunks = chunks;
    /* fused lm_head argmax: two partials per column tile of 64 or more */
    cudaFree(d->lm_part);
    d->lm_part = NULL;
    d->lm_part_bytes = (size_t)rows * 2 * ((d->V + 63) / 64) * 8;
    CK(cudaMalloc(&d->lm_part, d->lm_part_bytes));
    d->ws_gen++;
    return 0;
}

static void ec_dev_free(ec_dev *d)
{
    if (!d) return;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(d->device);
    if (d->stream) cudaStreamSynchronize(d->stream);
    ec_free_work(d);
    if (d->lw) {
        for (int l = 0; l < d->L; l++) {
            ec_dlayer *W = &d->lw[l];
            cudaFree(W->n1g); cudaFree(W->n1b); cudaFree(W->n2g); cudaFree(W->n2b);
            ec_free_lin(&W->qkv); ec_free_lin(&W->o); ec_free_lin(&W->up); ec_free_lin(&W->down);
        }
        free(d->lw);
    }
    if (d->lm != d->wte) cudaFree(d->lm);
    cudaFree(d->wte); cudaFree(d->wpe); cudaFree(d->nfg); cudaFree(d->nfb);
    cudaFree(d->kc); cudaFree(d->vc); cudaFree(d->rope_cos); cudaFree(d->rope_sin);
    cudaFreeHost(d->h_pt); cudaFree(d->d_pt); free(d->free_pages); free(d->kv_undo);
    cudaFree(d->d_mk_layers); cudaFree(d->d_bar); cudaFree(d->d_mk_err);
    cudaFreeHost(d->h_res);
    cudaFree(d->amax_v); cudaFree(d->amax_i);
    cudaFree(d->attn_part); cudaFree(d->logits); cudaFree(d->amax_part); cudaFree(d->lm_part);
    cudaFree(d->d_hist); cudaFree(d->taps); cudaFree(d->d_counter);
    cudaFree(d->acc32); cudaFree(d->tile_cnt);
    for (int k = 0; k < 2; k++)
        if (d->bg[k].exec) cudaGraphExecDestroy(d->bg[k].exec);
    cudaFreeHost(d->h_logits);
    if (d->prof_ready)
        for (int i = 0; i < 2 * EC_PROF_MAX; i++) cudaEventDestroy(d->prof_ev[i]);
    if (d->own_stream) cudaStreamDestroy(d->own_stream);
    free(d);
    cudaSetDevice(cur);
}

static int ec_set_lm_shard(ec_dev *d, int v0, int v1)
{
    d->v0 = v0;
    d->v1 = v1;
    d->logit_rows = 0;
    cudaFree(d->logits);
    d->logits = NULL;
    d->ws_gen++;
    return 0;
}

static ec_lin ec_lm_lin(const ec_dev *d)
{
    ec_lin l;
    memset(&l, 0, sizeof l);
    l.w = (char *)d->lm + (size_t)d->v0 * d->Ep * 2;
    l.N = d->v1 - d->v0;
    l.K = d->E;
    l.Kp = d->Ep;
    l.ldw = d->Ep;   /* the embedding table: no metadata tail */
    l.wt = d->hwt;
    l.unit = 1;
    return l;
}

static int ec_dev_build(GPT2 *g, ec_dev *d)
{
    d->owner = g;
    CK(cudaGetDevice(&d->device));
    CK(cudaDeviceGetAttribute(&d->num_sms, cudaDevAttrMultiProcessorCount, d->device));
    CK(cudaStreamCreateWithFlags(&d->own_stream, cudaStreamNonBlocking));
    d->stream = d->own_stream;
    if (ec_kernels_init()) { ec_seterr("kernel init failed: %s", cudaGetErrorString(cudaGetLastError())); return -1; }
    d->arch = g->arch;
    d->prec = g->precision;
    d->wt = g->precision == 0 ? EC_W_I8 : (g->precision == 1 ? EC_W_F16 : EC_W_BF16);
    d->hwt = g->precision == 2 ? EC_W_BF16 : EC_W_F16;
    d->L = g->n_layer;
    d->E = g->n_embd;
    d->Ep = round16(g->n_embd);
    d->H = g->n_head;
    d->KVH = g->n_kv_head;
    d->hd = g->head_dim;
    d->kv = g->n_kv_embd;
    d->I = g->intermediate;
    d->V = g->vocab;
    d->C = gpt2_eff_ctx(g);
    d->B = g->batch_cap;
    d->eps = g->eps;
    d->window = g->arch == ARCH_QWEN2 ? g->sliding_window : 0;
    if (d->hd % 8 || d->hd > 256 || d->hd < 8) { ec_seterr("unsupported head_dim %d", d->hd); return -1; }
    if (d->E != d->H * d->hd) { ec_seterr("n_embd must equal n_head * head_dim"); return -1; }

    if (ec_upload_table(&d->wte, g->wte, d->V, d->E, d->Ep)) return -1;
    if (g->wpe && ec_upload_table(&d->wpe, g->wpe, g->n_ctx, d->E, d->Ep)) return -1;
    if (g->lm_head) {
        if (ec_upload_table(&d->lm, g->lm_head, d->V, d->E, d->Ep)) return -1;
    } else {
        d->lm = d->wte;
    }
    if (ec_upload_f32(&d->nfg, g->lnf_g, d->E) || ec_upload_f32(&d->nfb, g->lnf_b, d->E)) return -1;

    d->lw = calloc((size_t)d->L, sizeof *d->lw);
    const int E = d->E, kv = d->kv, I = d->I;
    for (int l = 0; l < d->L; l++) {
        const struct LayerW *S = &g->lw[l];
        ec_dlayer *W = &d->lw[l];
        if (ec_upload_f32(&W->n1g, S->ln1_g, E) || ec_upload_f32(&W->n2g, S->ln2_g, E)) return -1;
        if (d->arch == ARCH_GPT2) {
            if (ec_upload_f32(&W->n1b, S->ln1_b, E) || ec_upload_f32(&W->n2b, S->ln2_b, E)) return -1;
            if (ec_plain_lin(&W->qkv, d->wt, S->attn_w, S->attn_s, S->attn_b, 3 * E, E) ||
                ec_plain_lin(&W->o, d->wt, S->proj_w, S->proj_s, S->proj_b, E, E) ||
                ec_plain_lin(&W->up, d->wt, S->fc_w, S->fc_s, S->fc_b, 4 * E, E) ||
                ec_plain_lin(&W->down, d->wt, S->fc2_w, S->fc2_s, S->fc2_b, E, 4 * E)) return -1;
        } else {
            /* no biases: the reference passes NULL to every Qwen2 projection */
            if (ec_qkv_lin(&W->qkv, d->wt, S, E, kv, d->hd, d->H, d->KVH) ||
                ec_plain_lin(&W->o, d->wt, S->o_w, S->o_s, NULL, E, E) ||
                ec_gateup_lin(&W->up, d->wt, S, E, I) ||
                ec_plain_lin(&W->down, d->wt, S->down_w, S->down_s, NULL, E, I)) return -1;
        }
    }
    ec_set_lm_shard(d, 0, d->V);

    /* paged KV arena: every slot's full context by default; EDGECORE_KV_PAGES
     * sets a smaller pool that slots draw from as their positions grow */
    d->mp = (d->C + EC_KV_PAGE - 1) / EC_KV_PAGE;
    d->kv_pages = d->B * d->mp;
    {
        const char *env = getenv("EDGECORE_KV_PAGES");
        if (env && atoi(env) > 0 && atoi(env) < d->kv_pages) d->kv_pages = atoi(env);
    }
    d->layer_kv = (size_t)d->kv_pages * EC_KV_PAGE * d->kv;
    CK(cudaMalloc((void **)&d->kc, d->layer_kv * d->L * 2));
    CK(cudaMalloc((void **)&d->vc, d->layer_kv * d->L * 2));
    CK(cudaMemset(d->kc, 0, d->layer_kv * d->L * 2));
    CK(cudaMemset(d->vc, 0, d->layer_kv * d->L * 2));
    CK(cudaMallocHost((void **)&d->h_pt, (size_t)d->B * d->mp * 4));
    CK(cudaMalloc((void **)&d->d_pt, (size_t)d->B * d->mp * 4));
    d->free_pages = malloc((size_t)d->kv_pages * sizeof(int));
    d->kv_undo = malloc((size_t)d->B * d->mp * sizeof(int));
    if (!d->free_pages || !d->kv_undo) { ec_seterr("out of host memory"); return -1; }
    for (int i = 0; i < d->B * d->mp; i++) d->h_pt[i] = -1;
    for (int i = 0; i < d->kv_pages; i++) d->free_pages[i] = d->kv_pages - 1 - i;   /* pop 0, 1, 2, ... */
    d->nfree = d->kv_pages;
    CK(cudaMemcpy(d->d_pt, d->h_pt, (size_t)d->B * d->mp * 4, cudaMemcpyHostToDevice));
    if (d->arch == ARCH_QWEN2 && ec_rope_tables(d, g)) return -1;
    if (ec_mk_build(d)) return -1;
    if (ec_ensure(d, d->B > 8 ? d->B : 8)) return -1;
    CK(cudaDeviceSynchronize());
    return 0;
}

/* ------------------------------------------------------------------ */
/* load / free (reference src/gpt2.c:161-387)                          */
/* ------------------------------------------------------------------ */

static void *ec_shadow_alloc(size_t bytes)
{
    void *p = mmap(NULL, bytes ? bytes : 4096, PROT_READ | PROT_WRITE,
                   MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0);
    return p == MAP_FAILED ? NULL : p;
}

static size_t ec_shadow_bytes(const GPT2 *g)
{
    return (size_t)g->n_layer * g->batch_cap * gpt2_eff_ctx(g) * g->n_kv_embd * sizeof(uint16_t);
}

static void ec_host_free(GPT2 *g)
{
    if (g->tok.id_to_token && tokenizer_free) tokenizer_free(&g->tok);
    free(g->lw);
    const size_t kvb = ec_shadow_bytes(g);
    if (g->k_cache) munmap(g->k_cache, kvb ? kvb : 4096);
    if (g->v_cache) munmap(g->v_cache, kvb ? kvb : 4096);
    if (g->file_data) {
        if (g->file_mapped) munmap(g->file_data, g->file_size);
        else free(g->file_data);
    }
}

static void ec_defaults_qwen2(GPT2 *g)
{
    if (g->n_kv_head <= 0) g->n_kv_head = g->n_head;
    g->head_dim = g->n_embd / (g->n_head > 0 ? g->n_head : 1);
    g->n_kv_embd = g->n_kv_head * g->head_dim;
    if (g->intermediate <= 0) g->intermediate = 4 * g->n_embd;
    if (g->rope_theta <= 0) g->rope_theta = 10000.0;
    if (g->yarn_orig_max <= 0) g->yarn_orig_max = g->n_ctx;
    if (g->yarn_factor <= 0) g->yarn_factor = 1.0;
    if (g->yarn_attention_factor <= 0) g->yarn_attention_factor = 1.0;
}

static int ec_load_fail(EcmTensor *t, const char *msg, const char *arg)
{
    ec_seterr(msg, arg);
    fprintf(stderr, "%s\n", g_err);
    free(t);
    return -1;
}

static int ec_load_host(GPT2 *g, const char *path, int batch_cap, int max_ctx)
{
    memset(g, 0, sizeof *g);
    g->batch_cap = batch_cap < 1 ? 1 : batch_cap;
    g->max_ctx = max_ctx > 0 ? max_ctx : 0;
    g->eps = 1e-5;
    int fd = open(path, O_RDONLY);
    if (fd < 0) { perror("open model"); ec_seterr("cannot open %s", path); return -1; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) { close(fd); ec_seterr("empty model file"); return -1; }
    void *map = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) { perror("mmap model"); ec_seterr("mmap failed"); return -1; }
    g->file_data = map;
    g->file_size = (size_t)st.st_size;
    g->file_mapped = 1;

    /* The reference's table holds 512 entries (src/gpt2.c:180-181), too few
     * for a 28-layer Qwen2 with q/k/v biases (534 tensors, BASELINE config
     * 4's Qwen2.5-1.5B); this loader's holds EC_MAX_TENSORS. */
    EcmTensor *t = calloc(EC_MAX_TENSORS, sizeof *t);
    if (!t) { ec_seterr("out of host memory"); return -1; }
    const int n = ecm_parse(g->file_data, g->file_size, t, EC_MAX_TENSORS, g);
    if (n < 0) return ec_load_fail(t, "ecm: parse failed%s", "");
    const char *base = g->file_data;
    for (int i = 0; i < n; i++)
        if (t[i].offset + t[i].bytes > g->file_size) return ec_load_fail(t, "ecm: tensor %s past end of file", t[i].name);
    const EcmTensor *wte = ec_find(t, n, "wte"), *lnf = ec_find(t, n, "ln_f.g");
    if (!wte || !lnf) return ec_load_fail(t, "ecm: missing core tensors (wte, ln_f.g)%s", "");
    g->wte = (const uint16_t *)(base + wte->offset);
    g->lnf_g = (const float *)(base + lnf->offset);
    const char *lin0 = g->arch == ARCH_QWEN2 ? "blocks.0.q.w" : "blocks.0.attn.w";
    const EcmTensor *t0 = ec_find(t, n, lin0);
    if (!t0) return ec_load_fail(t, "ecm: missing %s", lin0);
    if (t0->dtype == 1) g->precision = 1;
    else if (t0->dtype == 2) g->precision = 0;
    else if (t0->dtype == 4) g->precision = 2;
    else return ec_load_fail(t, "ecm: unexpected linear weight dtype%s", "");
    if (g->arch == ARCH_QWEN2) ec_defaults_qwen2(g);
    if (g->arch == ARCH_GPT2) {
        const EcmTensor *wpe = ec_find(t, n, "wpe"), *lnb = ec_find(t, n, "ln_f.b");
        if (!wpe || !lnb) return ec_load_fail(t, "ecm: missing wpe / ln_f.b%s", "");
        g->wpe = (const uint16_t *)(base + wpe->offset);
        g->lnf_b = (const float *)(base + lnb->offset);
        g->n_kv_embd = g->n_embd;
        g->n_kv_head = g->n_head;
        g->intermediate = 4 * g->n_embd;
        g->head_dim = g->n_embd / (g->n_head > 0 ? g->n_head : 1);
    } else {
        const EcmTensor *lmh = ec_find(t, n, "lm_head.w");
        if (lmh && !g->tie_word_embeddings) g->lm_head = (const uint16_t *)(base + lmh->offset);
        if (g->tie_word_embeddings || !lmh) g->tie_word_embeddings = 1;
    }
    if (g->vocab <= 0 || g->n_layer <= 0 || g->n_embd <= 0 || g->n_head <= 0 || g->n_ctx <= 0)
        return ec_load_fail(t, "ecm: bad dimensions%s", "");
    if (wte->bytes < (size_t)g->vocab * g->n_embd * 2) return ec_load_fail(t, "ecm: wte smaller than vocab x n_embd%s", "");
    g->lw = calloc((size_t)g->n_layer, sizeof *g->lw);
    char nm[256];
    for (int l = 0; l < g->n_layer; l++) {
        struct LayerW *W = &g->lw[l];
        const float **nv[4] = {&W->ln1_g, &W->ln1_b, &W->ln2_g, &W->ln2_b};
        const char *nn[4] = {"ln_1.g", "ln_1.b", "ln_2.g", "ln_2.b"};
        for (int i = 0; i < 4; i++) {
            snprintf(nm, sizeof nm, "blocks.%d.%s", l, nn[i]);
            const EcmTensor *x = ec_find(t, n, nm);
            if (x) *nv[i] = (const float *)(base + x->offset);
        }
        if (!W->ln1_g || !W->ln2_g || (g->arch == ARCH_GPT2 && (!W->ln1_b || !W->ln2_b))) {
            snprintf(nm, sizeof nm, "blocks.%d.ln_*", l);
            return ec_load_fail(t, "ecm: missing norm tensors %s", nm);
        }
        const char *qn[7] = {"q", "k", "v", "o", "gate", "up", "down"};
        const void **qw[7] = {&W->q_w, &W->k_w, &W->v_w, &W->o_w, &W->gate_w, &W->up_w, &W->down_w};
        const float **qs[7] = {&W->q_s, &W->k_s, &W->v_s, &W->o_s, &W->gate_s, &W->up_s, &W->down_s};
        const float **qb[7] = {&W->q_b, &W->k_b, &W->v_b, &W->o_b, &W->gate_b, &W->up_b, &W->down_b};
        const char *gn[4] = {"attn", "proj", "fc", "fc2"};
        const void **gw[4] = {&W->attn_w, &W->proj_w, &W->fc_w, &W->fc2_w};
        const float **gs[4] = {&W->attn_s, &W->proj_s, &W->fc_s, &W->fc2_s};
        const float **gb[4] = {&W->attn_b, &W->proj_b, &W->fc_b, &W->fc2_b};
        const int cnt = g->arch == ARCH_QWEN2 ? 7 : 4;
        for (int s = 0; s < cnt; s++) {
            const char *sf = g->arch == ARCH_QWEN2 ? qn[s] : gn[s];
            snprintf(nm, sizeof nm, "blocks.%d.%s.w", l, sf);
            const EcmTensor *tw = ec_find(t, n, nm);
            snprintf(nm, sizeof nm, "blocks.%d.%s.s", l, sf);
            const EcmTensor *ts = ec_find(t, n, nm);
            snprintf(nm, sizeof nm, "blocks.%d.%s.b", l, sf);
            const EcmTensor *tb = ec_find(t, n, nm);
            if (!tw || (g->arch == ARCH_GPT2 && !tb) || (g->arch == ARCH_GPT2 && g->precision == 0 && !ts)) {
                snprintf(nm, sizeof nm, "blocks.%d.%s", l, sf);
                return ec_load_fail(t, "ecm: missing %s tensors", nm);
            }
            const void *wp = base + tw->offset;
            const float *sp = (g->precision == 0 && ts) ? (const float *)(base + ts->offset) : NULL;
            const float *bp = tb ? (const float *)(base + tb->offset) : NULL;
            if (g->arch == ARCH_QWEN2) { *qw[s] = wp; *qs[s] = sp; *qb[s] = bp; }
            else { *gw[s] = wp; *gs[s] = sp; *gb[s] = bp; }
        }
    }
    const size_t kvb = ec_shadow_bytes(g);
    g->k_cache = ec_shadow_alloc(kvb);
    g->v_cache = ec_shadow_alloc(kvb);
    if (!g->k_cache || !g->v_cache) return ec_load_fail(t, "host KV shadow allocation failed%s", "");
    if (tokenizer_load) {
        const EcmTensor *tv = ec_find(t, n, "tokenizer.vocab"), *tm = ec_find(t, n, "tokenizer.merges");
        if (!tv || !tm) return ec_load_fail(t, "ecm: tokenizer blobs missing%s", "");
        if (tokenizer_load(&g->tok, base + tv->offset, tv->bytes, base + tm->offset, tm->bytes, g->vocab,
                           g->arch == ARCH_QWEN2 ? 1 : 0) != 0)
            return ec_load_fail(t, "tokenizer_load failed%s", "");
    }
    free(t);
    return 0;
}

EC_EXPORT int gpt2_load(GPT2 *g, const char *path, int batch_cap, int max_ctx)
{
    g_err[0] = 0;
    if (ec_load_host(g, path, batch_cap, max_ctx)) {
        if (!g_err[0]) ec_seterr("load failed");
        fprintf(stderr, "edgecore_b200: %s\n", g_err);
        ec_host_free(g);
        memset(g, 0, sizeof *g);
        return -1;
    }
    ec_dev *d = calloc(1, sizeof *d);
    if (ec_dev_build(g, d) || ec_register(g, d)) {
        fprintf(stderr, "edgecore_b200: device setup failed: %s\n", g_err);
        ec_dev_free(d);
        ec_host_free(g);
        memset(g, 0, sizeof *g);
        return -1;
    }
    return 0;
}

EC_EXPORT void gpt2_free(GPT2 *g)
{
    if (!g) return;
    ec_dev *d = ec_lookup(g);
    if (d) {
        ec_unregister(g);
        ec_dev_free(d);
    }
    ec_host_free(g);
    memset(g, 0, sizeof *g);
}

/* ------------------------------------------------------------------ */
/* forward                                                              */
/* ------------------------------------------------------------------ */

static ec_tokens ec_tk(const ec_dev *d)
{
    ec_tokens tk;
    tk.tok = d->d_tok;
    tk.pos = d->d_pos;
    tk.slot = d->d_slot;
    return tk;
}

static ec_kvgeo ec_geo(const ec_dev *d, int l)
{
    ec_kvgeo g;
    g.kc = d->kc + d->layer_kv * l;
    g.vc = d->vc + d->layer_kv * l;
    g.pt = d->d_pt;
    g.mp = d->mp;
    g.B = d->B;
    g.C = d->C;
    g.kv = d->kv;
    g.E = d->E;
    g.hd = d->hd;
    g.rope_cos = d->rope_cos;
    g.rope_sin = d->rope_sin;
    return g;
}

/* Profiling marks: event pairs around every launch while prof_on. */
static int ec_prof_begin(ec_dev *d, int cls, double bytes)
{
    if (!d->prof_on || d->prof_n >= EC_PROF_MAX) return -1;
    const int i = d->prof_n++;
    d->prof_cls[i] = cls;
    d->prof_bytes[i] = bytes;
    cudaEventRecord(d->prof_ev[2 * i], d->stream);
    return i;
}

static void ec_prof_end(ec_dev *d, int i)
{
    if (i >= 0) cudaEventRecord(d->prof_ev[2 * i + 1], d->stream);
}

/* Algorithmic HBM bytes of one linear over M rows: weights (+scales, bias),
 * activations in, outputs out. */
static double ec_lin_bytes(const ec_lin *l, int M)
{
    const double elt = l->wt == EC_W_I8 ? 1.0 : 2.0;
    return (double)l->N * l->K * elt + (l->s ? 4.0 * l->N : 0.0) + (l->b ? 4.0 * l->N : 0.0) + 4.0 * M * l->K +
           4.0 * M * l->N;
}

/* Algorithmic HBM bytes of one decode step of M rows whose attention reads
 * `kv_positions` cached positions per row on average. */
static double ec_step_bytes(const ec_dev *d, int M, double kv_positions)
{
    double b = 0.0;
    for (int l = 0; l < d->L; l++) {
        const ec_dlayer *W = &d->lw[l];
        b += ec_lin_bytes(&W->qkv, M) + ec_lin_bytes(&W->o, M) + ec_lin_bytes(&W->up, M) + ec_lin_bytes(&W->down, M);
        b += 4.0 * 4 * d->E;                                         /* norm gains/biases */
    }
    const ec_lin lm = ec_lm_lin(d);
    b += ec_lin_bytes(&lm, M);
    b += (double)M * d->L * 2.0 * d->kv * 2.0 * kv_positions;       /* K and V reads */
    b += (double)M * d->L * 2.0 * d->kv * 2.0;                      /* K and V writes */
    b += (double)M * d->E * 2.0;                                     /* embedding row */
    return b;
}

/* One linear on the generic GEMM path (any M): out = X . W^T with epilogue.
 * X == NULL for int8 weights: the operand is already quantised in d->aq /
 * d->as (by a fused norm or SwiGLU kernel). */
/* The launch of ec_linear, its CUDA status returned (0: enqueued). */
static int ec_linear_rc(ec_dev *d, const ec_lin *l, const float *X, int ldx, int M, float *out, int ldo, int epi)
{
    cudaStream_t st = d->stream;
    ec_gemm_args g;
    memset(&g, 0, sizeof g);
    g.W = l->w; g.wscale = l->s; g.bias = l->b;
    g.wt = l->wt; g.N = l->N; g.K = l->K; g.Kp = l->Kp; g.ldw = l->ldw; g.M = M;
    int pi = ec_prof_begin(d, EC_PC_GEMM, ec_lin_bytes(l, M));
    if (l->wt == EC_W_I8) {
        if (X) CK(ec_launch_quant(d->aq, d->as, X, ldx, M, l->K, l->Kp, st));
        g.Aq = d->aq;
        g.a_scale = d->as;
    } else {
        g.X = X;
        g.ldx = ldx;
    }
    g.out = out; g.ldo = ldo; g.epi = epi;
    g.split = d->split; g.split_bytes = d->split_bytes;
    g.acc32 = d->acc32; g.acc32_elems = d->acc32_elems; g.tile_cnt = d->tile_cnt; g.cnt_elems = EC_TILE_CNT;
    const int rc = ec_launch_gemm(&g, st);
    ec_prof_end(d, pi);
    return rc;
}

static int ec_linear(ec_dev *d, const ec_lin *l, const float *X, int ldx, int M, float *out, int ldo, int epi)
{
    CK(ec_linear_rc(d, l, X, ldx, M, out, ldo, epi));
    return 0;
}

/* Per-layer kernels for rows already staged in d_tok/d_pos/d_slot: the
 * prefill path.  Leaves the normed final hidden state in d->h. */
static int ec_enqueue_body(ec_dev *d, int M, int maxlen)
{
    cudaStream_t st = d->stream;
    const int E = d->E, ldqkv = E + 2 * d->kv;
    int pi = ec_prof_begin(d, EC_PC_OTHER, 0.0);
    CK(ec_launch_embed(d->x, d->wte, d->wpe, d->Ep, d->prec == 2, ec_tk(d), M, E, d->V, d->C, st));
    ec_prof_end(d, pi);
    if (d->taps_on && d->taps && M <= d->taps_rows)
        CK(cudaMemcpyAsync(d->taps, d->x, (size_t)M * E * 4, cudaMemcpyDeviceToDevice, st));
    ec_attn_args at;
    memset(&at, 0, sizeof at);
    at.q = d->q; at.ldq = E; at.out = d->att; at.ldo = E;
    at.tk = ec_tk(d); at.H = d->H; at.KVH = d->KVH; at.M = M; at.window = d->window;
    at.part = d->attn_part; at.maxlen = maxlen; at.nsplit = ec_pick_nsplit(maxlen);
    at.blocks = d->nblk > 0 ? d->d_blk : NULL;
    at.nblocks = d->nblk;
    const int wact = d->arch == ARCH_QWEN2 ? d->I : 4 * E;
    /* int8 layers: the norms and SwiGLU write the int8 operand themselves */
    const int fuse_norm = d->wt == EC_W_I8 && (size_t)E * 4 <= 48 * 1024;
    const int fuse_swiglu = fuse_norm && d->arch == ARCH_QWEN2 && (size_t)d->I * 4 <= 48 * 1024;
    for (int l = 0; l < d->L; l++) {
        ec_dlayer *W = &d->lw[l];
        pi = ec_prof_begin(d, EC_PC_NORM, 8.0 * M * E);
        if (fuse_norm) CK(ec_launch_norm_quant(d->aq, d->as, W->qkv.Kp, d->x, W->n1g, W->n1b, M, E, d->eps, st));
        else CK(ec_launch_norm(d->h, d->x, W->n1g, W->n1b, M, E, d->eps, st));
        ec_prof_end(d, pi);
        if (ec_linear(d, &W->qkv, fuse_norm ? NULL : d->h, E, M, d->qkv, ldqkv, EC_EPI_STORE)) return -1;
        pi = ec_prof_begin(d, EC_PC_OTHER, 0.0);
        CK(ec_launch_qkv_split(d->q, d->qkv, ldqkv, ec_tk(d), ec_geo(d, l), d->H, d->KVH, d->arch == ARCH_QWEN2, M, st));
        ec_prof_end(d, pi);
        at.geo = ec_geo(d, l);
        pi = ec_prof_begin(d, EC_PC_ATTN, 0.0);
        CK(ec_launch_attention(&at, st));
        ec_prof_end(d, pi);
        if (ec_linear(d, &W->o, d->att, E, M, d->x, E, EC_EPI_RESID)) return -1;
        pi = ec_prof_begin(d, EC_PC_NORM, 8.0 * M * E);
        if (fuse_norm) CK(ec_launch_norm_quant(d->aq, d->as, W->up.Kp, d->x, W->n2g, W->n2b, M, E, d->eps, st));
        else CK(ec_launch_norm(d->h, d->x, W->n2g, W->n2b, M, E, d->eps, st));
        ec_prof_end(d, pi);
        if (d->arch == ARCH_QWEN2) {
            if (ec_linear(d, &W->up, fuse_norm ? NULL : d->h, E, M, d->big, 2 * d->I, EC_EPI_STORE)) return -1;
            if (fuse_swiglu) CK(ec_launch_swiglu_quant(d->aq, d->as, W->down.Kp, d->big, 2 * d->I, d->I, M, st));
            else CK(ec_launch_swiglu(d->act, d->I, d->big, 2 * d->I, d->I, M, st));
        } else {
            if (ec_linear(d, &W->up, fuse_norm ? NULL : d->h, E, M, d->act, wact, EC_EPI_GELU)) return -1;
        }
        if (ec_linear(d, &W->down, fuse_swiglu ? NULL : d->act, wact, M, d->x, E, EC_EPI_RESID)) return -1;
        if (d->taps_on && d->taps && M <= d->taps_rows)
            CK(cudaMemcpyAsync(d->taps + (size_t)(l + 1) * M * E, d->x, (size_t)M * E * 4, cudaMemcpyDeviceToDevice, st));
    }
    pi = ec_prof_begin(d, EC_PC_NORM, 8.0 * M * E);
    CK(ec_launch_norm(d->h, d->x, d->nfg, d->nfb, M, E, d->eps, st));
    ec_prof_end(d, pi);
    return 0;
}

/* lm_head rows [r0, r0+rows) of h -> d->logits [rows][v1-v0]. */
static int ec_enqueue_lm(ec_dev *d, int r0, int rows)
{
    const ec_lin lm = ec_lm_lin(d);
    return ec_linear(d, &lm, d->h + (size_t)r0 * d->E, d->E, rows, d->logits, d->v1 - d->v0, EC_EPI_STORE);
}

/* lm_head rows [r0, r0+rows) of h and their row argmax into d_ids / d_max
 * (ids offset by v0).  When the tensor-core GEMM takes the call, the argmax
 * runs in its epilogue (per-tile partials, then k_argmax_final) and no
 * logits are written; otherwise (fewer than 64 rows, or operands the
 * tensor-core path does not take) the logits, then the argmax kernels. */
static int ec_lm_argmax_rows(ec_dev *d, int r0, int rows)
{
    const int Vs = d->v1 - d->v0;
    /* from 64 rows (measured: 128 streams 2.17 -> 2.14 ms per step; 16 and 32
     * streams 1-3 % slower fused, the epilogue's compare chains being longer
     * than the stores and the argmax pass they replace) */
    const int nch = rows >= 64 ? ec_gemm_tc_argmax_chunks(d->hwt, rows, Vs) : 0;
    if (nch > 0 && d->lm_part && (size_t)rows * nch * 8 <= d->lm_part_bytes) {
        const ec_lin lm = ec_lm_lin(d);
        const int rc = ec_linear_rc(d, &lm, d->h + (size_t)r0 * d->E, d->E, rows, (float *)d->lm_part, nch,
                                    EC_EPI_ARGMAX);
        if (rc == 0) {
            CK(ec_launch_argmax_final(d->d_ids + r0, d->d_max + r0, d->lm_part, nch, rows, d->v0, d->stream));
            return 0;
        }
        if (rc != (int)cudaErrorNotSupported) CK(rc);
        cudaGetLastError();
    }
    if (ec_enqueue_lm(d, r0, rows)) return -1;
    CK(ec_launch_argmax(d->d_ids + r0, d->d_max + r0, d->logits, Vs, Vs, rows, d->v0, d->amax_part,
                        d->amax_chunks, d->stream));
    return 0;
}

/* Map KV pages for positions [0, end) of slot s (pages come off the free
 * stack in order); the table reaches the device with ec_kv_flush on the
 * model stream, ahead of the launches that use it.  Entries only go from
 * unmapped to mapped between releases, so a flush that runs later than it
 * was enqueued copies a superset of what that launch needs. */
static void ec_kv_begin(ec_dev *d) { d->nundo = 0; }

/* A call that fails maps none of its pages. */
static void ec_kv_undo(ec_dev *d)
{
    while (d->nundo > 0) {
        int *e = &d->h_pt[d->kv_undo[--d->nundo]];
        d->free_pages[d->nfree++] = *e;
        *e = -1;
    }
}

static int ec_kv_fail(ec_dev *d)
{
    ec_kv_undo(d);
    ec_seterr("KV arena full: all %d pages of %d positions are mapped (ec_kv_release frees a slot)",
              d->kv_pages, EC_KV_PAGE);
    return -1;
}

static int ec_kv_map(ec_dev *d, int s, int end)
{
    if (end > d->C) end = d->C;
    const int need = (end + EC_KV_PAGE - 1) / EC_KV_PAGE;
    for (int j = 0; j < need; j++) {
        const int idx = s * d->mp + j;
        int *e = &d->h_pt[idx];
        if (*e >= 0) continue;
        if (d->nfree == 0) return ec_kv_fail(d);
        *e = d->free_pages[--d->nfree];
        d->kv_undo[d->nundo++] = idx;
        d->pt_dirty = 1;
    }
    return 0;
}

static int ec_kv_flush(ec_dev *d)
{
    if (!d->pt_dirty) return 0;
    CK(cudaMemcpyAsync(d->d_pt, d->h_pt, (size_t)d->B * d->mp * 4, cudaMemcpyHostToDevice, d->stream));
    d->pt_dirty = 0;
    return 0;
}

/* Slots [0, M) mapped for positions [0, end). */
static int ec_kv_map_slots(ec_dev *d, int M, int end)
{
    ec_kv_begin(d);
    for (int s = 0; s < M && s < d->B; s++)
        if (ec_kv_map(d, s, end)) return -1;
    return ec_kv_flush(d);
}

/* Validate host inputs and stage tok/pos/slot into the pinned buffer. */
static int ec_stage_inputs(ec_dev *d, const int *tokens, const int *positions, const int *seqs, int M)
{
    if (M < 1) { ec_seterr("M must be >= 1 (got %d)", M); return -1; }
    if (!tokens || !positions) { ec_seterr("tokens/positions must not be NULL"); return -1; }
    if (ec_ensure(d, M)) return -1;
    CK(cudaStreamSynchronize(d->stream));   /* h_in may still feed a previous async copy */
    int *ht = d->h_in, *hp = d->h_in + M, *hs = d->h_in + 2 * M;
    ec_kv_begin(d);
    for (int m = 0; m < M; m++) {
        const int t = tokens[m], p = positions[m];
        int s = seqs ? seqs[m] : m;
        if (s >= d->B) s = d->B - 1;   /* reference clamp, src/gpt2.c:512-513 */
        if (t < 0 || t >= d->V || p < 0 || p >= d->C || s < 0) {
            ec_kv_fail(d);
            if (t < 0 || t >= d->V) ec_seterr("token id %d out of range [0,%d)", t, d->V);
            else if (p < 0 || p >= d->C) ec_seterr("position %d out of range [0,%d)", p, d->C);
            else ec_seterr("slot %d is negative", s);
            return -1;
        }
        ht[m] = t; hp[m] = p; hs[m] = s;
        if (ec_kv_map(d, s, p + 1)) return -1;
    }
    return ec_kv_flush(d);
}

static int ec_copy_inputs(ec_dev *d, int M)
{
    CK(cudaMemcpyAsync(d->d_tok, d->h_in, (size_t)M * 4, cudaMemcpyHostToDevice, d->stream));
    CK(cudaMemcpyAsync(d->d_pos, d->h_in + M, (size_t)M * 4, cudaMemcpyHostToDevice, d->stream));
    CK(cudaMemcpyAsync(d->d_slot, d->h_in + 2 * M, (size_t)M * 4, cudaMemcpyHostToDevice, d->stream));
    return 0;
}

static int ec_max_len(const ec_dev *d, int M)
{
    int mx = 1;
    for (int m = 0; m < M; m++) {
        const int p = d->h_in[M + m];
        int lo = d->window > 0 ? p - d->window + 1 : 0;
        if (lo < 0) lo = 0;
        if (p + 1 - lo > mx) mx = p + 1 - lo;
    }
    return mx;
}

/* Pinned host staging of at least `bytes` for logits copies. */
static int ec_host_logits(ec_dev *d, size_t bytes)
{
    if (bytes <= d->h_logits_cap) return 0;
    cudaFreeHost(d->h_logits);
    d->h_logits = NULL;
    d->h_logits_cap = 0;
    CK(cudaMallocHost((void **)&d->h_logits, bytes));
    d->h_logits_cap = bytes;
    return 0;
}

static int ec_check_kernel_error(ec_dev *d)
{
    int code = 0, mk = 0;
    CK(ec_kernel_error_take(d->stream, &code));
    CK(cudaMemcpy(&mk, d->d_mk_err, 4, cudaMemcpyDeviceToHost));
    if (mk) {
        CK(cudaMemset(d->d_mk_err, 0, 4));
        d->bar_reset = 1;   /* the abort flag may be set */
    }
    if (code || mk) {
        ec_seterr("device kernel reported error code %d/%d (bad index or bounded wait gave up)", code, mk);
        return -1;
    }
    return 0;
}

/* ---- the persistent decode kernel ---- */

/* Fill the kernel parameters for M rows attending at most maxlen positions;
 * returns -1 if the kernel cannot take this call (shared memory). */
static int ec_mk_plan(ec_dev *d, int M, int maxlen, ec_mk_params *p)
{
    if (!d->mk_grid || M < 1 || M > EC_MK_MT) return -1;
    /* 16-byte asynchronous copies of q rows and cached K/V rows */
    if (d->hd % 8 || d->kv % 8 || d->E % 4) return -1;
    memset(p, 0, sizeof *p);
    p->L = d->L;   /* the layer table, norm vectors, RoPE rows and owned residual rows */
    p->E = d->E;   /* are part of the shared-memory layout */
    p->hd = d->hd;
    p->own_rows = (d->E + d->mk_grid - 1) / d->mk_grid + 1;
    const int Kdown = d->lw[0].down.Kp, Kmax = d->Ep > Kdown ? d->Ep : Kdown;
    const int opb = d->wt == EC_W_I8 ? 1 : 4;
    int xbuf = M * Kmax * opb;
    if (M * d->Ep * 4 > xbuf) xbuf = M * d->Ep * 4;           /* lm_head fp32 planes */
    xbuf = (xbuf + 15) & ~15;
    int stage = M * d->E * 4;                                  /* norm rows */
    stage = (stage + 15) & ~15;
    const int limit = ec_mk_smem_limit();
    /* attention scratch (q row, scores, one K and one V chunk) overlays xbuf+stage */
    int ch = 256;
    while (ch > 8 && ch / 2 >= maxlen) ch /= 2;
    for (;;) {
        const int attn = 4 * ((d->hd + 3) & ~3) + 4 * ((maxlen + 3) & ~3) + ch * (d->hd + 8) * 2 + ch * d->hd * 2 + 64;
        p->xbuf_bytes = xbuf;
        p->stage_bytes = attn - xbuf > stage ? ((attn - xbuf + 15) & ~15) : stage;
        if ((int)ec_mk_smem_bytes(p) <= limit) break;
        if (ch <= 8) return -1;
        ch /= 2;
    }
    p->kvchunk = ch;
    const int want = (M * Kdown * 4 + 15) & ~15;               /* down-proj input staged */
    if (want > p->stage_bytes) {
        const int keep = p->stage_bytes;
        p->stage_bytes = want;
        if ((int)ec_mk_smem_bytes(p) > limit) p->stage_bytes = keep;
    }
    p->arch = d->arch;
    p->lwt = d->wt;
    p->hwt = d->hwt;
    p->L = d->L; p->E = d->E; p->H = d->H; p->KVH = d->KVH; p->hd = d->hd; p->kv = d->kv; p->I = d->I;
    p->V = d->V; p->C = d->C; p->B = d->B; p->window = d->window; p->M = M;
    p->eps = d->eps;
    p->wte = d->wte; p->wpe = d->wpe; p->ld_emb = d->Ep; p->emb_bf16 = d->prec == 2;
    p->nfg = d->nfg; p->nfb = d->nfb;
    const ec_lin lm = ec_lm_lin(d);
    p->lm = ec_mk_of(&lm);
    if (p->lm.tile_rows <= 0) return -1;
    p->v0 = d->v0;
    p->rope_cos = d->rope_cos; p->rope_sin = d->rope_sin;
    p->layers = d->d_mk_layers;
    p->x = d->x; p->q = d->q; p->att = d->att; p->act = d->act;
    p->amax_v = d->amax_v; p->amax_i = d->amax_i;
    p->tok = d->d_tok; p->pos = d->d_pos; p->slot = d->d_slot;
    p->pt = d->d_pt; p->mp = d->mp;
    p->bar = d->d_bar; p->abort_flag = d->d_abort; p->err = d->d_mk_err;
    p->maxlen = maxlen;
    p->taps = (d->taps_on && d->taps && M <= d->taps_rows) ? d->taps : NULL;
    return 0;
}

/* Launch the decode kernel on the counter of this launch; it zeroes the
 * other one for the next launch, so no reset is enqueued unless an error
 * was seen (bar_reset). */
static int ec_mk_run(ec_dev *d, const ec_mk_params *p, int n_steps)
{
    ec_mk_params q = *p;
    if (d->bar_reset) {
        CK(cudaMemsetAsync(d->d_bar, 0, 512, d->stream));   /* both counters and the abort flag */
        d->bar_reset = 0;
    }
    q.bar = d->d_bar + 32 * d->bar_par;
    q.bar_next = d->d_bar + 32 * (1 - d->bar_par);
    d->bar_par ^= 1;
    const int e = ec_mk_launch(&q, n_steps, d->mk_grid, d->stream);
    if (e) d->bar_reset = 1;   /* the next counter was not zeroed by a kernel */
    CK(e);
    return 0;
}

/* ---- host-array forward ---- */

static int ec_forward_impl(GPT2 *g, const int *tokens, const int *positions, const int *seqs, int M,
                           float *logits, int *ids, float *maxv)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded by this library"); return -1; }
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != d->device) CK(cudaSetDevice(d->device));
    if (ec_stage_inputs(d, tokens, positions, seqs, M)) return -1;
    const int maxlen = ec_len_bucket(d, ec_max_len(d, M));
    const int Vs = d->v1 - d->v0;
    ec_mk_params mp;
    if (ec_mk_plan(d, M, maxlen, &mp) == 0) {
        const size_t bytes = (size_t)M * Vs * 4;
        if (!ids && (ec_host_logits(d, bytes) || ec_ensure_logits(d, M))) return -1;
        const int mapped = d->h_res_dev != NULL;
        if (mapped) {
            /* inputs by value in the launch parameters; ids and the completion
             * word written by the kernel into pinned host memory; logits in
             * device memory and one copy (written in place by the kernel over
             * PCIe they cost more: its stores are scattered 16-byte pieces) */
            for (int m = 0; m < M; m++) {
                mp.in_tok[m] = d->h_in[m];
                mp.in_pos[m] = d->h_in[M + m];
                mp.in_slot[m] = d->h_in[2 * M + m];
            }
            mp.inline_in = 1;
            mp.logits = ids ? NULL : d->logits;
            mp.ids = d->h_res_dev + 1;
            mp.maxv = (float *)(d->h_res_dev + 1 + EC_MK_MT);
            d->res_seq = d->res_seq >= 0x3fffffff ? 1 : d->res_seq + 1;
            mp.done = d->h_res_dev;
            mp.seq = d->res_seq;
            ((volatile int *)d->h_res)[0] = 0;
        } else {
            if (ec_copy_inputs(d, M)) return -1;
            mp.logits = ids ? NULL : d->logits;
            mp.ids = d->d_ids;
            mp.maxv = d->d_max;
        }
        mp.advance = 0;
        if (ec_mk_run(d, &mp, 1)) return -1;
        if (mapped) {
            if (!ids) CK(cudaMemcpyAsync(d->h_logits, d->logits, bytes, cudaMemcpyDeviceToHost, d->stream));
            CK(cudaStreamSynchronize(d->stream));
            if (((volatile int *)d->h_res)[0] != mp.seq) {   /* aborted or an error recorded */
                if (ec_check_kernel_error(d)) return -1;
                d->bar_reset = 1;
                ec_seterr("decode kernel did not complete");
                return -1;
            }
            if (ids) {
                memcpy(ids, d->h_res + 1, (size_t)M * 4);
                if (maxv) memcpy(maxv, d->h_res + 1 + EC_MK_MT, (size_t)M * 4);
            } else {
                memcpy(logits, d->h_logits, bytes);
            }
            return 0;
        }
        if (ids) {
            CK(cudaMemcpyAsync(d->h_ids, d->d_ids, (size_t)M * 4, cudaMemcpyDeviceToHost, d->stream));
            CK(cudaMemcpyAsync(d->h_max, d->d_max, (size_t)M * 4, cudaMemcpyDeviceToHost, d->stream));
            CK(cudaStreamSynchronize(d->stream));
            memcpy(ids, d->h_ids, (size_t)M * 4);
            if (maxv) memcpy(maxv, d->h_max, (size_t)M * 4);
        } else {
            CK(cudaMemcpyAsync(d->h_logits, d->logits, bytes, cudaMemcpyDeviceToHost, d->stream));
            CK(cudaStreamSynchronize(d->stream));
            memcpy(logits, d->h_logits, bytes);
        }
        return ec_check_kernel_error(d);
    }
    /* prefill path: per-layer kernels, lm_head in row chunks */
    if (ec_copy_inputs(d, M)) return -1;
    if (ec_ensure_attn(d, M, maxlen)) return -1;
    /* blocks of up to EC_ATTN_RUN consecutive rows of one slot at consecutive
     * positions; when they average 8 rows or more (prefill), the block
     * attention kernel takes them (the copy is complete before h_blk is
     * written again: every host-array call synchronises the stream first) */
    int nb = 0;
    for (int m = 0; m < M;) {
        int n = 1;
        while (m + n < M && n < EC_ATTN_RUN && d->h_in[2 * M + m + n] == d->h_in[2 * M + m] &&
               d->h_in[M + m + n] == d->h_in[M + m] + n)
            n++;
        d->h_blk[2 * nb] = m;
        d->h_blk[2 * nb + 1] = n;
        nb++;
        m += n;
    }
    if (8 * nb <= M) {
        CK(cudaMemcpyAsync(d->d_blk, d->h_blk, (size_t)nb * 8, cudaMemcpyHostToDevice, d->stream));
        d->nblk = nb;
    }
    const int body = ec_enqueue_body(d, M, maxlen);
    d->nblk = 0;
    if (body) return -1;
    int chunk = (int)((256u << 20) / ((size_t)Vs * 4));
    if (chunk < 8) chunk = 8;
    if (chunk > M) chunk = M;
    if (ec_ensure_logits(d, chunk) || ec_ensure_amax(d, chunk)) return -1;
    const size_t hbytes = (size_t)chunk * Vs * 4;
    if (!ids && ec_host_logits(d, hbytes)) return -1;
    for (int r0 = 0; r0 < M; r0 += chunk) {
        const int rows = M - r0 < chunk ? M - r0 : chunk;
        if (ids) {
            if (ec_lm_argmax_rows(d, r0, rows)) return -1;
        } else {
            if (ec_enqueue_lm(d, r0, rows)) return -1;
            CK(cudaMemcpyAsync(d->h_logits, d->logits, (size_t)rows * Vs * 4, cudaMemcpyDeviceToHost, d->stream));
            CK(cudaStreamSynchronize(d->stream));
            memcpy(logits + (size_t)r0 * Vs, d->h_logits, (size_t)rows * Vs * 4);
        }
    }
    if (ids) {
        CK(cudaMemcpyAsync(d->h_ids, d->d_ids, (size_t)M * 4, cudaMemcpyDeviceToHost, d->stream));
        CK(cudaMemcpyAsync(d->h_max, d->d_max, (size_t)M * 4, cudaMemcpyDeviceToHost, d->stream));
    }
    CK(cudaStreamSynchronize(d->stream));
    if (ids) {
        memcpy(ids, d->h_ids, (size_t)M * 4);
        if (maxv) memcpy(maxv, d->h_max, (size_t)M * 4);
    }
    return ec_check_kernel_error(d);
}

EC_EXPORT void gpt2_forward(GPT2 *g, const int *tokens, const int *positions, const int *seqs, int M, float *logits)
{
    if (ec_forward_impl(g, tokens, positions, seqs, M, logits, NULL, NULL)) ec_fatal("gpt2_forward");
}

EC_EXPORT void qwen2_forward(GPT2 *g, const int *tokens, const int *positions, const int *seqs, int M, float *logits)
{
    gpt2_forward(g, tokens, positions, seqs, M, logits);
}

/* ------------------------------------------------------------------ */
/* extensions                                                           */
/* ------------------------------------------------------------------ */

EC_EXPORT GPT2 *ec_model_open(const char *path, int batch_cap, int max_ctx)
{
    GPT2 *g = calloc(1, sizeof *g);
    if (!g) { ec_seterr("out of memory"); return NULL; }
    if (gpt2_load(g, path, batch_cap, max_ctx)) { free(g); return NULL; }
    return g;
}

EC_EXPORT void ec_model_close(GPT2 *g)
{
    if (!g) return;
    gpt2_free(g);
    free(g);
}

EC_EXPORT int ec_model_info(const GPT2 *g, int *o)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    const int v[16] = {g->arch, g->precision, g->n_layer, g->n_head, g->n_kv_head, g->n_embd, g->head_dim,
                       g->intermediate, g->vocab, g->n_ctx, gpt2_eff_ctx(g), g->batch_cap, g->n_kv_embd,
                       g->tie_word_embeddings, d->device, 0};
    memcpy(o, v, sizeof v);
    return 0;
}

EC_EXPORT int ec_model_set_stream(GPT2 *g, void *stream)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    cudaStream_t s = stream ? (cudaStream_t)stream : d->own_stream;
    if (s != d->stream) {
        CK(cudaStreamSynchronize(d->stream));
        d->stream = s;
    }
    return 0;
}

EC_EXPORT int ec_forward_device(GPT2 *g, const int *d_tokens, const int *d_positions, const int *d_seqs, int M,
                                float *d_logits)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    if (M < 1 || M > EC_MK_MT) { ec_seterr("ec_forward_device: 1 <= M <= %d", EC_MK_MT); return -1; }
    if (ec_ensure(d, M)) return -1;
    /* device-resident slots and positions: every slot fully mapped */
    if (ec_kv_map_slots(d, d->B, d->C)) return -1;
    ec_mk_params mp;
    if (ec_mk_plan(d, M, d->C, &mp)) { ec_seterr("ec_forward_device: eff_ctx too long for the decode kernel"); return -1; }
    CK(cudaStreamSynchronize(d->stream));   /* h_in reuse */
    CK(cudaMemcpyAsync(d->d_tok, d_tokens, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
    CK(cudaMemcpyAsync(d->d_pos, d_positions, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
    if (d_seqs) {
        CK(cudaMemcpyAsync(d->d_slot, d_seqs, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
    } else {
        for (int m = 0; m < M; m++) d->h_in[2 * M + m] = m < d->B ? m : d->B - 1;
        CK(cudaMemcpyAsync(d->d_slot, d->h_in + 2 * M, (size_t)M * 4, cudaMemcpyHostToDevice, d->stream));
    }
    mp.logits = d_logits;
    mp.advance = 0;
    return ec_mk_run(d, &mp, 1);
}

EC_EXPORT int ec_forward_argmax(GPT2 *g, const int *tokens, const int *positions, const int *seqs, int M,
                                int *out_ids, float *out_max)
{
    if (!out_ids) { ec_seterr("out_ids must not be NULL"); return -1; }
    return ec_forward_impl(g, tokens, positions, seqs, M, NULL, out_ids, out_max);
}

EC_EXPORT int ec_forward_shard_argmax(GPT2 *g, const int *tokens, const int *positions, const int *seqs, int M,
                                      int *out_ids, float *out_max)
{
    return ec_forward_argmax(g, tokens, positions, seqs, M, out_ids, out_max);
}

/* Stage a decode run: tokens from device, positions start_pos, slots 0..M-1. */
/* Rows m < M decode from slot m at start_pos on; positions up to end - 1. */
static int ec_decode_setup(ec_dev *d, int *d_tokens, int start_pos, int M, int end)
{
    if (ec_ensure(d, M)) return -1;
    if (ec_kv_map_slots(d, M, end)) return -1;
    CK(cudaStreamSynchronize(d->stream));   /* h_in reuse */
    for (int m = 0; m < M; m++) {
        d->h_in[M + m] = start_pos;
        d->h_in[2 * M + m] = m;
    }
    CK(cudaMemcpyAsync(d->d_tok, d_tokens, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
    CK(cudaMemcpyAsync(d->d_pos, d->h_in + M, (size_t)M * 4, cudaMemcpyHostToDevice, d->stream));
    CK(cudaMemcpyAsync(d->d_slot, d->h_in + 2 * M, (size_t)M * 4, cudaMemcpyHostToDevice, d->stream));
    return 0;
}

EC_EXPORT int ec_decode_greedy_cycle(GPT2 *g, int *d_tokens, int start_pos, int period, int n_steps,
                                     int *d_out_ids)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    const int M = d->B;
    if (M > EC_MK_MT) { ec_seterr("ec_decode_greedy: batch_cap must be <= %d (got %d)", EC_MK_MT, M); return -1; }
    const int span = period > 0 && period < n_steps ? period : n_steps;
    if (n_steps < 0 || period < 0 || start_pos < 0 || start_pos + span > d->C) {
        ec_seterr("decode range [%d, %d) exceeds eff_ctx %d", start_pos, start_pos + span, d->C);
        return -1;
    }
    if (n_steps == 0) return 0;
    int max_len = start_pos + span;
    if (d->window > 0 && max_len > d->window) max_len = d->window;
    ec_mk_params mp;
    if (ec_mk_plan(d, M, ec_len_bucket(d, max_len), &mp)) {
        ec_seterr("decode range too long for the decode kernel's shared memory");
        return -1;
    }
    if (d_out_ids && d->hist_cap < n_steps * M) {
        CK(cudaStreamSynchronize(d->stream));
        cudaFree(d->d_hist);
        d->d_hist = NULL;
        d->ws_gen++;
        CK(cudaMalloc((void **)&d->d_hist, (size_t)n_steps * M * 4));
        d->hist_cap = n_steps * M;
    }
    if (ec_decode_setup(d, d_tokens, start_pos, M, start_pos + span)) return -1;
    mp.hist = d_out_ids ? d->d_hist : NULL;
    mp.advance = 1;
    mp.wrap_lo = period > 0 ? start_pos : 0;
    mp.wrap_hi = period > 0 ? start_pos + period : 0;
    if (ec_mk_run(d, &mp, n_steps)) return -1;
    if (d_out_ids)
        CK(cudaMemcpyAsync(d_out_ids, d->d_hist, (size_t)n_steps * M * 4, cudaMemcpyDeviceToDevice, d->stream));
    CK(cudaMemcpyAsync(d_tokens, d->d_tok, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
    return 0;
}

EC_EXPORT int ec_decode_greedy(GPT2 *g, int *d_tokens, int start_pos, int n_steps, int *d_out_ids)
{
    return ec_decode_greedy_cycle(g, d_tokens, start_pos, 0, n_steps, d_out_ids);
}

/* ------------------------------------------------------------------ */
/* batched decode: any number of token rows, per-layer kernels           */
/* ------------------------------------------------------------------ */

/* Rows of lm_head logits computed per chunk (<= 512 MB of logits). */
static int ec_lm_chunk(const ec_dev *d, int M)
{
    const int Vs = d->v1 - d->v0;
    int chunk = (int)((512u << 20) / ((size_t)Vs * 4));
    if (chunk < EC_TC_MIN_M) chunk = EC_TC_MIN_M;
    return chunk < M ? chunk : M;
}

/* lm_head of the vocab shard over rows [0, M) of d->h and the row argmax
 * into d_ids / d_max (global vocab ids), chunk rows at a time. */
static int ec_enqueue_lm_argmax(ec_dev *d, int M, int chunk)
{
    const int Vs = d->v1 - d->v0;
    for (int r0 = 0; r0 < M; r0 += chunk) {
        const int rows = M - r0 < chunk ? M - r0 : chunk;
        if (ec_lm_argmax_rows(d, r0, rows)) return -1;
    }
    return 0;
}

/* Workspaces of a batched call of M rows (slot m = row m) attending at most
 * maxlen positions, with lm_head chunks of `chunk` rows; kernel set-up done
 * here so that nothing allocates or sets attributes during graph capture. */
static int ec_batch_prepare(ec_dev *d, int M, int maxlen, int chunk)
{
    if (ec_ensure(d, M) || ec_ensure_attn(d, M, maxlen)) return -1;
    if (chunk > 0 && (ec_ensure_logits(d, chunk) || ec_ensure_amax(d, chunk))) return -1;
    if (!d->d_counter) CK(cudaMalloc((void **)&d->d_counter, 16));
    const int tc = ec_tc_init();
    if (tc && tc != (int)cudaErrorNotSupported) { ec_seterr("tensor-core set-up failed: %s", cudaGetErrorString((cudaError_t)tc)); return -1; }
    cudaGetLastError();
    CK(cudaStreamSynchronize(d->stream));   /* h_in reuse */
    for (int m = 0; m < M; m++) d->h_in[2 * M + m] = m;
    CK(cudaMemcpyAsync(d->d_slot, d->h_in + 2 * M, (size_t)M * 4, cudaMemcpyHostToDevice, d->stream));
    return 0;
}

/* The captured graph of kind k (0: body + lm_head argmax + token/position
 * advance; 1: body only, normed rows left in d->h), rebuilt when the shape or
 * a workspace changed. */
static int ec_bgraph(ec_dev *d, int kind, int M, int maxlen, int chunk, int hist, cudaGraphExec_t *out)
{
    if (d->bg[kind].exec && d->bg[kind].M == M && d->bg[kind].maxlen == maxlen && d->bg[kind].chunk == chunk &&
        d->bg[kind].hist == hist && d->bg[kind].gen == d->ws_gen) {
        *out = d->bg[kind].exec;
        return 0;
    }
    if (d->bg[kind].exec) {
        cudaGraphExecDestroy(d->bg[kind].exec);
        d->bg[kind].exec = NULL;
    }
    cudaGraph_t gr = NULL;
    CK(cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal));
    int rc = 0;
    rc = ec_enqueue_body(d, M, maxlen);
    if (!rc && kind == 0) rc = ec_enqueue_lm_argmax(d, M, chunk);
    if (!rc && kind == 0 &&
        ec_launch_step_advance(d->d_tok, d->d_pos, d->d_ids, M, hist ? d->d_hist : NULL, hist ? d->d_counter : NULL,
                               0, 0, d->stream))
        rc = -1;
    const cudaError_t ee = cudaStreamEndCapture(d->stream, &gr);
    if (rc || ee != cudaSuccess) {
        if (gr) cudaGraphDestroy(gr);
        cudaGetLastError();
        if (!rc) ec_seterr("stream capture failed: %s", cudaGetErrorString(ee));
        return -1;
    }
    size_t nn = 0;
    int nk = 0;
    if (cudaGraphGetNodes(gr, NULL, &nn) == cudaSuccess && nn > 0) {
        cudaGraphNode_t *nodes = malloc(nn * sizeof *nodes);
        if (nodes && cudaGraphGetNodes(gr, nodes, &nn) == cudaSuccess)
            for (size_t i = 0; i < nn; i++) {
                enum cudaGraphNodeType ty;
                if (cudaGraphNodeGetType(nodes[i], &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) nk++;
            }
        free(nodes);
    }
    const cudaError_t ei = cudaGraphInstantiate(&d->bg[kind].exec, gr, 0);
    cudaGraphDestroy(gr);
    if (ei != cudaSuccess) {
        d->bg[kind].exec = NULL;
        ec_seterr("cudaGraphInstantiate: %s", cudaGetErrorString(ei));
        return -1;
    }
    d->bg[kind].M = M;
    d->bg[kind].maxlen = maxlen;
    d->bg[kind].chunk = chunk;
    d->bg[kind].hist = hist;
    d->bg[kind].gen = d->ws_gen;
    d->bg[kind].kernels = nk;
    *out = d->bg[kind].exec;
    return 0;
}

/* Attended-length bucket for rows whose positions are < max_pos_end. */
static int ec_batch_len(const ec_dev *d, int max_pos_end)
{
    int len = max_pos_end;
    if (d->window > 0 && len > d->window) len = d->window;
    return ec_len_bucket(d, len);
}

EC_EXPORT int ec_decode_batch(GPT2 *g, int *d_tokens, int *d_positions, int n_steps, int *d_out_ids)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    if (n_steps < 0) { ec_seterr("n_steps must be >= 0"); return -1; }
    if (n_steps == 0) return 0;
    const int M = d->B;
    if (ec_ensure(d, M)) return -1;
    CK(cudaStreamSynchronize(d->stream));
    CK(cudaMemcpy(d->h_in + M, d_positions, (size_t)M * 4, cudaMemcpyDeviceToHost));
    int maxp = 0;
    ec_kv_begin(d);
    for (int m = 0; m < M; m++) {
        const int p = d->h_in[M + m];
        if (p < 0 || p + n_steps > d->C) {
            ec_kv_undo(d);
            ec_seterr("slot %d: positions [%d, %d) exceed eff_ctx %d", m, p, p + n_steps, d->C);
            return -1;
        }
        if (p + n_steps > maxp) maxp = p + n_steps;
        if (ec_kv_map(d, m, p + n_steps)) return -1;
    }
    if (ec_kv_flush(d)) return -1;
    if (M < EC_TC_MIN_M) {   /* up to 7 streams: the persistent decode kernel, one launch for all steps;
                               from 8 the per-layer graph with tensor-core GEMMs is faster */
        int max_len = maxp;
        if (d->window > 0 && max_len > d->window) max_len = d->window;
        ec_mk_params mp;
        if (ec_mk_plan(d, M, ec_len_bucket(d, max_len), &mp) == 0) {
            if (d_out_ids && d->hist_cap < n_steps * M) {
                cudaFree(d->d_hist);
                d->d_hist = NULL;
                d->ws_gen++;
                CK(cudaMalloc((void **)&d->d_hist, (size_t)n_steps * M * 4));
                d->hist_cap = n_steps * M;
            }
            for (int m = 0; m < M; m++) d->h_in[2 * M + m] = m;
            CK(cudaMemcpyAsync(d->d_tok, d_tokens, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
            CK(cudaMemcpyAsync(d->d_pos, d->h_in + M, (size_t)M * 4, cudaMemcpyHostToDevice, d->stream));
            CK(cudaMemcpyAsync(d->d_slot, d->h_in + 2 * M, (size_t)M * 4, cudaMemcpyHostToDevice, d->stream));
            mp.hist = d_out_ids ? d->d_hist : NULL;
            mp.advance = 1;
            if (ec_mk_run(d, &mp, n_steps)) return -1;
            CK(cudaMemcpyAsync(d_tokens, d->d_tok, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
            CK(cudaMemcpyAsync(d_positions, d->d_pos, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
            if (d_out_ids)
                CK(cudaMemcpyAsync(d_out_ids, d->d_hist, (size_t)n_steps * M * 4, cudaMemcpyDeviceToDevice,
                                   d->stream));
            return 0;
        }
    }
    const int maxlen = ec_batch_len(d, maxp);
    const int chunk = ec_lm_chunk(d, M);
    if (d_out_ids && d->hist_cap < n_steps * M) {
        cudaFree(d->d_hist);
        d->d_hist = NULL;
        CK(cudaMalloc((void **)&d->d_hist, (size_t)n_steps * M * 4));
        d->hist_cap = n_steps * M;
        d->ws_gen++;
    }
    if (ec_batch_prepare(d, M, maxlen, chunk)) return -1;
    CK(cudaMemcpyAsync(d->d_tok, d_tokens, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
    CK(cudaMemcpyAsync(d->d_pos, d_positions, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
    if (d_out_ids) CK(cudaMemsetAsync(d->d_counter, 0, 4, d->stream));
    cudaGraphExec_t ex;
    if (ec_bgraph(d, 0, M, maxlen, chunk, d_out_ids != NULL, &ex)) return -1;
    for (int s = 0; s < n_steps; s++) CK(cudaGraphLaunch(ex, d->stream));
    CK(cudaMemcpyAsync(d_tokens, d->d_tok, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
    CK(cudaMemcpyAsync(d_positions, d->d_pos, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
    if (d_out_ids)
        CK(cudaMemcpyAsync(d_out_ids, d->d_hist, (size_t)n_steps * M * 4, cudaMemcpyDeviceToDevice, d->stream));
    return 0;
}

EC_EXPORT int ec_batch_hidden(GPT2 *g, const int *d_tokens, const int *d_positions, int M, int max_pos_end,
                              float *d_hidden)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    if (M < 1 || M > d->B) { ec_seterr("ec_batch_hidden: 1 <= M <= batch_cap (%d), got %d", d->B, M); return -1; }
    if (max_pos_end < 1 || max_pos_end > d->C) { ec_seterr("ec_batch_hidden: max_pos_end %d outside [1, %d]", max_pos_end, d->C); return -1; }
    const int maxlen = ec_batch_len(d, max_pos_end);
    if (ec_kv_map_slots(d, M, max_pos_end)) return -1;
    if (ec_batch_prepare(d, M, maxlen, 0)) return -1;
    CK(cudaMemcpyAsync(d->d_tok, d_tokens, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
    CK(cudaMemcpyAsync(d->d_pos, d_positions, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
    cudaGraphExec_t ex;
    if (ec_bgraph(d, 1, M, maxlen, 0, 0, &ex)) return -1;
    CK(cudaGraphLaunch(ex, d->stream));
    CK(cudaMemcpyAsync(d_hidden, d->h, (size_t)M * d->E * 4, cudaMemcpyDeviceToDevice, d->stream));
    return 0;
}

EC_EXPORT int ec_lm_shard_keys(GPT2 *g, const float *d_hidden, int rows, long long *d_keys)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    if (rows < 1) { ec_seterr("ec_lm_shard_keys: rows must be >= 1"); return -1; }
    const int chunk = ec_lm_chunk(d, rows);
    if (ec_ensure(d, rows) || ec_ensure_logits(d, chunk) || ec_ensure_amax(d, chunk)) return -1;
    const int tc = ec_tc_init();
    if (tc && tc != (int)cudaErrorNotSupported) { ec_seterr("tensor-core set-up failed"); return -1; }
    cudaGetLastError();
    CK(cudaMemcpyAsync(d->h, d_hidden, (size_t)rows * d->E * 4, cudaMemcpyDeviceToDevice, d->stream));
    if (ec_enqueue_lm_argmax(d, rows, chunk)) return -1;
    CK(ec_launch_pack_keys(d->d_ids, d->d_max, rows, d_keys, d->stream));
    return 0;
}

EC_EXPORT int ec_kv_release(GPT2 *g, int slot)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    if (slot >= d->B) { ec_seterr("ec_kv_release: slot %d >= batch_cap %d", slot, d->B); return -1; }
    CK(cudaStreamSynchronize(d->stream));   /* no launch in flight still reads the pages */
    for (int s = slot < 0 ? 0 : slot; s < (slot < 0 ? d->B : slot + 1); s++)
        for (int j = 0; j < d->mp; j++) {
            int *e = &d->h_pt[(size_t)s * d->mp + j];
            if (*e < 0) continue;
            d->free_pages[d->nfree++] = *e;
            *e = -1;
            d->pt_dirty = 1;
        }
    return ec_kv_flush(d);
}

EC_EXPORT int ec_kv_info(const GPT2 *g, int *info4)
{
    ec_dev *d = ec_lookup(g);
    if (!d || !info4) { ec_seterr("ec_kv_info: no model or NULL info"); return -1; }
    info4[0] = d->kv_pages;
    info4[1] = d->nfree;
    info4[2] = EC_KV_PAGE;
    info4[3] = d->mp;
    return 0;
}

EC_EXPORT long long ec_model_packed(const GPT2 *g, int layer, int which, void *out, size_t cap, int *info5)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    if (which < 0 || which > 4 || (which < 4 && (layer < 0 || layer >= d->L))) {
        ec_seterr("ec_model_packed: bad layer %d / which %d", layer, which);
        return -1;
    }
    ec_lin lm;
    const ec_lin *l;
    if (which == 4) {
        lm = ec_lm_lin(d);
        l = &lm;
    } else {
        const ec_dlayer *W = &d->lw[layer];
        l = which == 0 ? &W->qkv : which == 1 ? &W->o : which == 2 ? &W->up : &W->down;
    }
    const int elt = l->wt == EC_W_I8 ? 1 : 2;
    if (info5) { info5[0] = l->N; info5[1] = l->K; info5[2] = l->Kp; info5[3] = l->ldw; info5[4] = elt; }
    const size_t bytes = (size_t)l->N * l->ldw * elt;
    if (!out) return (long long)bytes;
    if (cap < bytes) { ec_seterr("ec_model_packed: %zu bytes needed", bytes); return -1; }
    CK(cudaStreamSynchronize(d->stream));
    CK(cudaMemcpy(out, l->w, bytes, cudaMemcpyDeviceToHost));
    return (long long)bytes;
}

EC_EXPORT int ec_batch_graph_kernels(GPT2 *g, int kind)
{
    ec_dev *d = ec_lookup(g);
    if (!d || kind < 0 || kind > 1) { ec_seterr("ec_batch_graph_kernels: no model or bad kind"); return -1; }
    return d->bg[kind].exec ? d->bg[kind].kernels : 0;
}

EC_EXPORT int ec_keys_advance(GPT2 *g, const long long *d_keys, int M, int *d_tokens, int *d_positions)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    if (M < 1) { ec_seterr("ec_keys_advance: M must be >= 1"); return -1; }
    CK(ec_launch_keys_advance(d_keys, M, d_tokens, d_positions, NULL, d->stream));
    return 0;
}

/* Instrumented decode: each step is one launch of the persistent kernel with
 * an event pair around it (class 0), so out[0..2] = {ms, algorithmic bytes,
 * launches} of that kernel.  Models the kernel cannot take fall back to the
 * per-layer kernels with an event pair around every launch. */
EC_EXPORT int ec_decode_profile(GPT2 *g, int *d_tokens, int start_pos, int n_steps, double *out)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    const int M = d->B;
    if (n_steps < 1 || start_pos < 0 || start_pos + n_steps > d->C) { ec_seterr("bad profile range"); return -1; }
    if (!d->prof_ready) {
        for (int i = 0; i < 2 * EC_PROF_MAX; i++) CK(cudaEventCreate(&d->prof_ev[i]));
        d->prof_ready = 1;
    }
    for (int i = 0; i < 16; i++) out[i] = 0.0;
    const int maxlen = ec_len_bucket(d, start_pos + n_steps);
    ec_mk_params mp;
    if (ec_mk_plan(d, M, maxlen, &mp) == 0) {
        if (ec_decode_setup(d, d_tokens, start_pos, M, start_pos + n_steps)) return -1;
        mp.advance = 1;
        for (int st = 0; st < n_steps; st++) {
            if (d->bar_reset) {   /* outside the timed interval */
                CK(cudaMemsetAsync(d->d_bar, 0, 512, d->stream));
                d->bar_reset = 0;
            }
            CK(cudaEventRecord(d->prof_ev[0], d->stream));
            if (ec_mk_run(d, &mp, 1)) return -1;
            CK(cudaEventRecord(d->prof_ev[1], d->stream));
            CK(cudaStreamSynchronize(d->stream));
            float ms = 0.0f;
            CK(cudaEventElapsedTime(&ms, d->prof_ev[0], d->prof_ev[1]));
            out[EC_PC_STEP * 3 + 0] += ms;
            out[EC_PC_STEP * 3 + 1] += ec_step_bytes(d, M, start_pos + st + 1);
            out[EC_PC_STEP * 3 + 2] += 1.0;
        }
    } else {
        const int chunk = ec_lm_chunk(d, M);
        if (ec_decode_setup(d, d_tokens, start_pos, M, start_pos + n_steps) || ec_ensure_logits(d, chunk) ||
            ec_ensure_amax(d, chunk) ||
            ec_ensure_attn(d, M, maxlen)) return -1;
        for (int st = 0; st < n_steps; st++) {
            d->prof_on = 1;
            d->prof_n = 0;
            int rc = ec_enqueue_body(d, M, maxlen);
            for (int r0 = 0; !rc && r0 < M; r0 += chunk) {   /* lm_head (GEMM class) + argmax (other) */
                const int rows = M - r0 < chunk ? M - r0 : chunk;
                rc = ec_enqueue_lm(d, r0, rows);
                const int pa = ec_prof_begin(d, EC_PC_OTHER, 0.0);
                if (!rc && ec_launch_argmax(d->d_ids + r0, d->d_max + r0, d->logits, d->v1 - d->v0, d->v1 - d->v0,
                                            rows, d->v0, d->amax_part, d->amax_chunks, d->stream))
                    rc = -1;
                ec_prof_end(d, pa);
            }
            int pi = ec_prof_begin(d, EC_PC_OTHER, 0.0);
            if (!rc && ec_launch_step_advance(d->d_tok, d->d_pos, d->d_ids, M, NULL, NULL, 0, 0, d->stream)) rc = -1;
            ec_prof_end(d, pi);
            d->prof_on = 0;
            if (rc) return -1;
            CK(cudaStreamSynchronize(d->stream));
            for (int i = 0; i < d->prof_n; i++) {
                float ms = 0.0f;
                CK(cudaEventElapsedTime(&ms, d->prof_ev[2 * i], d->prof_ev[2 * i + 1]));
                out[d->prof_cls[i] * 3 + 0] += ms;
                out[d->prof_cls[i] * 3 + 1] += d->prof_bytes[i];
                out[d->prof_cls[i] * 3 + 2] += 1.0;
            }
        }
    }
    out[15] = n_steps;
    CK(cudaMemcpyAsync(d_tokens, d->d_tok, (size_t)M * 4, cudaMemcpyDeviceToDevice, d->stream));
    CK(cudaStreamSynchronize(d->stream));
    return ec_check_kernel_error(d);
}

/* One decode launch of n_steps with the timeline of CTA 0 recorded: host
 * `out[cap]` receives (code << 56) | globaltimer-ns entries, those of the
 * consumer thread first, then those of the producer thread; returns the
 * number of entries or -1. */
EC_EXPORT int ec_decode_trace(GPT2 *g, int *d_tokens, int start_pos, int n_steps, unsigned long long *out, int cap)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    if (!ec_mk_traced()) {
        ec_seterr("decode timeline not compiled in (build with EDGECORE_B200_TRACE=1: "
                  "libedgecore_b200_trace.so)");
        return -1;
    }
    const int M = d->B;
    if (M > EC_MK_MT || n_steps < 1 || cap < 1 || start_pos < 0 || start_pos + n_steps > d->C) {
        ec_seterr("bad trace range");
        return -1;
    }
    ec_mk_params mp;
    if (ec_mk_plan(d, M, ec_len_bucket(d, start_pos + n_steps), &mp)) { ec_seterr("decode kernel not applicable"); return -1; }
    unsigned long long *dt = NULL;
    CK(cudaMalloc((void **)&dt, (size_t)cap * 8));
    CK(cudaMemsetAsync(dt, 0, (size_t)cap * 8, d->stream));
    if (ec_decode_setup(d, d_tokens, start_pos, M, start_pos + n_steps)) { cudaFree(dt); return -1; }
    mp.advance = 1;
    mp.trace = dt;
    mp.trace_cap = cap;
    int rc = ec_mk_run(d, &mp, n_steps);
    if (!rc && cudaMemcpyAsync(out, dt, (size_t)cap * 8, cudaMemcpyDeviceToHost, d->stream) != cudaSuccess) rc = -1;
    if (!rc && cudaStreamSynchronize(d->stream) != cudaSuccess) rc = -1;
    cudaFree(dt);
    if (rc) { ec_seterr("traced decode failed"); return -1; }
    /* compact the two halves (consumer thread, producer thread) */
    const int half = cap / 2;
    int n = 0;
    for (int i = 0; i < half && out[i]; ++i) n++;
    for (int i = half; i < cap && out[i]; ++i) out[n++] = out[i];
    for (int i = n; i < cap; ++i) out[i] = 0;
    return ec_check_kernel_error(d) ? -1 : n;
}

EC_EXPORT int ec_model_set_taps(GPT2 *g, int enable)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    d->taps_on = enable > 0;
    if (d->taps_on && (!d->taps || d->taps_rows < enable)) {
        CK(cudaStreamSynchronize(d->stream));
        cudaFree(d->taps);
        d->taps = NULL;
        CK(cudaMalloc((void **)&d->taps, (size_t)(d->L + 1) * enable * d->E * 4));
        d->taps_rows = enable;
    }
    return 0;
}

EC_EXPORT int ec_model_get_taps(GPT2 *g, float *out, int M)
{
    ec_dev *d = ec_lookup(g);
    if (!d || !d->taps || M > d->taps_rows) { ec_seterr("taps not enabled for %d rows", M); return -1; }
    CK(cudaStreamSynchronize(d->stream));
    CK(cudaMemcpy(out, d->taps, (size_t)(d->L + 1) * M * d->E * 4, cudaMemcpyDeviceToHost));
    return 0;
}

EC_EXPORT int ec_model_set_vocab_shard(GPT2 *g, int v_begin, int v_end)
{
    ec_dev *d = ec_lookup(g);
    if (!d) { ec_seterr("model not loaded"); return -1; }
    if (v_begin < 0 || v_end > d->V || v_begin >= v_end) { ec_seterr("bad vocab shard [%d,%d)", v_begin, v_end); return -1; }
    CK(cudaStreamSynchronize(d->stream));
    return ec_set_lm_shard(d, v_begin, v_end);
}

/* (max, idx) -> key: unsigned order = larger value first, then lower index. */
EC_EXPORT uint64_t ec_argmax_key(float maxv, int idx)
{
    uint32_t b;
    if (maxv == 0.0f) maxv = 0.0f;   /* -0 and +0 compare equal in the reference's '>' scan */
    memcpy(&b, &maxv, 4);
    if (maxv != maxv) b = 0u;        /* NaN never wins a '>' comparison: below every number */
    else b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);   /* order-preserving float bits */
    return ((uint64_t)b << 32) | (uint32_t)(0x7fffffff - idx);
}

EC_EXPORT void ec_argmax_key_decode(uint64_t key, float *maxv, int *idx)
{
    uint32_t b = (uint32_t)(key >> 32);
    b = (b & 0x80000000u) ? (b & 0x7fffffffu) : ~b;
    if (maxv) memcpy(maxv, &b, 4);
    if (idx) *idx = 0x7fffffff - (int)(uint32_t)(key & 0xffffffffu);
}
