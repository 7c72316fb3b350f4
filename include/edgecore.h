/*
 * edgecore.h -- drop-in replacement header for EdgeCore's C inference runtime,
 * backed by the B200 (sm_100a) library libedgecore_b200.so.
 *
 * Every type and prototype here is layout- and signature-identical to the
 * reference header (EdgeCore src/edgecore.h).  That identity is the whole
 * point: the reference's unmodified src/runtime_main.c and src/tokenizer.c
 * compile against this header, or link their existing objects, against
 * libedgecore_b200.so instead of src/gpt2.c + src/kernels.c.  The device state
 * of a loaded model is therefore NOT a struct field; the library keeps it in an
 * internal table keyed by the GPT2 address (so a GPT2 must not be moved or
 * copied between gpt2_load and gpt2_free, which the reference callers never do).
 *
 * Pointer semantics of the replacements:
 *   - gemm_fp16_fp32 / gemm_bf16_fp32 / gemm_int8 accept host OR device
 *     pointers (classified per call).  Host operands are staged through the
 *     device; the call returns with C written, like the CPU version.
 *   - gpt2_forward / qwen2_forward take host tokens/positions/seqs and write
 *     host logits [M][vocab], exactly as the reference does.
 *
 * Extensions that have no reference counterpart live in edgecore_b200.h.
 */
#ifndef EDGECORE_H
#define EDGECORE_H

#include <stdint.h>
#include <stddef.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <float.h>

#ifdef _OPENMP
#include <omp.h>   /* runtime_main.c calls omp_set_num_threads through this header */
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define ECM_MAGIC "ECM1\n"

/* `arch` meta values (reference src/edgecore.h:23-24). */
#define ARCH_GPT2  0
#define ARCH_QWEN2 1

/* `rope_type` meta values (reference src/edgecore.h:27-28). */
#define ROPE_DEFAULT 0
#define ROPE_YARN    1

/* ------------------------------------------------------------------ */
/* Half-precision helpers (reference src/edgecore.h:34-109).           */
/* Portable restatements: binary16 decode is exact, encode rounds to   */
/* nearest-even (what F16C's _mm_cvtps_ph(.,0) does), bf16 decode is a */
/* 16-bit shift.                                                       */
/* ------------------------------------------------------------------ */

static inline float fp16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t mag = (uint32_t)(h & 0x7fffu);
    uint32_t bits;
    if (mag >= 0x7c00u) {                 /* inf / nan */
        bits = sign | 0x7f800000u | ((mag & 0x3ffu) << 13);
    } else if (mag >= 0x0400u) {          /* normal: rebias exponent 15 -> 127 */
        bits = sign | ((mag << 13) + ((uint32_t)(127 - 15) << 23));
    } else {                              /* zero / subnormal: mag * 2^-24 is exact */
        float f = (float)mag * 5.9604644775390625e-08f;
        memcpy(&bits, &f, 4);
        bits |= sign;
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

static inline uint16_t f32_to_fp16(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);          /* nan (quiet) */
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);         /* rounds to inf */
    if (ax < 0x38800000u) {                                          /* result subnormal or 0 */
        /* value / 2^-24, rounded to nearest-even, is the subnormal payload */
        float a;
        memcpy(&a, &ax, 4);
        float scaled = a * 16777216.0f;          /* exact: power-of-two scaling */
        uint32_t q = (uint32_t)scaled;
        float rem = scaled - (float)q;
        if (rem > 0.5f || (rem == 0.5f && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    /* normal: keep 10 mantissa bits, round-to-nearest-even on the 13 dropped bits */
    uint32_t r = ax + 0x0fffu + ((ax >> 13) & 1u);
    r -= (uint32_t)(127 - 15) << 23;
    return (uint16_t)(sign | (r >> 13));
}

static inline float bf16_to_f32(uint16_t b)
{
    uint32_t bits = (uint32_t)b << 16;
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

/* ------------------------------------------------------------------ */
/* GEMM entry points (reference src/edgecore.h:119-136,                */
/* implemented in reference src/kernels.c:129-168).                    */
/* ------------------------------------------------------------------ */

/* C[M][N] = A[M][K] (fp32) . B[N][K]^T (fp16 row-major), fp32 accumulate. */
void gemm_fp16_fp32(float *C, const float *A, const uint16_t *B,
                    int M, int K, int N);

/* Same with B stored as bfloat16. */
void gemm_bf16_fp32(float *C, const float *A, const uint16_t *B,
                    int M, int K, int N);

/* C[m][n] = bias[n] + ((float)sum_k A[m][k]*B[n][k]) * a_scale[m] * b_scale[n]
 * with A int8 [M][K], B int8 [N][K]; b_scale and bias may be NULL. */
void gemm_int8(float *C, const int8_t *A, const float *a_scale,
               const int8_t *B, const float *b_scale, const float *bias,
               int M, int K, int N);

/* ------------------------------------------------------------------ */
/* Tokenizer (reference src/edgecore.h:142-164).  The implementation    */
/* stays the reference's src/tokenizer.c; this library only calls       */
/* tokenizer_load / tokenizer_free when that object is linked in.       */
/* ------------------------------------------------------------------ */

typedef struct {
    char **id_to_token;
    int32_t *byte_to_id;
    int32_t *cp_to_byte;
    uint32_t *merge_l, *merge_r, *merge_m;
    int n_merges;
    int vocab_size;
    int variant;
    int eos_id;
    char **sp_tok;
    uint32_t *sp_len;
    int32_t *sp_id;
    int n_sp;
} Tokenizer;

int tokenizer_load(Tokenizer *t, const void *vocab_blob, size_t vocab_bytes,
                   const void *merges_blob, size_t merges_bytes, int vocab_size,
                   int variant);
void tokenizer_free(Tokenizer *t);
int tokenizer_encode(const Tokenizer *t, const char *text, int *out, int max_out);
char *tokenizer_decode(const Tokenizer *t, const int *ids, int n);

/* ------------------------------------------------------------------ */
/* Model (reference src/edgecore.h:170-244).  Field order and types    */
/* are kept exactly so the struct has the reference's layout.           */
/* ------------------------------------------------------------------ */

typedef struct {
    char model_name[64];
    int n_layer, n_head, n_embd, n_ctx, vocab;
    int n_kv_head;
    int n_kv_embd;
    int intermediate;
    int head_dim;
    int arch;
    size_t n_params;
    double eps;

    double rope_theta;
    int rope_type;
    double yarn_factor, yarn_orig_max, yarn_attention_factor;
    int sliding_window;
    int tie_word_embeddings;
    int eos_token_id;

    const uint16_t *wte;        /* host view of the .ecm [vocab][n_embd] */
    const uint16_t *wpe;

    struct LayerW {
        const float *ln1_g, *ln1_b;
        const void *attn_w;
        const float *attn_s, *attn_b;
        const void *proj_w;
        const float *proj_s, *proj_b;
        const float *ln2_g, *ln2_b;
        const void *fc_w;
        const float *fc_s, *fc_b;
        const void *fc2_w;
        const float *fc2_s, *fc2_b;

        const void *q_w, *k_w, *v_w, *o_w;
        const float *q_s, *k_s, *v_s, *o_s;
        const float *q_b, *k_b, *v_b, *o_b;
        const void *gate_w, *up_w, *down_w;
        const float *gate_s, *up_s, *down_s;
        const float *gate_b, *up_b, *down_b;
    } *lw;

    const float *lnf_g, *lnf_b;
    const uint16_t *lm_head;

    int precision;              /* 0 = int8, 1 = fp16, 2 = bf16 */

    /* Host KV buffers.  In this library the live KV cache is a device arena;
     * these stay valid, full-size host buffers so that callers which reset
     * them with memset (reference src/runtime_main.c:312-316) keep working. */
    uint16_t *k_cache, *v_cache;
    int batch_cap;
    int max_ctx;

    /* Host workspaces of the CPU runtime.  Unused (NULL) in this library. */
    float *ws_x, *ws_tmp, *ws_qkv, *ws_attn, *ws_scores;
    int8_t *ws_q;
    float *ws_qs;
    size_t ws_q_cols;

    Tokenizer tok;

    void *file_data;            /* the mmap'd .ecm file */
    size_t file_size;
    int file_mapped;
} GPT2;

typedef struct {
    char name[128];
    int dtype;                  /* 0=fp32 1=fp16 2=int8 3=text 4=bf16 */
    size_t nelems;
    size_t bytes;
    size_t offset;
    size_t dims[4];
    int ndims;
} EcmTensor;

/* Load: returns 0, or -1 with a message on stderr (reference gpt2.c:161-366). */
int gpt2_load(GPT2 *g, const char *path, int batch_cap, int max_ctx);
void gpt2_free(GPT2 *g);

/* Forward M tokens; logits [M][vocab] fp32 host.  seqs == NULL: token m is in
 * slot m; else slot seqs[m] at positions[m] (reference gpt2.c:470-581). */
void gpt2_forward(GPT2 *g, const int *tokens, const int *positions,
                  const int *seqs, int M, float *logits);

/* Qwen2 decoder forward (reference gpt2.c:667-805). */
void qwen2_forward(GPT2 *g, const int *tokens, const int *positions,
                   const int *seqs, int M, float *logits);

static inline int gpt2_eff_ctx(const GPT2 *g) {
    return (g->max_ctx > 0 && g->max_ctx < g->n_ctx) ? g->max_ctx : g->n_ctx;
}

/* Parse the .ecm header; returns the tensor count or -1 (reference gpt2.c:34-136). */
int ecm_parse(const void *data, size_t size, EcmTensor *out, int max,
              GPT2 *meta_out);

/* Utilities defined by the runtime driver (reference runtime_main.c:10-28). */
float peak_rss_gb(void);
double now_sec(void);

#ifdef __cplusplus
}
#endif

#endif /* EDGECORE_H */
