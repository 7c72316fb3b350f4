/*
 * ref_shim.c -- TEST INFRASTRUCTURE ONLY.  Compiled (by oracle/Makefile) with
 * the reference's own src/gpt2.c textually included, so that the reference's
 * static helpers (linear, layernorm_rows, rmsnorm_rows, qwen_inv_freq, ...)
 * can be called from the tests and the golden-vector generator through plain
 * C entry points.  The output, oracle/_ref/libecref.so, is the reference
 * itself built from source; it is never linked into the product library.
 *
 * Built only where the reference sources are present (see oracle/Makefile).
 */
#include "gpt2.c"   /* resolved with -I<reference>/src */

#define REF_API __attribute__((visibility("default")))

REF_API void ref_set_threads(int n)
{
#ifdef _OPENMP
    omp_set_num_threads(n > 0 ? n : 1);
#else
    (void)n;
#endif
}

REF_API GPT2 *ref_open(const char *path, int batch_cap, int max_ctx)
{
    GPT2 *g = calloc(1, sizeof *g);
    if (!g) return NULL;
    if (gpt2_load(g, path, batch_cap, max_ctx) != 0) { free(g); return NULL; }
    return g;
}

REF_API void ref_close(GPT2 *g)
{
    if (!g) return;
    gpt2_free(g);
    free(g);
}

/* The KV reset the reference driver performs before every run
 * (src/runtime_main.c:312-316). */
REF_API void ref_reset_kv(GPT2 *g)
{
    size_t kv = (size_t)g->n_layer * g->batch_cap * gpt2_eff_ctx(g) * g->n_kv_embd;
    memset(g->k_cache, 0, kv * sizeof(uint16_t));
    memset(g->v_cache, 0, kv * sizeof(uint16_t));
}

REF_API void ref_info(const GPT2 *g, int *o)
{
    int v[16] = {g->arch, g->precision, g->n_layer, g->n_head, g->n_kv_head, g->n_embd,
                 g->head_dim, g->intermediate, g->vocab, g->n_ctx, gpt2_eff_ctx(g),
                 g->batch_cap, g->n_kv_embd, g->tie_word_embeddings, 0, 0};
    memcpy(o, v, sizeof v);
}

REF_API void ref_forward(GPT2 *g, const int *tok, const int *pos, const int *seqs, int M, float *logits)
{
    gpt2_forward(g, tok, pos, seqs, M, logits);
}

/* Run the forward truncated to the first `nl` layers and copy the residual
 * stream it leaves in ws_x ([M][n_embd]) to `x_out`: the per-layer tap. */
REF_API void ref_forward_layers(GPT2 *g, int nl, const int *tok, const int *pos,
                                const int *seqs, int M, float *logits, float *x_out)
{
    int keep = g->n_layer;
    g->n_layer = nl;
    gpt2_forward(g, tok, pos, seqs, M, logits);
    g->n_layer = keep;
    memcpy(x_out, g->ws_x, (size_t)M * g->n_embd * sizeof(float));
}

/* The reference linear() on a standalone weight: precision 0 (int8, with its
 * activation quantisation), 1 (fp16) or 2 (bf16).  q_out/qs_out (may be NULL)
 * receive the quantised activations of the int8 branch. */
REF_API void ref_linear(int precision, const void *w, const float *scale, const float *bias,
                        const float *in, float *out, int M, int K, int N,
                        int8_t *q_out, float *qs_out)
{
    GPT2 g;
    memset(&g, 0, sizeof g);
    g.precision = precision;
    g.n_ctx = M;
    g.batch_cap = 1;
    g.ws_q_cols = (size_t)K;
    g.ws_q = malloc((size_t)M * K);
    g.ws_qs = malloc((size_t)M * sizeof(float));
    linear(&g, w, scale, bias, in, out, M, K, N);
    if (q_out) memcpy(q_out, g.ws_q, (size_t)M * K);
    if (qs_out) memcpy(qs_out, g.ws_qs, (size_t)M * sizeof(float));
    free(g.ws_q);
    free(g.ws_qs);
}

REF_API void ref_layernorm(float *out, const float *in, const float *g, const float *b, int M, int N, double eps)
{
    layernorm_rows(out, in, g, b, M, N, eps);
}

REF_API void ref_rmsnorm(float *out, const float *in, const float *g, int M, int N, double eps)
{
    rmsnorm_rows(out, in, g, M, N, eps);
}

REF_API void ref_rope(double *inv_out, double *cos_out, double *sin_out, int half, int pos,
                      double theta, int rope_type, double yarn_factor, double yarn_orig_max,
                      double attn_scale)
{
    GPT2 g;
    memset(&g, 0, sizeof g);
    g.rope_theta = theta;
    g.rope_type = rope_type;
    g.yarn_factor = yarn_factor;
    g.yarn_orig_max = yarn_orig_max;
    qwen_inv_freq(inv_out, half, &g);
    qwen_rope_cos_sin(inv_out, half, pos, attn_scale, cos_out, sin_out);
}

REF_API float ref_gelu(float x) { return gelu_new(x); }
REF_API float ref_silu(float x) { return qwen_silu(x); }
REF_API uint16_t ref_f32_to_fp16(float x) { return f32_to_fp16(x); }
REF_API float ref_fp16_to_f32(uint16_t h) { return fp16_to_f32(h); }
