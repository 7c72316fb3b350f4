/*
 * ec_launch.h -- internal C interface between the host code (ec_host.c,
 * ec_abi.c; plain C11) and the sm_100a kernels (*.cu).  Every launcher
 * enqueues on `stream` and returns a cudaError_t-compatible int (0 = ok).
 */
#ifndef EC_LAUNCH_H
#define EC_LAUNCH_H

#include <stdint.h>
#include <stddef.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Weight element types. */
enum { EC_W_I8 = 0, EC_W_F16 = 1, EC_W_BF16 = 2 };

/* GEMV / GEMM epilogues. */
enum {
    EC_EPI_STORE = 0,   /* out[m][n] = v                                     */
    EC_EPI_RESID = 1,   /* out[m][n] = out[m][n] + v   (residual add)        */
    EC_EPI_GELU = 2,    /* out[m][n] = gelu_new(v)                           */
    EC_EPI_SWIGLU = 3,  /* pair blocks: out[m][j] = silu(v_j) * v_{j+P}      */
    EC_EPI_QKV = 4,     /* q -> out, k/v -> fp16 KV cache (+RoPE on pairs)   */
    EC_EPI_ARGMAX = 5   /* tensor-core GEMMs only: out is float2 [M][ldo],
                           per (row, column tile, half) {max of v, first
                           column index} for k_argmax_final; ldo >=
                           ec_gemm_tc_argmax_chunks(wt, M, N)              */
};

/* One row block of a weight matrix: rows [row0, row0+nrows) and, when pair>0,
 * also [row0+pair, row0+pair+nrows) (staged right after the first range). */
typedef struct { int row0, nrows, pair, kind; } ec_block;

/* Block kinds for EC_EPI_QKV. */
enum { EC_BK_PLAIN = 0, EC_BK_ROPE = 1 };

/* Per-step token inputs, all device arrays of length M. */
typedef struct {
    const int *tok;     /* token ids                      */
    const int *pos;     /* absolute positions             */
    const int *slot;    /* KV slot (already clamped)      */
} ec_tokens;

/* Positions per page of the paged KV arena (ec_kv_row in ec_common.cuh). */
#define EC_KV_PAGE 64

/* KV-cache / attention geometry for the QKV epilogue and attention. */
typedef struct {
    uint16_t *kc, *vc;        /* this layer's paged fp16 caches [pages][64][kv] */
    const int *pt;            /* page table [B][mp] (see ec_kv_row)            */
    int mp;                   /* pages per slot                                */
    int B;                    /* batch_cap (slots)                             */
    int C;                    /* eff_ctx                                       */
    int kv;                   /* n_kv_embd                                     */
    int E;                    /* n_embd (q rows of the fused qkv)              */
    int hd;                   /* head_dim                                      */
    const double *rope_cos;   /* [C][hd/2] scaled cos (NULL: no RoPE)          */
    const double *rope_sin;
} ec_kvgeo;

typedef struct {
    const void *W;            /* [N][ldw] weights (type wt), row-major         */
    const float *wscale;      /* [N] per-row scale (int8 only)                 */
    const float *bias;        /* [N] or NULL                                   */
    int wt, N, K, Kp;
    int ldw;                  /* row stride in elements (>= Kp; 0 means Kp)    */
    const ec_block *blocks;   /* device table                                   */
    int nblocks;
    int block_rows;           /* max staged rows per block (nrows * (pair?2:1)) */
    const float *X;           /* [M][ldx] fp32 activations                     */
    const int8_t *Xq;         /* or pre-quantised int8 [M][ldx] ...            */
    const float *xscale;      /* ... with per-row scales (int8 weights only)   */
    int ldx, M;
    float *out;               /* epilogue target                                */
    int ldo;
    int epi;
    ec_tokens tk;             /* EC_EPI_QKV only                               */
    ec_kvgeo geo;             /* EC_EPI_QKV only                               */
} ec_gemv_args;

/* Decode-shaped (M <= 8) weight-streaming GEMV with fused activation
 * quantisation (int8) and epilogue. */
int ec_launch_gemv(const ec_gemv_args *a, int num_sms, cudaStream_t stream);

/* 1 when ec_launch_gemv can take these arguments (M, block rows, K alignment
 * and the shared memory of one staged block plus the activation rows), else 0. */
int ec_gemv_fits(const ec_gemv_args *a);

/* Generic GEMM for any M: A int8 [M][Kp] + a_scale[M] (int8 weights) or
 * A fp32 [M][ldx] (16-bit weights); plain/resid/gelu epilogues only. */
typedef struct {
    const void *W; const float *wscale; const float *bias;
    int wt, N, K, Kp;
    int ldw;                                  /* W row stride (0: Kp)  */
    const int8_t *Aq; const float *a_scale;   /* int8 weights */
    const float *X; int ldx;                  /* 16-bit weights */
    int M;
    float *out; int ldo; int epi;
    void *split; size_t split_bytes;          /* 16-bit weights on tensor cores: workspace
                                                 of ec_gemm_tc_split_bytes() bytes,
                                                 256-byte aligned (NULL: SIMT kernel) */
    int *acc32; size_t acc32_elems;           /* int8 on tensor cores, split over K when the
                                                 output has few tiles: int32 [M][N] sums, all
                                                 zero between calls (NULL: no split) */
    unsigned *tile_cnt; int cnt_elems;        /* per-tile split counters, zero between calls */
} ec_gemm_args;
int ec_launch_gemm(const ec_gemm_args *a, cudaStream_t stream);

/* The GEMMs on tcgen05 tensor cores (ec_tc.cu), used by ec_launch_gemm for
 * M >= EC_TC_MIN_M: int8 weights directly, fp16/bf16 weights with the
 * activations split into 16-bit parts in the `split` workspace;
 * cudaErrorNotSupported when the operands miss its alignment rules.
 * ec_tc_error_take reads and clears its error word. */
#define EC_TC_MIN_M 8
int ec_launch_gemm_tc(const ec_gemm_args *a, cudaStream_t stream);

/* One-time set-up of the tensor-core GEMMs on the current device (driver
 * entry point of the tensor-map encoder, kernel shared-memory attributes,
 * SM count), so that no later launch does it; cudaErrorNotSupported when the
 * driver has no tensor-map encoder (ec_launch_gemm then uses the SIMT kernels). */
int ec_tc_init(void);
size_t ec_gemm_tc_split_bytes(int wt, int M, int Kp);
/* Partials per row that the tensor-core GEMM writes for EC_EPI_ARGMAX (two
 * per column tile of the configuration it picks for M x N); 0 below
 * EC_TC_MIN_M rows. */
int ec_gemm_tc_argmax_chunks(int wt, int M, int N);
int ec_tc_error_take(int *code);

/* Per-row symmetric int8 quantisation of X [M][ldx] (K used, Kp written). */
int ec_launch_quant(int8_t *q, float *scale, const float *X, int ldx, int M, int K, int Kp,
                    cudaStream_t stream);

/* x[m][:E] = h2f(wte[tok[m]]) (+ h2f(wpe[pos[m]])); table rows have stride ld. */
int ec_launch_embed(float *x, const uint16_t *wte, const uint16_t *wpe, int ld, int is_bf16,
                    ec_tokens tk, int M, int E, int V, int C, cudaStream_t stream);

/* Norm rows then their int8 quantisation (k_norm + k_quant in one pass):
 * q [M][Kp], scale [M]; cudaErrorNotSupported when E floats exceed 48 KB. */
int ec_launch_norm_quant(int8_t *q, float *scale, int Kp, const float *x, const float *gamma, const float *beta,
                         int M, int E, double eps, cudaStream_t stream);

/* SwiGLU of interleaved gate|up rows then their int8 quantisation: q [M][Kp],
 * scale [M]; cudaErrorNotSupported when I floats exceed 48 KB. */
int ec_launch_swiglu_quant(int8_t *q, float *scale, int Kp, const float *gu, int ldg, int I, int M,
                           cudaStream_t stream);

/* LayerNorm (beta != NULL) or RMSNorm (beta == NULL) rows, fp64 statistics. */
int ec_launch_norm(float *out, const float *x, const float *gamma, const float *beta,
                   int M, int E, double eps, cudaStream_t stream);

/* Split the q|k|v rows of a GEMM output [M][ldq] (Qwen2 packed layout when
 * packed != 0): RoPE, q -> q_out [M][E] in head order, k/v -> fp16 cache. */
int ec_launch_qkv_split(float *q_out, const float *qkv, int ldq, ec_tokens tk, ec_kvgeo geo, int H,
                        int KVH, int packed, int M, cudaStream_t stream);

/* out[m][j] = silu(gu[m][2j]) * gu[m][2j+1] (gate|up interleaved). */
int ec_launch_swiglu(float *out, int ldo, const float *gu, int ldg, int I, int M,
                     cudaStream_t stream);

/* x[i] = gelu_new(x[i]) */
int ec_launch_gelu_inplace(float *x, size_t n, cudaStream_t stream);

/* Attention for M query rows against the fp16 KV cache (GQA / MHA).
 * q [M][ldq] (head h at column h*hd), out [M][E]; split over positions. */
typedef struct {
    const float *q; int ldq;
    float *out; int ldo;
    ec_tokens tk; ec_kvgeo geo;
    int H, KVH, M, window;        /* window > 0: sliding window */
    float *part;                  /* scratch: [M][H][nsplit][hd + 2] */
    int nsplit;
    int maxlen;                   /* upper bound on attended positions per row */
    int per_head;                 /* set by the launcher: one CTA per (head, row)
                                     instead of per (KV head, row) */
    const int *blocks;            /* or NULL: nblocks pairs {first row, rows}, each
                                     up to EC_ATTN_RUN consecutive rows of one slot
                                     at consecutive positions (prefill): the block
                                     kernel may be used */
    int nblocks;
} ec_attn_args;
#define EC_ATTN_RUN 32            /* rows per block of the block kernel at most */
/* Chooses the exact-order kernels (reference summation order): the block
 * kernel when the caller passes a block table (one CTA per query head and
 * block of up to 32 rows, each cached K / V row staged once per block), else
 * one CTA per (token, KV head) holding
 * all scores in shared memory when maxlen fits, else the split kernel
 * (flash-decoding order, within 1e-6 of the reference). */
int ec_launch_attention(const ec_attn_args *a, cudaStream_t stream);
/* 1: every ec_launch_attention uses the split kernels (tests, measurement). */
void ec_attention_set_force_split(int on);
size_t ec_attention_scratch_floats(int M, int H, int hd, int nsplit);
/* 1 if the exact-order kernel handles rows of up to maxlen positions. */
int ec_attention_exact_fits(int H, int KVH, int hd, int maxlen);

/* Row-wise argmax (lowest index on ties) of logits [M][ld] over [0, N),
 * reporting ids offset by id_base.  part is scratch of 2*M*nchunk words. */
int ec_launch_argmax(int *ids, float *maxv, const float *logits, int ld, int N, int M,
                     int id_base, void *part, int nchunk, cudaStream_t stream);
/* The merge step alone, over partials float2 [M][nchunk] (EC_EPI_ARGMAX). */
int ec_launch_argmax_final(int *ids, float *maxv, const void *part, int nchunk, int M, int id_base,
                           cudaStream_t stream);

/* Device-side decode bookkeeping for a captured step: tok[m] = ids[m];
 * pos[m] += 1, wrapping to wrap_lo when it reaches wrap_hi (wrap_hi <= 0: no
 * wrap); optionally record ids into hist[step][M] with step read from and
 * incremented in *counter. */
int ec_launch_step_advance(int *tok, int *pos, const int *ids, int M, int *hist, int *counter,
                           int wrap_lo, int wrap_hi, cudaStream_t stream);

/* keys[m] = signed 64-bit argmax key of (maxv[m], ids[m]): larger logit,
 * then lower index, wins a signed max (see ec_argmax_key). */
int ec_launch_pack_keys(const int *ids, const float *maxv, int M, long long *keys, cudaStream_t stream);

/* tok[m] = index of keys[m]; pos[m] += 1 (pos may be NULL); ids[m] = index
 * (ids may be NULL). */
int ec_launch_keys_advance(const long long *keys, int M, int *tok, int *pos, int *ids, cudaStream_t stream);

/* e[i] = expf(x[i]), t[i] = tanhf(x[i]) with the device restatements of the
 * reference's libm functions (ec_common.cuh); e or t may be NULL. */
int ec_launch_reference_math(const float *x, float *e, float *t, int n, cudaStream_t stream);

/* The library-wide device error word (bounded waits that gave up, bad
 * indices skipped).  Read and cleared by ec_kernel_error_take. */
int ec_kernel_error_take(cudaStream_t stream, int *code);

/* One-time per-device kernel attribute setup (dynamic shared memory limits). */
int ec_kernels_init(void);

/* Text for ec_last_error() of the calling thread (ec_host.c). */
void ec_set_error_text(const char *msg);

#ifdef __cplusplus
}
#endif

#endif /* EC_LAUNCH_H */
