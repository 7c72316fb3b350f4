/*
 * ec_decode.h -- parameters of the persistent decode kernel (ec_decode.cu),
 * shared by the C host code.  One launch runs `n_steps` forward steps of M
 * token rows (M <= EC_MK_MT) through every layer and the lm_head.
 *
 * Weight layout ("packed"): every layer linear is [N][ldw] row-major: Kp
 * weights (K rounded up to a multiple of 16, zero padded) followed by a
 * 16-byte tail {fp32 scale, fp32 bias, 0, 0}, so one bulk copy of a row
 * brings its epilogue constants along.  Qwen2 q|k|v has the rows of each q and k head
 * reordered so that the RoPE partners (i, i + head_dim/2) are adjacent
 * (packed row 2i+t <- original row i + t*head_dim/2), v rows unchanged;
 * Qwen2 gate|up is interleaved (packed row 2j <- gate j, 2j+1 <- up j).
 * GPT-2 matrices keep the file's order.  Scales and biases follow the rows.
 */
#ifndef EC_DECODE_H
#define EC_DECODE_H

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EC_MK_MT 8              /* max token rows per launch               */
#define EC_MK_STAGES 4          /* weight ring slots                       */
#define EC_MK_TILE 32768        /* bytes per ring slot                     */
#define EC_MK_MAX_TILE_ROWS 64  /* rows per tile                           */
#define EC_MK_CONS_WARPS 8
#define EC_MK_THREADS (32 * (EC_MK_CONS_WARPS + 1))

typedef struct {
    const void *w;              /* packed [N][ldw]                         */
    int N, K, Kp;
    int ldw;                    /* row stride in elements (>= Kp)          */
    int meta;                   /* row tail after Kp weights holds fp32
                                   {scale, bias}: bit 0 scale used, bit 1
                                   bias used (0: no tail)                  */
    int unit;                   /* 1, or 2 for pair-packed rows            */
    int tile_rows;              /* rows per ring tile (multiple of unit)   */
} ec_mk_mat;

typedef struct {
    ec_mk_mat qkv, o, up, down;
    const float *n1g, *n1b, *n2g, *n2b;
    uint16_t *kc, *vc;          /* this layer's paged fp16 caches          */
} ec_mk_layer;

typedef struct {
    int arch, lwt, hwt;         /* ARCH_*, layer / lm_head weight types    */
    int L, E, H, KVH, hd, kv, I, V, C, B, window, M;
    double eps;
    const uint16_t *wte, *wpe;
    int ld_emb, emb_bf16;
    const float *nfg, *nfb;
    ec_mk_mat lm;
    int v0;                     /* lm row 0 is vocab id v0 (vocab shard)   */
    const double *rope_cos, *rope_sin;
    const ec_mk_layer *layers;  /* device array [L]                        */
    float *x, *q, *att, *act;   /* [M][E] x3, [M][I or 4E]                 */
    float *logits;              /* [M][lm.N] or NULL                       */
    float *amax_v;              /* [grid][M] per-CTA argmax partials       */
    int *amax_i;
    int *tok, *pos, *slot;      /* [M] token state                         */
    const int *pt;              /* KV page table [B][mp] (ec_kv_row)       */
    int mp;
    int *ids;                   /* [M] argmax ids of the last step or NULL */
    float *maxv;                /* [M] their logits or NULL                */
    int *hist;                  /* [n_steps][M] or NULL                    */
    int advance;                /* 1: feed argmax back, advance positions  */
    int wrap_lo, wrap_hi;       /* position cycle (wrap_hi <= 0: none)     */
    float *taps;                /* [L+1][M][E] or NULL                     */
    unsigned *bar;              /* grid barrier counter, zero at launch    */
    unsigned *bar_next;         /* the other counter of a pair: CTA 0 zeroes
                                   it for the next launch (or NULL)        */
    int *abort_flag;            /* set by any CTA that gives up            */
    int *err;
    int in_tok[EC_MK_MT];       /* inline_in: the rows' token, position and */
    int in_pos[EC_MK_MT];       /* slot passed by value (tok / pos / slot   */
    int in_slot[EC_MK_MT];      /* are then not read)                       */
    int inline_in;
    int *done;                  /* host-mapped word or NULL: CTA 0 writes seq
                                   at a clean end, -1 if an error was recorded */
    int seq;
    int maxlen;                 /* max attended positions per row          */
    int own_rows;               /* >= residual rows owned by one CTA       */
    int kvchunk;                /* cached positions staged per attention
                                   chunk (K and V buffers in shared memory) */
    int xbuf_bytes;             /* activation smem: operand buffer ...      */
    int stage_bytes;            /* ... and fp32 staging                    */
    unsigned long long *trace;  /* optional timeline of CTA 0, (code << 56) |  */
    int trace_cap;              /* globaltimer ns; consumers fill the first
                                   half, the producer the second half       */
} ec_mk_params;

/* Trace codes: a phase's grid barrier passed, its operand built, its tiles
 * done; attention done; lm_head done; argmax merged; per weight tile: data
 * arrived, ring slot released, epilogue done; producer issued a tile copy. */
enum { EC_TR_SYNC = 1, EC_TR_PROLOGUE = 2, EC_TR_TILES = 3, EC_TR_ATTN = 4, EC_TR_LM = 5, EC_TR_ARGMAX = 6,
       EC_TR_TILE_IN = 7, EC_TR_TILE_FREE = 8, EC_TR_TILE_DONE = 9, EC_TR_ISSUE = 10,
       EC_TR_STAGED = 11,    /* a prologue's or attention item's inputs arrived in shared memory */
       EC_TR_STATS = 12,     /* norm statistics reduced */
       EC_TR_SCORES = 13,    /* attention scores and their max done */
       EC_TR_SOFTMAX = 14,   /* attention weights normalised */
       EC_TR_PHASE_IN = 15 }; /* a weight phase entered */

/* Dynamic shared memory of the kernel for these parameters. */
size_t ec_mk_smem_bytes(const ec_mk_params *p);

/* Max dynamic shared memory available to one CTA of the kernel. */
int ec_mk_smem_limit(void);

/* Launch (cooperative, one CTA per SM).  The barrier counter must be zero. */
int ec_mk_launch(const ec_mk_params *p, int n_steps, int grid, cudaStream_t stream);
/* 1 when the decode kernel was compiled with its timeline (EC_DECODE_TRACE). */
int ec_mk_traced(void);

#ifdef __cplusplus
}
#endif

#endif /* EC_DECODE_H */
