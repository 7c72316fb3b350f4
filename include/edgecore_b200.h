/*
 * edgecore_b200.h -- entry points of libedgecore_b200.so beyond the reference
 * EdgeCore ABI (which is declared, unchanged, in edgecore.h).
 *
 * All functions are plain C: pointers and sizes, no torch or CUDA types.
 * A `stream` argument is a cudaStream_t passed as void* (NULL = the model's
 * own stream / the legacy default stream for the standalone ops).
 * Functions returning int return 0 on success and -1 on failure; the reason
 * is available from ec_last_error().  Functions that mirror a `void` reference
 * entry point abort the process on a CUDA error, like the reference aborts on
 * a workspace overflow (reference src/gpt2.c:442-445).
 */
#ifndef EDGECORE_B200_H
#define EDGECORE_B200_H

#include "edgecore.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- library ---------------------------------------------------------- */

/* Text of the last error recorded on this thread ("" if none). */
const char *ec_last_error(void);

/* Library version string, e.g. "edgecore_b200 0.1 sm_100a". */
const char *ec_version(void);

/* ---- model handle for FFI callers that cannot allocate a GPT2 ---------- */

/* calloc a GPT2 and gpt2_load() it on the current CUDA device; NULL on error.
 * Mirrors reference src/runtime_main.c:650-655 (stack GPT2 + gpt2_load). */
GPT2 *ec_model_open(const char *path, int batch_cap, int max_ctx);

/* gpt2_free() + free() of a handle from ec_model_open. */
void ec_model_close(GPT2 *g);

/* Copy scalar model metadata into out[0..15]:
 * {arch, precision, n_layer, n_head, n_kv_head, n_embd, head_dim, intermediate,
 *  vocab, n_ctx, eff_ctx, batch_cap, n_kv_embd, tie_word_embeddings, device, 0}. */
int ec_model_info(const GPT2 *g, int *out16);

/* Bind all subsequent work of the model to `stream` (NULL = its own stream). */
int ec_model_set_stream(GPT2 *g, void *stream);

/* ---- forward variants --------------------------------------------------- */

/* gpt2_forward with DEVICE tokens/positions/seqs and DEVICE logits [M][vocab],
 * enqueued on the model stream without a host synchronisation. */
int ec_forward_device(GPT2 *g, const int *d_tokens, const int *d_positions,
                      const int *d_seqs, int M, float *d_logits);

/* Greedy forward: like gpt2_forward but returns only, per token row m, the
 * argmax over the vocab (lowest index on ties, as reference
 * src/runtime_main.c:213-219) and its logit.  Host pointers. */
int ec_forward_argmax(GPT2 *g, const int *tokens, const int *positions,
                      const int *seqs, int M, int *out_ids, float *out_max);

/* Device-resident greedy decode of `n_steps` tokens for the batch_cap slots
 * (batch_cap <= 8).  d_tokens[batch_cap] holds the current token of every
 * slot and is updated in place; step i runs at position start_pos + i for all
 * slots; the sampled ids are written to d_out_ids[n_steps][batch_cap] (may be
 * NULL).  All n_steps steps run inside one launch of the persistent decode
 * kernel, the argmax of each step feeding the next (reference decode loop:
 * src/runtime_main.c:336-352 with sample_token's greedy branch). */
int ec_decode_greedy(GPT2 *g, int *d_tokens, int start_pos, int n_steps,
                     int *d_out_ids);

/* ec_decode_greedy with the positions cycling through [start_pos,
 * start_pos + period): after the step at start_pos + period - 1 the next step
 * runs at start_pos again, i.e. a new continuation of the same cached prefix.
 * Lets a long measurement keep the context length of a short decode. */
int ec_decode_greedy_cycle(GPT2 *g, int *d_tokens, int start_pos, int period, int n_steps,
                           int *d_out_ids);

/* ---- batched decode: any number of independent streams ------------------ */

/* Device-resident greedy decode of n_steps tokens for every one of the
 * batch_cap slots, each at its own position: DEVICE d_tokens[batch_cap] and
 * d_positions[batch_cap] hold each slot's current token and position and are
 * updated in place; the sampled ids go to DEVICE d_out_ids[n_steps][batch_cap]
 * (may be NULL).  Up to 7 slots run the persistent decode kernel, one
 * launch for all steps; from 8, every step runs the per-layer kernels
 * (tcgen05 GEMMs, attention of each slot over its own KV rows, the lm_head
 * and a row argmax with the lowest index on ties) captured once into a CUDA
 * graph and replayed.  The call reads the positions once (synchronising the model
 * stream) and returns with the steps enqueued.  Reference: the batched decode
 * loop of src/runtime_main.c:336-352 with sample_token's greedy branch
 * (:213-219). */
int ec_decode_batch(GPT2 *g, int *d_tokens, int *d_positions, int n_steps, int *d_out_ids);

/* The column-split lm_head across ranks, in three steps a caller interleaves
 * with its own collectives (all on the model stream):
 *   ec_batch_hidden  -- rows m < M (slot m, DEVICE tokens / positions, every
 *                       position < max_pos_end) through every layer and the
 *                       final norm; normed rows [M][n_embd] fp32 into DEVICE
 *                       d_hidden (reference src/gpt2.c:797-798);
 *   ec_lm_shard_keys -- the lm_head of this model's vocab shard
 *                       (ec_model_set_vocab_shard) over `rows` DEVICE hidden
 *                       rows, each row's argmax packed as a signed 64-bit key
 *                       (ec_argmax_key with the top bit flipped) into DEVICE
 *                       d_keys[rows]: the signed max over all shards is the
 *                       reference's greedy pick (src/runtime_main.c:213-219);
 *   ec_keys_advance  -- d_tokens[m] = the index in d_keys[m], d_positions[m]
 *                       += 1 for m < M (DEVICE arrays). */
int ec_batch_hidden(GPT2 *g, const int *d_tokens, const int *d_positions, int M, int max_pos_end,
                    float *d_hidden);
int ec_lm_shard_keys(GPT2 *g, const float *d_hidden, int rows, long long *d_keys);
int ec_keys_advance(GPT2 *g, const long long *d_keys, int M, int *d_tokens, int *d_positions);

/* Kernel launches in the last captured step graph of ec_decode_batch
 * (kind 0) or ec_batch_hidden (kind 1); 0 if none was captured. */
int ec_batch_graph_kernels(GPT2 *g, int kind);

/* Paged KV arena.  Each layer's K and V caches are pools of pages of 64
 * positions; slot s keeps positions [64 j, 64 j + 64) in the page its table
 * entry j names.  Pages are mapped as calls reach new positions of a slot
 * (host-visible positions: the rows of gpt2_forward / ec_forward_argmax,
 * start_pos + n_steps of the decode loops, max_pos_end of
 * ec_batch_hidden; ec_forward_device maps every slot fully) and stay mapped
 * until ec_kv_release(slot) (slot < 0: every slot) returns them.  The pool
 * holds batch_cap * ceil(eff_ctx / 64) pages by default, so no call can run
 * out; the environment variable EDGECORE_KV_PAGES at gpt2_load sets a
 * smaller pool, and a call that needs more pages than are free fails with
 * "KV arena full".  ec_kv_info: {pages, free pages, positions per page,
 * pages per slot}. */
int ec_kv_release(GPT2 *g, int slot);
int ec_kv_info(const GPT2 *g, int *info4);

/* The device copy of one linear as gpt2_load packed it (replaces reading the
 * reference's host LayerW arrays, src/edgecore.h:119-136, for a check of the
 * load-time repack).  which: 0 q|k|v, 1 o, 2 gate|up (Qwen2) / fc (GPT-2),
 * 3 down / fc2, 4 lm_head (layer ignored).  info5 = {N rows, K, Kp, ldw,
 * element bytes}; a packed row is Kp weights (K..Kp-1 zero) then, except for
 * the lm_head, a 16-byte fp32 tail {scale, bias, 0, 0} (scale 1 / bias 0
 * where the model has none).  Row order: Qwen2 q|k|v puts the RoPE partners
 * i and i + head_dim/2 of every q and k head at rows 2i, 2i+1 (then the v
 * rows in file order); Qwen2 gate|up interleaves gate j and up j at rows 2j,
 * 2j+1; everything else is in file order.  out == NULL returns the byte
 * count only; otherwise out must hold N * ldw * element bytes (cap). */
long long ec_model_packed(const GPT2 *g, int layer, int which, void *out, size_t cap, int *info5);

/* Instrumented greedy decode for measurement: n_steps steps, one kernel
 * launch per step, with a CUDA event pair around every kernel launch on the
 * model stream.  out[16]: for kernel class c in {0 persistent decode step,
 * 1 GEMM (activation quantisation included; the lm_head too), 2 attention,
 * 3 norms, 4 other} (classes 1-4 when the persistent kernel cannot take the
 * batch: batch_cap > 8 or shared memory): out[3c] = total ms, out[3c+1] =
 * total algorithmic HBM bytes, out[3c+2] = launches; out[15] = steps. */
int ec_decode_profile(GPT2 *g, int *d_tokens, int start_pos, int n_steps, double *out16);

/* Decode n_steps (as ec_decode_greedy) recording the timeline of CTA 0 of the
 * persistent decode kernel: out[cap] receives entries (code << 56) |
 * globaltimer-ns, first those of one consumer thread (codes 1 barrier passed,
 * 2 operand built, 3 weight tiles done, 4 attention done, 5 lm_head done,
 * 6 argmax merged, 7 tile data arrived, 8 ring slot released, 9 tile epilogue
 * done, 11 a prologue's or attention item's inputs staged in shared memory,
 * 12 norm statistics reduced, 13 attention scores and their max done,
 * 14 attention weights normalised), then those of the producer thread
 * (10 tile copy issued), each part
 * holding at most cap/2 entries.  Returns the number of entries, or -1. */
int ec_decode_trace(GPT2 *g, int *d_tokens, int start_pos, int n_steps,
                    unsigned long long *out, int cap);

/* Per-layer taps of the last forward: copies the residual stream after the
 * embedding and after every layer, [n_layer+1][M][n_embd] fp32, to host
 * `out`.  Only valid after a forward with taps enabled by ec_model_set_taps. */
int ec_model_set_taps(GPT2 *g, int enable);
int ec_model_get_taps(GPT2 *g, float *out, int M);

/* ---- vocab-sharded lm_head (column split across ranks) ----------------- */

/* Restrict the model's lm_head to rows [v_begin, v_end) of the vocab.  After
 * this, ec_forward_shard_argmax returns per-row (max logit, global argmax)
 * of the shard; ranks combine them with ec_argmax_combine or a collective. */
int ec_model_set_vocab_shard(GPT2 *g, int v_begin, int v_end);
int ec_forward_shard_argmax(GPT2 *g, const int *tokens, const int *positions,
                            const int *seqs, int M, int *out_ids, float *out_max);

/* Encode (max, idx) as a 64-bit key whose unsigned order is "larger logit,
 * then lower index": combining shards with an unsigned max gives the
 * reference tie rule.  -0.0 is encoded as +0.0 (the reference's '>' scan
 * treats them as equal) and NaN below every number (it never wins a '>').
 * Decode inverts it (a NaN comes back as a NaN, -0.0 as +0.0). */
uint64_t ec_argmax_key(float maxv, int idx);
void ec_argmax_key_decode(uint64_t key, float *maxv, int *idx);

/* ---- standalone ops (host or device pointers) --------------------------- */

/* Per-row symmetric int8 activation quantisation, bit-exact with the int8
 * branch of reference linear() (src/gpt2.c:446-461). */
int ec_quantize_rows(int8_t *q, float *scale, const float *x, int M, int K);

/* W8A8 linear: quantise X rows then gemm_int8 (reference src/gpt2.c:437-462). */
int ec_linear_int8(float *C, const float *X, const int8_t *W,
                   const float *w_scale, const float *bias, int M, int K, int N);

/* The device exp and tanh every kernel of this library uses: restatements
 * of the reference's host libm expf / tanhf (glibc 2.39: ARM
 * optimized-routines expf, fdlibm tanhf / expm1f) that round exactly as the
 * host functions.  Applies them to n DEVICE floats (d_exp or d_tanh may be
 * NULL), enqueued on `stream`; for checking against the host library. */
int ec_reference_math(const float *d_x, float *d_exp, float *d_tanh, int n, void *stream);

/* Attention of the per-layer path (prefill, batched decode; the persistent
 * decode kernel has its own): 1 = always the split kernels (flash-decoding
 * partial sums over position blocks, then a combine), which otherwise run
 * only when a row's scores do not fit the exact-order kernel's shared memory
 * (tens of thousands of positions); 0 = the default choice.  Process-wide,
 * for tests and measurement.  The reference's order is the exact kernel's;
 * the split kernels agree with it to rounding of the partial sums. */
int ec_attention_force_split(int on);

/* gemm_int8 (wt 0: A int8 [M][K] with a_scale[M]), gemm_fp16_fp32 (wt 1)
 * or gemm_bf16_fp32 (wt 2: A fp32 [M][K]) on DEVICE operands of the current
 * device, enqueued on `stream` with no host synchronisation: the
 * reference's gemm_* (src/kernels.c:129-168) for GPU callers that keep their
 * data resident.  K must be a multiple of 16 (rows are read in place).
 * M < 8 runs the weight-streaming GEMV, larger M the tcgen05 GEMM kernels
 * (16-bit weights there use a library workspace allocated on first use).  Device-side errors: ec_device_error_take. */
int ec_gemm_async(int wt, float *C, const void *A, const float *a_scale, const void *B,
                  const float *b_scale, const float *bias, int M, int K, int N, void *stream);

/* Device-side error of the standalone ops: synchronises `stream`, then reads
 * and clears the library's device error words into *code (0 none, 1 a
 * bounded wait inside a kernel gave up, 2 an out-of-range index was
 * skipped).  The entry points that return before their kernels finish
 * (ec_linear_int8_noalloc, ec_forward_device) report such errors only here. */
int ec_device_error_take(void *stream, int *code);

/* ec_linear_int8 that allocates no device memory: no counterpart in the
 * reference (whose CPU op needs none).  For callers that cannot allocate on
 * the request path -- HBM handed to a caching allocator, or a decode loop
 * that must not be stalled by cudaMalloc's device synchronisation.  The
 * int8 activations and their scales live in a fixed 4 MiB per-device static
 * buffer: requires M*K + 4*M (rounded up to 256) <= 4 MiB, K % 16 == 0 and
 * device pointers only; larger sizes are rejected with an error.  M < 8
 * uses the weight-streaming GEMV when a W row plus the M activation rows fit
 * its shared memory (K up to about 113,000 at M = 1), else the GEMM kernels.
 * The first call on a device does the set-up (scratch address lookup,
 * kernel attributes, tensor-map encoder, loading) and should come before any
 * stream capture.  Device-side errors: ec_device_error_take.  Work
 * is enqueued on `stream` (cudaStream_t, NULL = legacy default) without a
 * host wait.  Calls that can overlap on the device share the one buffer and
 * race: order them on one stream or with events.  Returns 0 or -1 (reason
 * in ec_last_error()). */
int ec_linear_int8_noalloc(float *C, const float *X, const int8_t *W,
                           const float *w_scale, const float *bias, int M, int K, int N,
                           void *stream);

#ifdef __cplusplus
}
#endif

#endif /* EDGECORE_B200_H */
