// ec_decode.cu -- persistent decode kernel: a whole forward step (embedding,
// every layer, final norm, lm_head, greedy argmax) for M <= 8 token rows in
// one cooperative launch, optionally looping over many decode steps.
//
// One CTA per SM, 9 warps:
//   warp 0      producer: streams this CTA's share of every weight matrix, in
//               execution order, through a ring of EC_MK_STAGES x 32 KB shared
//               memory slots with bulk TMA copies (cp.async.bulk, this GPU's
//               own memory only).  Weights do not depend on activations, so
//               the producer runs ahead across phase and layer boundaries,
//               bounded only by the ring.
//   warps 1-8   consumers: the dependent chain of phases, separated by grid
//               barriers (arrival counter in global memory):
//     A  norm(x) -> int8 quantise -> q|k|v rows  -> RoPE, q, fp16 KV store
//     B  exact-order attention, one (token, head) item per CTA
//     C  quantise(attn) -> o rows -> residual add into x
//     D  norm(x) -> quantise -> gate|up rows -> SwiGLU (GELU for GPT-2)
//     E  quantise(act) -> down rows -> residual add into x
//     F  final norm -> lm_head rows -> logits, per-CTA argmax
//     G  every CTA merges the argmax partials -> next token
//   Each CTA owns a contiguous slice of every matrix's rows; o and down share
//   their partition, so a residual row of x is only ever written by its owner.
//
// Code size is kept small on purpose (the whole step runs from the
// instruction cache): the token count is a template parameter (1, 2, 4 or 8
// rows), and the tile loop, the norm and the operand builder exist once per
// kernel as non-inlined functions shared by all phases.
//
// Numerics are those of the reference (src/gpt2.c, src/kernels.c): exact
// int32 dots and the (bias + ((float)dot*as)*ws) epilogue, fp64 norm
// statistics, fp64 RoPE, the exact-order attention of k_attn_exact, and
// the host libm's exp/tanh (ec_expf / ec_tanhf).  Every wait is bounded; a CTA that gives up
// raises the shared abort flag so the others leave instead of spinning.
#include "ec_common.cuh"
#include "ec_launch.h"
#include "ec_decode.h"

#include <float.h>

#include <atomic>

namespace {

constexpr int MT = EC_MK_MT;
constexpr int NCW = EC_MK_CONS_WARPS;
constexpr int NCT = NCW * 32;
constexpr int STAGES = EC_MK_STAGES;
constexpr int TILE = EC_MK_TILE;
constexpr int ARCH_Q2 = 1;                        // ARCH_QWEN2
constexpr long long SPIN_CYCLES = 4000000000LL;   // ~2 s: bound on any grid-barrier wait
constexpr int ERR_TIMEOUT = 1, ERR_INDEX = 2;
constexpr uint32_t T_ABORT = 0xffffffffu;         // tile counter value meaning "aborted"
constexpr unsigned PRODUCER_BACKOFF_NS = 128;      // producer sleep between empty-slot polls

// Phase kinds of the shared tile loop, and the five matrix shapes whose
// per-CTA row ranges are computed once per launch.
enum { PK_QKV = 0, PK_RESID = 1, PK_UP = 2 };
enum { MI_QKV = 0, MI_O = 1, MI_UP = 2, MI_DOWN = 3, MI_LM = 4, MI_N = 5 };

// Loop over the token rows m < p.M with compile-time indices (bounded by the
// kernel's MM), so per-token arrays stay in registers.
// Every user declares `const int nM = p.M;` (a register, not a reload).
#define FOR_TOK(m) _Pragma("unroll") for (int m = 0; m < MM; ++m) if (m < nM)

// Loop over k = ct, ct + NCT, ... < n, deliberately not unrolled: these loops
// run one to a few iterations per thread (K / 256), and on B200 the unrolled
// form (guarded copies, more code per phase) measured slower than the plain
// loop (decode step 0.935 -> 0.893 ms for this change alone).
#define FOR_K(k, n) _Pragma("unroll 1") for (int k = ct; k < (n); k += NCT)

struct Lay {
    uint32_t ring, xbuf, stage, nrm, rope, xown, redd, redf, redi, asc, ints, lpt, bars, lays, par, total;
};

// KV page-table rows of the token rows' slots kept in shared memory (fixed
// for a launch: the host maps every page a launch touches beforehand) when a
// slot has at most PT_SMEM pages; else read from global memory.
constexpr int PT_SMEM = 64;

__host__ __device__ inline uint32_t al16(uint32_t v) { return (v + 15u) & ~15u; }

__host__ __device__ inline Lay mk_layout(int xbuf_bytes, int stage_bytes, int n_layer, int E, int hd, int own_rows) {
    Lay L;
    // fixed-size regions first, at compile-time offsets (no address arithmetic
    // in the helpers), then the regions sized by the model
    uint32_t o = 0;
    L.ints = o;  o += al16((3 * MT + 4 + 2 * MI_N) * 4);
    L.lpt = o;   o += MT * PT_SMEM * 4;
    L.bars = o;  o += 2 * STAGES * 8;
    L.redd = o;  o += 2 * NCW * MT * 8;
    L.redf = o;  o += 2 * NCW * MT * 4;
    L.redi = o;  o += NCW * MT * 4;
    L.asc = o;   o += MT * 4;
    o = (o + 127u) & ~127u;
    L.ring = o;  o += STAGES * TILE;
    L.xbuf = o;  o += al16((uint32_t)xbuf_bytes);
    L.stage = o; o += al16((uint32_t)stage_bytes);
    L.nrm = o;   o += 2u * al16((uint32_t)E * 4u);
    L.rope = o;  o += al16((uint32_t)MT * (uint32_t)hd * 8u);          // cos, sin rows of each token's position
    L.xown = o;  o += al16((uint32_t)MT * (uint32_t)own_rows * 4u);    // residual rows owned by this CTA
    L.lays = o;  o += al16((uint32_t)n_layer * (uint32_t)sizeof(ec_mk_layer));
    L.par = o;   o += al16((uint32_t)sizeof(ec_mk_params));
    L.total = o;
    return L;
}

extern __shared__ __align__(128) unsigned char g_smem[];

struct Rg { int r0, r1; };

struct Sm {
    unsigned char *ring, *xbuf;
    float *stage;
    float *nrm;               // norm gain [E] and bias [E] of the running norm
    double *rope;             // [MT][hd/2] cos then [MT][hd/2] sin at each token's position
    float *xown;              // [MT][own_rows] residual rows owned by this CTA (also in p.x)
    double *redd;             // [2][NCW][MT]: two slots, see red_sum_d
    float *redf;              // [2][NCW][MT]
    int *redi;
    float *asc;
    int *ltok, *lpos, *lslot;
    int *lpt;                 // [MT][PT_SMEM] page-table rows of the token rows' slots
    volatile int *flag;       // [0]: abort
    int *tcount;              // [2]: trace entries written (consumer, producer)
    Rg *rg;                   // [MI_N]: this CTA's row range of each matrix shape
    uint64_t *full, *empty;
    const ec_mk_layer *lay;   // shared-memory copy of the layer descriptors
    ec_mk_params *par;        // shared-memory copy of the kernel parameters
};

__device__ __forceinline__ Sm sm_of(const ec_mk_params &p) {
    const Lay L = mk_layout(p.xbuf_bytes, p.stage_bytes, p.L, p.E, p.hd, p.own_rows);
    Sm S;
    S.ring = g_smem + L.ring;
    S.xbuf = g_smem + L.xbuf;
    S.stage = reinterpret_cast<float *>(g_smem + L.stage);
    S.nrm = reinterpret_cast<float *>(g_smem + L.nrm);
    S.rope = reinterpret_cast<double *>(g_smem + L.rope);
    S.xown = reinterpret_cast<float *>(g_smem + L.xown);
    S.redd = reinterpret_cast<double *>(g_smem + L.redd);
    S.redf = reinterpret_cast<float *>(g_smem + L.redf);
    S.redi = reinterpret_cast<int *>(g_smem + L.redi);
    S.asc = reinterpret_cast<float *>(g_smem + L.asc);
    int *ints = reinterpret_cast<int *>(g_smem + L.ints);
    S.ltok = ints;
    S.lpos = ints + MT;
    S.lslot = ints + 2 * MT;
    S.lpt = reinterpret_cast<int *>(g_smem + L.lpt);
    S.flag = ints + 3 * MT;
    S.tcount = ints + 3 * MT + 1;
    S.rg = reinterpret_cast<Rg *>(ints + 3 * MT + 4);
    S.full = reinterpret_cast<uint64_t *>(g_smem + L.bars);
    S.empty = S.full + STAGES;
    S.lay = reinterpret_cast<const ec_mk_layer *>(g_smem + L.lays);
    S.par = reinterpret_cast<ec_mk_params *>(g_smem + L.par);
    return S;
}

// Arena row of position `pos` of token row q (slot `slot`).
__device__ __forceinline__ size_t kv_row_q(const ec_mk_params &p, const Sm &S, int q, int slot, int pos) {
    const int pg = p.mp <= PT_SMEM ? S.lpt[q * PT_SMEM + (pos >> 6)] : __ldg(p.pt + (size_t)slot * p.mp + (pos >> 6));
    return (size_t)(pg < 0 ? 0 : pg) * EC_KV_PAGE + (size_t)(pos & (EC_KV_PAGE - 1));
}

__device__ __forceinline__ Rg mk_range(const ec_mk_mat &m, int c, int G) {
    const int U = m.N / m.unit;
    const int u0 = (int)(((long long)c * U) / G), u1 = (int)(((long long)(c + 1) * U) / G);
    return Rg{u0 * m.unit, u1 * m.unit};
}

__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory"); }

// Consumer barrier that also ORs a predicate over the NCT consumer threads,
// so that every warp takes the same abort decision.
__device__ __forceinline__ bool cons_sync_or(bool v) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.s32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\t"
        "selp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((int)v), "n"(NCT)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(ec_smem_u32(bar)) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int ld_relaxed_i(const int *p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int elt_of(int wt) { return wt == EC_W_I8 ? 1 : 2; }

// 16-byte asynchronous global -> shared copy through L2 (data written by
// other SMs before the last grid barrier).
__device__ __forceinline__ void cpa16(void *dst_smem, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(ec_smem_u32(dst_smem)), "l"(src) : "memory");
}

__device__ __forceinline__ void cpa_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Issue the copy of n floats global -> shared with every 16-byte piece in
// flight at once (scalar loads for a ragged tail or an unaligned source).
// Completion: cpa_wait_all() by every issuing thread, then a consumer barrier.
__device__ __forceinline__ void stage_issue(float *dst, const float *src, int n, int ct) {
    int done = 0;
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        const int n4 = n >> 2;
#pragma unroll 1
        for (int i = ct; i < n4; i += NCT) cpa16(dst + 4 * i, src + 4 * i);
        done = 4 * n4;
    }
#pragma unroll 1
    for (int i = done + ct; i < n; i += NCT) dst[i] = __ldcg(src + i);
}

// Timeline of CTA 0 when p.trace is set, in builds with EC_DECODE_TRACE
// defined (the product build has none: even a not-taken check of p.trace at
// every mark cost ~5 % of the decode step): consumer thread 0 writes the
// first half of the buffer, the producer thread the second half, entries
// (code << 56) | globaltimer ns.  Each half has its own count in shared memory.
#ifdef EC_DECODE_TRACE
__device__ __noinline__ void tmark_rec(const ec_mk_params &p, int *tcount, int who, int code) {
    const int half = p.trace_cap / 2, cap = who ? p.trace_cap - half : half;
    int &n = tcount[who];
    if (n < cap) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        p.trace[(size_t)who * half + n++] = ((unsigned long long)code << 56) | (t & 0x00ffffffffffffffull);
    }
}

// The check stays inline, the recording out of line.
__device__ __forceinline__ void tmark(const ec_mk_params &p, const Sm &S, int who, int code) {
    if (p.trace && blockIdx.x == 0) tmark_rec(p, S.tcount, who, code);
}
#else
__device__ __forceinline__ void tmark(const ec_mk_params &, const Sm &, int, int) {}
#endif

// ---------------------------------------------------------------------------
// producer
// ---------------------------------------------------------------------------

__device__ __noinline__ uint32_t mk_produce(const ec_mk_params &p, const ec_mk_mat &m, int wt, Rg rg, uint32_t t) {
    const Sm S = sm_of(p);
    const uint32_t row_bytes = (uint32_t)m.ldw * (uint32_t)elt_of(wt);
    const uint64_t pol = ec_l2_evict_first();
    for (int r = rg.r0; r < rg.r1; r += m.tile_rows) {
        const int nr = min(m.tile_rows, rg.r1 - r);
        const int s = (int)(t % STAGES);
        const uint32_t k = t / STAGES;
        if (k > 0) {
            bool ok = false;
            for (uint32_t i = 0; i < EC_WAIT_LIMIT; ++i) {
                if (ec_mbar_try_wait(&S.empty[s], (k - 1) & 1)) { ok = true; break; }
                if (S.flag[0]) return T_ABORT;
                // The producer runs ahead of the consumers and waits here most
                // of the time: sleep between polls so that it takes no issue
                // slots or shared-memory bandwidth from the consumer warps.
                __nanosleep(PRODUCER_BACKOFF_NS);
            }
            if (!ok) { S.flag[0] = 1; atomicCAS(p.err, 0, ERR_TIMEOUT); return T_ABORT; }
        }
        const uint32_t bytes = (uint32_t)nr * row_bytes;
        ec_mbar_expect_tx(&S.full[s], bytes);
        ec_bulk_g2s_hint(S.ring + (size_t)s * TILE, static_cast<const unsigned char *>(m.w) + (size_t)r * row_bytes,
                         bytes, &S.full[s], pol);
        tmark(p, S, 1, EC_TR_ISSUE);
        ++t;
    }
    return t;
}

// ---------------------------------------------------------------------------
// consumers: reductions over the NCT consumer threads (fixed order: lanes by
// xor tree, warps in index order; every thread gets the totals)
// ---------------------------------------------------------------------------

// CTA-wide reductions over the NCT consumer threads: lanes by xor tree (or
// redux), warps in index order, every thread gets the totals.  Each call
// site uses its own slot of the reduction buffers, and every buffer slot is
// read before a consumer barrier that precedes its next write, so one
// barrier per reduction suffices.
template <int MM>
__device__ __forceinline__ void red_sum_d(const ec_mk_params &p, const Sm &S, double v[MM], int ct, int slot) {
    const int nM = p.M;
    const int lane = ct & 31, w = ct >> 5;
    double *buf = S.redd + slot * NCW * MT;
    FOR_TOK(m) v[m] = ec_warp_sum_d(v[m]);
    if (lane == 0) FOR_TOK(m) buf[w * MT + m] = v[m];
    cons_sync();
    FOR_TOK(m) {
        double t = 0.0;
        for (int i = 0; i < NCW; ++i) t = __dadd_rn(t, buf[i * MT + m]);
        v[m] = t;
    }
}

// Max of non-negative, non-NaN values: their bit patterns order like the
// values, so one redux instruction reduces a warp.
template <int MM>
__device__ __forceinline__ void red_max_f(const ec_mk_params &p, const Sm &S, float v[MM], int ct, int slot) {
    const int nM = p.M;
    const int lane = ct & 31, w = ct >> 5;
    float *buf = S.redf + slot * NCW * MT;
    FOR_TOK(m) v[m] = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v[m])));
    if (lane == 0) FOR_TOK(m) buf[w * MT + m] = v[m];
    cons_sync();
    FOR_TOK(m) {
        float t = buf[m];
        for (int i = 1; i < NCW; ++i) t = ec_max_keep(t, buf[i * MT + m]);
        v[m] = t;
    }
}

__device__ __forceinline__ void am_merge(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

template <int MM>
__device__ __forceinline__ void red_argmax(const ec_mk_params &p, const Sm &S, float bv[MM], int bi[MM], int ct) {
    const int nM = p.M;
    const int lane = ct & 31, w = ct >> 5;
    FOR_TOK(m) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv[m], o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi[m], o);
            am_merge(bv[m], bi[m], ov, oi);
        }
    }
    if (lane == 0) FOR_TOK(m) { S.redf[w * MT + m] = bv[m]; S.redi[w * MT + m] = bi[m]; }
    cons_sync();
    FOR_TOK(m) {
        float v = S.redf[m];
        int i = S.redi[m];
        for (int k = 1; k < NCW; ++k) am_merge(v, i, S.redf[k * MT + m], S.redi[k * MT + m]);
        bv[m] = v;
        bi[m] = i;
    }
}

// ---------------------------------------------------------------------------
// consumers: prologues
// ---------------------------------------------------------------------------

__device__ __forceinline__ float mk_embed(const ec_mk_params &p, int tok, int pos, int k) {
    const bool bf = p.emb_bf16 != 0;
    float e = ec_h2f(p.wte[(size_t)tok * p.ld_emb + k], bf);
    if (p.wpe) e = __fadd_rn(e, ec_h2f(p.wpe[(size_t)pos * p.ld_emb + k], bf));
    return e;
}

// Norm of the residual rows (or of the embedding, for layer 0) into S.stage
// [M][E] fp32: LayerNorm when beta != NULL, else RMSNorm (reference
// src/gpt2.c:398-414, :592-604), fp64 statistics.  The rows and the gains
// come in with one round of asynchronous copies.
template <int MM>
__device__ __noinline__ void mk_norm(const ec_mk_params &p, bool from_embed, const float *g, const float *b, int ct) {
    const Sm S = sm_of(p);
    const int nM = p.M;
    const int E = p.E;
    float *st = S.stage;
    float *gs = S.nrm, *bs = S.nrm + ((E + 3) & ~3);
    stage_issue(gs, g, E, ct);
    if (b) stage_issue(bs, b, E, ct);
    if (!from_embed) stage_issue(st, p.x, nM * E, ct);
    else FOR_TOK(m) for (int k = ct; k < E; k += NCT) st[m * E + k] = mk_embed(p, S.ltok[m], S.lpos[m], k);
    cpa_wait_all();
    cons_sync();
    double s1[MM];
    FOR_TOK(m) {
        s1[m] = 0.0;
        FOR_K(k, E) {
            const double d = (double)st[m * E + k];
            s1[m] = b ? __dadd_rn(s1[m], d) : __dadd_rn(s1[m], __dmul_rn(d, d));
        }
    }
    red_sum_d<MM>(p, S, s1, ct, 0);
    double mean[MM], rstd[MM];
    if (b) {
        double s2[MM];
        FOR_TOK(m) {
            s2[m] = 0.0;
            mean[m] = __ddiv_rn(s1[m], (double)E);
            FOR_K(k, E) {
                const double d = __dsub_rn((double)st[m * E + k], mean[m]);
                s2[m] = __dadd_rn(s2[m], __dmul_rn(d, d));
            }
        }
        red_sum_d<MM>(p, S, s2, ct, 1);
        FOR_TOK(m) rstd[m] = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(s2[m], (double)E), p.eps)));
    } else {
        FOR_TOK(m) {
            mean[m] = 0.0;
            rstd[m] = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(s1[m], (double)E), p.eps)));
        }
    }
    FOR_TOK(m) {
        FOR_K(k, E) {
            const double d = b ? __dsub_rn((double)st[m * E + k], mean[m]) : (double)st[m * E + k];
            const float t = (float)__dmul_rn(d, rstd[m]);
            st[m * E + k] = b ? __fadd_rn(__fmul_rn(t, gs[k]), bs[k]) : __fmul_rn(t, gs[k]);
        }
    }
    cons_sync();
}

// Build the GEMV operand for K-wide rows: int8 quantised rows (reference
// src/gpt2.c:446-461) with scales in S.asc, or fp32 planes for 16-bit weights.
// Source: S.stage (src == NULL) or global rows `src` with row stride K.
template <int MM>
__device__ __noinline__ void mk_operand(const ec_mk_params &p, const float *src, int K, int Kp, int wt, int ct) {
    const Sm S = sm_of(p);
    const int nM = p.M;
    const bool fits = (size_t)p.M * K * 4 <= (size_t)p.stage_bytes;
    float *st = S.stage;
    if (src && fits) {   // one round of asynchronous copies into the staging area
        stage_issue(st, src, nM * K, ct);
        cpa_wait_all();
        cons_sync();
    }
    const bool from_stage = !src || fits;
    const bool vec = from_stage && (K & 3) == 0;   // rows as float4 (Kp is a multiple of 16)
    if (wt == EC_W_I8) {
        float mx[MM];
        FOR_TOK(m) {
            mx[m] = 0.0f;
            if (vec) {
                const float4 *r4 = reinterpret_cast<const float4 *>(st + (size_t)m * K);
                FOR_K(c, K >> 2) {
                    const float4 v = r4[c];
                    mx[m] = ec_max_keep(ec_max_keep(ec_max_keep(ec_max_keep(mx[m], fabsf(v.x)), fabsf(v.y)), fabsf(v.z)), fabsf(v.w));
                }
            } else {
                for (int k = ct; k < K; k += NCT)
                    mx[m] = ec_max_keep(mx[m], fabsf(from_stage ? st[m * K + k] : __ldcg(src + (size_t)m * K + k)));
            }
        }
        red_max_f<MM>(p, S, mx, ct, 0);
        int8_t *xq = reinterpret_cast<int8_t *>(S.xbuf);
        FOR_TOK(m) {
            const float s = mx[m] > 0.0f ? __fdiv_rn(mx[m], 127.0f) : 1.0f;
            const float r = __fdiv_rn(1.0f, s);
            if (ct == 0) S.asc[m] = s;
            if (vec) {
                const float4 *r4 = reinterpret_cast<const float4 *>(st + (size_t)m * K);
                char4 *q4 = reinterpret_cast<char4 *>(xq + (size_t)m * Kp);
                FOR_K(c, Kp >> 2) {
                    char4 o = make_char4(0, 0, 0, 0);
                    if (4 * c < K) {
                        const float4 v = r4[c];
                        o = make_char4((signed char)ec_quant_fast(v.x, s, r), (signed char)ec_quant_fast(v.y, s, r),
                                       (signed char)ec_quant_fast(v.z, s, r), (signed char)ec_quant_fast(v.w, s, r));
                    }
                    q4[c] = o;
                }
            } else {
                for (int k = ct; k < Kp; k += NCT) {
                    const float v = k < K ? (from_stage ? st[m * K + k] : __ldcg(src + (size_t)m * K + k)) : 0.0f;
                    xq[(size_t)m * Kp + k] = (int8_t)(k < K ? ec_quant_fast(v, s, r) : 0);
                }
            }
        }
    } else {
        float *xs = reinterpret_cast<float *>(S.xbuf);
        FOR_TOK(m) {
            float *xm = xs + (size_t)m * Kp;
            FOR_K(k, Kp) {
                const float v = k < K ? (from_stage ? st[m * K + k] : __ldcg(src + (size_t)m * K + k)) : 0.0f;
                const int c = k >> 3, e = k & 7;
                xm[(e >> 2) * (Kp >> 1) + c * 4 + (e & 3)] = v;
            }
        }
    }
    cons_sync();
}

// mk_prep for 4 or 8 token rows: the same arithmetic in the same order, but
// the element loops run over one token row at a time and the per-row
// statistics, scales and reciprocals pass through shared memory, so that no
// per-row array lives in registers across an element loop (with 8 rows
// unrolled the register form spilled to local memory inside those loops,
// ~20-70 us per phase).
template <int MM>
__device__ __noinline__ void mk_prep_rows(const ec_mk_params &p, const float *src, int K, int Kp, bool from_embed,
                                          const float *g, const float *b, int ct) {
    const Sm S = sm_of(p);
    const int nM = p.M;
    const int lane = ct & 31, w = ct >> 5;
    float *st = S.stage;
    float *gs = S.nrm, *bs = S.nrm + ((K + 3) & ~3);
    float *pmax = S.redf;                       // [NCW][MT] per-warp maxima
    if (!g && !from_embed && (size_t)nM * K * 4 > (size_t)p.stage_bytes) {
        // rows wider than the staging area holds together (the down
        // projection's input): one row at a time
        int8_t *xq = reinterpret_cast<int8_t *>(S.xbuf);
#pragma unroll 1
        for (int m = 0; m < nM; ++m) {
            stage_issue(st, src + (size_t)m * K, K, ct);
            cpa_wait_all();
            cons_sync();
            float mx = 0.0f;
            const float4 *r4 = reinterpret_cast<const float4 *>(st);
            FOR_K(c, K >> 2) {
                const float4 v = r4[c];
                mx = ec_max_keep(ec_max_keep(ec_max_keep(ec_max_keep(mx, fabsf(v.x)), fabsf(v.y)), fabsf(v.z)), fabsf(v.w));
            }
            mx = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(mx)));
            if (lane == 0) pmax[w * MT + m] = mx;
            cons_sync();
            float t = pmax[m];
            for (int i = 1; i < NCW; ++i) t = ec_max_keep(t, pmax[i * MT + m]);
            const float sc = t > 0.0f ? __fdiv_rn(t, 127.0f) : 1.0f;
            const float r = __fdiv_rn(1.0f, sc);
            if (ct == 0) S.asc[m] = sc;
            char4 *q4 = reinterpret_cast<char4 *>(xq + (size_t)m * Kp);
            FOR_K(c, Kp >> 2) {
                char4 o = make_char4(0, 0, 0, 0);
                if (4 * c < K) {
                    const float4 v = r4[c];
                    o = make_char4((signed char)ec_quant_fast(v.x, sc, r), (signed char)ec_quant_fast(v.y, sc, r),
                                   (signed char)ec_quant_fast(v.z, sc, r), (signed char)ec_quant_fast(v.w, sc, r));
                }
                q4[c] = o;
            }
            cons_sync();   // the staging area takes the next row
        }
        return;
    }
    if (g) {
        stage_issue(gs, g, K, ct);
        if (b) stage_issue(bs, b, K, ct);
    }
    if (!from_embed) stage_issue(st, src, nM * K, ct);
    else FOR_TOK(m) FOR_K(k, K) st[m * K + k] = mk_embed(p, S.ltok[m], S.lpos[m], k);
    cpa_wait_all();
    cons_sync();
    double *part = S.redd;                      // [NCW][MT] per-warp partial sums
    double *mean = S.redd + NCW * MT, *rstd = mean + MT;
    float *rcp = S.redf + NCW * MT;
    if (g) {
#pragma unroll 1
        for (int m = 0; m < nM; ++m) {
            double s1 = 0.0;
            FOR_K(k, K) {
                const double d = (double)st[m * K + k];
                s1 = b ? __dadd_rn(s1, d) : __dadd_rn(s1, __dmul_rn(d, d));
            }
            s1 = ec_warp_sum_d(s1);
            if (lane == 0) part[w * MT + m] = s1;
        }
        cons_sync();
        if (ct < nM) {
            double t = 0.0;
            for (int i = 0; i < NCW; ++i) t = __dadd_rn(t, part[i * MT + ct]);
            if (b) mean[ct] = __ddiv_rn(t, (double)K);
            else {
                mean[ct] = 0.0;
                rstd[ct] = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(t, (double)K), p.eps)));
            }
        }
        cons_sync();
        if (b) {
#pragma unroll 1
            for (int m = 0; m < nM; ++m) {
                const double mu = mean[m];
                double s2 = 0.0;
                FOR_K(k, K) {
                    const double d = __dsub_rn((double)st[m * K + k], mu);
                    s2 = __dadd_rn(s2, __dmul_rn(d, d));
                }
                s2 = ec_warp_sum_d(s2);
                if (lane == 0) part[w * MT + m] = s2;
            }
            cons_sync();
            if (ct < nM) {
                double t = 0.0;
                for (int i = 0; i < NCW; ++i) t = __dadd_rn(t, part[i * MT + ct]);
                rstd[ct] = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(t, (double)K), p.eps)));
            }
            cons_sync();
        }
#pragma unroll 1
        for (int m = 0; m < nM; ++m) {
            const double mu = mean[m], rs = rstd[m];
            float mx = 0.0f;
            float4 *r4 = reinterpret_cast<float4 *>(st + (size_t)m * K);
            FOR_K(c, K >> 2) {
                float e[4];
                *reinterpret_cast<float4 *>(e) = r4[c];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int k = 4 * c + j;
                    const double d = b ? __dsub_rn((double)e[j], mu) : (double)e[j];
                    const float t = (float)__dmul_rn(d, rs);
                    e[j] = b ? __fadd_rn(__fmul_rn(t, gs[k]), bs[k]) : __fmul_rn(t, gs[k]);
                    mx = ec_max_keep(mx, fabsf(e[j]));
                }
                r4[c] = *reinterpret_cast<const float4 *>(e);
            }
            mx = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(mx)));
            if (lane == 0) pmax[w * MT + m] = mx;
        }
    } else {
#pragma unroll 1
        for (int m = 0; m < nM; ++m) {
            float mx = 0.0f;
            const float4 *r4 = reinterpret_cast<const float4 *>(st + (size_t)m * K);
            FOR_K(c, K >> 2) {
                const float4 v = r4[c];
                mx = ec_max_keep(ec_max_keep(ec_max_keep(ec_max_keep(mx, fabsf(v.x)), fabsf(v.y)), fabsf(v.z)), fabsf(v.w));
            }
            mx = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(mx)));
            if (lane == 0) pmax[w * MT + m] = mx;
        }
    }
    cons_sync();
    if (ct < nM) {
        float t = pmax[ct];
        for (int i = 1; i < NCW; ++i) t = ec_max_keep(t, pmax[i * MT + ct]);
        const float sc = t > 0.0f ? __fdiv_rn(t, 127.0f) : 1.0f;
        S.asc[ct] = sc;
        rcp[ct] = __fdiv_rn(1.0f, sc);
    }
    cons_sync();
    int8_t *xq = reinterpret_cast<int8_t *>(S.xbuf);
#pragma unroll 1
    for (int m = 0; m < nM; ++m) {
        const float sc = S.asc[m], r = rcp[m];
        const float4 *r4 = reinterpret_cast<const float4 *>(st + (size_t)m * K);
        char4 *q4 = reinterpret_cast<char4 *>(xq + (size_t)m * Kp);
        FOR_K(c, Kp >> 2) {
            char4 o = make_char4(0, 0, 0, 0);
            if (4 * c < K) {
                const float4 v = r4[c];
                o = make_char4((signed char)ec_quant_fast(v.x, sc, r), (signed char)ec_quant_fast(v.y, sc, r),
                               (signed char)ec_quant_fast(v.z, sc, r), (signed char)ec_quant_fast(v.w, sc, r));
            }
            q4[c] = o;
        }
    }
    cons_sync();
}

// Int8 operand of one phase in a single pass, shared by the four per-layer
// call sites so that one copy of the code serves them all: the K-wide rows
// come from `src` (o / down inputs) or are the norm of the residual rows
// (q|k|v and gate|up inputs; the embedding for layer 0), then quantise into
// S.xbuf with scales in S.asc.  Same arithmetic, in the same order, as
// mk_norm followed by mk_operand; the max of |x| is taken while the
// normalised values are written, which saves a pass and a barrier.
template <int MM>
__device__ __noinline__ void mk_prep(const ec_mk_params &p, const float *src, int K, int Kp, bool from_embed,
                                     const float *g, const float *b, int ct) {
    if constexpr (MM >= 4) {
        mk_prep_rows<MM>(p, src, K, Kp, from_embed, g, b, ct);
        return;
    }
    const Sm S = sm_of(p);
    const int nM = p.M;
    float *st = S.stage;
    float *gs = S.nrm, *bs = S.nrm + ((K + 3) & ~3);
    if (g) {
        stage_issue(gs, g, K, ct);
        if (b) stage_issue(bs, b, K, ct);
    }
    if (!from_embed) stage_issue(st, src, nM * K, ct);
    else FOR_TOK(m) FOR_K(k, K) st[m * K + k] = mk_embed(p, S.ltok[m], S.lpos[m], k);
    cpa_wait_all();
    cons_sync();
    if (ct == 0) tmark(p, S, 0, EC_TR_STAGED);
    float mx[MM];
    FOR_TOK(m) mx[m] = 0.0f;
    if (g) {
        double s1[MM], mean[MM], rstd[MM];
        FOR_TOK(m) {
            s1[m] = 0.0;
            FOR_K(k, K) {
                const double d = (double)st[m * K + k];
                s1[m] = b ? __dadd_rn(s1[m], d) : __dadd_rn(s1[m], __dmul_rn(d, d));
            }
        }
        red_sum_d<MM>(p, S, s1, ct, 0);
        if (ct == 0) tmark(p, S, 0, EC_TR_STATS);
        if (b) {
            double s2[MM];
            FOR_TOK(m) {
                s2[m] = 0.0;
                mean[m] = __ddiv_rn(s1[m], (double)K);
                FOR_K(k, K) {
                    const double d = __dsub_rn((double)st[m * K + k], mean[m]);
                    s2[m] = __dadd_rn(s2[m], __dmul_rn(d, d));
                }
            }
            red_sum_d<MM>(p, S, s2, ct, 1);
            FOR_TOK(m) rstd[m] = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(s2[m], (double)K), p.eps)));
        } else {
            FOR_TOK(m) {
                mean[m] = 0.0;
                rstd[m] = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(s1[m], (double)K), p.eps)));
            }
        }
        FOR_TOK(m) {
            float4 *r4 = reinterpret_cast<float4 *>(st + (size_t)m * K);
            FOR_K(c, K >> 2) {
                float e[4];
                *reinterpret_cast<float4 *>(e) = r4[c];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int k = 4 * c + j;
                    const double d = b ? __dsub_rn((double)e[j], mean[m]) : (double)e[j];
                    const float t = (float)__dmul_rn(d, rstd[m]);
                    e[j] = b ? __fadd_rn(__fmul_rn(t, gs[k]), bs[k]) : __fmul_rn(t, gs[k]);
                    mx[m] = ec_max_keep(mx[m], fabsf(e[j]));
                }
                r4[c] = *reinterpret_cast<const float4 *>(e);
            }
        }
    } else {
        FOR_TOK(m) {
            const float4 *r4 = reinterpret_cast<const float4 *>(st + (size_t)m * K);
            FOR_K(c, K >> 2) {
                const float4 v = r4[c];
                mx[m] = ec_max_keep(ec_max_keep(ec_max_keep(ec_max_keep(mx[m], fabsf(v.x)), fabsf(v.y)), fabsf(v.z)), fabsf(v.w));
            }
        }
    }
    red_max_f<MM>(p, S, mx, ct, 0);   // its barrier also orders the writes above before the reads below
    int8_t *xq = reinterpret_cast<int8_t *>(S.xbuf);
    FOR_TOK(m) {
        const float s = mx[m] > 0.0f ? __fdiv_rn(mx[m], 127.0f) : 1.0f;
        const float r = __fdiv_rn(1.0f, s);
        if (ct == 0) S.asc[m] = s;
        const float4 *r4 = reinterpret_cast<const float4 *>(st + (size_t)m * K);
        char4 *q4 = reinterpret_cast<char4 *>(xq + (size_t)m * Kp);
        FOR_K(c, Kp >> 2) {
            char4 o = make_char4(0, 0, 0, 0);
            if (4 * c < K) {
                const float4 v = r4[c];
                o = make_char4((signed char)ec_quant_fast(v.x, s, r), (signed char)ec_quant_fast(v.y, s, r),
                               (signed char)ec_quant_fast(v.z, s, r), (signed char)ec_quant_fast(v.w, s, r));
            }
            q4[c] = o;
        }
    }
    cons_sync();
}

// ---------------------------------------------------------------------------
// consumers: one phase's weight tiles -> dots -> epilogue (shared by all
// phases; one copy per weight type and token bound)
// ---------------------------------------------------------------------------

template <int WT> struct AccT { typedef float T; };
template <> struct AccT<EC_W_I8> { typedef int T; };

constexpr int RB = 4;   // weight rows a consumer warp reduces together

// Sum of each of the V = RB*MM per-lane values over the warp, transposed:
// the values are halved between lane pairs at offsets 16, 8, ... (each lane
// keeps one half and adds its partner's copy of that half), so V values take
// V-1 shuffles instead of 5*V; the remaining offsets add duplicates.  Lane L
// ends with the total of value vidx<V>(L); lanes differing only in their low
// log2(32/V) bits hold the same total.  Integer sums are exact; float sums
// are deterministic (every step is a commutative pair sum).
template <int V, typename T>
__device__ __forceinline__ T tr_reduce(T (&a)[V], int lane) {
    static_assert(V >= 1 && V <= 32 && (V & (V - 1)) == 0, "V must be a power of two <= 32");
    int n = V;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        if (n > 1) {
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int v = 0; v < V / 2; ++v) {
                if (v < n / 2) {
                    const T send = up ? a[v] : a[v + n / 2];
                    const T keep = up ? a[v + n / 2] : a[v];
                    a[v] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            n >>= 1;
        } else {
            a[0] = a[0] + __shfl_xor_sync(0xffffffffu, a[0], o);
        }
    }
    return a[0];
}

template <int V>
__device__ __forceinline__ int vidx(int lane) {
    int idx = 0, w = V >> 1;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        if (w >= 1) {
            if (lane & o) idx += w;
            w >>= 1;
        }
    }
    return idx;
}

// Final value of one output row (staged bytes at `row`, metadata tail after
// Kp weights) for token q: reference gemm_int8 epilogue
// bias + ((float)dot * a_scale) * w_scale (src/kernels.c), or dot + bias.
template <int WT>
__device__ __forceinline__ float mk_fin(int Kp, int meta, const Sm &S, const unsigned char *row,
                                        typename AccT<WT>::T d, int q) {
    const float *tail = reinterpret_cast<const float *>(row + (size_t)Kp * (WT == EC_W_I8 ? 1 : 2));
    if (WT == EC_W_I8) {
        const float t = __fmul_rn(__fmul_rn(__int2float_rn((int)d), S.asc[q]), (meta & 1) ? tail[0] : 1.0f);
        return (meta & 2) ? __fadd_rn(tail[1], t) : t;
    } else {
        return (meta & 2) ? __fadd_rn((float)d, tail[1]) : (float)d;
    }
}

// One phase's weight tiles.  Every consumer warp takes whole units (1 row,
// or 2 for pair-packed rows) of each staged tile, RB rows at a time, with the
// lanes splitting K (4 chunks of 16 bytes per lane per round, unrolled); the
// unit -> warp assignment rotates from tile to tile.  A warp reduces its dots
// with tr_reduce and applies the epilogue itself, one lane per (row, token),
// then releases the ring slot: there is no CTA-wide barrier per tile.  After
// an abort the remaining tiles are skipped and the next grid barrier returns
// for every warp.
template <int WT, int MM>
__device__ __noinline__ uint32_t mk_phase(const ec_mk_params &p, int kind, int layer, uint32_t t, int ct) {
    typedef typename AccT<WT>::T Acc;
    constexpr int ELT = WT == EC_W_I8 ? 1 : 2;
    constexpr int V = RB * MM;           // values reduced per group
    constexpr int D = 32 / V;            // lanes holding the same total
    const Sm S = sm_of(p);
    const int nM = p.M;
    const int cta = blockIdx.x;
    // layer: index of the layer (bit 16 set: the down projection of a
    // PK_RESID phase, else its o projection)
    const ec_mk_layer &ly = S.lay[layer & 0xffff];
    const int mi = kind == PK_QKV ? MI_QKV : kind == PK_UP ? MI_UP : (layer & 0x10000) ? MI_DOWN : MI_O;
    const ec_mk_mat &m = mi == MI_QKV ? ly.qkv : mi == MI_UP ? ly.up : mi == MI_DOWN ? ly.down : ly.o;
    const Rg rg = S.rg[mi];
    const int lane = ct & 31, cw = ct >> 5;
    const uint32_t row_bytes = (uint32_t)m.ldw * ELT;
    const int Kp = m.Kp, meta = m.meta, tile_rows = m.tile_rows, mN = m.N;
    const int nch = Kp * ELT / 16;
    const int unit = m.unit, gmax = RB / unit;
    const int half = p.hd >> 1;
    const int my = vidx<V>(lane);               // this lane's (row slot, token) after the reduction
    const int my_i = my / MM, my_q = my % MM;
    const bool my_lane = (lane & (D - 1)) == 0 && my_q < nM && (unit == 1 || (my_i & 1) == 0);
    if (ct == 0) tmark(p, S, 0, EC_TR_PHASE_IN);

    for (int row0 = rg.r0; row0 < rg.r1; row0 += tile_rows) {
        const int nr = min(tile_rows, rg.r1 - row0);
        const int U = nr / unit;
        const int s = (int)(t % STAGES);
        const uint32_t k = t / STAGES;
        ++t;
        if (S.flag[0]) continue;
        bool ok = false;
        for (uint32_t i = 0; i < EC_WAIT_LIMIT; ++i) {
            if (ec_mbar_try_wait(&S.full[s], k & 1)) { ok = true; break; }
            if (S.flag[0]) break;
        }
        if (!ok) {
            S.flag[0] = 1;
            atomicCAS(p.err, 0, ERR_TIMEOUT);
            continue;
        }
        if (ct == 0) tmark(p, S, 0, EC_TR_TILE_IN);
        const unsigned char *stg = S.ring + (size_t)s * TILE;
        const int rot = (unit == 2 ? (row0 - rg.r0) >> 1 : row0 - rg.r0) % NCW;
        for (int u0 = (cw - rot + NCW) % NCW; u0 < U; u0 += NCW * gmax) {
            int rr[RB];   // staged row of slot i, or -1 (warp-uniform)
#pragma unroll
            for (int i = 0; i < RB; ++i) {
                const int ug = u0 + (unit == 2 ? (i >> 1) : i) * NCW;
                rr[i] = ug < U ? ug * unit + (unit == 2 ? (i & 1) : 0) : -1;
            }
            Acc acc[V];
#pragma unroll
            for (int v = 0; v < V; ++v) acc[v] = 0;
            for (int cb = lane; cb < nch; cb += 128) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int c = cb + 32 * j;
                    if (c >= nch) break;
                    if (WT == EC_W_I8) {
                        uint4 w[RB];
#pragma unroll
                        for (int i = 0; i < RB; ++i)
                            if (rr[i] >= 0) w[i] = *reinterpret_cast<const uint4 *>(stg + (size_t)rr[i] * row_bytes + (size_t)c * 16);
                        const int8_t *xq = reinterpret_cast<const int8_t *>(S.xbuf);
                        FOR_TOK(q) {
                            const uint4 x = reinterpret_cast<const uint4 *>(xq + (size_t)q * Kp)[c];
#pragma unroll
                            for (int i = 0; i < RB; ++i) {
                                if (rr[i] < 0) continue;
                                int a = (int)acc[i * MM + q];
                                a = __dp4a((int)w[i].x, (int)x.x, a);
                                a = __dp4a((int)w[i].y, (int)x.y, a);
                                a = __dp4a((int)w[i].z, (int)x.z, a);
                                a = __dp4a((int)w[i].w, (int)x.w, a);
                                acc[i * MM + q] = a;
                            }
                        }
                    } else {
                        float f[RB][8];
#pragma unroll
                        for (int i = 0; i < RB; ++i) {
                            if (rr[i] < 0) continue;
                            const uint4 w = *reinterpret_cast<const uint4 *>(stg + (size_t)rr[i] * row_bytes + (size_t)c * 16);
                            const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                if (WT == EC_W_F16) {
                                    const float2 t2 = __half22float2(*reinterpret_cast<const __half2 *>(&u[e]));
                                    f[i][2 * e] = t2.x;
                                    f[i][2 * e + 1] = t2.y;
                                } else {
                                    f[i][2 * e] = __uint_as_float(u[e] << 16);
                                    f[i][2 * e + 1] = __uint_as_float(u[e] & 0xffff0000u);
                                }
                            }
                        }
                        const float *xs = reinterpret_cast<const float *>(S.xbuf);
                        FOR_TOK(q) {
                            const float *xm = xs + (size_t)q * Kp;
                            const float4 x0 = reinterpret_cast<const float4 *>(xm)[c];
                            const float4 x1 = reinterpret_cast<const float4 *>(xm + (Kp >> 1))[c];
#pragma unroll
                            for (int i = 0; i < RB; ++i) {
                                if (rr[i] < 0) continue;
                                float a = (float)acc[i * MM + q];
                                a = fmaf(f[i][0], x0.x, a); a = fmaf(f[i][1], x0.y, a);
                                a = fmaf(f[i][2], x0.z, a); a = fmaf(f[i][3], x0.w, a);
                                a = fmaf(f[i][4], x1.x, a); a = fmaf(f[i][5], x1.y, a);
                                a = fmaf(f[i][6], x1.z, a); a = fmaf(f[i][7], x1.w, a);
                                acc[i * MM + q] = a;
                            }
                        }
                    }
                }
            }
            const Acc tot = tr_reduce<V>(acc, lane);
            const Acc oth = __shfl_xor_sync(0xffffffffu, tot, 8);   // row slot my_i ^ 1, same token

            // ---- epilogue: one lane per (row slot, token) ----
            const int r0 = my_i == 0 ? rr[0] : my_i == 1 ? rr[1] : my_i == 2 ? rr[2] : rr[3];
            if (!my_lane || my_i >= gmax * unit || r0 < 0) continue;
            const int q = my_q;
            const unsigned char *row = stg + (size_t)r0 * row_bytes;
            const float v0 = mk_fin<WT>(Kp, meta, S, row, tot, q);
            const float v1 = unit == 2 ? mk_fin<WT>(Kp, meta, S, row + row_bytes, oth, q) : 0.0f;
            const int n = row0 + r0;   // matrix row of this lane's slot
            if (kind == PK_QKV) {
                const int pos = S.lpos[q], slot = S.lslot[q];
                const size_t kvo = kv_row_q(p, S, q, slot, pos) * p.kv;
                if (p.arch == ARCH_Q2) {
                    if (n < p.E + p.kv) {   // rotated pair (i, i + hd/2) of a q or k head
                        const int head = n / p.hd, i2 = (n % p.hd) >> 1;
                        const double c = S.rope[(size_t)q * half + i2], sn = S.rope[(size_t)(MT + q) * half + i2];
                        const float lo = (float)__dsub_rn(__dmul_rn((double)v0, c), __dmul_rn((double)v1, sn));
                        const float hi = (float)__dadd_rn(__dmul_rn((double)v0, sn), __dmul_rn((double)v1, c));
                        if (head < p.H) {
                            float *qr = p.q + (size_t)q * p.E + (size_t)head * p.hd;
                            qr[i2] = lo;
                            qr[i2 + half] = hi;
                        } else {
                            uint16_t *kr = ly.kc + kvo + (size_t)(head - p.H) * p.hd;
                            kr[i2] = ec_f2h(lo);
                            kr[i2 + half] = ec_f2h(hi);
                        }
                    } else {
                        const int col = n - p.E - p.kv;
                        ly.vc[kvo + col] = ec_f2h(v0);
                        ly.vc[kvo + col + 1] = ec_f2h(v1);
                    }
                } else {
                    if (n < p.E) p.q[(size_t)q * p.E + n] = v0;
                    else if (n < 2 * p.E) ly.kc[kvo + (n - p.E)] = ec_f2h(v0);
                    else ly.vc[kvo + (n - 2 * p.E)] = ec_f2h(v0);
                }
            } else if (kind == PK_RESID) {   // rows of this CTA's own residual slice
                float *xo = S.xown + (size_t)q * p.own_rows + (n - rg.r0);
                const float v = __fadd_rn(*xo, v0);
                *xo = v;
                p.x[(size_t)q * p.E + n] = v;
            } else if (kind == PK_UP) {
                if (p.arch == ARCH_Q2) p.act[(size_t)q * p.I + (n >> 1)] = __fmul_rn(ec_silu(v0), v1);
                else p.act[(size_t)q * (4 * p.E) + n] = ec_gelu(v0);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[s]);   // this warp no longer reads the slot
        if (ct == 0) tmark(p, S, 0, EC_TR_TILE_DONE);
    }
    return t;
}

// ---------------------------------------------------------------------------
// consumers: the lm_head, streamed straight from HBM into registers
// ---------------------------------------------------------------------------

// The lm_head rows of this CTA (its MI_LM range), 16-bit weights, streamed by
// the consumer warps without the ring: each warp takes groups of R rows
// (groups w, w+8, ...), every lane loads the 16-byte chunks lane, lane+32,
// ... of each row into registers (R*J loads in flight), and the warp sums
// its R*MM dots with one transposed reduction.  The per-row order (lane
// chunks in increasing order, 8 elements each, then the xor tree) is that of
// the standalone GEMV (ec_kernels.cu k_gemv), so the logits are the same bits
// as gemm_fp16_fp32 on the same rows.  Weights are read once per step:
// loaded with the L2 evict-first policy.  Each warp keeps a running argmax
// per token; the CTA's partial goes to amax_v / amax_i.
template <int WT, int MM>
__device__ __noinline__ void mk_lm(const ec_mk_params &p, int ct) {
    // rows per group and chunks per lane per row in flight: R * J = 16 loads
    // of 16 bytes per lane (64 KB per CTA), inside the 168 registers a thread
    // of a 9-warp CTA can have (4 sub-partitions of 16K registers, 3 warps on one)
    constexpr int R = MM >= 8 ? 2 : 4;
    constexpr int J = 4;
    constexpr int V = R * MM;            // values reduced per group (<= 32)
    constexpr int D = 32 / V;            // lanes ending with the same total
    static_assert(WT != EC_W_I8, "the lm_head has 16-bit weights");
    const Sm S = sm_of(p);
    const int nM = p.M;
    const int cta = blockIdx.x;
    const ec_mk_mat &m = p.lm;
    const Rg rg = S.rg[MI_LM];
    const int lane = ct & 31, cw = ct >> 5;
    const size_t row_bytes = (size_t)m.ldw * 2;
    const int Kp = m.Kp, nch = Kp / 8, mN = m.N;
    const int groups = (rg.r1 - rg.r0 + R - 1) / R;
    const uint64_t pol = ec_l2_evict_first();
    const unsigned char *W = static_cast<const unsigned char *>(m.w);
    const float *xs = reinterpret_cast<const float *>(S.xbuf);   // fp32 planes per token (mk_operand)
    const int my = ec_tr_vidx<V>(lane);
    const int my_r = my / MM, my_q = my % MM;
    const bool my_lane = (lane & (D - 1)) == 0 && my_q < nM;
    float bv = -INFINITY;   // running argmax of token my_q
    int bi = 0x7fffffff;
    // L2 prefetch of the row group a warp loads LMPF iterations later: more
    // bytes in flight than the registers of the loads hold
    constexpr int LMPF = 2;
    auto prefetch_group = [&](int gp) {
        if (gp >= groups) return;
        const int rows = min(R, rg.r1 - (rg.r0 + gp * R));
        const unsigned char *base = W + (size_t)(rg.r0 + gp * R) * row_bytes;
        const size_t bytes = (size_t)rows * row_bytes;
        for (size_t o = (size_t)lane * 128; o < bytes; o += 32 * 128)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(base + o));
    };
    for (int i = 1; i < LMPF; ++i) prefetch_group(cw + i * NCW);
    for (int g = cw; g < groups; g += NCW) {
        if (S.flag[0]) break;
        prefetch_group(g + LMPF * NCW);
        const int n0 = rg.r0 + g * R;
        float acc[V];
#pragma unroll
        for (int v = 0; v < V; ++v) acc[v] = 0.0f;
        for (int c0 = 0; c0 < nch; c0 += 32 * J) {
            uint4 w[R][J];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const unsigned char *rowp = W + (size_t)(n0 + r) * row_bytes;
#pragma unroll
                for (int j = 0; j < J; ++j) {
                    const int c = c0 + lane + 32 * j;
                    w[r][j] = (n0 + r < rg.r1 && c < nch) ? ec_ldg_stream16_hint(rowp + (size_t)c * 16, pol)
                                                          : make_uint4(0, 0, 0, 0);
                }
            }
#pragma unroll
            for (int j = 0; j < J; ++j) {
                const int c = c0 + lane + 32 * j;
                if (c >= nch) break;
                float4 x0[MM], x1[MM];
#pragma unroll
                for (int q = 0; q < MM; ++q) {
                    if (q >= nM) break;
                    const float *xm = xs + (size_t)q * Kp;
                    x0[q] = reinterpret_cast<const float4 *>(xm)[c];
                    x1[q] = reinterpret_cast<const float4 *>(xm + (Kp >> 1))[c];
                }
#pragma unroll
                for (int r = 0; r < R; ++r) {
#pragma unroll
                    for (int q = 0; q < MM; ++q) {
                        if (q >= nM) break;
                        acc[r * MM + q] = ec_dot8<WT == EC_W_BF16>(w[r][j], x0[q], x1[q], acc[r * MM + q]);
                    }
                }
            }
        }
        const float tot = ec_tr_reduce<V>(acc, lane);
        const int n = n0 + my_r;
        if (my_lane && n < rg.r1) {
            if (p.logits) p.logits[(size_t)my_q * mN + n] = tot;
            am_merge(bv, bi, tot, p.v0 + n);
        }
    }
    // lanes holding the same token: every xor offset except the token bits [D, D*MM)
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        if (o >= D && o < D * MM) continue;
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        am_merge(bv, bi, ov, oi);
    }
    cons_sync();
    if (my_r == 0 && (lane & (D - 1)) == 0) { S.redf[cw * MT + my_q] = bv; S.redi[cw * MT + my_q] = bi; }
    cons_sync();
    if (ct < nM) {
        float v = S.redf[ct];
        int i = S.redi[ct];
        for (int w = 1; w < NCW; ++w) am_merge(v, i, S.redf[w * MT + ct], S.redi[w * MT + ct]);
        p.amax_v[(size_t)cta * MT + ct] = v;
        p.amax_i[(size_t)cta * MT + ct] = i;
    }
}

// ---------------------------------------------------------------------------
// consumers: attention items (token m, head h), exact reference order
// ---------------------------------------------------------------------------

template <int MM>
__device__ __noinline__ void mk_attention(const ec_mk_params &p, int layer, int ct) {
    const Sm S = sm_of(p);
    const int nM = p.M;
    const ec_mk_layer &ly = S.lay[layer];
    const int G = gridDim.x, cta = blockIdx.x;
    const int hd = p.hd, kv = p.kv, H = p.H, E = p.E, CH = p.kvchunk;
    const int ks = hd + 8;      // padded K row stride (halves): per-position reads avoid bank conflicts
    const int per = hd >> 3;    // 16-byte pieces per cached row
    float *qs = reinterpret_cast<float *>(S.xbuf);
    float *sc = qs + ((hd + 3) & ~3);
    uint16_t *kch = reinterpret_cast<uint16_t *>(sc + ((p.maxlen + 3) & ~3));
    uint16_t *vch = kch + (size_t)CH * ks;
    const uint16_t *kc = ly.kc, *vc = ly.vc;
    const double inv_hd = 1.0 / sqrt((double)hd);
    for (int it = cta; it < nM * H; it += G) {
        const int m = it / H, h = it % H;
        const int kvh = h * p.KVH / H;
        const int pos = S.lpos[m], slot = S.lslot[m];
        int lo = 0;
        if (p.window > 0) { lo = pos - p.window + 1; if (lo < 0) lo = 0; }
        const int len = pos + 1 - lo;
        if (len > p.maxlen) {
            if (ct == 0) atomicCAS(p.err, 0, ERR_INDEX);
            continue;
        }
        // cached row of position lo + i: its page, then the row in the page
        const uint16_t *kb = kc + (size_t)kvh * hd, *vb = vc + (size_t)kvh * hd;
        // the q row and the first K and V chunks in flight together
        for (int d = ct; d < (hd >> 2); d += NCT) cpa16(qs + 4 * d, p.q + (size_t)m * E + (size_t)h * hd + 4 * d);
        {
            const int n0 = min(CH, len);
            for (int e = ct; e < n0 * per; e += NCT) {
                const int i = e / per, j = e - (e / per) * per;
                const size_t r = kv_row_q(p, S, m, slot, lo + i) * kv;
                cpa16(kch + (size_t)i * ks + 8 * j, kb + r + 8 * j);
                cpa16(vch + (size_t)i * hd + 8 * j, vb + r + 8 * j);
            }
        }
        cpa_wait_all();
        cons_sync();
        if (ct == 0) tmark(p, S, 0, EC_TR_STAGED);
        // scores: sequential fp32 dot per position, scaled in double
        float mx = -FLT_MAX;
        for (int c0 = 0; c0 < len; c0 += CH) {
            const int n = min(CH, len - c0);
            if (c0 > 0) {
                cons_sync();   // previous K chunk consumed
                for (int e = ct; e < n * per; e += NCT) {
                    const int i = e / per, j = e - (e / per) * per;
                    cpa16(kch + (size_t)i * ks + 8 * j, kb + kv_row_q(p, S, m, slot, lo + c0 + i) * kv + 8 * j);
                }
                cpa_wait_all();
                cons_sync();
            }
            for (int i = ct; i < n; i += NCT) {
                const uint16_t *kp = kch + (size_t)i * ks;
                float a = 0.0f;
#pragma unroll 4
                for (int d = 0; d < hd; d += 8) {
                    const uint4 w = *reinterpret_cast<const uint4 *>(kp + d);
                    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&u[j]));
                        a = __fadd_rn(a, __fmul_rn(qs[d + 2 * j], f.x));
                        a = __fadd_rn(a, __fmul_rn(qs[d + 2 * j + 1], f.y));
                    }
                }
                const float sv = (float)__dmul_rn((double)a, inv_hd);
                sc[c0 + i] = sv;
                mx = ec_max_keep(mx, sv);
            }
        }
        {
            const int lane = ct & 31, w = ct >> 5;
            mx = ec_warp_max(mx);
            if (lane == 0) S.redf[w * MT] = mx;
            cons_sync();
            float t = S.redf[0];
            for (int i = 1; i < NCW; ++i) t = ec_max_keep(t, S.redf[i * MT]);
            mx = t;
        }
        if (ct == 0) tmark(p, S, 0, EC_TR_SCORES);
        double sum = 0.0;
        for (int i = ct; i < len; i += NCT) {
            const float e = ec_expf(__fsub_rn(sc[i], mx));
            sc[i] = e;
            sum = __dadd_rn(sum, (double)e);
        }
        {
            const int lane = ct & 31, w = ct >> 5;
            sum = ec_warp_sum_d(sum);
            if (lane == 0) S.redd[w * MT] = sum;
            cons_sync();
            double t = 0.0;
            for (int i = 0; i < NCW; ++i) t = __dadd_rn(t, S.redd[i * MT]);
            sum = t;
        }
        const double isum = __ddiv_rn(1.0, sum);
        for (int i = ct; i < len; i += NCT) sc[i] = (float)__dmul_rn((double)sc[i], isum);
        cons_sync();
        if (ct == 0) tmark(p, S, 0, EC_TR_SOFTMAX);
        // P.V: sequential over positions for each output dimension
        float o = 0.0f;
        for (int c0 = 0; c0 < len; c0 += CH) {
            const int n = min(CH, len - c0);
            if (c0 > 0) {
                cons_sync();   // previous V chunk consumed
                for (int e = ct; e < n * per; e += NCT) {
                    const int i = e / per, j = e - (e / per) * per;
                    cpa16(vch + (size_t)i * hd + 8 * j, vb + kv_row_q(p, S, m, slot, lo + c0 + i) * kv + 8 * j);
                }
                cpa_wait_all();
                cons_sync();
            }
            if (ct < hd) {
                // products are independent; only the sum runs in position order
                int i = 0;
                for (; i + 8 <= n; i += 8) {
                    float pr[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        pr[j] = __fmul_rn(sc[c0 + i + j], __half2float(__ushort_as_half(vch[(size_t)(i + j) * hd + ct])));
#pragma unroll
                    for (int j = 0; j < 8; ++j) o = __fadd_rn(o, pr[j]);
                }
                for (; i < n; ++i)
                    o = __fadd_rn(o, __fmul_rn(sc[c0 + i], __half2float(__ushort_as_half(vch[(size_t)i * hd + ct]))));
            }
        }
        if (ct < hd) p.att[(size_t)m * E + (size_t)h * hd + ct] = o;
        cons_sync();
    }
}

// ---------------------------------------------------------------------------
// grid barrier among the consumers of all CTAs
// ---------------------------------------------------------------------------

__device__ __noinline__ bool mk_grid_sync(const ec_mk_params &p, unsigned target, int ct) {
    const Sm S = sm_of(p);
    if (cons_sync_or(S.flag[0] != 0)) {
        if (ct == 0) atomicExch(p.abort_flag, 1);
        return false;
    }
    if (ct == 0) {
        // arrive with release semantics: the CTA barrier above put every
        // warp's writes of this phase before this add (release is cumulative)
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar) : "memory");
        const long long t0 = clock64();
        for (unsigned it = 1;; ++it) {
            if (ld_acquire(p.bar) >= target) break;
            if ((it & 15u) != 0) continue;   // the abort flag and the clock: every 16th poll
            if (ld_relaxed_i(p.abort_flag)) { S.flag[0] = 1; break; }
            if (clock64() - t0 > SPIN_CYCLES) {
                S.flag[0] = 1;
                atomicCAS(p.err, 0, ERR_TIMEOUT);
                break;
            }
        }
        // no fence here: the acquire load that saw the count orders this
        // thread's later reads, and the CTA barrier below passes that order on
    }
    const bool stop = cons_sync_or(S.flag[0] != 0);
    if (stop && ct == 0) atomicExch(p.abort_flag, 1);
    return !stop;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

// Residual rows owned by this CTA after layer `slot - 1` -> taps[slot] (debug
// capture; out of line, off the hot path).
__device__ __noinline__ void mk_taps(const ec_mk_params &p, int slot, int ct) {
    const Sm S = sm_of(p);
    const Rg xr = S.rg[MI_O];
    const int xn = xr.r1 - xr.r0, M = p.M;
    for (int idx = ct; idx < xn * M; idx += NCT) {
        const int q = idx / xn, n = xr.r0 + idx % xn;
        p.taps[((size_t)slot * M + q) * p.E + n] = S.xown[(size_t)q * p.own_rows + (n - xr.r0)];
    }
}

template <int LWT, int HWT, int MM>
__global__ void __launch_bounds__(EC_MK_THREADS, 1) k_decode(const __grid_constant__ ec_mk_params pg, int n_steps) {
    const Lay L = mk_layout(pg.xbuf_bytes, pg.stage_bytes, pg.L, pg.E, pg.hd, pg.own_rows);
    const Sm S = sm_of(pg);
    const int G = gridDim.x, cta = blockIdx.x;
    const int M = pg.M;
    {   // parameters -> shared memory: the helpers below read them through a
        // reference, which for kernel-parameter space would be a slow generic load
        uint32_t *dst = reinterpret_cast<uint32_t *>(S.par);
        const uint32_t *src = reinterpret_cast<const uint32_t *>(&pg);
        for (int i = threadIdx.x; i < (int)(sizeof(ec_mk_params) / 4); i += blockDim.x) dst[i] = src[i];
    }
    const ec_mk_params &p = *S.par;
    const int nM = M;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ec_mbar_init(&S.full[s], 1);
            ec_mbar_init(&S.empty[s], NCW);
        }
        ec_fence_mbar_init();
        S.flag[0] = 0;
        S.tcount[0] = S.tcount[1] = 0;
        // the paired counter is unused by this launch; the next one starts on it
        if (cta == 0 && pg.bar_next) *pg.bar_next = 0u;
    }
    if (threadIdx.x < M) {
        S.ltok[threadIdx.x] = pg.inline_in ? pg.in_tok[threadIdx.x] : pg.tok[threadIdx.x];
        S.lpos[threadIdx.x] = pg.inline_in ? pg.in_pos[threadIdx.x] : pg.pos[threadIdx.x];
        S.lslot[threadIdx.x] = pg.inline_in ? pg.in_slot[threadIdx.x] : pg.slot[threadIdx.x];
    }
    {   // layer descriptors -> shared memory (read on every phase and tile)
        uint32_t *dst = reinterpret_cast<uint32_t *>(g_smem + L.lays);
        const uint32_t *src = reinterpret_cast<const uint32_t *>(pg.layers);
        const int words = (int)((size_t)pg.L * sizeof(ec_mk_layer) / 4);
        for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
    if (pg.mp <= PT_SMEM) {   // page-table rows of the rows' slots (slots are fixed for the launch)
        for (int i = threadIdx.x; i < M * pg.mp; i += blockDim.x) {
            const int q = i / pg.mp, jj = i - q * pg.mp;
            S.lpt[q * PT_SMEM + jj] = pg.pt[(size_t)S.lslot[q] * pg.mp + jj];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {   // row ranges: every layer has the same shapes
        S.rg[MI_QKV] = mk_range(S.lay[0].qkv, cta, G);
        S.rg[MI_O] = mk_range(S.lay[0].o, cta, G);
        S.rg[MI_UP] = mk_range(S.lay[0].up, cta, G);
        S.rg[MI_DOWN] = mk_range(S.lay[0].down, cta, G);
        S.rg[MI_LM] = mk_range(p.lm, cta, G);
    }
    __syncthreads();
    // Inputs are checked identically by every CTA before any work, so a bad
    // token / position / slot makes the whole grid return together.
    for (int q = 0; q < M; ++q) {
        const int tk = S.ltok[q], ps = S.lpos[q], sl = S.lslot[q];
        if (tk < 0 || tk >= p.V || ps < 0 || ps >= p.C || sl < 0 || sl >= p.B) {
            if (threadIdx.x == 0 && cta == 0) atomicCAS(p.err, 0, ERR_INDEX);
            return;
        }
    }

    if (threadIdx.x < 32) {
        // ---------------- producer ----------------
        if (threadIdx.x == 0) {
            uint32_t t = 0;
            for (int step = 0; t != T_ABORT && step < n_steps; ++step) {
                for (int l = 0; t != T_ABORT && l < p.L; ++l) {
                    const ec_mk_layer &ly = S.lay[l];
                    t = mk_produce(p, ly.qkv, LWT, S.rg[MI_QKV], t);
                    if (t != T_ABORT) t = mk_produce(p, ly.o, LWT, S.rg[MI_O], t);
                    if (t != T_ABORT) t = mk_produce(p, ly.up, LWT, S.rg[MI_UP], t);
                    if (t != T_ABORT) t = mk_produce(p, ly.down, LWT, S.rg[MI_DOWN], t);
                }
                // the lm_head is streamed by the consumers themselves (mk_lm);
                // meanwhile this loop already fills the ring for the next step
            }
            if (t == T_ABORT) {
                // give the copies already issued a bounded time to land
                for (int s = 0; s < STAGES; ++s)
                    for (uint32_t i = 0; i < (1u << 20); ++i)
                        if (ec_mbar_try_wait(&S.full[s], 0) || ec_mbar_try_wait(&S.full[s], 1)) break;
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const int ct = threadIdx.x - 32;
    uint32_t t = 0;
    unsigned target = 0;
    // int8 layers: the single-pass operand builder (its inputs must fit the staging area)
    // (4-8 rows: mk_prep_rows stages the down-projection input one row at a time)
    const bool I8P = LWT == EC_W_I8 &&
                     (size_t)(MM >= 4 ? 1 : M) * (size_t)S.lay[0].down.K * 4 <= (size_t)p.stage_bytes &&
                     (size_t)M * (size_t)p.E * 4 <= (size_t)p.stage_bytes && (p.E & 3) == 0 && (S.lay[0].down.K & 3) == 0;
    const Rg xr = S.rg[MI_O];   // residual rows owned by this CTA
    const int xn = xr.r1 - xr.r0;
#define SYNC_OR_RETURN()                                  \
    do {                                                  \
        target += (unsigned)G;                            \
        if (!mk_grid_sync(p, target, ct)) return;         \
        if (ct == 0) tmark(p, S, 0, EC_TR_SYNC);          \
    } while (0)
    for (int step = 0; step < n_steps; ++step) {
        // this step's RoPE rows, in flight while the embedding and the first
        // norm run (the norm's cp.async wait completes them)
        if (p.rope_cos) {
            const int half = p.hd >> 1, pairs = half >> 1;   // 16-byte pieces of one row
            for (int idx = ct; idx < 2 * M * pairs; idx += NCT) {
                const int tab = idx / (M * pairs), rem = idx % (M * pairs), q = rem / pairs, j = rem % pairs;
                const double *src = (tab ? p.rope_sin : p.rope_cos) + (size_t)S.lpos[q] * half + 2 * j;
                cpa16(S.rope + (size_t)(tab * MT + q) * half + 2 * j, src);
            }
        }
        // residual rows := embedding (reference src/gpt2.c:488-499, :690-700)
        for (int idx = ct; idx < xn * M; idx += NCT) {
            const int q = idx / xn, n = xr.r0 + idx % xn;
            const float e = mk_embed(p, S.ltok[q], S.lpos[q], n);
            S.xown[(size_t)q * p.own_rows + (n - xr.r0)] = e;
            p.x[(size_t)q * p.E + n] = e;
            if (p.taps) p.taps[(size_t)q * p.E + n] = e;
        }
        for (int l = 0; l < p.L; ++l) {
            const ec_mk_layer &ly = S.lay[l];
            // A: norm -> q|k|v
            if (l > 0) SYNC_OR_RETURN();
            if (I8P) mk_prep<MM>(p, p.x, p.E, ly.qkv.Kp, l == 0, ly.n1g, ly.n1b, ct);
            else { mk_norm<MM>(p, l == 0, ly.n1g, ly.n1b, ct); mk_operand<MM>(p, nullptr, p.E, ly.qkv.Kp, LWT, ct); }
            if (ct == 0) tmark(p, S, 0, EC_TR_PROLOGUE);
            t = mk_phase<LWT, MM>(p, PK_QKV, l, t, ct);
            if (ct == 0) tmark(p, S, 0, EC_TR_TILES);
            // B: attention
            SYNC_OR_RETURN();
            mk_attention<MM>(p, l, ct);
            if (ct == 0) tmark(p, S, 0, EC_TR_ATTN);
            // C: o + residual
            SYNC_OR_RETURN();
            if (I8P) mk_prep<MM>(p, p.att, p.E, ly.o.Kp, false, nullptr, nullptr, ct);
            else mk_operand<MM>(p, p.att, p.E, ly.o.Kp, LWT, ct);
            if (ct == 0) tmark(p, S, 0, EC_TR_PROLOGUE);
            t = mk_phase<LWT, MM>(p, PK_RESID, l, t, ct);
            if (ct == 0) tmark(p, S, 0, EC_TR_TILES);
            // D: norm -> gate|up / fc
            SYNC_OR_RETURN();
            if (I8P) mk_prep<MM>(p, p.x, p.E, ly.up.Kp, false, ly.n2g, ly.n2b, ct);
            else { mk_norm<MM>(p, false, ly.n2g, ly.n2b, ct); mk_operand<MM>(p, nullptr, p.E, ly.up.Kp, LWT, ct); }
            if (ct == 0) tmark(p, S, 0, EC_TR_PROLOGUE);
            t = mk_phase<LWT, MM>(p, PK_UP, l, t, ct);
            if (ct == 0) tmark(p, S, 0, EC_TR_TILES);
            // E: down / fc2 + residual
            SYNC_OR_RETURN();
            if (I8P) mk_prep<MM>(p, p.act, ly.down.K, ly.down.Kp, false, nullptr, nullptr, ct);
            else mk_operand<MM>(p, p.act, ly.down.K, ly.down.Kp, LWT, ct);
            if (ct == 0) tmark(p, S, 0, EC_TR_PROLOGUE);
            t = mk_phase<LWT, MM>(p, PK_RESID, l | 0x10000, t, ct);
            if (ct == 0) tmark(p, S, 0, EC_TR_TILES);
            if (p.taps) mk_taps(p, l + 1, ct);
        }
        // F: final norm -> lm_head (per-CTA argmax partial written inside)
        SYNC_OR_RETURN();
        mk_norm<MM>(p, false, p.nfg, p.nfb, ct);
        mk_operand<MM>(p, nullptr, p.E, p.lm.Kp, HWT, ct);
        if (ct == 0) tmark(p, S, 0, EC_TR_PROLOGUE);
        mk_lm<HWT, MM>(p, ct);
        if (ct == 0) tmark(p, S, 0, EC_TR_LM);
        // G: merge the per-CTA partials (CTA order, lowest index on ties)
        SYNC_OR_RETURN();
        float bv[MM];
        int bi[MM];
#pragma unroll
        for (int q = 0; q < MM; ++q) { bv[q] = -INFINITY; bi[q] = 0x7fffffff; }
        for (int c = ct; c < G; c += NCT)
            FOR_TOK(q) am_merge(bv[q], bi[q], __ldcg(p.amax_v + (size_t)c * MT + q), __ldcg(p.amax_i + (size_t)c * MT + q));
        red_argmax<MM>(p, S, bv, bi, ct);
        if (ct == 0) tmark(p, S, 0, EC_TR_ARGMAX);
        FOR_TOK(q) if (ct == q) {
            const int id = bi[q] == 0x7fffffff ? 0 : bi[q];
            if (cta == 0) {
                if (p.ids) p.ids[q] = id;
                if (p.maxv) p.maxv[q] = bv[q];
                if (p.hist) p.hist[(size_t)step * M + q] = id;
            }
            if (p.advance) {
                S.ltok[q] = id;
                const int np = S.lpos[q] + 1;
                S.lpos[q] = (p.wrap_hi > 0 && np >= p.wrap_hi) ? p.wrap_lo : np;
                if (cta == 0) { p.tok[q] = S.ltok[q]; p.pos[q] = S.lpos[q]; }
            }
        }
        cons_sync();
    }
    // clean end: errors recorded by any CTA before the last grid barrier
    // are visible here through that barrier's acquire
    if (p.done && cta == 0 && ct == 0) *(volatile int *)p.done = ld_relaxed_i(p.err) ? -1 : p.seq;
#undef SYNC_OR_RETURN
}

template <int LWT, int HWT, int MM>
int mk_launch_t(const ec_mk_params *p, int n_steps, int grid, cudaStream_t stream) {
    const Lay L = mk_layout(p->xbuf_bytes, p->stage_bytes, p->L, p->E, p->hd, p->own_rows);
    // the shared-memory opt-in is per device: raise it only when it grows
    static std::atomic<int> opted[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || opted[dev].load(std::memory_order_relaxed) < (int)L.total) {
        cudaError_t e = cudaFuncSetAttribute(k_decode<LWT, HWT, MM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)L.total);
        if (e != cudaSuccess) return (int)e;
        if (dev >= 0 && dev < 64) opted[dev].store((int)L.total, std::memory_order_relaxed);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(EC_MK_THREADS);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return (int)cudaLaunchKernelEx(&cfg, k_decode<LWT, HWT, MM>, *p, n_steps);
}

template <int LWT, int HWT>
int mk_launch_m(const ec_mk_params *p, int n_steps, int grid, cudaStream_t stream) {
    if (p->M <= 1) return mk_launch_t<LWT, HWT, 1>(p, n_steps, grid, stream);
    if (p->M <= 2) return mk_launch_t<LWT, HWT, 2>(p, n_steps, grid, stream);
    if (p->M <= 4) return mk_launch_t<LWT, HWT, 4>(p, n_steps, grid, stream);
    return mk_launch_t<LWT, HWT, 8>(p, n_steps, grid, stream);
}

}  // namespace

extern "C" int ec_mk_traced(void) {
#ifdef EC_DECODE_TRACE
    return 1;
#else
    return 0;
#endif
}

extern "C" size_t ec_mk_smem_bytes(const ec_mk_params *p) {
    return mk_layout(p->xbuf_bytes, p->stage_bytes, p->L, p->E, p->hd, p->own_rows).total;
}

extern "C" int ec_mk_smem_limit(void) {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    return v;
}

extern "C" int ec_mk_launch(const ec_mk_params *p, int n_steps, int grid, cudaStream_t stream) {
    if (p->M < 1 || p->M > EC_MK_MT || n_steps < 1 || grid < 1) return (int)cudaErrorInvalidValue;
    if (p->lwt == EC_W_I8 && p->hwt == EC_W_F16) return mk_launch_m<EC_W_I8, EC_W_F16>(p, n_steps, grid, stream);
    if (p->lwt == EC_W_F16 && p->hwt == EC_W_F16) return mk_launch_m<EC_W_F16, EC_W_F16>(p, n_steps, grid, stream);
    if (p->lwt == EC_W_BF16 && p->hwt == EC_W_BF16) return mk_launch_m<EC_W_BF16, EC_W_BF16>(p, n_steps, grid, stream);
    return (int)cudaErrorInvalidValue;
}
