// ec_tc.cu -- GEMMs on the 5th-generation tensor cores (tcgen05) for M >= EC_TC_MIN_M (8)
// rows (prefill, batched decode):
//
//   int8 weights (kind::i8):
//     out[m][n] = epi( bias[n] + ((float)(sum_k Aq[m][k] * W[n][k]) * a_scale[m]) * w_scale[n] )
//   Aq int8 [M][Kp] = the quantised activations; int32 accumulation in tensor
//   memory.  Products and sums are exact integers, so the result is
//   bit-identical to the reference gemm_int8 (src/kernels.c:153-168).
//
//   fp16 / bf16 weights (kind::f16):
//     out[m][n] = epi( (sum_k X[m][k] * W[n][k]) (+ bias[n]) )
//   with X fp32.  An MMA needs A and B of the same 16-bit type, so a pre-pass
//   (k_split16) writes each activation row as S 16-bit parts whose sum is the
//   fp32 value: fp16 weights -> hi + lo fp16 of the row scaled by an exact
//   power of two (max |x| in [2^13, 2^14)), ~2^-22 relative; bf16 weights ->
//   three bf16 parts, ~2^-27.  Every part is one more MMA against the same W
//   tile; fp32 accumulation; the epilogue multiplies the power of two back
//   exactly.  The result differs from the reference's fp32 dot (8-lane AVX2
//   order, src/kernels.c:29-64) only by summation order, like the SIMT path.
//
// Persistent CTAs (one per SM) walk 128 x BN output tiles over K in 128-byte
// stages:
//   warp 0     TMA producer: the A part boxes [128][128 B] and the W box
//              [BN][128 B] with the 128-byte swizzle into a ring that runs
//              across tiles
//   warp 1     allocates 2 x BN TMEM columns = two accumulators; one thread
//              issues the MMAs of a tile into the free accumulator and
//              commits stages back to the producer, the accumulator to the
//              epilogue
//   warps 2-9  epilogue of the other accumulator meanwhile: tcgen05.ld (warp
//              w reads TMEM lanes 32*(w%4)..+31 = tile rows; warps w and w+4
//              split the columns), scale and bias per element, transpose
//              through shared memory, coalesced 16-byte stores (store,
//              residual add or GELU)
// int8 GEMMs whose output has few tiles (decode-sized M) split K over
// `ksplit` CTAs per tile: each adds its int32 partial tile into a zeroed
// int32 workspace with atomics (integer sums: exact, in any order), and the
// CTA that finishes a tile last (a per-tile counter) applies the epilogue to
// the total and zeroes the workspace and the counter again.
// Loads never use cluster multicast; every wait is bounded and TMEM is freed
// on every path.
#include "ec_common.cuh"
#include "ec_launch.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <pthread.h>
#include <string.h>

namespace {

constexpr int BM = 128, BKB = 128;                     // tile rows, K bytes per stage
constexpr int THREADS = 320;                           // producer, MMA, 8 epilogue warps
constexpr int EPI_WARPS = 8, EPI_COLS = 16;           // two warps per TMEM lane group, 16-column chunks
constexpr int EPI_LD = 20;                             // staging row stride (floats): 16-byte rows, no bank conflicts
constexpr int EPI_BYTES = EPI_WARPS * 32 * EPI_LD * 4;
constexpr int A_BYTES = BM * BKB;                      // one A part per stage: 16 KB

// Per configuration (the weight type, and for int8 a narrow variant): weight
// type, A parts, tile columns, ring depth, instruction descriptor.
// Instruction descriptor fields: [4,6) D format (1 f32, 2 s32), [7,10) A and
// [10,13) B format (i8: 1 = signed; f16 kind: 0 = f16, 1 = bf16), bits 15/16
// K-major (0), [17,23) N >> 3, [24,29) M >> 4.
constexpr int TC_I8_NARROW = 3;   // int8 with 64-column tiles: 4x the CTAs for one row of tiles
template <int CF> struct TcCfg;
template <> struct TcCfg<EC_W_I8> {
    static constexpr int WT = EC_W_I8, S = 1, BN = 256, STAGES = 4, ELT = 1;
    static constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
};
template <> struct TcCfg<EC_W_F16> {
    static constexpr int WT = EC_W_F16, S = 2, BN = 256, STAGES = 3, ELT = 2;
    static constexpr uint32_t IDESC = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
};
template <> struct TcCfg<EC_W_BF16> {
    static constexpr int WT = EC_W_BF16, S = 3, BN = 128, STAGES = 3, ELT = 2;
    static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
};
template <> struct TcCfg<TC_I8_NARROW> {
    static constexpr int WT = EC_W_I8, S = 1, BN = 64, STAGES = 8, ELT = 1;
    static constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
};

template <int CF> __host__ __device__ constexpr int b_bytes() { return TcCfg<CF>::BN * BKB; }
template <int CF> __host__ __device__ constexpr int stage_bytes() { return TcCfg<CF>::S * A_BYTES + b_bytes<CF>(); }
template <int CF> __host__ __device__ constexpr int cst_bytes() { return EPI_WARPS * 2 * (TcCfg<CF>::BN / 2) * 4; }
template <int CF> __host__ __device__ constexpr int smem_bytes() {
    return 1024 /* alignment slack */ + TcCfg<CF>::STAGES * stage_bytes<CF>() + EPI_BYTES + cst_bytes<CF>() + 256;
}
static_assert(smem_bytes<EC_W_I8>() <= 232448 && smem_bytes<EC_W_F16>() <= 232448 && smem_bytes<EC_W_BF16>() <= 232448 &&
              smem_bytes<TC_I8_NARROW>() <= 232448, "shared memory per CTA");

__device__ int g_tc_err;

// Shared-memory matrix descriptor of a K-major tile stored as 128-byte rows
// with the 128-byte swizzle (8-row atoms of 1024 bytes): start >> 4,
// leading byte offset 1 (unused for swizzled K-major), stride byte offset
// 1024 >> 4, descriptor version 1, swizzle mode 2 (128 B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(map), "r"(bar), "r"(x), "r"(y) : "memory");
}

template <int CF>
__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    if (TcCfg<CF>::WT == EC_W_I8)
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
            ::"r"(tmem_d), "l"(da), "l"(db), "r"(TcCfg<CF>::IDESC), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
            ::"r"(tmem_d), "l"(da), "l"(db), "r"(TcCfg<CF>::IDESC), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float epi_apply(int epi, float o, float v) {
    return epi == EC_EPI_RESID ? __fadd_rn(o, v) : epi == EC_EPI_GELU ? ec_gelu(v) : v;
}

// Bounded wait on an mbarrier phase; false (and the error word set) if it
// never completes or another role has already given up.
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *stop) {
    for (uint32_t i = 0; i < EC_WAIT_LIMIT; ++i) {
        if (ec_mbar_try_wait(bar, parity)) return true;
        if (*stop) return false;
    }
    *stop = 1;
    atomicCAS(&g_tc_err, 0, EC_KERR_WAIT_TIMEOUT);
    return false;
}

struct TcMaps {
    CUtensorMap a[3];   // A parts (one for int8)
    CUtensorMap b;      // weights
};

// AND of `v` over the 256 epilogue threads (named barrier 1): every
// epilogue warp takes the same decision, so that none of them waits at a
// later named barrier for a warp that has left.
__device__ __forceinline__ bool epi_all(bool v) {
    int r;
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.s32 p, %1, 0;\n\tbar.red.and.pred p, 1, 256, p;\n\t"
                 "selp.s32 %0, 1, 0, p;\n\t}" : "=r"(r) : "r"((int)v) : "memory");
    return r != 0;
}

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Split-K, part 1: this warp's rows (TMEM lane group lg) and column half ch
// of the int32 partial tile at `taddr`, transposed through `st`, added into
// a.acc32 [M][N] with coalesced atomics.
template <int BN>
__device__ __forceinline__ void split_tile_add(const ec_gemm_args &a, uint32_t taddr, int m0, int n0, int lg, int ch,
                                               int lane, float *st) {
    constexpr int HALF = BN / 2;
    int *sti = reinterpret_cast<int *>(st);
    for (int c0 = ch * HALF; c0 < (ch + 1) * HALF && n0 + c0 < a.N; c0 += EPI_COLS) {
        uint32_t r[16];
        tmem_ld16(taddr + (uint32_t)c0, r);
#pragma unroll
        for (int j = 0; j < EPI_COLS; j += 4)
            *reinterpret_cast<int4 *>(sti + lane * EPI_LD + j) = make_int4((int)r[j], (int)r[j + 1], (int)r[j + 2], (int)r[j + 3]);
        __syncwarp();
#pragma unroll
        for (int pass = 0; pass < 4; ++pass) {
            const int row = pass * 8 + (lane >> 2), c4 = (lane & 3) * 4;
            const int m = m0 + lg * 32 + row, n = n0 + c0 + c4;
            if (m >= a.M) continue;
            int *dst = a.acc32 + (size_t)m * a.N + n;
            for (int e = 0; e < 4 && n + e < a.N; ++e)
                asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(dst + e), "r"(sti[row * EPI_LD + c4 + e]) : "memory");
        }
        __syncwarp();
    }
    __threadfence();   // this thread's additions before the tile counter below
}

// Split-K, part 2 (all 256 epilogue threads, et = 0..255): count this CTA's
// part of the tile; the CTA that completes it applies the int8 epilogue of
// the non-split path to the int32 totals, bit for bit, and zeroes the
// workspace and the counter for the next call.
__device__ __forceinline__ void split_tile_finish(const ec_gemm_args &a, const float *row_scale, int tile, int m0,
                                                  int n0, int bn, int ksplit, volatile int *flag_last, int et) {
    epi_sync();
    if (et == 0) *flag_last = atomicAdd(a.tile_cnt + tile, 1u) == (unsigned)(ksplit - 1);
    epi_sync();
    if (!*flag_last) return;
    __threadfence();
    // thread et: column et % bn of the tile, rows et / bn, + 256 / bn, ...;
    // eight rows' loads in flight per thread
    const int rows = min(BM, a.M - m0);
    const int c = et % bn, r0 = et / bn, rstep = 256 / bn, n = n0 + c;
    if (n < a.N) {
        const float ws = a.wscale ? __ldg(a.wscale + n) : 1.0f;
        const float bs = a.bias ? __ldg(a.bias + n) : 0.0f;
        for (int rb = r0; rb < rows; rb += 8 * rstep) {
            int acc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = rb + i * rstep;
                acc[i] = r < rows ? __ldcg(a.acc32 + (size_t)(m0 + r) * a.N + n) : 0;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = rb + i * rstep;
                if (r >= rows) break;
                const int m = m0 + r;
                __stcg(a.acc32 + (size_t)m * a.N + n, 0);
                const float v = __fadd_rn(bs, __fmul_rn(__fmul_rn(__int2float_rn(acc[i]), __ldg(row_scale + m)), ws));
                float *o = a.out + (size_t)m * a.ldo + n;
                *o = epi_apply(a.epi, a.epi == EC_EPI_RESID ? *o : 0.0f, v);
            }
        }
    }
    epi_sync();
    if (et == 0) a.tile_cnt[tile] = 0u;
}

// row_scale: a_scale (int8) or the power-of-two row scale of the split (16-bit)
template <int CF>
__global__ void __launch_bounds__(THREADS, 1)
k_gemm_tc(const __grid_constant__ TcMaps maps, const ec_gemm_args a, const float *row_scale,
          int flags,     // bit 0: 16-byte aligned output rows
          int ksplit) {  // CTAs per output tile over K (int8 only; 1: no split)
    constexpr int WT = TcCfg<CF>::WT;
    constexpr int S = TcCfg<CF>::S, BN = TcCfg<CF>::BN, STAGES = TcCfg<CF>::STAGES;
    constexpr int SB = stage_bytes<CF>();
    constexpr int KSTEP = 32;                                      // bytes of K per MMA instruction (both kinds)
    constexpr int TMEM_COLS = 2 * BN;                              // two accumulators
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = ec_smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;                  // 1024-byte aligned (128-byte swizzle atoms)
    unsigned char *gbase = smem_raw + (base - raw);
    // stage s: A parts at base + s*SB + p*A_BYTES, W at base + s*SB + S*A_BYTES
    float *stage_out = reinterpret_cast<float *>(gbase + STAGES * SB);
    float *cst = reinterpret_cast<float *>(gbase + STAGES * SB + EPI_BYTES);
    uint64_t *bars = reinterpret_cast<uint64_t *>(gbase + STAGES * SB + EPI_BYTES + cst_bytes<CF>());
    uint64_t *full = bars, *empty = bars + STAGES;
    uint64_t *accf = bars + 2 * STAGES, *acce = accf + 2, *drain = acce + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *stop = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *issued = const_cast<int *>(stop) + 1;   // k-blocks whose TMA loads were issued ...
    int *consumed = issued + 1;                  // ... and whose loads the MMA thread waited for
    volatile int *flag_last = consumed + 1;      // split-K: this CTA completed the tile

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kbytes = a.Kp * TcCfg<CF>::ELT;
    const int nk = (kbytes + BKB - 1) / BKB;
    const int kel = BKB / TcCfg<CF>::ELT;                          // K elements per stage
    const int mt = (a.M + BM - 1) / BM, nt = (a.N + BN - 1) / BN;
    const int tiles = mt * nt, items = tiles * ksplit;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ec_mbar_init(&full[s], 1);
            ec_mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            ec_mbar_init(&accf[b], 1);
            ec_mbar_init(&acce[b], EPI_WARPS);   // one arrival per epilogue warp
        }
        ec_mbar_init(drain, 1);
        *stop = 0;
        *issued = *consumed = 0;
        ec_fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(ec_smem_u32(tmem_slot)), "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // The weights do not depend on the previous kernel on the stream, which
    // may still be finishing (programmatic dependent launch): the producer
    // issues the weight tiles of the first ring stages before waiting for it,
    // their activation tiles right after; every other global access follows
    // the wait.
    int pre = 0;
    if (warp == 0 && lane == 0 && (int)blockIdx.x < items) {
        const int tile = blockIdx.x / ksplit, sp = blockIdx.x - tile * ksplit;
        const int kb0 = sp * nk / ksplit, kb1 = (sp + 1) * nk / ksplit;
        pre = kb1 - kb0 < STAGES ? kb1 - kb0 : STAGES;
        for (int j = 0; j < pre; ++j) {
            ec_mbar_expect_tx(&full[j], (uint32_t)SB);
            tma_load_2d(base + (uint32_t)(j * SB) + S * A_BYTES, &maps.b, ec_smem_u32(&full[j]), (kb0 + j) * kel,
                        (tile % nt) * BN);
        }
    }
    EC_PDL_ENTER();
    if (pre > 0) {
        const int tile = blockIdx.x / ksplit, sp = blockIdx.x - tile * ksplit;
        const int kb0 = sp * nk / ksplit;
        for (int j = 0; j < pre; ++j)
#pragma unroll
            for (int p = 0; p < S; ++p)
                tma_load_2d(base + (uint32_t)(j * SB) + p * A_BYTES, &maps.a[p], ec_smem_u32(&full[j]), (kb0 + j) * kel,
                            (tile / nt) * BM);
        *issued = pre;
    }

    if (warp == 0) {
        if (lane == 0) {   // TMA producer, one ring across all tiles of this CTA
            int g = 0;
            for (int it = blockIdx.x; it < items && !*stop; it += gridDim.x) {
                const int tile = it / ksplit, sp = it - tile * ksplit;
                const int m0 = (tile / nt) * BM, n0 = (tile % nt) * BN;
                const int kb0 = sp * nk / ksplit, kb1 = (sp + 1) * nk / ksplit;
                for (int kb = kb0; kb < kb1; ++kb, ++g) {
                    if (g < pre) continue;   // issued above
                    const int s = g % STAGES;
                    if (g >= STAGES && !tc_wait(&empty[s], (uint32_t)((g / STAGES - 1) & 1), stop)) break;
                    const uint32_t st = base + (uint32_t)(s * SB);
                    ec_mbar_expect_tx(&full[s], (uint32_t)SB);
#pragma unroll
                    for (int p = 0; p < S; ++p) tma_load_2d(st + p * A_BYTES, &maps.a[p], ec_smem_u32(&full[s]), kb * kel, m0);
                    tma_load_2d(st + S * A_BYTES, &maps.b, ec_smem_u32(&full[s]), kb * kel, n0);
                    *issued = g + 1;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {   // MMA issuer
            int g = 0, tc = 0;
            for (int it = blockIdx.x; it < items && !*stop; it += gridDim.x, ++tc) {
                const int sp = it % ksplit;
                const int kb0 = sp * nk / ksplit, kb1 = (sp + 1) * nk / ksplit;
                const int b = tc & 1;
                if (tc >= 2 && !tc_wait(&acce[b], (uint32_t)((tc / 2 - 1) & 1), stop)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(b * BN);
                bool ok = true;
                for (int kb = kb0; kb < kb1; ++kb, ++g) {
                    const int s = g % STAGES;
                    if (!tc_wait(&full[s], (uint32_t)((g / STAGES) & 1), stop)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t st = base + (uint32_t)(s * SB);
                    const uint64_t db = sw128_desc(st + S * A_BYTES);
#pragma unroll
                    for (int k = 0; k < BKB / KSTEP; ++k)     // +2 in 16-byte units per 32 bytes of K
#pragma unroll
                        for (int p = 0; p < S; ++p)
                            mma<CF>(d, sw128_desc(st + p * A_BYTES) + 2 * k, db + 2 * k, ((kb - kb0) | k | p) != 0);
                    mma_commit(ec_smem_u32(&empty[s]));   // stage reusable once these MMAs have read it
                    *consumed = g + 1;
                }
                if (!ok) break;
                mma_commit(ec_smem_u32(&accf[b]));
            }
            // every MMA this thread issued is complete once `drain` fires
            mma_commit(ec_smem_u32(drain));
            tc_wait(drain, 0, stop);
        }
    } else {   // epilogue: warps 2..9
        const int lg = warp & 3;                 // TMEM lane group this warp may access
        const int ch = (warp - 2) >> 2;          // column half of the tile
        constexpr int HALF = BN / 2;
        float *st = stage_out + (size_t)(warp - 2) * 32 * EPI_LD;
        float *cws = cst + (size_t)(warp - 2) * BN, *cb = cws + HALF;   // this warp's columns
        const bool vec_out = flags & 1;
        int tc = 0;
        for (int it = blockIdx.x; it < items; it += gridDim.x, ++tc) {
            const int tile = it / ksplit;
            const int m0 = (tile / nt) * BM, n0 = (tile % nt) * BN;
            const int b = tc & 1;
            if (WT == EC_W_I8 && ksplit > 1) {
                int ready = 0;
                if (lane == 0) ready = tc_wait(&accf[b], (uint32_t)((tc / 2) & 1), stop) && !*stop;
                ready = __shfl_sync(0xffffffffu, ready, 0);
                if (!epi_all(ready != 0)) break;
                tc_fence_after();
                split_tile_add<BN>(a, tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)(b * BN), m0, n0, lg, ch, lane, st);
                // this warp is done with accumulator b
                tc_fence_before();
                __syncwarp();
                if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(ec_smem_u32(&acce[b])) : "memory");
                split_tile_finish(a, row_scale, tile, m0, n0, BN, ksplit, flag_last, (int)threadIdx.x - 64);
                continue;
            }
            // Issue the tile's constants before waiting for its accumulator, so
            // their latency hides behind the MMAs: the row scale of this lane
            // and w_scale / bias of the warp's columns (lane j: j, j+32, ...).
            const int mrow = m0 + lg * 32 + lane;          // this lane's row in the TMEM read
            const float rs = mrow < a.M ? __ldg(row_scale + mrow) : 0.0f;
            float cw[HALF / 32], cbv[HALF / 32];
#pragma unroll
            for (int q = 0; q < HALF / 32; ++q) {
                const int n = n0 + ch * HALF + lane + 32 * q;
                cw[q] = WT == EC_W_I8 && a.wscale && n < a.N ? __ldg(a.wscale + n) : 1.0f;
                cbv[q] = a.bias && n < a.N ? __ldg(a.bias + n) : 0.0f;
            }
            int ready = 0;   // one lane waits; the warp takes its answer (tcgen05.ld is warp-collective)
            if (lane == 0) ready = tc_wait(&accf[b], (uint32_t)((tc / 2) & 1), stop) && !*stop;
            ready = __shfl_sync(0xffffffffu, ready, 0);
            if (!ready) break;
            tc_fence_after();
#pragma unroll
            for (int q = 0; q < HALF / 32; ++q) {
                cws[lane + 32 * q] = cw[q];
                cb[lane + 32 * q] = cbv[q];
            }
            __syncwarp();
            // EC_EPI_ARGMAX: this lane's row, max and first index over the
            // warp's columns, in four independent chains (columns e mod 4)
            const bool amx = a.epi == EC_EPI_ARGMAX;
            float bv[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            int bi[4] = {0x7fffffff, 0x7fffffff, 0x7fffffff, 0x7fffffff};
            for (int c0 = ch * HALF; c0 < (ch + 1) * HALF && n0 + c0 < a.N; c0 += EPI_COLS) {
                uint32_t r[16];
                tmem_ld16(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)(b * BN + c0), r);
                // scale + bias in the row-per-lane layout; the column constants
                // are the same for every lane (broadcast reads, 4 at a time)
#pragma unroll
                for (int j = 0; j < EPI_COLS; j += 4) {
                    const int cc = c0 - ch * HALF + j;              // column within this warp's half
                    const float4 ws4 = *reinterpret_cast<const float4 *>(cws + cc);
                    const float4 bs4 = *reinterpret_cast<const float4 *>(cb + cc);
                    const float ws[4] = {ws4.x, ws4.y, ws4.z, ws4.w}, bs[4] = {bs4.x, bs4.y, bs4.z, bs4.w};
                    float vv[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        if (WT == EC_W_I8) {
                            vv[e] = __fadd_rn(bs[e], __fmul_rn(__fmul_rn(__int2float_rn((int)r[j + e]), rs), ws[e]));
                        } else {
                            const float dot = __fmul_rn(__uint_as_float(r[j + e]), rs);   // exact: power of two
                            vv[e] = a.bias ? __fadd_rn(dot, bs[e]) : dot;
                        }
                    }
                    if (amx) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int n = n0 + c0 + j + e;
                            if (n < a.N && (vv[e] > bv[e] || (vv[e] == bv[e] && n < bi[e]))) { bv[e] = vv[e]; bi[e] = n; }
                        }
                    } else {
                        *reinterpret_cast<float4 *>(st + lane * EPI_LD + j) = make_float4(vv[0], vv[1], vv[2], vv[3]);
                    }
                }
                if (amx) continue;
                __syncwarp();
                // coalesced: 4 lanes per row (16 bytes each), 8 rows per pass
#pragma unroll
                for (int pass = 0; pass < 4; ++pass) {
                    const int row = pass * 8 + (lane >> 2), c4 = (lane & 3) * 4;
                    const int m = m0 + lg * 32 + row, n = n0 + c0 + c4;
                    if (m >= a.M || n >= a.N) continue;
                    const float4 v = *reinterpret_cast<const float4 *>(st + row * EPI_LD + c4);
                    float *o = a.out + (size_t)m * a.ldo + n;
                    if (vec_out && n + 3 < a.N) {
                        float4 w = v;
                        if (a.epi == EC_EPI_RESID) {
                            const float4 q = *reinterpret_cast<const float4 *>(o);
                            w = make_float4(__fadd_rn(q.x, v.x), __fadd_rn(q.y, v.y), __fadd_rn(q.z, v.z), __fadd_rn(q.w, v.w));
                        } else if (a.epi == EC_EPI_GELU) {
                            w = make_float4(ec_gelu(v.x), ec_gelu(v.y), ec_gelu(v.z), ec_gelu(v.w));
                        }
                        *reinterpret_cast<float4 *>(o) = w;
                    } else {
                        const float *vp = reinterpret_cast<const float *>(&v);
                        for (int e = 0; e < 4 && n + e < a.N; ++e) o[e] = epi_apply(a.epi, o[e], vp[e]);
                    }
                }
                __syncwarp();
            }
            if (amx && mrow < a.M) {   // partial (row, column tile, half) in the layout k_argmax_final merges
#pragma unroll
                for (int e = 1; e < 4; ++e)
                    if (bv[e] > bv[0] || (bv[e] == bv[0] && bi[e] < bi[0])) { bv[0] = bv[e]; bi[0] = bi[e]; }
                reinterpret_cast<float2 *>(a.out)[(size_t)mrow * a.ldo + (size_t)(n0 / BN) * 2 + ch] =
                    make_float2(bv[0], __int_as_float(bi[0]));
            }
            // this warp is done with accumulator b (and with its constants)
            tc_fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(ec_smem_u32(&acce[b])) : "memory");
        }
    }
    // After an abort: let TMA loads that nobody waited for land (bounded)
    // before the CTA's shared memory goes away.
    if (warp == 0 && lane == 0 && *stop)
        for (int g = *consumed; g < *issued; ++g)
            for (uint32_t i = 0; i < (1u << 20); ++i)
                if (ec_mbar_try_wait(&full[g % STAGES], (uint32_t)((g / STAGES) & 1))) break;
    // Every role is done with the accumulators; warp 1 frees the columns.
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

// Activation rows fp32 [M][ldx] -> S 16-bit parts [S][M][Kp] (zero padded
// past K) whose sum is the row times 2^-e, and rscale[m] = 2^e (see the file
// comment).  One CTA per row.
template <int WT>
__global__ void __launch_bounds__(256) k_split16(uint16_t *parts, float *rscale, const float *X, int ldx, int M, int K,
                                                 int Kp) {
    EC_PDL_ENTER();
    const int m = blockIdx.x;
    const float *x = X + (size_t)m * ldx;
    __shared__ float red[8];
    float sm = 1.0f, rs = 1.0f;
    if (WT == EC_W_F16) {
        float mx = 0.0f;
        for (int k = threadIdx.x; k < K; k += blockDim.x) mx = ec_max_keep(mx, fabsf(x[k]));
        mx = ec_warp_max(mx);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
        __syncthreads();
        mx = red[0];
        for (int i = 1; i < 8; ++i) mx = ec_max_keep(mx, red[i]);
        if (mx > 0.0f && mx < INFINITY) {   // max |x| * 2^-e in [2^13, 2^14)
            int ex;
            frexpf(mx, &ex);
            sm = ldexpf(1.0f, 14 - ex);
            rs = ldexpf(1.0f, ex - 14);
        }
    }
    if (threadIdx.x == 0) rscale[m] = rs;
    const size_t plane = (size_t)M * Kp;
    uint16_t *p0 = parts + (size_t)m * Kp;
    for (int k = threadIdx.x; k < Kp; k += blockDim.x) {
        const float v = k < K ? __fmul_rn(x[k], sm) : 0.0f;
        if (WT == EC_W_F16) {
            const __half h = __float2half_rn(v);
            const float r = __fsub_rn(v, __half2float(h));
            p0[k] = __half_as_ushort(h);
            p0[plane + k] = __half_as_ushort(__float2half_rn(r));
        } else {
            const __nv_bfloat16 b0 = __float2bfloat16_rn(v);
            const float r1 = __fsub_rn(v, __bfloat162float(b0));
            const __nv_bfloat16 b1 = __float2bfloat16_rn(r1);
            const float r2 = __fsub_rn(r1, __bfloat162float(b1));
            p0[k] = __bfloat16_as_ushort(b0);
            p0[plane + k] = __bfloat16_as_ushort(b1);
            p0[2 * plane + k] = __bfloat16_as_ushort(__float2bfloat16_rn(r2));
        }
    }
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
pthread_once_t g_once = PTHREAD_ONCE_INIT;
int g_attr_set[4][64];
int g_sms[64];

void resolve_encode() {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

// 2-D map of a [rows][inner] matrix of 1- or 2-byte elements with row stride
// `stride` bytes, box [box_rows][128 bytes], 128-byte swizzle; out-of-range
// elements read as 0.
int make_map(CUtensorMap *map, const void *ptr, int elt, int inner, int rows, int stride, int box_rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)stride};
    const cuuint32_t box[2] = {(cuuint32_t)(BKB / elt), (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = g_encode(map, elt == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 2,
                                const_cast<void *>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

template <int CF>
int set_attr(int dev) {
    if (!g_attr_set[CF][dev]) {
        const cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<CF>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes<CF>());
        if (e != cudaSuccess) return (int)e;
        g_attr_set[CF][dev] = 1;
    }
    return 0;
}

template <int CF>
int launch(const ec_gemm_args &a, const void *const *aparts, const float *row_scale, int dev, cudaStream_t stream) {
    constexpr int WT = TcCfg<CF>::WT;
    constexpr int S = TcCfg<CF>::S, BN = TcCfg<CF>::BN, ELT = TcCfg<CF>::ELT;
    {
        const int e = set_attr<CF>(dev);
        if (e) return e;
    }
    TcMaps maps;
    memset(&maps, 0, sizeof maps);
    int rc = 0;
    for (int p = 0; p < S && !rc; ++p) rc = make_map(&maps.a[p], aparts[p], ELT, a.Kp, a.M, a.Kp * ELT, BM);
    if (!rc) rc = make_map(&maps.b, a.W, ELT, a.Kp, a.N, a.ldw * ELT, BN);
    if (rc) return rc;
    const long long tiles = (long long)((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
    if (tiles > 0x7fffffffLL) return (int)cudaErrorInvalidValue;
    const int sms = g_sms[dev];
    // split K when the output is one row of tiles (M <= 64) and has fewer
    // tiles than half the SMs: at least 4 k-blocks of 128 bytes per split, at
    // most 8 splits and one CTA per SM in total.  Every split adds its whole
    // partial tile with atomics, so more rows or splits cost more than they
    // save (measured: decode of 32 streams 2.93 -> 2.76 ms per step, of 128
    // streams 3.03 -> 3.83 ms).
    int ksplit = 1;
    const int nk = (a.Kp * ELT + BKB - 1) / BKB;
    if (WT == EC_W_I8 && a.epi != EC_EPI_ARGMAX && a.M <= 64 && a.acc32 && a.tile_cnt && 2 * tiles <= sms &&
        tiles <= a.cnt_elems &&
        (size_t)a.M * a.N <= a.acc32_elems) {
        ksplit = sms / (int)tiles;
        if (ksplit > nk / 4) ksplit = nk / 4;
        if (ksplit > 8) ksplit = 8;
        if (ksplit < 1) ksplit = 1;
    }
    const long long items = tiles * ksplit;
    const int grid = (int)(items < (long long)sms ? items : sms);
    const int flags = (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 && (a.ldo & 3) == 0 ? 1 : 0;
    ec_launch_k(k_gemm_tc<CF>, dim3(grid), dim3(THREADS), (size_t)smem_bytes<CF>(), stream, maps, a, row_scale, flags,
                ksplit);
    return (int)cudaGetLastError();
}

}  // namespace

extern "C" int ec_gemm_tc_argmax_chunks(int wt, int M, int N) {
    if (M < EC_TC_MIN_M || N <= 0) return 0;
    int BN = wt == EC_W_F16 ? TcCfg<EC_W_F16>::BN : wt == EC_W_BF16 ? TcCfg<EC_W_BF16>::BN : TcCfg<EC_W_I8>::BN;
    if (wt == EC_W_I8) {   // the launcher's narrow-tile rule
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
        if (!g_sms[dev] && cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
        const long long wide_tiles = (long long)((M + BM - 1) / BM) * ((N + BN - 1) / BN);
        if (2 * wide_tiles <= g_sms[dev]) BN = TcCfg<TC_I8_NARROW>::BN;
    }
    return 2 * ((N + BN - 1) / BN);
}

extern "C" size_t ec_gemm_tc_split_bytes(int wt, int M, int Kp) {
    if (wt == EC_W_I8) return 0;
    const size_t S = wt == EC_W_F16 ? 2 : 3;
    return (S * (size_t)M * Kp * 2 + 255) / 256 * 256 + (size_t)M * 4;
}

// Tensor-core path (M >= EC_TC_MIN_M); cudaErrorNotSupported when the
// operands miss its alignment rules or a 16-bit GEMM has no split workspace
// (the caller then uses the SIMT kernel).
extern "C" int ec_launch_gemm_tc(const ec_gemm_args *args, cudaStream_t stream) {
    ec_gemm_args a = *args;
    if (a.M <= 0 || a.N <= 0) return 0;
    if (a.ldw == 0) a.ldw = a.Kp;
    const int elt = a.wt == EC_W_I8 ? 1 : 2;
    if (a.Kp % 16 || (a.ldw * elt) % 16 || a.ldw < a.Kp || (reinterpret_cast<uintptr_t>(a.W) & 15) ||
        (a.epi != EC_EPI_STORE && a.epi != EC_EPI_RESID && a.epi != EC_EPI_GELU && a.epi != EC_EPI_ARGMAX))
        return (int)cudaErrorNotSupported;
    if (a.epi == EC_EPI_ARGMAX && a.ldo < ec_gemm_tc_argmax_chunks(a.wt, a.M, a.N)) return (int)cudaErrorInvalidValue;
    if (a.wt == EC_W_I8) {
        if (!a.Aq || !a.a_scale || (reinterpret_cast<uintptr_t>(a.Aq) & 15)) return (int)cudaErrorNotSupported;
    } else {
        if (!a.X || !a.split || a.split_bytes < ec_gemm_tc_split_bytes(a.wt, a.M, a.Kp) ||
            (reinterpret_cast<uintptr_t>(a.split) & 255))
            return (int)cudaErrorNotSupported;
    }
    pthread_once(&g_once, resolve_encode);
    if (!g_encode) return (int)cudaErrorNotSupported;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return (int)cudaErrorNotSupported;
    if (!g_sms[dev]) {
        e = cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return (int)e;
    }
    if (a.wt == EC_W_I8) {
        const void *parts[1] = {a.Aq};
        // 256-column tiles that would occupy fewer than half the SMs:
        // 64-column tiles, four times the CTAs
        const long long wide_tiles = (long long)((a.M + BM - 1) / BM) * ((a.N + TcCfg<EC_W_I8>::BN - 1) / TcCfg<EC_W_I8>::BN);
        if (2 * wide_tiles <= g_sms[dev]) return launch<TC_I8_NARROW>(a, parts, a.a_scale, dev, stream);
        return launch<EC_W_I8>(a, parts, a.a_scale, dev, stream);
    }
    // 16-bit weights: split the activations first (Kp % 16 == 0 keeps every
    // part 16-byte aligned)
    const size_t plane = (size_t)a.M * a.Kp;
    uint16_t *parts16 = static_cast<uint16_t *>(a.split);
    float *rscale = reinterpret_cast<float *>(static_cast<unsigned char *>(a.split) +
                                              ((a.wt == EC_W_F16 ? 2 : 3) * plane * 2 + 255) / 256 * 256);
    const void *parts[3] = {parts16, parts16 + plane, parts16 + 2 * plane};
    if (a.wt == EC_W_F16) {
        ec_launch_k(k_split16<EC_W_F16>, dim3(a.M), dim3(256), 0, stream, parts16, rscale, a.X, a.ldx, a.M, a.K, a.Kp);
        e = cudaGetLastError();
        if (e != cudaSuccess) return (int)e;
        return launch<EC_W_F16>(a, parts, rscale, dev, stream);
    }
    ec_launch_k(k_split16<EC_W_BF16>, dim3(a.M), dim3(256), 0, stream, parts16, rscale, a.X, a.ldx, a.M, a.K, a.Kp);
    e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    return launch<EC_W_BF16>(a, parts, rscale, dev, stream);
}

extern "C" int ec_tc_init(void) {
    pthread_once(&g_once, resolve_encode);
    if (!g_encode) return (int)cudaErrorNotSupported;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return (int)cudaErrorNotSupported;
    if (!g_sms[dev]) {
        e = cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return (int)e;
    }
    int rc = set_attr<EC_W_I8>(dev);
    if (!rc) rc = set_attr<TC_I8_NARROW>(dev);
    if (!rc) rc = set_attr<EC_W_F16>(dev);
    if (!rc) rc = set_attr<EC_W_BF16>(dev);
    return rc;
}

extern "C" int ec_tc_error_take(int *code) {
    int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(code, g_tc_err, sizeof(int));
    if (e == cudaSuccess && *code) e = cudaMemcpyToSymbol(g_tc_err, &zero, sizeof(int));
    return (int)e;
}
