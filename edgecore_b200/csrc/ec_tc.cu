// ec_tc.cu -- W8A8 GEMM on the 5th-generation tensor cores (tcgen05):
//   out[m][n] = epi( bias[n] + ((float)(sum_k Aq[m][k] * W[n][k]) * a_scale[m]) * w_scale[n] )
// with Aq int8 [M][Kp] (row stride Kp), W int8 [N][ldw] (K-major rows, the
// packed layout of the host code), int32 accumulation in tensor memory.  The
// int8 x int8 products and their int32 sums are exact, so the result is
// bit-identical to the reference gemm_int8 (src/kernels.c:153-168) and to the
// SIMT kernels, whatever the order of the tensor core's additions.
//
// Persistent CTAs (one per SM) walk 128 x 256 output tiles
// (tcgen05.mma.cta_group::1.kind::i8, M = 128, N = 256, K = 32 per
// instruction) over K in 128-byte stages:
//   warp 0     TMA producer: A [128][128 B] and W [256][128 B] boxes with the
//              128-byte swizzle into a 4-stage ring that runs across tiles
//   warp 1     allocates all 512 TMEM columns = two 256-column accumulators;
//              one thread issues the MMAs of a tile into the free accumulator
//              and commits stages back to the producer, the accumulator to
//              the epilogue
//   warps 2-9  epilogue of the other accumulator meanwhile: tcgen05.ld (warp
//              w reads TMEM lanes 32*(w%4)..+31 = tile rows; warps w and w+4
//              split the 256 columns), scale and bias per element, transpose
//              through shared memory, coalesced 16-byte stores (store,
//              residual add or GELU)
// Loads never use cluster multicast; every wait is bounded and TMEM is freed
// on every path.
#include "ec_common.cuh"
#include "ec_launch.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <pthread.h>

namespace {

constexpr int BM = 128, BN = 256, BKB = 128;          // tile rows, tile cols, K bytes per stage
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BKB, B_BYTES = BN * BKB;  // 16 KB + 32 KB per stage
constexpr int THREADS = 320;                           // producer, MMA, 8 epilogue warps
constexpr int TMEM_COLS = 512;                         // two 256-column accumulators
constexpr int EPI_WARPS = 8, EPI_COLS = 16;           // two warps per TMEM lane group, 16-column chunks
constexpr int EPI_LD = 20;                             // staging row stride (floats): 16-byte rows, no bank conflicts
constexpr int EPI_BYTES = EPI_WARPS * 32 * EPI_LD * 4;
constexpr int CST_BYTES = EPI_WARPS * 2 * (BN / 2) * 4;      // per epilogue warp: w_scale and bias of its 128 columns
constexpr int SMEM_BYTES = 1024 /* alignment slack */ + STAGES * (A_BYTES + B_BYTES) + EPI_BYTES + CST_BYTES + 256;

// Instruction descriptor, kind::i8: D = s32, A = B = signed 8-bit, both
// K-major, N = 256, M = 128.
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

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

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(IDESC), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

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

__global__ void __launch_bounds__(THREADS, 1)
k_gemm_tc_i8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const ec_gemm_args a,
             int flags) {   // bit 0: 16-byte aligned output rows
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = ec_smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;                       // 1024-byte aligned (128-byte swizzle atoms)
    unsigned char *gbase = smem_raw + (base - raw);
    const uint32_t sA = base, sB = base + STAGES * A_BYTES;
    float *stage_out = reinterpret_cast<float *>(gbase + STAGES * (A_BYTES + B_BYTES));
    float *cst = reinterpret_cast<float *>(gbase + STAGES * (A_BYTES + B_BYTES) + EPI_BYTES);
    uint64_t *bars = reinterpret_cast<uint64_t *>(gbase + STAGES * (A_BYTES + B_BYTES) + EPI_BYTES + CST_BYTES);
    uint64_t *full = bars, *empty = bars + STAGES;
    uint64_t *accf = bars + 2 * STAGES, *acce = accf + 2, *drain = acce + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *stop = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *issued = const_cast<int *>(stop) + 1;   // k-blocks whose TMA loads were issued ...
    int *consumed = issued + 1;                  // ... and whose loads the MMA thread waited for

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = (a.Kp + BKB - 1) / BKB;
    const int mt = (a.M + BM - 1) / BM, nt = (a.N + BN - 1) / BN;
    const int tiles = mt * nt;

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

    if (warp == 0) {
        if (lane == 0) {   // TMA producer, one ring across all tiles of this CTA
            int g = 0;
            for (int tile = blockIdx.x; tile < tiles && !*stop; tile += gridDim.x) {
                const int m0 = (tile / nt) * BM, n0 = (tile % nt) * BN;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % STAGES;
                    if (g >= STAGES && !tc_wait(&empty[s], (uint32_t)((g / STAGES - 1) & 1), stop)) break;
                    ec_mbar_expect_tx(&full[s], A_BYTES + B_BYTES);
                    tma_load_2d(sA + s * A_BYTES, &tmA, ec_smem_u32(&full[s]), kb * BKB, m0);
                    tma_load_2d(sB + s * B_BYTES, &tmB, ec_smem_u32(&full[s]), kb * BKB, n0);
                    *issued = g + 1;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {   // MMA issuer
            int g = 0, tc = 0;
            for (int tile = blockIdx.x; tile < tiles && !*stop; tile += gridDim.x, ++tc) {
                const int b = tc & 1;
                if (tc >= 2 && !tc_wait(&acce[b], (uint32_t)((tc / 2 - 1) & 1), stop)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(b * BN);
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % STAGES;
                    if (!tc_wait(&full[s], (uint32_t)((g / STAGES) & 1), stop)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t da = sw128_desc(sA + s * A_BYTES), db = sw128_desc(sB + s * B_BYTES);
#pragma unroll
                    for (int k = 0; k < BKB / 32; ++k)   // 32 bytes of K per instruction: +2 in 16-byte units
                        mma_i8(d, da + 2 * k, db + 2 * k, (kb | k) != 0);
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
        float *st = stage_out + (size_t)(warp - 2) * 32 * EPI_LD;
        float *cws = cst + (size_t)(warp - 2) * BN, *cb = cws + BN / 2;   // this warp's 128 columns
        const bool vec_out = flags & 1;
        int tc = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++tc) {
            const int m0 = (tile / nt) * BM, n0 = (tile % nt) * BN;
            const int b = tc & 1;
            // Issue the tile's constants before waiting for its accumulator, so
            // their latency hides behind the MMAs: the row scale of this lane
            // and w_scale / bias of the warp's columns (lane j: j, j+32, ...).
            const int mrow = m0 + lg * 32 + lane;          // this lane's row in the TMEM read
            const float as = mrow < a.M ? __ldg(a.a_scale + mrow) : 0.0f;
            float cw[4], cbv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int n = n0 + ch * (BN / 2) + lane + 32 * q;
                cw[q] = a.wscale && n < a.N ? __ldg(a.wscale + n) : 1.0f;
                cbv[q] = a.bias && n < a.N ? __ldg(a.bias + n) : 0.0f;
            }
            int ready = 0;   // one lane waits; the warp takes its answer (tcgen05.ld is warp-collective)
            if (lane == 0) ready = tc_wait(&accf[b], (uint32_t)((tc / 2) & 1), stop) && !*stop;
            ready = __shfl_sync(0xffffffffu, ready, 0);
            if (!ready) break;
            tc_fence_after();
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                cws[lane + 32 * q] = cw[q];
                cb[lane + 32 * q] = cbv[q];
            }
            __syncwarp();
            for (int c0 = ch * (BN / 2); c0 < (ch + 1) * (BN / 2) && n0 + c0 < a.N; c0 += EPI_COLS) {
                uint32_t r[16];
                tmem_ld16(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)(b * BN + c0), r);
                // scale + bias in the row-per-lane layout; the column constants
                // are the same for every lane (broadcast loads, 4 at a time)
#pragma unroll
                for (int j = 0; j < EPI_COLS; j += 4) {
                    const int cc = c0 - ch * (BN / 2) + j;           // column within this warp's half
                    const float4 ws4 = *reinterpret_cast<const float4 *>(cws + cc);   // broadcast reads
                    const float4 bs4 = *reinterpret_cast<const float4 *>(cb + cc);
                    const float ws[4] = {ws4.x, ws4.y, ws4.z, ws4.w}, bs[4] = {bs4.x, bs4.y, bs4.z, bs4.w};
                    float4 v;
                    v.x = __fadd_rn(bs[0], __fmul_rn(__fmul_rn(__int2float_rn((int)r[j + 0]), as), ws[0]));
                    v.y = __fadd_rn(bs[1], __fmul_rn(__fmul_rn(__int2float_rn((int)r[j + 1]), as), ws[1]));
                    v.z = __fadd_rn(bs[2], __fmul_rn(__fmul_rn(__int2float_rn((int)r[j + 2]), as), ws[2]));
                    v.w = __fadd_rn(bs[3], __fmul_rn(__fmul_rn(__int2float_rn((int)r[j + 3]), as), ws[3]));
                    *reinterpret_cast<float4 *>(st + lane * EPI_LD + j) = v;
                }
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
                        const float *vv = reinterpret_cast<const float *>(&v);
                        for (int e = 0; e < 4 && n + e < a.N; ++e) o[e] = epi_apply(a.epi, o[e], vv[e]);
                    }
                }
                __syncwarp();
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

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
pthread_once_t g_once = PTHREAD_ONCE_INIT;
int g_attr_set[64];

void resolve_encode() {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

// 2-D map of an int8 [rows][inner] matrix with row stride `stride` bytes, box
// [box_rows][128 bytes], 128-byte swizzle; out-of-range elements read as 0.
int make_map(CUtensorMap *map, const void *ptr, int inner, int rows, int stride, int box_rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)stride};
    const cuuint32_t box[2] = {(cuuint32_t)BKB, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(ptr), dims, strides, box, es,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

}  // namespace

// Tensor-core path for int8 weights; returns cudaErrorNotSupported when the
// operands do not meet its alignment rules (the caller then uses the SIMT
// kernel).
extern "C" int ec_launch_gemm_tc(const ec_gemm_args *args, cudaStream_t stream) {
    ec_gemm_args a = *args;
    if (a.M <= 0 || a.N <= 0) return 0;
    if (a.ldw == 0) a.ldw = a.Kp;
    if (a.wt != EC_W_I8 || !a.Aq || !a.a_scale || a.Kp % 16 || a.ldw % 16 || a.ldw < a.Kp ||
        (reinterpret_cast<uintptr_t>(a.Aq) & 15) || (reinterpret_cast<uintptr_t>(a.W) & 15) ||
        (a.epi != EC_EPI_STORE && a.epi != EC_EPI_RESID && a.epi != EC_EPI_GELU))
        return (int)cudaErrorNotSupported;
    pthread_once(&g_once, resolve_encode);
    if (!g_encode) return (int)cudaErrorNotSupported;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev >= 0 && dev < 64 && !g_attr_set[dev]) {
        e = cudaFuncSetAttribute(k_gemm_tc_i8, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return (int)e;
        g_attr_set[dev] = 1;
    }
    CUtensorMap ta, tb;
    int rc = make_map(&ta, a.Aq, a.Kp, a.M, a.Kp, BM);
    if (!rc) rc = make_map(&tb, a.W, a.Kp, a.N, a.ldw, BN);
    if (rc) return rc;
    static int sms[64];
    if (dev >= 0 && dev < 64 && !sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    const long long tiles = (long long)((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
    if (tiles > 0x7fffffffLL) return (int)cudaErrorInvalidValue;
    const int grid = (int)(tiles < (long long)sms[dev] ? tiles : sms[dev]);
    const int flags = (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 && (a.ldo & 3) == 0 ? 1 : 0;
    k_gemm_tc_i8<<<grid, THREADS, SMEM_BYTES, stream>>>(ta, tb, a, flags);
    return (int)cudaGetLastError();
}

extern "C" int ec_tc_error_take(int *code) {
    int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(code, g_tc_err, sizeof(int));
    if (e == cudaSuccess && *code) e = cudaMemcpyToSymbol(g_tc_err, &zero, sizeof(int));
    return (int)e;
}
