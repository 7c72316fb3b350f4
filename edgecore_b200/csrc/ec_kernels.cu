// ec_kernels.cu -- the sm_100a kernels of the decode/prefill path.
//
//   k_gemv        weight-streaming GEMV for M <= 8 token rows: every lane keeps
//                 R rows x J 16-byte chunks of the [N][ldw] weight matrix in
//                 flight with L1-bypassing loads, the activations sit in shared
//                 memory, and a transposed shuffle reduction finishes each row.
//                 int8 weights: exact int32 dp4a dot + the reference epilogue
//                 (bias + ((float)dot*as)*ws).
//   k_gemm_i8, k_gemm_f  SIMT tiled GEMMs for 8 < M < 32 and for operands the
//                 tcgen05 path (ec_tc.cu) cannot take, same numerics.
//   k_quant       per-row activation quantisation (reference gpt2.c:446-461).
//   k_embed, k_norm, k_norm_quant, k_qkv_split, k_swiglu, k_swiglu_quant, k_gelu,
//   k_attn_exact, k_attn_part/combine,
//   k_argmax*, k_step_advance.
//
// Every index that comes from the caller (token ids, positions, slots) is
// bounds-checked on the device; a bad one is skipped and recorded in the
// library error word instead of being dereferenced.
#include "ec_common.cuh"
#include "ec_launch.h"

#include <float.h>

__device__ int g_ec_err;

#define GEMV_THREADS 256
#define GEMV_WARPS (GEMV_THREADS / 32)
#define GEMV_MT 8          // max token rows per GEMV launch

// ---------------------------------------------------------------------------
// GEMV: weight streaming for M <= 8 token rows
//
// Every warp owns groups of R consecutive weight rows (group g, g + W, ... for
// the W warps of the grid, so that the rows in flight at one time are close
// together in HBM).  Lane l reads the 16-byte chunks l, l+32, l+64, l+96 of
// each of the R rows straight into registers (up to 4R loads in flight per
// lane, no shared-memory staging of weights), multiplies them with the
// activation chunks held in shared memory, and the warp sums its R*MM
// partial dots with one transposed shuffle reduction.  A row's result does not
// depend on which warp or slot computes it: lane l always accumulates its
// chunks in increasing order (8 elements per chunk in element order) and the
// lane sum is the xor tree 16, 8, 4, 2, 1.
// ---------------------------------------------------------------------------

template <int WT> struct GemvAcc;
template <> struct GemvAcc<EC_W_I8> { typedef int T; };
template <> struct GemvAcc<EC_W_F16> { typedef float T; };
template <> struct GemvAcc<EC_W_BF16> { typedef float T; };

EC_DEV void ec_f16x8_to_f32(const uint4 w, float f[8]) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __half22float2(*reinterpret_cast<const __half2 *>(&u[i]));
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

EC_DEV void prefetch_l2(const void *p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// Shared memory of one CTA: the activation operand, int8 [M][Kp] or fp32
// planes [M][Kp] (elements 0-3 and 4-7 of every 8-element chunk in two
// planes, so 16-byte reads by consecutive lanes are conflict-free).
__host__ __device__ inline size_t gemv_smem_bytes(int wt, int M, int Kp) {
    return (size_t)M * (size_t)Kp * (wt == EC_W_I8 ? 1u : 4u);
}

template <int WT, int MM, int R, int J>
__global__ void __launch_bounds__(GEMV_THREADS, 2) k_gemv(const ec_gemv_args a) {
    EC_PDL_ENTER();
    typedef typename GemvAcc<WT>::T Acc;
    constexpr int ELT = WT == EC_W_I8 ? 1 : 2;
    constexpr int V = R * MM;   // values reduced per row group: [r][m]
    constexpr int D = 32 / V;   // lanes ending with the same total
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ float asc[GEMV_MT];
    __shared__ float red[GEMV_WARPS][GEMV_MT];
    const int M = a.M, Kp = a.Kp, K = a.K, N = a.N;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ldw = a.ldw ? a.ldw : Kp;
    const size_t row_bytes = (size_t)ldw * ELT;
    const int nch = Kp * ELT / 16;
    const int groups = (N + R - 1) / R;
    const int nw = (int)gridDim.x * GEMV_WARPS;
    const int gw = (int)blockIdx.x * GEMV_WARPS + warp;
    const unsigned char *W = static_cast<const unsigned char *>(a.W);

    // this warp's first row group into L2 while the activations are prepared
    if (gw < groups) {
        const int rows = min(R, N - gw * R);
        const unsigned char *g0 = W + (size_t)gw * R * row_bytes;
        const size_t bytes = (size_t)(rows - 1) * row_bytes + (size_t)Kp * ELT;
        for (size_t o = (size_t)lane * 128; o < bytes; o += 32 * 128) prefetch_l2(g0 + o);
    }

    // ---- activation operand -------------------------------------------------
    if (WT == EC_W_I8) {
        int8_t *xs = reinterpret_cast<int8_t *>(smem);
        if (a.Xq) {
            if (tid < M) asc[tid] = a.xscale[tid];
            for (int m = 0; m < M; ++m)
                for (int k = tid; k < Kp; k += GEMV_THREADS)
                    xs[(size_t)m * Kp + k] = k < K ? a.Xq[(size_t)m * a.ldx + k] : (int8_t)0;
        } else {
            // reference activation quantisation (src/gpt2.c:446-461), per CTA
            float mx[MM];
#pragma unroll
            for (int m = 0; m < MM; ++m) mx[m] = 0.0f;
            for (int k = tid; k < K; k += GEMV_THREADS) {
#pragma unroll
                for (int m = 0; m < MM; ++m)
                    if (m < M) mx[m] = ec_max_keep(mx[m], fabsf(a.X[(size_t)m * a.ldx + k]));
            }
#pragma unroll
            for (int m = 0; m < MM; ++m) {
                const float w = ec_warp_max(mx[m]);
                if (lane == 0) red[warp][m] = w;
            }
            __syncthreads();
            if (tid < M) {
                float w = 0.0f;
                for (int i = 0; i < GEMV_WARPS; ++i) w = ec_max_keep(w, red[i][tid]);
                asc[tid] = w > 0.0f ? __fdiv_rn(w, 127.0f) : 1.0f;
            }
            __syncthreads();
            for (int m = 0; m < M; ++m) {
                const float s = asc[m], r = __fdiv_rn(1.0f, s);
                const float *xr = a.X + (size_t)m * a.ldx;
                for (int k = tid; k < Kp; k += GEMV_THREADS)
                    xs[(size_t)m * Kp + k] = (int8_t)(k < K ? ec_quant_fast(xr[k], s, r) : 0);
            }
        }
    } else {
        float *xs = reinterpret_cast<float *>(smem);
        for (int m = 0; m < M; ++m) {
            const float *xr = a.X + (size_t)m * a.ldx;
            float *xm = xs + (size_t)m * Kp;
            for (int k = tid; k < Kp; k += GEMV_THREADS) {
                const float v = k < K ? xr[k] : 0.0f;
                const int c = k >> 3, e = k & 7;
                xm[(e >> 2) * (Kp >> 1) + c * 4 + (e & 3)] = v;
            }
        }
    }
    __syncthreads();

    // ---- row groups ---------------------------------------------------------
    const int my = ec_tr_vidx<V>(lane);
    const int my_r = my / MM, my_m = my % MM;
    const bool my_lane = (lane & (D - 1)) == 0 && my_m < M;
    for (int g = gw; g < groups; g += nw) {
        const int n0 = g * R;
        Acc acc[V];
#pragma unroll
        for (int v = 0; v < V; ++v) acc[v] = 0;
        for (int c0 = 0; c0 < nch; c0 += 32 * J) {
            uint4 w[R][J];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const unsigned char *rowp = W + (size_t)(n0 + r) * row_bytes;
#pragma unroll
                for (int j = 0; j < J; ++j) {
                    const int c = c0 + lane + 32 * j;
                    w[r][j] = (n0 + r < N && c < nch) ? ec_ldg_stream16(rowp + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
                }
            }
#pragma unroll
            for (int j = 0; j < J; ++j) {
                const int c = c0 + lane + 32 * j;
                if (c >= nch) break;
                if (WT == EC_W_I8) {
                    const int8_t *xs = reinterpret_cast<const int8_t *>(smem);
#pragma unroll
                    for (int m = 0; m < MM; ++m) {
                        if (m >= M) break;
                        const uint4 x = reinterpret_cast<const uint4 *>(xs + (size_t)m * Kp)[c];
#pragma unroll
                        for (int r = 0; r < R; ++r) {
                            int t = (int)acc[r * MM + m];
                            t = __dp4a((int)w[r][j].x, (int)x.x, t);
                            t = __dp4a((int)w[r][j].y, (int)x.y, t);
                            t = __dp4a((int)w[r][j].z, (int)x.z, t);
                            t = __dp4a((int)w[r][j].w, (int)x.w, t);
                            acc[r * MM + m] = t;
                        }
                    }
                } else {
                    const float *xs = reinterpret_cast<const float *>(smem);
#pragma unroll
                    for (int m = 0; m < MM; ++m) {
                        if (m >= M) break;
                        const float *xm = xs + (size_t)m * Kp;
                        const float4 x0 = reinterpret_cast<const float4 *>(xm)[c];
                        const float4 x1 = reinterpret_cast<const float4 *>(xm + (Kp >> 1))[c];
#pragma unroll
                        for (int r = 0; r < R; ++r)
                            acc[r * MM + m] = ec_dot8<WT == EC_W_BF16>(w[r][j], x0, x1, (float)acc[r * MM + m]);
                    }
                }
            }
        }
        const Acc tot = ec_tr_reduce<V>(acc, lane);
        const int n = n0 + my_r;
        if (!my_lane || n >= N) continue;
        float v;
        if (WT == EC_W_I8) {
            // reference gemm_int8 epilogue: bias + ((float)dot * a_scale) * b_scale (src/kernels.c:153-168)
            const float t = __fmul_rn(__fmul_rn(__int2float_rn((int)tot), asc[my_m]), a.wscale ? a.wscale[n] : 1.0f);
            v = __fadd_rn(a.bias ? a.bias[n] : 0.0f, t);
        } else {
            v = (float)tot;
            if (a.bias) v = __fadd_rn(v, a.bias[n]);
        }
        float *o = a.out + (size_t)my_m * a.ldo + n;
        if (a.epi == EC_EPI_RESID) *o = __fadd_rn(*o, v);
        else if (a.epi == EC_EPI_GELU) *o = ec_gelu(v);
        else *o = v;
    }
}

static int g_ec_max_optin_smem = 0;

extern "C" int ec_kernels_init(void) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    e = cudaDeviceGetAttribute(&g_ec_max_optin_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return (int)e;
    ec_attention_exact_fits(1, 1, 8, 1);   // sets the exact-attention smem attribute outside any capture
    return (int)cudaGetLastError();
}

// The GEMV takes M <= 8 rows, plain / residual / GELU epilogues, no row
// blocks, K a multiple of 16 and the activation operand in shared memory.
static size_t gemv_need(const ec_gemv_args *a) {
    if (a->M <= 0 || a->M > GEMV_MT || a->blocks || a->Kp % 16 || a->K > a->Kp) return 0;
    if (a->epi != EC_EPI_STORE && a->epi != EC_EPI_RESID && a->epi != EC_EPI_GELU) return 0;
    const int ldw = a->ldw ? a->ldw : a->Kp;
    if (ldw < a->Kp || (ldw * (a->wt == EC_W_I8 ? 1 : 2)) % 16 != 0) return 0;
    return gemv_smem_bytes(a->wt, a->M, a->Kp) + 16;
}

extern "C" int ec_gemv_fits(const ec_gemv_args *a) {
    if (g_ec_max_optin_smem == 0 && ec_kernels_init() != 0) return 0;
    const size_t need = gemv_need(a);
    return need > 0 && need <= (size_t)g_ec_max_optin_smem;
}

template <int WT, int MM, int R, int J>
static int gemv_launch(const ec_gemv_args *a, int num_sms, size_t smem, cudaStream_t stream) {
    auto kern = k_gemv<WT, MM, R, J>;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
    }
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, GEMV_THREADS, smem) != cudaSuccess || occ < 1) {
        cudaGetLastError();
        occ = 1;
    }
    const long long groups = ((long long)a->N + R - 1) / R;
    long long grid = (groups + GEMV_WARPS - 1) / GEMV_WARPS;
    const long long cap = (long long)num_sms * occ;
    if (grid > cap) grid = cap;
    kern<<<(int)grid, GEMV_THREADS, smem, stream>>>(*a);
    return (int)cudaGetLastError();
}

// R rows of J chunks per lane in flight (R * J = 16 loads of 16 bytes):
// 8 rows of 2 chunks when a row has at most 64 chunks, else 4 rows of 4;
// 8 token rows keep R * MM <= 32 values per reduction (and 16-bit weights
// their registers) with fewer rows per group.
template <int WT>
static int gemv_launch_r(const ec_gemv_args *a, int num_sms, size_t smem, cudaStream_t stream) {
    const int nch = a->Kp * (WT == EC_W_I8 ? 1 : 2) / 16;
    const bool short_rows = nch <= 64;
    if constexpr (WT == EC_W_I8) {
        if (a->M <= 1) return short_rows ? gemv_launch<WT, 1, 8, 2>(a, num_sms, smem, stream)
                                         : gemv_launch<WT, 1, 4, 4>(a, num_sms, smem, stream);
        if (a->M <= 2) return short_rows ? gemv_launch<WT, 2, 8, 2>(a, num_sms, smem, stream)
                                         : gemv_launch<WT, 2, 4, 4>(a, num_sms, smem, stream);
        if (a->M <= 4) return short_rows ? gemv_launch<WT, 4, 8, 2>(a, num_sms, smem, stream)
                                         : gemv_launch<WT, 4, 4, 4>(a, num_sms, smem, stream);
        return gemv_launch<WT, 8, 4, 4>(a, num_sms, smem, stream);
    } else {
        if (a->M <= 1) return short_rows ? gemv_launch<WT, 1, 8, 2>(a, num_sms, smem, stream)
                                         : gemv_launch<WT, 1, 4, 4>(a, num_sms, smem, stream);
        if (a->M <= 2) return gemv_launch<WT, 2, 4, 4>(a, num_sms, smem, stream);
        if (a->M <= 4) return gemv_launch<WT, 4, 4, 4>(a, num_sms, smem, stream);
        return gemv_launch<WT, 8, 2, 4>(a, num_sms, smem, stream);
    }
}

extern "C" int ec_launch_gemv(const ec_gemv_args *a, int num_sms, cudaStream_t stream) {
    if (a->M <= 0 || a->N <= 0) return 0;
    if (g_ec_max_optin_smem == 0) {
        const int e = ec_kernels_init();
        if (e) return e;
    }
    const size_t need = gemv_need(a);
    if (need == 0 || need > (size_t)g_ec_max_optin_smem) return (int)cudaErrorInvalidValue;
    const size_t smem = gemv_smem_bytes(a->wt, a->M, a->Kp);
    switch (a->wt) {
    case EC_W_I8: return gemv_launch_r<EC_W_I8>(a, num_sms, smem, stream);
    case EC_W_F16: return gemv_launch_r<EC_W_F16>(a, num_sms, smem, stream);
    default: return gemv_launch_r<EC_W_BF16>(a, num_sms, smem, stream);
    }
}

// ---------------------------------------------------------------------------
// Generic tiled GEMM (any M).  C[m][n] over a 64x64 tile per CTA, 256 threads,
// each thread a 4x4 micro-tile.  int8: exact int32 dp4a accumulation and the
// reference epilogue; 16-bit weights: fp32 FMA accumulation.
// ---------------------------------------------------------------------------

#define GT_BM 64
#define GT_BN 64
#define GT_BK 64

EC_DEV float gemm_finish(const ec_gemm_args &a, int m, int n, float acc_f, int acc_i) {
    float v;
    if (a.wt == EC_W_I8) {
        float t = __fmul_rn(__fmul_rn(__int2float_rn(acc_i), a.a_scale[m]), a.wscale ? a.wscale[n] : 1.0f);
        v = __fadd_rn(a.bias ? a.bias[n] : 0.0f, t);
    } else {
        v = acc_f;
        if (a.bias) v = __fadd_rn(v, a.bias[n]);
    }
    return v;
}

EC_DEV void gemm_apply(const ec_gemm_args &a, int m, int n, float v) {
    float *o = a.out + (size_t)m * a.ldo + n;
    if (a.epi == EC_EPI_RESID) *o = __fadd_rn(*o, v);
    else if (a.epi == EC_EPI_GELU) *o = ec_gelu(v);
    else *o = v;
}

__global__ void __launch_bounds__(256) k_gemm_i8(const ec_gemm_args a) {
    EC_PDL_ENTER();
    __shared__ __align__(16) int8_t As[GT_BM][GT_BK + 16];
    __shared__ __align__(16) int8_t Ws[GT_BN][GT_BK + 16];
    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * GT_BM, n0 = blockIdx.x * GT_BN;
    const int tm = (tid / 16) * 4, tn = (tid % 16) * 4;
    int acc[4][4] = {};
    for (int k0 = 0; k0 < a.Kp; k0 += GT_BK) {
        // 64 rows x 64 bytes per operand = 256 x 16 B
        {
            const int r = tid / 4, c = (tid % 4) * 16;
            uint4 va = make_uint4(0, 0, 0, 0), vw = make_uint4(0, 0, 0, 0);
            if (m0 + r < a.M && k0 + c < a.Kp)
                va = *reinterpret_cast<const uint4 *>(a.Aq + (size_t)(m0 + r) * a.Kp + k0 + c);
            if (n0 + r < a.N && k0 + c < a.Kp)
                vw = *reinterpret_cast<const uint4 *>(static_cast<const int8_t *>(a.W) + (size_t)(n0 + r) * a.ldw + k0 + c);
            *reinterpret_cast<uint4 *>(&As[r][c]) = va;
            *reinterpret_cast<uint4 *>(&Ws[r][c]) = vw;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < GT_BK; kk += 4) {
            int av[4], wv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = *reinterpret_cast<const int *>(&As[tm + i][kk]);
#pragma unroll
            for (int j = 0; j < 4; ++j) wv[j] = *reinterpret_cast<const int *>(&Ws[tn + j][kk]);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = __dp4a(av[i], wv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int m = m0 + tm + i, n = n0 + tn + j;
            if (m < a.M && n < a.N) gemm_apply(a, m, n, gemm_finish(a, m, n, 0.0f, acc[i][j]));
        }
}

template <int WT>
__global__ void __launch_bounds__(256) k_gemm_f(const ec_gemm_args a) {
    EC_PDL_ENTER();
    __shared__ float As[GT_BK / 2][GT_BM + 4];   // [k][m]
    __shared__ float Ws[GT_BK / 2][GT_BN + 4];   // [k][n]
    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * GT_BM, n0 = blockIdx.x * GT_BN;
    const int tm = (tid / 16) * 4, tn = (tid % 16) * 4;
    const int BK = GT_BK / 2;
    float acc[4][4] = {};
    const uint16_t *W = static_cast<const uint16_t *>(a.W);
    for (int k0 = 0; k0 < a.Kp; k0 += BK) {
        for (int e = tid; e < GT_BM * BK; e += 256) {
            const int r = e / BK, c = e % BK;
            const int k = k0 + c;
            As[c][r] = (m0 + r < a.M && k < a.K) ? a.X[(size_t)(m0 + r) * a.ldx + k] : 0.0f;
            Ws[c][r] = (n0 + r < a.N && k < a.Kp) ? ec_h2f(W[(size_t)(n0 + r) * a.ldw + k], WT == EC_W_BF16) : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < BK; ++kk) {
            float av[4], wv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = As[kk][tm + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) wv[j] = Ws[kk][tn + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int m = m0 + tm + i, n = n0 + tn + j;
            if (m < a.M && n < a.N) gemm_apply(a, m, n, gemm_finish(a, m, n, acc[i][j], 0));
        }
}

extern "C" int ec_launch_gemm(const ec_gemm_args *args, cudaStream_t stream) {
    ec_gemm_args a = *args;
    if (a.M <= 0 || a.N <= 0) return 0;
    if (a.ldw == 0) a.ldw = a.Kp;
    if (a.Kp % 16 || a.ldw < a.Kp || (a.ldw * (a.wt == EC_W_I8 ? 1 : 2)) % 16) return (int)cudaErrorInvalidValue;
    if (a.M >= EC_TC_MIN_M) {   // tensor cores unless the operands miss their alignment rules
        const int rc = ec_launch_gemm_tc(&a, stream);
        if (rc != (int)cudaErrorNotSupported || a.epi == EC_EPI_ARGMAX) return rc;
        cudaGetLastError();
    }
    if (a.epi == EC_EPI_ARGMAX) return (int)cudaErrorNotSupported;   // tensor cores only
    dim3 grid((a.N + GT_BN - 1) / GT_BN, (a.M + GT_BM - 1) / GT_BM);
    if (grid.y > 65535) return (int)cudaErrorInvalidValue;
    if (a.wt == EC_W_I8) k_gemm_i8<<<grid, 256, 0, stream>>>(a);
    else if (a.wt == EC_W_F16) k_gemm_f<EC_W_F16><<<grid, 256, 0, stream>>>(a);
    else k_gemm_f<EC_W_BF16><<<grid, 256, 0, stream>>>(a);
    return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Row-wise ops
// ---------------------------------------------------------------------------

template <typename T>
EC_DEV T block_reduce_sum(T v, T *sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    T t = 0;
    for (int i = 0; i < nw; ++i) t += sh[i];   // fixed order: deterministic
    return t;
}

EC_DEV float block_reduce_max(float v, float *sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = ec_warp_max(v);
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < nw; ++i) t = ec_max_keep(t, sh[i]);
    return t;
}

// Per-row activation quantisation: q[m][k] (k < Kp, zero padding), scale[m].
__global__ void __launch_bounds__(256) k_quant(int8_t *q, float *scale, const float *X, int ldx, int K, int Kp) {
    EC_PDL_ENTER();
    __shared__ float sh[32];
    const int m = blockIdx.x;
    const float *xr = X + (size_t)m * ldx;
    float mx = 0.0f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) mx = ec_max_keep(mx, fabsf(xr[k]));
    mx = block_reduce_max(mx, sh);
    const float s = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
    if (threadIdx.x == 0) scale[m] = s;
    for (int k = threadIdx.x; k < Kp; k += blockDim.x)
        q[(size_t)m * Kp + k] = (int8_t)(k < K ? ec_quant1(xr[k], s) : 0);
}

extern "C" int ec_launch_quant(int8_t *q, float *scale, const float *X, int ldx, int M, int K, int Kp,
                               cudaStream_t stream) {
    if (M <= 0) return 0;
    k_quant<<<M, 256, 0, stream>>>(q, scale, X, ldx, K, Kp);
    return (int)cudaGetLastError();
}

__global__ void __launch_bounds__(256) k_embed(float *x, const uint16_t *wte, const uint16_t *wpe, int ld,
                                               int bf16, ec_tokens tk, int E, int V, int C) {
    EC_PDL_ENTER();
    const int m = blockIdx.x;
    const int t = tk.tok[m];
    const int p = tk.pos ? tk.pos[m] : 0;
    if (t < 0 || t >= V || (wpe && (p < 0 || p >= C))) {
        if (threadIdx.x == 0) atomicCAS(&g_ec_err, 0, EC_KERR_BAD_INDEX);
        return;
    }
    for (int d = threadIdx.x; d < E; d += blockDim.x) {
        float e = ec_h2f(wte[(size_t)t * ld + d], bf16);
        if (wpe) e = __fadd_rn(e, ec_h2f(wpe[(size_t)p * ld + d], bf16));
        x[(size_t)m * E + d] = e;
    }
}

extern "C" int ec_launch_embed(float *x, const uint16_t *wte, const uint16_t *wpe, int ld, int is_bf16,
                               ec_tokens tk, int M, int E, int V, int C, cudaStream_t stream) {
    if (M <= 0) return 0;
    k_embed<<<M, 256, 0, stream>>>(x, wte, wpe, ld, is_bf16, tk, E, V, C);
    return (int)cudaGetLastError();
}

// LayerNorm (beta != NULL) / RMSNorm (beta == NULL) with fp64 statistics,
// products rounded separately as in the reference's -ffp-contract=off build.
__global__ void __launch_bounds__(256) k_norm(float *out, const float *x, const float *g, const float *b,
                                              int E, double eps) {
    EC_PDL_ENTER();
    __shared__ double sh[32];
    const int m = blockIdx.x;
    const float *xr = x + (size_t)m * E;
    float *orow = out + (size_t)m * E;
    if (b) {
        double s = 0.0;
        for (int i = threadIdx.x; i < E; i += blockDim.x) s = __dadd_rn(s, (double)xr[i]);
        const double mean = __ddiv_rn(block_reduce_sum(s, sh), (double)E);
        double v = 0.0;
        for (int i = threadIdx.x; i < E; i += blockDim.x) {
            const double d = __dsub_rn((double)xr[i], mean);
            v = __dadd_rn(v, __dmul_rn(d, d));
        }
        const double var = __ddiv_rn(block_reduce_sum(v, sh), (double)E);
        const double rstd = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(var, eps)));
        for (int i = threadIdx.x; i < E; i += blockDim.x) {
            const float t = (float)__dmul_rn(__dsub_rn((double)xr[i], mean), rstd);
            orow[i] = __fadd_rn(__fmul_rn(t, g[i]), b[i]);
        }
    } else {
        double s = 0.0;
        for (int i = threadIdx.x; i < E; i += blockDim.x) {
            const double d = (double)xr[i];
            s = __dadd_rn(s, __dmul_rn(d, d));
        }
        const double ms = block_reduce_sum(s, sh);
        const double rstd = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ms, (double)E), eps)));
        for (int i = threadIdx.x; i < E; i += blockDim.x)
            orow[i] = __fmul_rn((float)__dmul_rn((double)xr[i], rstd), g[i]);
    }
}

extern "C" int ec_launch_norm(float *out, const float *x, const float *gamma, const float *beta,
                              int M, int E, double eps, cudaStream_t stream) {
    if (M <= 0) return 0;
    k_norm<<<M, 256, 0, stream>>>(out, x, gamma, beta, E, eps);
    return (int)cudaGetLastError();
}

// The row's int8 quantisation (k_quant) of `row` [K] held in shared memory,
// with this thread's running max |value|: q[Kp] (zero past K) and *scale.
__device__ __forceinline__ void quant_smem_row(int8_t *q, float *scale, const float *row, int K, int Kp, float mx,
                                               float *sh) {
    mx = block_reduce_max(mx, sh);   // its barriers also publish the row
    const float s = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
    if (threadIdx.x == 0) *scale = s;
    for (int k = threadIdx.x; k < Kp; k += blockDim.x) q[k] = (int8_t)(k < K ? ec_quant1(row[k], s) : 0);
}

// k_norm then k_quant in one pass, the same arithmetic in the same order: the
// int8 operand of the q|k|v and gate|up linears (the fp32 normed rows are not
// needed there).  Dynamic shared memory: E floats.
__global__ void __launch_bounds__(256) k_norm_quant(int8_t *q, float *scale, int Kp, const float *x, const float *g,
                                                    const float *b, int E, double eps) {
    EC_PDL_ENTER();
    extern __shared__ float nq_row[];
    __shared__ double sh[32];
    __shared__ float shf[32];
    const int m = blockIdx.x;
    const float *xr = x + (size_t)m * E;
    float mx = 0.0f;
    if (b) {
        double s = 0.0;
        for (int i = threadIdx.x; i < E; i += blockDim.x) s = __dadd_rn(s, (double)xr[i]);
        const double mean = __ddiv_rn(block_reduce_sum(s, sh), (double)E);
        double v = 0.0;
        for (int i = threadIdx.x; i < E; i += blockDim.x) {
            const double d = __dsub_rn((double)xr[i], mean);
            v = __dadd_rn(v, __dmul_rn(d, d));
        }
        const double var = __ddiv_rn(block_reduce_sum(v, sh), (double)E);
        const double rstd = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(var, eps)));
        for (int i = threadIdx.x; i < E; i += blockDim.x) {
            const float t = (float)__dmul_rn(__dsub_rn((double)xr[i], mean), rstd);
            const float o = __fadd_rn(__fmul_rn(t, g[i]), b[i]);
            nq_row[i] = o;
            mx = ec_max_keep(mx, fabsf(o));
        }
    } else {
        double s = 0.0;
        for (int i = threadIdx.x; i < E; i += blockDim.x) {
            const double d = (double)xr[i];
            s = __dadd_rn(s, __dmul_rn(d, d));
        }
        const double ms = block_reduce_sum(s, sh);
        const double rstd = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ms, (double)E), eps)));
        for (int i = threadIdx.x; i < E; i += blockDim.x) {
            const float o = __fmul_rn((float)__dmul_rn((double)xr[i], rstd), g[i]);
            nq_row[i] = o;
            mx = ec_max_keep(mx, fabsf(o));
        }
    }
    quant_smem_row(q + (size_t)m * Kp, scale + m, nq_row, E, Kp, mx, shf);
}

extern "C" int ec_launch_norm_quant(int8_t *q, float *scale, int Kp, const float *x, const float *gamma,
                                    const float *beta, int M, int E, double eps, cudaStream_t stream) {
    if (M <= 0) return 0;
    if ((size_t)E * 4 > 48 * 1024) return (int)cudaErrorNotSupported;
    k_norm_quant<<<M, 256, (size_t)E * 4, stream>>>(q, scale, Kp, x, gamma, beta, E, eps);
    return (int)cudaGetLastError();
}

// Split the q|k|v rows of a GEMM output [M][ldq] (packed layout: RoPE
// partners adjacent for Qwen2 when packed != 0, file order for GPT-2): RoPE
// q and k (fp64, reference src/gpt2.c:656-665), q -> q_out [M][E] in head
// order, k and v -> fp16 KV cache at (slot, pos).
__global__ void __launch_bounds__(256) k_qkv_split(float *q_out, const float *qkv, int ldq, ec_tokens tk,
                                                   ec_kvgeo g, int H, int KVH, int packed) {
    EC_PDL_ENTER();
    const int m = blockIdx.x;
    const int pos = tk.pos[m], slot = tk.slot[m];
    if (pos < 0 || pos >= g.C || slot < 0 || slot >= g.B) {
        if (threadIdx.x == 0) atomicCAS(&g_ec_err, 0, EC_KERR_BAD_INDEX);
        return;
    }
    const float *row = qkv + (size_t)m * ldq;
    float *qo = q_out + (size_t)m * g.E;
    const size_t kvo = ec_kv_row(g.pt, g.mp, slot, pos) * g.kv;
    uint16_t *kr = g.kc + kvo;
    uint16_t *vr = g.vc + kvo;
    if (packed) {
        const int half = g.hd >> 1;
        const int npairs = (H + KVH) * half;
        for (int idx = threadIdx.x; idx < npairs; idx += blockDim.x) {
            const int h = idx / half, i = idx % half;
            const float *v = row + (size_t)h * g.hd + 2 * i;
            const double c = g.rope_cos[(size_t)pos * half + i], s = g.rope_sin[(size_t)pos * half + i];
            const double av = (double)v[0], bv = (double)v[1];
            const float lo = (float)__dsub_rn(__dmul_rn(av, c), __dmul_rn(bv, s));
            const float hi = (float)__dadd_rn(__dmul_rn(av, s), __dmul_rn(bv, c));
            if (h < H) {
                qo[h * g.hd + i] = lo;
                qo[h * g.hd + i + half] = hi;
            } else {
                kr[(h - H) * g.hd + i] = ec_f2h(lo);
                kr[(h - H) * g.hd + i + half] = ec_f2h(hi);
            }
        }
        for (int d = threadIdx.x; d < g.kv; d += blockDim.x) vr[d] = ec_f2h(row[g.E + g.kv + d]);
    } else {
        for (int n = threadIdx.x; n < g.E; n += blockDim.x) qo[n] = row[n];
        for (int d = threadIdx.x; d < g.kv; d += blockDim.x) {
            kr[d] = ec_f2h(row[g.E + d]);
            vr[d] = ec_f2h(row[g.E + g.kv + d]);
        }
    }
}

extern "C" int ec_launch_qkv_split(float *q_out, const float *qkv, int ldq, ec_tokens tk, ec_kvgeo geo, int H,
                                   int KVH, int packed, int M, cudaStream_t stream) {
    if (M <= 0) return 0;
    k_qkv_split<<<M, 256, 0, stream>>>(q_out, qkv, ldq, tk, geo, H, KVH, packed);
    return (int)cudaGetLastError();
}

// out[m][j] = silu(gate) * up with gate|up interleaved: gu[m][2j], gu[m][2j+1].
__global__ void k_swiglu(float *out, int ldo, const float *gu, int ldg, int I, int M) {
    EC_PDL_ENTER();
    const size_t n = (size_t)M * I;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const size_t m = idx / I, j = idx % I;
        const float g = gu[m * ldg + 2 * j], u = gu[m * ldg + 2 * j + 1];
        out[m * ldo + j] = __fmul_rn(ec_silu(g), u);
    }
}

extern "C" int ec_launch_swiglu(float *out, int ldo, const float *gu, int ldg, int I, int M, cudaStream_t stream) {
    if (M <= 0) return 0;
    const size_t n = (size_t)M * I;
    const int grid = (int)((n + 255) / 256 > 65535 ? 65535 : (n + 255) / 256);
    k_swiglu<<<grid, 256, 0, stream>>>(out, ldo, gu, ldg, I, M);
    return (int)cudaGetLastError();
}

// k_swiglu then k_quant in one pass (one CTA per row): the int8 operand of
// the down projection.  Dynamic shared memory: I floats.
__global__ void __launch_bounds__(256) k_swiglu_quant(int8_t *q, float *scale, int Kp, const float *gu, int ldg, int I) {
    EC_PDL_ENTER();
    extern __shared__ float sq_row[];
    __shared__ float shf[32];
    const int m = blockIdx.x;
    const float *row = gu + (size_t)m * ldg;
    float mx = 0.0f;
    for (int j = threadIdx.x; j < I; j += blockDim.x) {
        const float a = __fmul_rn(ec_silu(row[2 * j]), row[2 * j + 1]);
        sq_row[j] = a;
        mx = ec_max_keep(mx, fabsf(a));
    }
    quant_smem_row(q + (size_t)m * Kp, scale + m, sq_row, I, Kp, mx, shf);
}

extern "C" int ec_launch_swiglu_quant(int8_t *q, float *scale, int Kp, const float *gu, int ldg, int I, int M,
                                      cudaStream_t stream) {
    if (M <= 0) return 0;
    if ((size_t)I * 4 > 48 * 1024) return (int)cudaErrorNotSupported;
    k_swiglu_quant<<<M, 256, (size_t)I * 4, stream>>>(q, scale, Kp, gu, ldg, I);
    return (int)cudaGetLastError();
}

__global__ void k_gelu(float *x, size_t n) {
    EC_PDL_ENTER();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        x[i] = ec_gelu(x[i]);
}

extern "C" int ec_launch_gelu_inplace(float *x, size_t n, cudaStream_t stream) {
    if (!n) return 0;
    const int grid = (int)((n + 255) / 256 > 65535 ? 65535 : (n + 255) / 256);
    k_gelu<<<grid, 256, 0, stream>>>(x, n);
    return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Attention: split over key positions (flash-decoding), then combine.
// Part layout: [M][H][nsplit][hd + 2] = partial output (unnormalised), max, sum.
// ---------------------------------------------------------------------------

#define ATT_THREADS 128
#define ATT_MAX_CHUNK 1024

extern "C" size_t ec_attention_scratch_floats(int M, int H, int hd, int nsplit) {
    return (size_t)M * H * nsplit * (hd + 2);
}

__global__ void __launch_bounds__(ATT_THREADS) k_attn_part(const ec_attn_args a) {
    EC_PDL_ENTER();
    __shared__ float qs[256];
    __shared__ float sc[ATT_MAX_CHUNK];
    __shared__ float red[ATT_THREADS / 32];
    __shared__ double redd[ATT_THREADS / 32];
    const int s = blockIdx.x, h = blockIdx.y, m = blockIdx.z;
    const ec_kvgeo &g = a.geo;
    const int hd = g.hd;
    const int pos = a.tk.pos[m], slot = a.tk.slot[m];
    float *part = a.part + (((size_t)m * a.H + h) * a.nsplit + s) * (hd + 2);
    if (pos < 0 || pos >= g.C || slot < 0 || slot >= g.B) {
        if (threadIdx.x == 0) atomicCAS(&g_ec_err, 0, EC_KERR_BAD_INDEX);
        return;
    }
    int lo = 0;
    if (a.window > 0) { lo = pos - a.window + 1; if (lo < 0) lo = 0; }
    const int len = pos + 1 - lo;
    const int chunk = (len + a.nsplit - 1) / a.nsplit;
    const int p0 = lo + s * chunk;
    const int p1 = min(pos + 1, p0 + chunk);
    if (p0 >= p1 || chunk > ATT_MAX_CHUNK) {
        if (chunk > ATT_MAX_CHUNK && threadIdx.x == 0) atomicCAS(&g_ec_err, 0, EC_KERR_BAD_INDEX);
        if (threadIdx.x == 0) { part[hd] = -FLT_MAX; part[hd + 1] = 0.0f; }
        for (int d = threadIdx.x; d < hd; d += blockDim.x) part[d] = 0.0f;
        return;
    }
    const int kvh = h * a.KVH / a.H;
    const uint16_t *kb = g.kc + (size_t)kvh * hd;   // + the arena row of each position
    const uint16_t *vb = g.vc + (size_t)kvh * hd;
    const float *q = a.q + (size_t)m * a.ldq + (size_t)h * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) qs[d] = q[d];
    __syncthreads();
    const double inv_hd = 1.0 / sqrt((double)hd);
    // scores: one position per thread, the reference's sequential fp32 dot
    float mx = -FLT_MAX;
    for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
        const uint16_t *kp = kb + ec_kv_row(g.pt, g.mp, slot, p) * g.kv;
        float acc = 0.0f;
        for (int d = 0; d < hd; d += 8) {
            const uint4 w = *reinterpret_cast<const uint4 *>(kp + d);
            float f[8];
            ec_f16x8_to_f32(w, f);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc = __fadd_rn(acc, __fmul_rn(qs[d + e], f[e]));
        }
        const float sv = (float)__dmul_rn((double)acc, inv_hd);
        sc[p - p0] = sv;
        mx = ec_max_keep(mx, sv);
    }
    {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        float w = mx;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) { float t = __shfl_xor_sync(0xffffffffu, w, o); w = t > w ? t : w; }
        if (lane == 0) red[warp] = w;
        __syncthreads();
        mx = red[0];
        for (int i = 1; i < ATT_THREADS / 32; ++i) mx = red[i] > mx ? red[i] : mx;
    }
    double sum = 0.0;
    for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
        const float e = ec_expf(sc[p - p0] - mx);
        sc[p - p0] = e;
        sum += (double)e;
    }
    {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        sum = ec_warp_sum_d(sum);
        if (lane == 0) redd[warp] = sum;
        __syncthreads();
        sum = 0.0;
        for (int i = 0; i < ATT_THREADS / 32; ++i) sum += redd[i];
    }
    // unnormalised P.V: one output dim per thread, sequential over positions
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = 0.0f;
        for (int p = p0; p < p1; ++p)
            o = __fadd_rn(o, __fmul_rn(sc[p - p0],
                                       __half2float(__ushort_as_half(vb[ec_kv_row(g.pt, g.mp, slot, p) * g.kv + d]))));
        part[d] = o;
    }
    if (threadIdx.x == 0) { part[hd] = mx; part[hd + 1] = (float)sum; }
}

__global__ void k_attn_combine(const ec_attn_args a) {
    EC_PDL_ENTER();
    const int h = blockIdx.x, m = blockIdx.y;
    const int hd = a.geo.hd;
    const float *part = a.part + ((size_t)m * a.H + h) * a.nsplit * (hd + 2);
    float M = -FLT_MAX;
    for (int s = 0; s < a.nsplit; ++s) M = ec_max_keep(M, part[s * (hd + 2) + hd]);
    double L = 0.0;
    for (int s = 0; s < a.nsplit; ++s) {
        const float ls = part[s * (hd + 2) + hd + 1];
        if (ls > 0.0f) L += (double)ls * exp((double)part[s * (hd + 2) + hd] - (double)M);
    }
    const double invL = L > 0.0 ? 1.0 / L : 0.0;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        double o = 0.0;
        for (int s = 0; s < a.nsplit; ++s) {
            const float ls = part[s * (hd + 2) + hd + 1];
            if (ls > 0.0f) o += (double)part[s * (hd + 2) + d] * exp((double)part[s * (hd + 2) + hd] - (double)M);
        }
        a.out[(size_t)m * a.ldo + (size_t)h * hd + d] = (float)(o * invL);
    }
}

// Exact-order attention: the reference's arithmetic step for step
// (src/gpt2.c:743-777, :527-557) for all query heads of one KV head and one
// token row.  Scores are the sequential fp32 dot over head_dim (products and
// sums rounded separately), scaled in fp64; the max is global; weights are
// (float)(exp(s - max) * (1 / sum)) with the sum in fp64; the output is the
// sequential fp32 sum over positions of w * v, in position order.  Only the
// fp64 sums are reassociated (they round to the same fp32 weights except in
// ~2^-29 of cases).  One CTA per (KV head, token); scores live in shared
// memory (maxlen * heads_per_group floats), and V comes through shared memory
// ATTX_VCH positions at a time with coalesced 16-byte loads.
#define ATTX_THREADS 256
#define ATTX_MAX_GROUP 16
#define ATTX_VCH 64
#define ATTX_OPT 16   // (head, d) output pairs per thread at most: G * hd <= 16 * 256

__host__ __device__ inline size_t attx_v_offset(int G, int hd, int maxlen) {
    return (((size_t)G * hd + (size_t)G * maxlen) * sizeof(float) + 15) & ~(size_t)15;
}

__host__ __device__ inline size_t attx_smem_bytes(int G, int hd, int maxlen) {
    return attx_v_offset(G, hd, maxlen) + (size_t)ATTX_VCH * hd * 2;
}

__global__ void __launch_bounds__(ATTX_THREADS) k_attn_exact(const ec_attn_args a) {
    EC_PDL_ENTER();
    extern __shared__ __align__(16) float attx_smem[];
    const int m = blockIdx.y;
    const ec_kvgeo &geo = a.geo;
    const int hd = geo.hd;
    // the query heads of this CTA: one (per_head) or all of KV head g's
    const int g = a.per_head ? (int)blockIdx.x * a.KVH / a.H : (int)blockIdx.x;
    const int h0 = a.per_head ? (int)blockIdx.x : (g * a.H + a.KVH - 1) / a.KVH;
    const int h1 = a.per_head ? h0 + 1 : ((g + 1) * a.H + a.KVH - 1) / a.KVH;
    const int G = h1 - h0;
    const int pos = a.tk.pos[m], slot = a.tk.slot[m];
    if (pos < 0 || pos >= geo.C || slot < 0 || slot >= geo.B || G <= 0 || G > ATTX_MAX_GROUP) {
        if (threadIdx.x == 0) atomicCAS(&g_ec_err, 0, EC_KERR_BAD_INDEX);
        return;
    }
    int lo = 0;
    if (a.window > 0) { lo = pos - a.window + 1; if (lo < 0) lo = 0; }
    const int len = pos + 1 - lo;
    if (len > a.maxlen) {
        if (threadIdx.x == 0) atomicCAS(&g_ec_err, 0, EC_KERR_BAD_INDEX);
        return;
    }
    float *qs = attx_smem;                 // [G][hd]
    float *sc = attx_smem + G * hd;        // [G][maxlen]
    const uint16_t *kb = geo.kc + (size_t)g * hd;   // + the arena row of each position
    const uint16_t *vb = geo.vc + (size_t)g * hd;
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x)
        qs[i] = a.q[(size_t)m * a.ldq + (size_t)(h0 + i / hd) * hd + (i % hd)];
    __syncthreads();
    const double inv_hd = 1.0 / sqrt((double)hd);

    // scores, one position per thread, all heads of the group
    for (int p = lo + (int)threadIdx.x; p <= pos; p += blockDim.x) {
        const uint16_t *kp = kb + ec_kv_row(geo.pt, geo.mp, slot, p) * geo.kv;
        float acc[ATTX_MAX_GROUP];
#pragma unroll
        for (int hh = 0; hh < ATTX_MAX_GROUP; ++hh) acc[hh] = 0.0f;
        for (int d = 0; d < hd; d += 8) {
            float f[8];
            ec_f16x8_to_f32(*reinterpret_cast<const uint4 *>(kp + d), f);
#pragma unroll
            for (int hh = 0; hh < ATTX_MAX_GROUP; ++hh) {
                if (hh < G) {
                    // q in two 16-byte broadcast loads (qs rows are 32-byte aligned: hd % 8 == 0)
                    const float4 q0 = *reinterpret_cast<const float4 *>(qs + hh * hd + d);
                    const float4 q1 = *reinterpret_cast<const float4 *>(qs + hh * hd + d + 4);
                    const float q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                    float t = acc[hh];
#pragma unroll
                    for (int e = 0; e < 8; ++e) t = __fadd_rn(t, __fmul_rn(q[e], f[e]));
                    acc[hh] = t;
                }
            }
        }
#pragma unroll
        for (int hh = 0; hh < ATTX_MAX_GROUP; ++hh)
            if (hh < G) sc[hh * a.maxlen + (p - lo)] = (float)__dmul_rn((double)acc[hh], inv_hd);
    }
    __syncthreads();

    // softmax weights, one warp per head
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int hh = warp; hh < G; hh += ATTX_THREADS / 32) {
        float *s = sc + hh * a.maxlen;
        float mx = -FLT_MAX;
        for (int i = lane; i < len; i += 32) mx = ec_max_keep(mx, s[i]);
        mx = ec_warp_max(mx);
        double sum = 0.0;
        for (int i = lane; i < len; i += 32) {
            const float e = ec_expf(__fsub_rn(s[i], mx));
            s[i] = e;
            sum = __dadd_rn(sum, (double)e);
        }
        sum = ec_warp_sum_d(sum);
        const double isum = __ddiv_rn(1.0, sum);
        __syncwarp();
        for (int i = lane; i < len; i += 32) s[i] = (float)__dmul_rn((double)s[i], isum);
    }
    __syncthreads();

    // output: sequential fp32 accumulation over positions for every (head, d),
    // V staged ATTX_VCH positions at a time; each pair keeps its running sum
    // across chunks, so the order is the reference's
    uint16_t *vs = reinterpret_cast<uint16_t *>(reinterpret_cast<unsigned char *>(attx_smem) +
                                                attx_v_offset(G, hd, a.maxlen));
    const int npair = G * hd, per = hd >> 3;
    float o[ATTX_OPT];
#pragma unroll
    for (int k = 0; k < ATTX_OPT; ++k) o[k] = 0.0f;
    for (int c0 = 0; c0 < len; c0 += ATTX_VCH) {
        const int n = min(ATTX_VCH, len - c0);
        __syncthreads();   // the previous chunk is consumed
        for (int e = threadIdx.x; e < n * per; e += blockDim.x) {
            const int i = e / per, j = e - i * per;
            const uint16_t *src = vb + ec_kv_row(geo.pt, geo.mp, slot, lo + c0 + i) * geo.kv + 8 * j;
            *reinterpret_cast<uint4 *>(vs + (size_t)i * hd + 8 * j) = __ldg(reinterpret_cast<const uint4 *>(src));
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < ATTX_OPT; ++k) {
            const int idx = (int)threadIdx.x + k * ATTX_THREADS;
            if (idx >= npair) break;
            const int hh = idx / hd, d = idx - hh * hd;
            const float *w = sc + hh * a.maxlen + c0;
            const uint16_t *vd = vs + d;
            float acc = o[k];
            int i = 0;
            if (((a.maxlen | c0) & 3) == 0)   // weights 16-byte aligned: four per broadcast load
                for (; i + 4 <= n; i += 4) {
                    const float4 w4 = *reinterpret_cast<const float4 *>(w + i);
                    acc = __fadd_rn(acc, __fmul_rn(w4.x, __half2float(__ushort_as_half(vd[(size_t)i * hd]))));
                    acc = __fadd_rn(acc, __fmul_rn(w4.y, __half2float(__ushort_as_half(vd[(size_t)(i + 1) * hd]))));
                    acc = __fadd_rn(acc, __fmul_rn(w4.z, __half2float(__ushort_as_half(vd[(size_t)(i + 2) * hd]))));
                    acc = __fadd_rn(acc, __fmul_rn(w4.w, __half2float(__ushort_as_half(vd[(size_t)(i + 3) * hd]))));
                }
            for (; i < n; ++i)
                acc = __fadd_rn(acc, __fmul_rn(w[i], __half2float(__ushort_as_half(vd[(size_t)i * hd]))));
            o[k] = acc;
        }
    }
#pragma unroll
    for (int k = 0; k < ATTX_OPT; ++k) {
        const int idx = (int)threadIdx.x + k * ATTX_THREADS;
        if (idx >= npair) break;
        const int hh = idx / hd, d = idx - hh * hd;
        a.out[(size_t)m * a.ldo + (size_t)(h0 + hh) * hd + d] = o[k];
    }
}

// Exact-order attention for runs of query rows (prefill): the arithmetic of
// k_attn_exact, value for value, for a block of up to ATTP_QB consecutive
// rows of one slot at consecutive positions (the host's block table) and
// one query head, so that every cached K and V row is brought into shared
// memory once per block instead of once per row.
// Scores are kept transposed, scT[t - lo0][r] (row stride ATTP_QBP floats:
// 16-byte aligned, and the score writes of a warp fall on distinct banks).
// Per (row, d) the output is the sequential fp32 sum over positions t in
// [lo_r, pos_r], ascending, as in the reference (src/gpt2.c:757-775).
#define ATTP_QB EC_ATTN_RUN
#define ATTP_QBP 36
#define ATTP_THREADS 256
#define ATTP_KCH 64

__host__ __device__ inline int attp_span_cap(int maxlen) { return (maxlen + ATTP_QB - 1 + 3) & ~3; }

__host__ __device__ inline size_t attp_smem_bytes(int hd, int span_cap) {
    return (size_t)ATTP_QB * hd * 4 + (size_t)span_cap * ATTP_QBP * 4 + (size_t)ATTP_KCH * (hd + 8) * 2 +
           (size_t)ATTP_KCH * hd * 2;
}

__global__ void __launch_bounds__(ATTP_THREADS) k_attn_prefill(const ec_attn_args a) {
    EC_PDL_ENTER();
    extern __shared__ __align__(16) float attp_smem[];
    const ec_kvgeo &geo = a.geo;
    const int hd = geo.hd, h = blockIdx.x;
    const int r0 = a.blocks[2 * blockIdx.y], nr = a.blocks[2 * blockIdx.y + 1];
    if (r0 < 0 || nr < 1 || nr > ATTP_QB || r0 + nr > a.M) {
        if (threadIdx.x == 0) atomicCAS(&g_ec_err, 0, EC_KERR_BAD_INDEX);
        return;
    }
    const int g = h * a.KVH / a.H;   // the KV head of query head h
    const int pos0 = a.tk.pos[r0], slot = a.tk.slot[r0];
    const int pend = pos0 + nr - 1;
    int lo0 = 0;
    if (a.window > 0) { lo0 = pos0 - a.window + 1; if (lo0 < 0) lo0 = 0; }
    const int span = pend + 1 - lo0, cap = attp_span_cap(a.maxlen);
    if (pos0 < 0 || pend >= geo.C || slot < 0 || slot >= geo.B || span > cap || hd > 128) {
        if (threadIdx.x == 0) atomicCAS(&g_ec_err, 0, EC_KERR_BAD_INDEX);
        return;
    }
    float *qs = attp_smem;                                   // [QB][hd]
    float *scT = qs + ATTP_QB * hd;                          // [cap][QBP]
    uint16_t *kch = reinterpret_cast<uint16_t *>(scT + (size_t)cap * ATTP_QBP);   // [KCH][hd + 8]
    uint16_t *vch = kch + (size_t)ATTP_KCH * (hd + 8);                            // [KCH][hd]
    const uint16_t *kb = geo.kc + (size_t)g * hd, *vb = geo.vc + (size_t)g * hd;
    const int per = hd >> 3;   // 16-byte pieces of a cached row
    for (int i = threadIdx.x; i < nr * hd; i += blockDim.x)
        qs[i] = a.q[(size_t)(r0 + i / hd) * a.ldq + (size_t)h * hd + (i % hd)];
    const double inv_hd = 1.0 / sqrt((double)hd);

    // scores: thread (r, ib) takes positions ib, ib + 8, ... of each K chunk
    {
        const int r = threadIdx.x >> 3, ib = threadIdx.x & 7;
        for (int c0 = lo0; c0 <= pend; c0 += ATTP_KCH) {
            const int n = min(ATTP_KCH, pend + 1 - c0);
            __syncthreads();   // q staged / the previous chunk consumed
            for (int e = threadIdx.x; e < n * per; e += blockDim.x) {
                const int i = e / per, j = e - i * per;
                const uint16_t *src = kb + ec_kv_row(geo.pt, geo.mp, slot, c0 + i) * geo.kv + 8 * j;
                *reinterpret_cast<uint4 *>(kch + (size_t)i * (hd + 8) + 8 * j) = __ldg(reinterpret_cast<const uint4 *>(src));
            }
            __syncthreads();
            if (r < nr) {
                float acc[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
                for (int d = 0; d < hd; d += 8) {
                    const float4 q0 = *reinterpret_cast<const float4 *>(qs + r * hd + d);
                    const float4 q1 = *reinterpret_cast<const float4 *>(qs + r * hd + d + 4);
                    const float q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int i = ib + 8 * j;
                        if (i < n) {
                            float f[8];
                            ec_f16x8_to_f32(*reinterpret_cast<const uint4 *>(kch + (size_t)i * (hd + 8) + d), f);
                            float t = acc[j];
#pragma unroll
                            for (int e = 0; e < 8; ++e) t = __fadd_rn(t, __fmul_rn(q[e], f[e]));
                            acc[j] = t;
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int i = ib + 8 * j;
                    if (i < n) scT[(size_t)(c0 - lo0 + i) * ATTP_QBP + r] = (float)__dmul_rn((double)acc[j], inv_hd);
                }
            }
        }
    }
    __syncthreads();

    // softmax weights, one warp per row (the order of k_attn_exact)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int r = warp; r < nr; r += ATTP_THREADS / 32) {
        const int pr = pos0 + r;
        int lr = 0;
        if (a.window > 0) { lr = pr - a.window + 1; if (lr < 0) lr = 0; }
        const int len = pr + 1 - lr;
        float *s = scT + (size_t)(lr - lo0) * ATTP_QBP + r;
        float mx = -FLT_MAX;
        for (int i = lane; i < len; i += 32) mx = ec_max_keep(mx, s[(size_t)i * ATTP_QBP]);
        mx = ec_warp_max(mx);
        double sum = 0.0;
        for (int i = lane; i < len; i += 32) {
            const float e = ec_expf(__fsub_rn(s[(size_t)i * ATTP_QBP], mx));
            s[(size_t)i * ATTP_QBP] = e;
            sum = __dadd_rn(sum, (double)e);
        }
        sum = ec_warp_sum_d(sum);
        const double isum = __ddiv_rn(1.0, sum);
        __syncwarp();
        for (int i = lane; i < len; i += 32) s[(size_t)i * ATTP_QBP] = (float)__dmul_rn((double)s[(size_t)i * ATTP_QBP], isum);
    }

    // P.V: thread (rows 8*rq .. 8*rq + 7; dimensions d0 and d0 + 64), positions ascending
    const int rq = threadIdx.x >> 6, d0 = threadIdx.x & 63;
    int lor[8], hir[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int r = 8 * rq + j, pr = pos0 + r;
        int lr = 0;
        if (a.window > 0) { lr = pr - a.window + 1; if (lr < 0) lr = 0; }
        lor[j] = lr;
        hir[j] = r < nr ? pr : -1;
    }
    const int tfull = a.window > 0 ? -1 : pos0 + 8 * rq;   // every row of the thread active up to here
    float o[2][8];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int j = 0; j < 8; ++j) o[u][j] = 0.0f;
    for (int c0 = lo0; c0 <= pend; c0 += ATTP_KCH) {
        const int n = min(ATTP_KCH, pend + 1 - c0);
        __syncthreads();   // weights final / the previous chunk consumed
        for (int e = threadIdx.x; e < n * per; e += blockDim.x) {
            const int i = e / per, j = e - i * per;
            const uint16_t *src = vb + ec_kv_row(geo.pt, geo.mp, slot, c0 + i) * geo.kv + 8 * j;
            *reinterpret_cast<uint4 *>(vch + (size_t)i * hd + 8 * j) = __ldg(reinterpret_cast<const uint4 *>(src));
        }
        __syncthreads();
        if (8 * rq >= nr) continue;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int d = d0 + 64 * u;
            if (d >= hd) break;
            for (int i = 0; i < n; ++i) {
                const int t = c0 + i;
                const float *wp = scT + (size_t)(t - lo0) * ATTP_QBP + 8 * rq;
                const float4 w0 = *reinterpret_cast<const float4 *>(wp);
                const float4 w1 = *reinterpret_cast<const float4 *>(wp + 4);
                const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                const float v = __half2float(__ushort_as_half(vch[(size_t)i * hd + d]));
                if (t <= tfull) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) o[u][j] = __fadd_rn(o[u][j], __fmul_rn(w[j], v));
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (t >= lor[j] && t <= hir[j]) o[u][j] = __fadd_rn(o[u][j], __fmul_rn(w[j], v));
                }
            }
        }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int d = d0 + 64 * u;
        if (d >= hd) break;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int r = 8 * rq + j;
            if (r < nr) a.out[(size_t)(r0 + r) * a.ldo + (size_t)h * hd + d] = o[u][j];
        }
    }
}

static int g_attx_max_smem = 0;

extern "C" int ec_attention_exact_fits(int H, int KVH, int hd, int maxlen) {
    if (KVH <= 0 || H % KVH) return 0;
    const int G = H / KVH;
    if (G > ATTX_MAX_GROUP || maxlen < 1 || G * hd > ATTX_OPT * ATTX_THREADS) return 0;
    if (g_attx_max_smem == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_attx_max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaFuncSetAttribute(k_attn_exact, cudaFuncAttributeMaxDynamicSharedMemorySize, g_attx_max_smem);
    }
    return attx_smem_bytes(G, hd, maxlen) <= (size_t)g_attx_max_smem;
}

static int g_attp_max_smem = 0;

// 1 if k_attn_prefill takes this geometry (hd % 8 == 0 checked by the caller).
static int attp_fits(const ec_attn_args *a) {
    if (a->geo.hd > 128 || a->KVH <= 0 || a->H % a->KVH || a->maxlen < 1) return 0;
    if (g_attp_max_smem == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_attp_max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (cudaFuncSetAttribute(k_attn_prefill, cudaFuncAttributeMaxDynamicSharedMemorySize, g_attp_max_smem) !=
            cudaSuccess) {
            cudaGetLastError();
            g_attp_max_smem = 48 * 1024;   // the default limit stays
        }
    }
    return attp_smem_bytes(a->geo.hd, attp_span_cap(a->maxlen)) <= (size_t)g_attp_max_smem;
}

static int g_attn_force_split = 0;

extern "C" void ec_attention_set_force_split(int on) { g_attn_force_split = on != 0; }

extern "C" int ec_launch_attention(const ec_attn_args *a, cudaStream_t stream) {
    if (a->M <= 0) return 0;
    if (a->geo.hd > 256 || a->geo.hd % 8 || a->nsplit < 1) return (int)cudaErrorInvalidValue;
    if (!g_attn_force_split && a->blocks && a->nblocks > 0 && attp_fits(a)) {
        dim3 g(a->H, a->nblocks);
        k_attn_prefill<<<g, ATTP_THREADS, attp_smem_bytes(a->geo.hd, attp_span_cap(a->maxlen)), stream>>>(*a);
        return (int)cudaGetLastError();
    }
    if (!g_attn_force_split && ec_attention_exact_fits(a->H, a->KVH, a->geo.hd, a->maxlen)) {
        // few rows: one CTA per query head (its KV rows are read once per
        // head instead of once per group) so that the grid fills the GPU
        static int sms = 0;
        if (!sms) {
            int dev = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        }
        ec_attn_args b = *a;
        b.per_head = a->M * a->KVH < sms && a->H > a->KVH;   // measured: 32 rows 0.47 -> 0.39 ms per step; 128 rows slower
        const int G = b.per_head ? 1 : a->H / a->KVH;
        dim3 g(b.per_head ? a->H : a->KVH, a->M);
        k_attn_exact<<<g, ATTX_THREADS, attx_smem_bytes(G, a->geo.hd, a->maxlen), stream>>>(b);
        return (int)cudaGetLastError();
    }
    dim3 g1(a->nsplit, a->H, a->M);
    k_attn_part<<<g1, ATT_THREADS, 0, stream>>>(*a);
    dim3 g2(a->H, a->M);
    k_attn_combine<<<g2, 128, 0, stream>>>(*a);
    return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Argmax (lowest index among equal maxima) and decode bookkeeping
// ---------------------------------------------------------------------------

EC_DEV void argmax_merge(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

__global__ void __launch_bounds__(256) k_argmax_part(const float *logits, int ld, int N, int nchunk, float2 *part) {
    EC_PDL_ENTER();
    __shared__ float sv[8];
    __shared__ int si[8];
    const int c = blockIdx.x, m = blockIdx.y;
    const int per = (N + nchunk - 1) / nchunk;
    const int b = c * per, e = min(N, b + per);
    const float *row = logits + (size_t)m * ld;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = b + threadIdx.x; i < e; i += blockDim.x) argmax_merge(bv, bi, row[i], i);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, ov, oi);
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        bv = sv[0]; bi = si[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) argmax_merge(bv, bi, sv[w], si[w]);
        part[(size_t)m * nchunk + c] = make_float2(bv, __int_as_float(bi));
    }
}

__global__ void k_argmax_final(const float2 *part, int nchunk, int M, int id_base, int *ids, float *maxv) {
    EC_PDL_ENTER();
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= M) return;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = 0; c < nchunk; ++c) {
        const float2 p = part[(size_t)m * nchunk + c];
        argmax_merge(bv, bi, p.x, __float_as_int(p.y));
    }
    if (bi == 0x7fffffff) bi = 0;   // all NaN / empty: the reference keeps index 0
    if (ids) ids[m] = bi + id_base;
    if (maxv) maxv[m] = bv;
}

extern "C" int ec_launch_argmax(int *ids, float *maxv, const float *logits, int ld, int N, int M,
                                int id_base, void *part, int nchunk, cudaStream_t stream) {
    if (M <= 0) return 0;
    dim3 g(nchunk, M);
    k_argmax_part<<<g, 256, 0, stream>>>(logits, ld, N, nchunk, static_cast<float2 *>(part));
    k_argmax_final<<<(M + 127) / 128, 128, 0, stream>>>(static_cast<const float2 *>(part), nchunk, M, id_base, ids, maxv);
    return (int)cudaGetLastError();
}

extern "C" int ec_launch_argmax_final(int *ids, float *maxv, const void *part, int nchunk, int M, int id_base,
                                      cudaStream_t stream) {
    if (M <= 0) return 0;
    k_argmax_final<<<(M + 127) / 128, 128, 0, stream>>>(static_cast<const float2 *>(part), nchunk, M, id_base, ids, maxv);
    return (int)cudaGetLastError();
}

__global__ void k_step_advance(int *tok, int *pos, const int *ids, int M, int *hist, int *counter,
                               int wrap_lo, int wrap_hi) {
    EC_PDL_ENTER();
    const int step = counter ? *counter : 0;
    for (int m = threadIdx.x; m < M; m += blockDim.x) {
        tok[m] = ids[m];
        const int np = pos[m] + 1;
        pos[m] = (wrap_hi > 0 && np >= wrap_hi) ? wrap_lo : np;
        if (hist) hist[(size_t)step * M + m] = ids[m];
    }
    __syncthreads();
    if (threadIdx.x == 0 && counter) *counter = step + 1;
}

extern "C" int ec_launch_step_advance(int *tok, int *pos, const int *ids, int M, int *hist, int *counter,
                                      int wrap_lo, int wrap_hi, cudaStream_t stream) {
    k_step_advance<<<1, 256, 0, stream>>>(tok, pos, ids, M, hist, counter, wrap_lo, wrap_hi);
    return (int)cudaGetLastError();
}

// Signed 64-bit argmax keys: the order-preserving bits of the max logit
// (-0 as +0, NaN below every number) above (0x7fffffff - index), top bit
// flipped, so that the signed max over vocab shards is "larger logit, then
// lower index" -- the reference's greedy tie rule (src/runtime_main.c:213-219).
// Same encoding as ec_argmax_key (ec_host.c) with the sign bit flipped.
__device__ __forceinline__ long long argmax_key(float v, int idx) {
    if (v == 0.0f) v = 0.0f;
    uint32_t b = __float_as_uint(v);
    if (v != v) b = 0u;
    else b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    const unsigned long long k = ((unsigned long long)b << 32) | (uint32_t)(0x7fffffff - idx);
    return (long long)(k ^ 0x8000000000000000ull);
}

__global__ void k_pack_keys(const int *ids, const float *maxv, int M, long long *keys) {
    EC_PDL_ENTER();
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m < M) keys[m] = argmax_key(maxv[m], ids[m]);
}

extern "C" int ec_launch_pack_keys(const int *ids, const float *maxv, int M, long long *keys, cudaStream_t stream) {
    k_pack_keys<<<(M + 255) / 256, 256, 0, stream>>>(ids, maxv, M, keys);
    return (int)cudaGetLastError();
}

// tok[m] = the index in keys[m], pos[m] += 1; optionally ids[m] = the index.
__global__ void k_keys_advance(const long long *keys, int M, int *tok, int *pos, int *ids) {
    EC_PDL_ENTER();
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= M) return;
    const unsigned long long k = (unsigned long long)keys[m] ^ 0x8000000000000000ull;
    const int id = 0x7fffffff - (int)(uint32_t)(k & 0xffffffffu);
    tok[m] = id;
    if (pos) pos[m] += 1;
    if (ids) ids[m] = id;
}

extern "C" int ec_launch_keys_advance(const long long *keys, int M, int *tok, int *pos, int *ids,
                                      cudaStream_t stream) {
    k_keys_advance<<<(M + 255) / 256, 256, 0, stream>>>(keys, M, tok, pos, ids);
    return (int)cudaGetLastError();
}

__global__ void k_reference_math(const float *x, float *e, float *t, int n) {
    EC_PDL_ENTER();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        if (e) e[i] = ec_expf(x[i]);
        if (t) t[i] = ec_tanhf(x[i]);
    }
}

extern "C" int ec_launch_reference_math(const float *x, float *e, float *t, int n, cudaStream_t stream) {
    if (n <= 0) return 0;
    const int grid = (n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096;
    k_reference_math<<<grid, 256, 0, stream>>>(x, e, t, n);
    return (int)cudaGetLastError();
}

extern "C" int ec_kernel_error_take(cudaStream_t stream, int *code) {
    int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(code, g_ec_err, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return (int)e;
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return (int)e;
    if (*code) e = cudaMemcpyToSymbolAsync(g_ec_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess && !*code) e = (cudaError_t)ec_tc_error_take(code);
    return (int)e;
}
