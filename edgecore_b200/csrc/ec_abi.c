/*
 * ec_abi.c -- the standalone GEMM entry points of the reference ABI
 * (gemm_fp16_fp32, gemm_bf16_fp32, gemm_int8: reference src/edgecore.h:119-136,
 * src/kernels.c:129-168) and the op-level extensions ec_quantize_rows /
 * ec_linear_int8, on the GPU.
 *
 * Operands may be host or device pointers; each is classified per call.  Host
 * operands (and device weights whose row length is not a multiple of 16
 * elements) are staged into per-device scratch buffers.  Work runs on the
 * legacy default stream, so it is ordered after the caller's default-stream
 * work, and every call returns with C complete, as the CPU version does.
 */
#include "edgecore.h"
#include "edgecore_b200.h"
#include "ec_launch.h"

#include <cuda_runtime_api.h>
#include <pthread.h>

#define EC_EXPORT __attribute__((visibility("default")))
#define EC_MAX_DEV 16

enum { S_A, S_AS, S_B, S_BS, S_BIAS, S_C, S_Q, S_QS, S_SPLIT, S_N };

static pthread_mutex_t g_abi_mu = PTHREAD_MUTEX_INITIALIZER;
static struct { void *p[S_N]; size_t cap[S_N]; int sms; } g_scr[EC_MAX_DEV];

static int is_device_ptr(const void *p)
{
    if (!p) return 0;
    struct cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

static void *scratch(int dev, int slot, size_t bytes)
{
    if (g_scr[dev].cap[slot] < bytes) {
        cudaFree(g_scr[dev].p[slot]);
        g_scr[dev].p[slot] = NULL;
        g_scr[dev].cap[slot] = 0;
        if (cudaMalloc(&g_scr[dev].p[slot], bytes) != cudaSuccess) return NULL;
        g_scr[dev].cap[slot] = bytes;
    }
    return g_scr[dev].p[slot];
}

static int round16(int k) { return (k + 15) & ~15; }

typedef struct {
    int dev;
    char err[256];
} abi_ctx;

static int ctx_init(abi_ctx *c)
{
    c->err[0] = 0;
    if (cudaGetDevice(&c->dev) != cudaSuccess || c->dev < 0 || c->dev >= EC_MAX_DEV) {
        snprintf(c->err, sizeof c->err, "no usable CUDA device");
        return -1;
    }
    if (!g_scr[c->dev].sms) cudaDeviceGetAttribute(&g_scr[c->dev].sms, cudaDevAttrMultiProcessorCount, c->dev);
    return 0;
}

#define ACK(call)                                                                              \
    do {                                                                                       \
        cudaError_t e_ = (cudaError_t)(call);                                                  \
        if (e_ != cudaSuccess) {                                                               \
            snprintf(c->err, sizeof c->err, "%s: %s", #call, cudaGetErrorString(e_));          \
            return -1;                                                                         \
        }                                                                                      \
    } while (0)

/* Device view of a dense [rows][cols] operand with row stride ld_out elements
 * (elt bytes each); copies when the operand is on the host or has the wrong
 * stride. */
static int dev_view(abi_ctx *c, int slot, const void *src, int rows, int cols, int ld_out, int elt,
                    const void **out)
{
    if (!src) { *out = NULL; return 0; }
    if (is_device_ptr(src) && cols == ld_out) { *out = src; return 0; }
    void *dst = scratch(c->dev, slot, (size_t)rows * ld_out * elt + 16);
    if (!dst) { snprintf(c->err, sizeof c->err, "scratch allocation failed"); return -1; }
    if (ld_out != cols) ACK(cudaMemsetAsync(dst, 0, (size_t)rows * ld_out * elt, 0));
    ACK(cudaMemcpy2DAsync(dst, (size_t)ld_out * elt, src, (size_t)cols * elt, (size_t)cols * elt, (size_t)rows,
                          cudaMemcpyDefault, 0));
    *out = dst;
    return 0;
}

/* Weight-side linear over [N][Kp] with the GEMV (M < EC_TC_MIN_M) or GEMM kernels. */
static int run_linear(abi_ctx *c, int wt, float *C, const float *X, const int8_t *Aq, const float *a_scale,
                      const void *B, const float *b_scale, const float *bias, int M, int K, int N, int quantise)
{
    const int Kp = round16(K);
    const int elt = wt == EC_W_I8 ? 1 : 2;
    const void *dB, *dbs = NULL, *dbias = NULL;
    if (dev_view(c, S_B, B, N, K, Kp, elt, &dB)) return -1;
    if (b_scale && dev_view(c, S_BS, b_scale, 1, N, N, 4, &dbs)) return -1;
    if (bias && dev_view(c, S_BIAS, bias, 1, N, N, 4, &dbias)) return -1;
    float *dC = C;
    const int c_dev = is_device_ptr(C);
    if (!c_dev) {
        dC = scratch(c->dev, S_C, (size_t)M * N * 4);
        if (!dC) { snprintf(c->err, sizeof c->err, "scratch allocation failed"); return -1; }
    }
    for (int m0 = 0; m0 < M;) {
        int rows = M - m0;
        if (M < EC_TC_MIN_M) {
            ec_gemv_args g;
            memset(&g, 0, sizeof g);
            g.W = dB; g.wscale = dbs; g.bias = dbias; g.wt = wt; g.N = N; g.K = K; g.Kp = Kp;
            int R = (N + 2 * g_scr[c->dev].sms - 1) / (2 * g_scr[c->dev].sms);
            int maxr = (32 * 1024) / (Kp * elt);
            if (maxr < 1) maxr = 1;
            if (R > maxr) R = maxr;
            if (R > 128) R = 128;
            if (R < 1) R = 1;
            g.blocks = NULL; g.block_rows = R; g.nblocks = (N + R - 1) / R;
            g.M = rows; g.out = dC; g.ldo = N; g.epi = EC_EPI_STORE;
            if (wt == EC_W_I8 && !quantise) {
                const void *dA, *das;
                if (dev_view(c, S_A, Aq, M, K, K, 1, &dA) || dev_view(c, S_AS, a_scale, 1, M, M, 4, &das)) return -1;
                g.Xq = dA; g.xscale = das; g.ldx = K;
            } else {
                const void *dX;
                if (dev_view(c, S_A, X, M, K, K, 4, &dX)) return -1;
                g.X = dX; g.ldx = K;
            }
            if (ec_gemv_fits(&g)) {   /* else rows too long for its shared memory: the GEMM below */
                ACK(ec_launch_gemv(&g, g_scr[c->dev].sms, 0));
                m0 += rows;
                continue;
            }
        }
        ec_gemm_args g;
        memset(&g, 0, sizeof g);
        g.W = dB; g.wscale = dbs; g.bias = dbias; g.wt = wt; g.N = N; g.K = K; g.Kp = Kp; g.M = M;
        g.out = dC; g.ldo = N; g.epi = EC_EPI_STORE;
        if (wt == EC_W_I8) {
            const void *dA, *das;
            if (quantise) {
                const void *dX;
                if (dev_view(c, S_A, X, M, K, K, 4, &dX)) return -1;
                int8_t *q = scratch(c->dev, S_Q, (size_t)M * Kp);
                float *qs = scratch(c->dev, S_QS, (size_t)M * 4);
                if (!q || !qs) { snprintf(c->err, sizeof c->err, "scratch allocation failed"); return -1; }
                ACK(ec_launch_quant(q, qs, dX, K, M, K, Kp, 0));
                dA = q;
                das = qs;
            } else {
                if (dev_view(c, S_A, Aq, M, K, Kp, 1, &dA) || dev_view(c, S_AS, a_scale, 1, M, M, 4, &das)) return -1;
            }
            g.Aq = dA; g.a_scale = das;
        } else {
            const void *dX;
            if (dev_view(c, S_A, X, M, K, K, 4, &dX)) return -1;
            g.X = dX; g.ldx = K;
            if (M >= EC_TC_MIN_M) {   /* tensor cores: activation parts workspace */
                g.split_bytes = ec_gemm_tc_split_bytes(wt, M, Kp);
                g.split = scratch(c->dev, S_SPLIT, g.split_bytes);
                if (!g.split) g.split_bytes = 0;
            }
        }
        ACK(ec_launch_gemm(&g, 0));
        m0 = M;
    }
    if (!c_dev) ACK(cudaMemcpyAsync(C, dC, (size_t)M * N * 4, cudaMemcpyDeviceToHost, 0));
    ACK(cudaStreamSynchronize(0));
    int code = 0;
    ACK(ec_kernel_error_take(0, &code));
    if (code) { snprintf(c->err, sizeof c->err, "kernel error code %d", code); return -1; }
    return 0;
}

EC_EXPORT int ec_gemm_async(int wt, float *C, const void *A, const float *a_scale, const void *B,
                            const float *b_scale, const float *bias, int M, int K, int N, void *stream)
{
    if (M <= 0 || N <= 0) return 0;
    char msg[200];
    if ((wt != EC_W_I8 && wt != EC_W_F16 && wt != EC_W_BF16) || K <= 0 || K % 16) {
        snprintf(msg, sizeof msg, "ec_gemm_async: wt=%d K=%d (wt 0/1/2, K a positive multiple of 16)", wt, K);
        ec_set_error_text(msg);
        return -1;
    }
    if (!is_device_ptr(C) || !is_device_ptr(A) || !is_device_ptr(B) || (b_scale && !is_device_ptr(b_scale)) ||
        (bias && !is_device_ptr(bias)) || (wt == EC_W_I8 && !is_device_ptr(a_scale))) {
        ec_set_error_text("ec_gemm_async: all operands must be device memory");
        return -1;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= EC_MAX_DEV) {
        cudaGetLastError();
        ec_set_error_text("ec_gemm_async: no usable CUDA device");
        return -1;
    }
    pthread_mutex_lock(&g_abi_mu);
    if (!g_scr[dev].sms) cudaDeviceGetAttribute(&g_scr[dev].sms, cudaDevAttrMultiProcessorCount, dev);
    const int sms = g_scr[dev].sms;
    cudaStream_t st = (cudaStream_t)stream;
    int e = 0;
    ec_gemv_args v;
    memset(&v, 0, sizeof v);
    v.W = B; v.wscale = b_scale; v.bias = bias; v.wt = wt; v.N = N; v.K = K; v.Kp = K; v.ldw = K;
    v.M = M; v.out = C; v.ldo = N; v.epi = EC_EPI_STORE;
    if (wt == EC_W_I8) { v.Xq = (const int8_t *)A; v.xscale = a_scale; v.ldx = K; }
    else { v.X = (const float *)A; v.ldx = K; }
    if (M < EC_TC_MIN_M && ec_gemv_fits(&v)) {   /* from EC_TC_MIN_M rows the tensor cores are faster */
        e = ec_launch_gemv(&v, sms, st);
    } else {
        ec_gemm_args g;
        memset(&g, 0, sizeof g);
        g.W = B; g.wscale = b_scale; g.bias = bias; g.wt = wt; g.N = N; g.K = K; g.Kp = K; g.ldw = K; g.M = M;
        g.out = C; g.ldo = N; g.epi = EC_EPI_STORE;
        if (wt == EC_W_I8) {
            g.Aq = (const int8_t *)A; g.a_scale = a_scale;
        } else {
            g.X = (const float *)A; g.ldx = K;
            if (M >= EC_TC_MIN_M) {   /* tensor cores: activation parts workspace (allocated once, cached) */
                g.split_bytes = ec_gemm_tc_split_bytes(wt, M, K);
                g.split = scratch(dev, S_SPLIT, g.split_bytes);
                if (!g.split) g.split_bytes = 0;
            }
        }
        e = ec_launch_gemm(&g, st);
    }
    pthread_mutex_unlock(&g_abi_mu);
    if (e) {
        snprintf(msg, sizeof msg, "ec_gemm_async: launch failed: CUDA error %d (%s)", e, cudaGetErrorString((cudaError_t)e));
        ec_set_error_text(msg);
        return -1;
    }
    return 0;
}

EC_EXPORT int ec_reference_math(const float *d_x, float *d_exp, float *d_tanh, int n, void *stream)
{
    const int e = ec_launch_reference_math(d_x, d_exp, d_tanh, n, (cudaStream_t)stream);
    if (e) {
        ec_set_error_text("ec_reference_math: launch failed");
        return -1;
    }
    return 0;
}

EC_EXPORT int ec_attention_force_split(int on)
{
    ec_attention_set_force_split(on);
    return 0;
}

EC_EXPORT int ec_device_error_take(void *stream, int *code)
{
    if (!code) { ec_set_error_text("ec_device_error_take: code must not be NULL"); return -1; }
    *code = 0;
    const int e = ec_kernel_error_take((cudaStream_t)stream, code);
    if (e) {
        char msg[160];
        snprintf(msg, sizeof msg, "ec_device_error_take: CUDA error %d (%s)", e, cudaGetErrorString((cudaError_t)e));
        ec_set_error_text(msg);
        return -1;
    }
    return 0;
}

static void abi_fail(const char *fn, const abi_ctx *c)
{
    fprintf(stderr, "edgecore_b200: %s: %s\n", fn, c->err);
    abort();
}

EC_EXPORT void gemm_fp16_fp32(float *C, const float *A, const uint16_t *B, int M, int K, int N)
{
    if (M <= 0 || N <= 0) return;
    abi_ctx c;
    pthread_mutex_lock(&g_abi_mu);
    int rc = ctx_init(&c) || run_linear(&c, EC_W_F16, C, A, NULL, NULL, B, NULL, NULL, M, K, N, 0);
    pthread_mutex_unlock(&g_abi_mu);
    if (rc) abi_fail("gemm_fp16_fp32", &c);
}

EC_EXPORT void gemm_bf16_fp32(float *C, const float *A, const uint16_t *B, int M, int K, int N)
{
    if (M <= 0 || N <= 0) return;
    abi_ctx c;
    pthread_mutex_lock(&g_abi_mu);
    int rc = ctx_init(&c) || run_linear(&c, EC_W_BF16, C, A, NULL, NULL, B, NULL, NULL, M, K, N, 0);
    pthread_mutex_unlock(&g_abi_mu);
    if (rc) abi_fail("gemm_bf16_fp32", &c);
}

EC_EXPORT void gemm_int8(float *C, const int8_t *A, const float *a_scale, const int8_t *B, const float *b_scale,
                         const float *bias, int M, int K, int N)
{
    if (M <= 0 || N <= 0) return;
    abi_ctx c;
    pthread_mutex_lock(&g_abi_mu);
    int rc = ctx_init(&c) || run_linear(&c, EC_W_I8, C, NULL, A, a_scale, B, b_scale, bias, M, K, N, 0);
    pthread_mutex_unlock(&g_abi_mu);
    if (rc) abi_fail("gemm_int8", &c);
}

EC_EXPORT int ec_linear_int8(float *C, const float *X, const int8_t *W, const float *w_scale, const float *bias,
                             int M, int K, int N)
{
    if (M <= 0 || N <= 0) return 0;
    abi_ctx c;
    pthread_mutex_lock(&g_abi_mu);
    int rc = ctx_init(&c) || run_linear(&c, EC_W_I8, C, X, NULL, NULL, W, w_scale, bias, M, K, N, 1);
    pthread_mutex_unlock(&g_abi_mu);
    if (rc) {
        fprintf(stderr, "edgecore_b200: ec_linear_int8: %s\n", c.err);
        return -1;
    }
    return 0;
}

EC_EXPORT int ec_quantize_rows(int8_t *q, float *scale, const float *x, int M, int K)
{
    if (M <= 0) return 0;
    abi_ctx c;
    int rc = 0;
    pthread_mutex_lock(&g_abi_mu);
    if (ctx_init(&c)) {
        rc = -1;
    } else {
        const void *dX = NULL;
        int8_t *dq = q;
        float *ds = scale;
        const int qd = is_device_ptr(q), sd = is_device_ptr(scale);
        if (dev_view(&c, S_A, x, M, K, K, 4, &dX)) rc = -1;
        if (!rc && !qd) dq = scratch(c.dev, S_Q, (size_t)M * K + 16);
        if (!rc && !sd) ds = scratch(c.dev, S_QS, (size_t)M * 4);
        if (!rc && (!dq || !ds)) { snprintf(c.err, sizeof c.err, "scratch allocation failed"); rc = -1; }
        if (!rc && ec_launch_quant(dq, ds, dX, K, M, K, K, 0)) { snprintf(c.err, sizeof c.err, "launch failed"); rc = -1; }
        if (!rc && !qd && cudaMemcpyAsync(q, dq, (size_t)M * K, cudaMemcpyDeviceToHost, 0)) rc = -1;
        if (!rc && !sd && cudaMemcpyAsync(scale, ds, (size_t)M * 4, cudaMemcpyDeviceToHost, 0)) rc = -1;
        if (!rc && cudaStreamSynchronize(0) != cudaSuccess) { snprintf(c.err, sizeof c.err, "sync failed"); rc = -1; }
    }
    pthread_mutex_unlock(&g_abi_mu);
    if (rc) fprintf(stderr, "edgecore_b200: ec_quantize_rows: %s\n", c.err);
    return rc;
}
