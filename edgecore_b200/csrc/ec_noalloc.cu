// ec_noalloc.cu -- ec_linear_int8_noalloc: the W8A8 linear of ec_linear_int8
// for device operands, with its activation scratch in a fixed, statically
// allocated device buffer instead of memory obtained at call time.
//
// Why a caller may be unable to allocate: a serving process usually hands
// nearly all of HBM to a caching allocator up front (PyTorch's reserves it
// for tensors), so a cudaMalloc on the request path can fail even though the
// op itself needs only a few MB; and cudaMalloc / cudaFree synchronise the
// device, which stalls every other stream of a latency-sensitive decode
// loop.  Such callers need an op whose device memory footprint is fixed
// when the library is loaded.
//
// Contract:
//  * All of C, X, W, w_scale (and bias, if given) are device pointers of the
//    current device; K is a multiple of 16 (W rows are read in place).
//  * Scratch: EC_NOALLOC_SCRATCH_BYTES (4 MiB) per device, holding the
//    per-row activation scales (M floats, padded to 256 bytes) and the
//    int8 activation rows (M x K bytes).  Larger M*K is rejected with an
//    error, before anything is launched.  Nothing in the scratch has to start
//    at zero: the quantisation kernel writes every scale and every byte of
//    every row before the GEMV / GEMM reads them.
//  * The first call on each device does the set-up: it looks up the scratch
//    address with cudaGetSymbolAddress, sets the shared-memory attributes of
//    the GEMV and of the tensor-core GEMMs and resolves the driver's
//    tensor-map encoder, and the CUDA runtime loads the kernels it launches.
//    Make that first call before starting any stream capture on that device.
//  * M < 8 runs the weight-streaming GEMV when one staged W row plus the M
//    int8 activation rows fit the GEMV's shared memory (K up to about
//    113,000 at M = 1, 28,000 at M = 7); otherwise, and for M >= 8, the
//    GEMM kernels run (tcgen05 tensor cores from 8 rows).
//  * Device-side failures (a bounded wait that gave up inside a kernel) are
//    not visible in the return code, which only covers the checks and the
//    launches: after synchronising the stream, ec_device_error_take() reads
//    and clears the library's device error words.
//  * The work is enqueued on `stream` and the call returns without waiting.
//    There is ONE scratch buffer per device: calls whose work can overlap on
//    the device (different streams without ordering between them, or several
//    host threads) race on it and corrupt each other's activations.  Order
//    them on one stream or with events.
#include "ec_launch.h"

#include <cuda_runtime_api.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#define EC_NOALLOC_SCRATCH_BYTES (4u << 20)
#define EC_NOALLOC_MAX_DEV 16

// The scratch: file scope, fixed size, part of the module image on every
// device the library runs on.
static __device__ __align__(256) unsigned char g_noalloc_scratch[EC_NOALLOC_SCRATCH_BYTES];

namespace {

pthread_mutex_t g_setup_mu = PTHREAD_MUTEX_INITIALIZER;
unsigned char *g_scratch_ptr[EC_NOALLOC_MAX_DEV];
int g_sms[EC_NOALLOC_MAX_DEV];

bool is_device_ptr(const void *p, int dev) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice && at.device == dev;
}

int fail(const char *msg) {
    ec_set_error_text(msg);
    return -1;
}

// Text for a code returned by the launch helpers (cudaError_t values).
void code_text(char *buf, size_t n, int code) {
    const char *name = cudaGetErrorName((cudaError_t)code);
    snprintf(buf, n, "CUDA error %d (%s: %s)", code, name ? name : "?",
             cudaGetErrorString((cudaError_t)code));
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int ec_linear_int8_noalloc(
    float *C, const float *X, const int8_t *W, const float *w_scale, const float *bias, int M, int K, int N,
    void *stream) {
    char msg[256];
    if (M <= 0 || N <= 0) return 0;
    if (K <= 0 || K % 16 != 0) {
        snprintf(msg, sizeof msg, "ec_linear_int8_noalloc: K=%d must be a positive multiple of 16", K);
        return fail(msg);
    }
    const size_t scale_bytes = ((size_t)M * 4 + 255) & ~(size_t)255;
    const size_t need = scale_bytes + (size_t)M * (size_t)K;
    if (need > EC_NOALLOC_SCRATCH_BYTES) {
        snprintf(msg, sizeof msg,
                 "ec_linear_int8_noalloc: M=%d x K=%d needs %zu bytes of scratch, above the fixed %u bytes "
                 "(M*K + 4*M rounded up to 256 must fit)",
                 M, K, need, EC_NOALLOC_SCRATCH_BYTES);
        return fail(msg);
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= EC_NOALLOC_MAX_DEV) {
        cudaGetLastError();
        return fail("ec_linear_int8_noalloc: no usable CUDA device");
    }
    if (!is_device_ptr(C, dev) || !is_device_ptr(X, dev) || !is_device_ptr(W, dev) || !is_device_ptr(w_scale, dev) ||
        (bias && !is_device_ptr(bias, dev)))
        return fail("ec_linear_int8_noalloc: C, X, W, w_scale and bias must be device memory of the current device");

    // per-device set-up, once
    pthread_mutex_lock(&g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        int e = (int)cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e == 0) e = (int)cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e == 0) e = ec_kernels_init();
        if (e == 0) {
            e = ec_tc_init();
            if (e == (int)cudaErrorNotSupported) e = 0;   // no encoder: the GEMM falls back to SIMT kernels
        }
        if (e != 0) {
            pthread_mutex_unlock(&g_setup_mu);
            char ct[160];
            code_text(ct, sizeof ct, e);
            snprintf(msg, sizeof msg, "ec_linear_int8_noalloc: set-up failed: %s", ct);
            return fail(msg);
        }
        g_scratch_ptr[dev] = static_cast<unsigned char *>(p);
    }
    unsigned char *scr = g_scratch_ptr[dev];
    const int sms = g_sms[dev];
    pthread_mutex_unlock(&g_setup_mu);

    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float *a_scale = reinterpret_cast<float *>(scr);
    int8_t *aq = reinterpret_cast<int8_t *>(scr + scale_bytes);
    int e = ec_launch_quant(aq, a_scale, X, K, M, K, K, st);
    if (e == 0) {
        ec_gemv_args g;
        memset(&g, 0, sizeof g);
        bool gemv = false;
        if (M < EC_TC_MIN_M) {
            g.W = W; g.wscale = w_scale; g.bias = bias;
            g.wt = EC_W_I8; g.N = N; g.K = K; g.Kp = K; g.ldw = K;
            int R = (N + 2 * sms - 1) / (2 * sms);   // about two row blocks per SM
            int maxr = (32 * 1024) / K;
            if (maxr < 1) maxr = 1;
            if (R > maxr) R = maxr;
            if (R > 128) R = 128;
            if (R < 1) R = 1;
            g.block_rows = R;
            g.nblocks = (N + R - 1) / R;
            g.Xq = aq; g.xscale = a_scale; g.ldx = K;
            g.M = M; g.out = C; g.ldo = N; g.epi = EC_EPI_STORE;
            gemv = ec_gemv_fits(&g) != 0;   // long rows: the GEMM below instead
        }
        if (gemv) {
            e = ec_launch_gemv(&g, sms, st);
        } else {
            ec_gemm_args g;
            memset(&g, 0, sizeof g);
            g.W = W; g.wscale = w_scale; g.bias = bias;
            g.wt = EC_W_I8; g.N = N; g.K = K; g.Kp = K; g.ldw = K; g.M = M;
            g.Aq = aq; g.a_scale = a_scale;
            g.out = C; g.ldo = N; g.epi = EC_EPI_STORE;
            e = ec_launch_gemm(&g, st);
        }
    }
    if (e != 0) {
        char ct[160];
        code_text(ct, sizeof ct, e);
        snprintf(msg, sizeof msg, "ec_linear_int8_noalloc: launch failed: %s", ct);
        return fail(msg);
    }
    return 0;
}
