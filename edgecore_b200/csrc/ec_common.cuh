// ec_common.cuh -- device helpers shared by the sm_100a kernels: bulk-copy
// (TMA, non-tensor) staging with mbarriers, bounded waits, warp reductions and
// the exact-rounding arithmetic the reference numerics need.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define EC_DEV __device__ __forceinline__

// Error codes written to the library error word (first error wins).
enum { EC_KERR_NONE = 0, EC_KERR_WAIT_TIMEOUT = 1, EC_KERR_BAD_INDEX = 2 };

// Upper bound on mbarrier polls before a wait gives up (~seconds at GPU rates).
#define EC_WAIT_LIMIT (1u << 26)

EC_DEV uint32_t ec_smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

EC_DEV void ec_mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(ec_smem_u32(bar)), "r"(count));
}

EC_DEV void ec_fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Arrive on `bar` announcing `bytes` of transaction traffic to come.
EC_DEV void ec_mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(ec_smem_u32(bar)), "r"(bytes) : "memory");
}

// One bulk global->shared copy (16-byte aligned addresses, size % 16 == 0)
// completing on `bar`.  The global source is this GPU's own memory.
EC_DEV void ec_bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(ec_smem_u32(dst)), "l"(src), "r"(bytes), "r"(ec_smem_u32(bar)) : "memory");
}

EC_DEV bool ec_mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(ec_smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Bounded wait for phase `parity` of `bar`.  Returns false (and records
// EC_KERR_WAIT_TIMEOUT in *err) if the phase never completes.
EC_DEV bool ec_mbar_wait(uint64_t *bar, uint32_t parity, int *err) {
    for (uint32_t i = 0; i < EC_WAIT_LIMIT; ++i)
        if (ec_mbar_try_wait(bar, parity)) return true;
    if (err) atomicCAS(err, 0, EC_KERR_WAIT_TIMEOUT);
    return false;
}

EC_DEV float ec_warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

EC_DEV int ec_warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

EC_DEV double ec_warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// max that never lets a NaN in (mirrors `if (a > m) m = a`).
EC_DEV float ec_max_keep(float m, float a) { return a > m ? a : m; }

EC_DEV float ec_warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = ec_max_keep(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <int WT> struct ec_wtraits;
template <> struct ec_wtraits<0> { typedef int8_t T; static constexpr int kPer16 = 16; };
template <> struct ec_wtraits<1> { typedef __half T; static constexpr int kPer16 = 8; };
template <> struct ec_wtraits<2> { typedef __nv_bfloat16 T; static constexpr int kPer16 = 8; };

EC_DEV float ec_h2f(uint16_t h, bool bf16) {
    return bf16 ? __uint_as_float((uint32_t)h << 16) : __half2float(__ushort_as_half(h));
}

// fp32 -> binary16 bits, round to nearest even (the F16C conversion the
// reference KV store uses).
EC_DEV uint16_t ec_f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Exact reference activation quantisation of one value: lrintf(x / s) clamped.
EC_DEV int ec_quant1(float x, float s) {
    int q = __float2int_rn(__fdiv_rn(x, s));
    return q > 127 ? 127 : (q < -128 ? -128 : q);
}

// ec_quant1 without a division per element: r = 1/s correctly rounded, so
// t = x*r is within 2^-16 of the exact x/s for |x/s| <= 127.5, and so is the
// rounded quotient x/s.  Unless t lies within 2^-12 of a half-integer, both
// round to the same integer; near a tie (or for out-of-range t) the exact
// division decides.
EC_DEV int ec_quant_fast(float x, float s, float r) {
    const float t = __fmul_rn(x, r);
    const float n = rintf(t);
    if (fabsf(fabsf(t - n) - 0.5f) < 0x1p-12f || !(fabsf(t) <= 127.5f)) return ec_quant1(x, s);
    return (int)n;
}

// Correctly rounded fp32 exp and tanh: the fp64 function (error < 1 ulp of
// fp64) rounded once to fp32.  The reference calls the host libm's expf /
// tanhf, which are not correctly rounded; every int8 quantisation downstream
// is discontinuous, so this library pins the rounding of these functions to
// the one well-defined choice and the oracle has a matching build.
EC_DEV float ec_expf(float x) { return __double2float_rn(exp((double)x)); }
EC_DEV float ec_tanhf(float x) { return __double2float_rn(tanh((double)x)); }

// Reference gelu_new (src/gpt2.c:393-396) with its evaluation order kept.
EC_DEV float ec_gelu(float x) {
    float c = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
    float t = ec_tanhf(__fmul_rn(0.7978845608028654f, __fadd_rn(x, c)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}

// Reference SiLU (src/gpt2.c:587-590).
EC_DEV float ec_silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, ec_expf(-x))); }
