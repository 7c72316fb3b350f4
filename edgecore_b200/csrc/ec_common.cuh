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

// L2 policy for data read once per pass (weight streams): evicted first, so
// that the KV cache and the activations exchanged between SMs stay in L2.
EC_DEV uint64_t ec_l2_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// ec_bulk_g2s with an L2 cache policy.
EC_DEV void ec_bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(ec_smem_u32(dst)), "l"(src), "r"(bytes), "r"(ec_smem_u32(bar)), "l"(pol) : "memory");
}

// 16 bytes of read-only data read once: no L1 allocation, 256-byte L2 fetch.
EC_DEV uint4 ec_ldg_stream16(const void *p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// ec_ldg_stream16 under an L2 cache policy.
EC_DEV uint4 ec_ldg_stream16_hint(const void *p, uint64_t pol) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p), "l"(pol));
    return v;
}

// Transposed warp sum of each of the V per-lane values: values are halved
// between lane pairs at offsets 16, 8, ... (each lane keeps one half and adds
// its partner's copy of it), so V values cost V-1 shuffles plus one per
// remaining offset.  Every value is summed by the same xor tree 16, 8, 4, 2, 1
// (pair sums are commutative), so a value's total does not depend on the
// slot it sits in.  Lane L ends with the total of value ec_tr_vidx<V>(L);
// lanes differing only in their low log2(32/V) bits hold the same total.
template <int V, typename T>
EC_DEV T ec_tr_reduce(T (&a)[V], int lane) {
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
EC_DEV int ec_tr_vidx(int lane) {
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

// fp32 dot contribution of one 16-byte chunk of 16-bit weights (8 elements,
// in element order) with its activations x0 (elements 0-3) and x1 (4-7).
template <bool BF16>
EC_DEV float ec_dot8(const uint4 w, const float4 x0, const float4 x1, float t) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (BF16) {
            f[2 * i] = __uint_as_float(u[i] << 16);
            f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
        } else {
            const float2 h = __half22float2(*reinterpret_cast<const __half2 *>(&u[i]));
            f[2 * i] = h.x;
            f[2 * i + 1] = h.y;
        }
    }
    t = fmaf(f[0], x0.x, t); t = fmaf(f[1], x0.y, t);
    t = fmaf(f[2], x0.z, t); t = fmaf(f[3], x0.w, t);
    t = fmaf(f[4], x1.x, t); t = fmaf(f[5], x1.y, t);
    t = fmaf(f[6], x1.z, t); t = fmaf(f[7], x1.w, t);
    return t;
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
