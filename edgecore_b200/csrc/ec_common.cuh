// ec_common.cuh -- device helpers shared by the sm_100a kernels: bulk-copy
// (TMA, non-tensor) staging with mbarriers, bounded waits, warp reductions and
// the exact-rounding arithmetic the reference numerics need.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "ec_launch.h"

#define EC_DEV __device__ __forceinline__

// Programmatic dependent launch.  The tensor-core GEMMs (ec_launch_k) may
// start while their predecessor on the stream is still finishing, so that
// their set-up and first weight tiles overlap its tail.  EC_PDL_ENTER()
// waits (griddepcontrol.wait) until the predecessor has completed and its
// writes are visible -- a no-op for a kernel launched without the attribute
// -- and lets the next kernel start early (griddepcontrol.launch_dependents,
// which only matters when that kernel is launched with the attribute).  It
// comes before the kernel's first global-memory access.  Every kernel of the
// library enters through it; only the GEMMs are launched with the attribute
// (per-step batched decode: 1.94 -> 1.84 ms at 32 streams; launching every
// kernel so was slower than launching none).
#define EC_PDL_WAIT() asm volatile("griddepcontrol.wait;" ::: "memory")
#define EC_PDL_NEXT() asm volatile("griddepcontrol.launch_dependents;" ::: "memory")
#define EC_PDL_ENTER() do { EC_PDL_WAIT(); EC_PDL_NEXT(); } while (0)

// Launch with programmatic stream serialisation (see EC_PDL_ENTER); the
// kernel must begin with EC_PDL_ENTER() or EC_PDL_WAIT().
template <typename... KArgs, typename... Args>
static inline cudaError_t ec_launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                      cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

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

// Paged KV arena: a layer's K (or V) cache is [pages][EC_KV_PAGE][kv] fp16,
// and pt[slot * mp + pos / EC_KV_PAGE] is the physical page holding
// positions [64 j, 64 j + 64) of a slot (the host maps pages before every
// launch that touches them; EC_KV_PAGE is 64, ec_launch.h).  Row of (slot,
// pos) in the arena:
EC_DEV size_t ec_kv_row(const int *pt, int mp, int slot, int pos) {
    const int pg = __ldg(pt + (size_t)slot * mp + (pos >> 6));
    return (size_t)(pg < 0 ? 0 : pg) * EC_KV_PAGE + (size_t)(pos & (EC_KV_PAGE - 1));
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

// The reference's exp and tanh.  The reference calls the host C library's
// expf / tanhf (glibc 2.39 on the x86-64 build hosts of this project), which
// are not correctly rounded; every int8 activation quantisation downstream is
// discontinuous, so a last-bit difference in exp can move a W8A8 model's
// residual stream by ~1e-2.  These are restatements of glibc's published
// algorithms, checked bit for bit against the host library on all 2^32 float
// inputs (oracle/libm_check.c):
//  * expf: ARM optimized-routines (glibc sysdeps/ieee754/flt-32/e_expf.c):
//    k = round(x * 32/ln2), exp(x) = 2^(k/32) * p(r) with a 32-entry table of
//    2^(i/32) and a cubic in double; the fused multiply-adds are those of the
//    FMA-capable x86-64 build the library dispatches to on AVX2/FMA hosts.
//  * tanhf: fdlibm (s_tanhf.c): 1 - 2/(expm1(2|x|) + 2) for |x| >= 1,
//    -expm1(-2|x|)/(expm1(-2|x|) + 2) below, with fdlibm's expm1f (reduction by
//    ln2 in hi/lo parts and its 5-term rational correction), in float.
// Every operation is written with an explicit-rounding intrinsic so that the
// compiler contracts nothing the host build does not.

// 2^(i/32) as the bits of the nearest double, minus i << 47 (the exponent
// adjustment the reconstruction adds back).
static __device__ const unsigned long long ec_exp2f_tab[32] = {
    0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL, 0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL, 0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL, 0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL, 0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL, 0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL, 0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL, 0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL};

EC_DEV float ec_expf(float x) {
    constexpr double C0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32, C1 = 0x1.ebfce50fac4f3p-3 / 32 / 32,
                     C2 = 0x1.62e42ff0c52d6p-1 / 32, INVLN2N = 0x1.71547652b82fep+0 * 32, SHIFT = 0x1.8p+52;
    const uint32_t ux = __float_as_uint(x);
    const uint32_t abstop = (ux >> 20) & 0x7ffu;
    if (abstop >= 0x42bu) {                       // |x| >= 88, inf or nan
        if (ux == 0xff800000u) return 0.0f;
        if (abstop >= 0x7f8u) return __fadd_rn(x, x);
        if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double xd = (double)x;
    const double z = __dmul_rn(INVLN2N, xd);
    double kd = __dadd_rn(z, SHIFT);
    const unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
    kd = __dsub_rn(kd, SHIFT);
    const double r = __fma_rn(INVLN2N, xd, -kd);
    const double s = __longlong_as_double((long long)(ec_exp2f_tab[ki % 32] + (ki << 47)));
    const double p = __fma_rn(C0, r, C1);
    const double r2 = __dmul_rn(r, r);
    double y = __fma_rn(C2, r, 1.0);
    y = __fma_rn(p, r2, y);
    return __double2float_rn(__dmul_rn(y, s));
}

EC_DEV float ec_expm1f(float x) {
    constexpr float ln2_hi = 6.9313812256e-01f, ln2_lo = 9.0580006145e-06f, invln2 = 1.4426950216e+00f;
    constexpr float Q1 = -3.3333335072e-02f, Q2 = 1.5873016091e-03f, Q3 = -7.9365076090e-05f,
                    Q4 = 4.0082177293e-06f, Q5 = -2.0109921195e-07f;
    float hi, lo, c = 0.0f, t, e, y;
    int k;
    uint32_t hx = __float_as_uint(x);
    const uint32_t xsb = hx & 0x80000000u;
    hx &= 0x7fffffffu;
    if (hx >= 0x4195b844u) {                      // |x| >= 27 ln2
        if (hx >= 0x42b17218u) {
            if (hx > 0x7f800000u) return __fadd_rn(x, x);
            if (hx == 0x7f800000u) return xsb == 0 ? x : -1.0f;
            if (x > 8.8721679688e+01f) return __int_as_float(0x7f800000);
        }
        if (xsb != 0) return -1.0f;
    }
    if (hx > 0x3eb17218u) {                       // |x| > 0.5 ln2
        if (hx < 0x3f851592u) {                   // and < 1.5 ln2
            if (xsb == 0) { hi = __fsub_rn(x, ln2_hi); lo = ln2_lo; k = 1; }
            else { hi = __fadd_rn(x, ln2_hi); lo = -ln2_lo; k = -1; }
        } else {
            k = __float2int_rz(__fadd_rn(__fmul_rn(invln2, x), xsb == 0 ? 0.5f : -0.5f));
            t = __int2float_rn(k);
            hi = __fsub_rn(x, __fmul_rn(t, ln2_hi));
            lo = __fmul_rn(t, ln2_lo);
        }
        x = __fsub_rn(hi, lo);
        c = __fsub_rn(__fsub_rn(hi, x), lo);
    } else if (hx < 0x33000000u) {                // |x| < 2^-25
        return x;
    } else {
        k = 0;
    }
    const float hfx = __fmul_rn(0.5f, x);
    const float hxs = __fmul_rn(x, hfx);
    float q = __fadd_rn(Q4, __fmul_rn(hxs, Q5));
    q = __fadd_rn(Q3, __fmul_rn(hxs, q));
    q = __fadd_rn(Q2, __fmul_rn(hxs, q));
    q = __fadd_rn(Q1, __fmul_rn(hxs, q));
    const float r1 = __fadd_rn(1.0f, __fmul_rn(hxs, q));
    t = __fsub_rn(3.0f, __fmul_rn(r1, hfx));
    e = __fmul_rn(hxs, __fdiv_rn(__fsub_rn(r1, t), __fsub_rn(6.0f, __fmul_rn(x, t))));
    if (k == 0) return __fsub_rn(x, __fsub_rn(__fmul_rn(x, e), hxs));
    e = __fsub_rn(__fmul_rn(x, __fsub_rn(e, c)), c);
    e = __fsub_rn(e, hxs);
    if (k == -1) return __fsub_rn(__fmul_rn(0.5f, __fsub_rn(x, e)), 0.5f);
    if (k == 1) {
        if (x < -0.25f) return __fmul_rn(-2.0f, __fsub_rn(e, __fadd_rn(x, 0.5f)));
        return __fadd_rn(1.0f, __fmul_rn(2.0f, __fsub_rn(x, e)));
    }
    if (k <= -2 || k > 56) {
        y = __fsub_rn(1.0f, __fsub_rn(e, x));
        if (k == 128) y = __fmul_rn(__fmul_rn(y, 2.0f), 0x1p127f);
        else y = __uint_as_float(__float_as_uint(y) + ((uint32_t)k << 23));
        return __fsub_rn(y, 1.0f);
    }
    if (k < 23) {
        t = __uint_as_float(0x3f800000u - (0x1000000u >> k));
        y = __fsub_rn(t, __fsub_rn(e, x));
    } else {
        t = __uint_as_float((uint32_t)(0x7f - k) << 23);
        y = __fsub_rn(x, __fadd_rn(e, t));
        y = __fadd_rn(y, 1.0f);
    }
    return __uint_as_float(__float_as_uint(y) + ((uint32_t)k << 23));
}

EC_DEV float ec_tanhf(float x) {
    const uint32_t jx = __float_as_uint(x), ix = jx & 0x7fffffffu;
    float t, z;
    if (ix >= 0x7f800000u)                                   // inf or nan
        return (int)jx >= 0 ? __fadd_rn(__fdiv_rn(1.0f, x), 1.0f) : __fsub_rn(__fdiv_rn(1.0f, x), 1.0f);
    if (ix < 0x41b00000u) {                                  // |x| < 22
        if (ix == 0) return x;
        if (ix < 0x24000000u) return __fmul_rn(x, __fadd_rn(1.0f, x));
        if (ix >= 0x3f800000u) {                             // |x| >= 1
            t = ec_expm1f(__fmul_rn(2.0f, fabsf(x)));
            z = __fsub_rn(1.0f, __fdiv_rn(2.0f, __fadd_rn(t, 2.0f)));
        } else {
            t = ec_expm1f(__fmul_rn(-2.0f, fabsf(x)));
            z = __fdiv_rn(-t, __fadd_rn(t, 2.0f));
        }
    } else {
        z = __fsub_rn(1.0f, 1.0e-30f);
    }
    return (int)jx >= 0 ? z : -z;
}

// Reference gelu_new (src/gpt2.c:393-396) with its evaluation order kept.
EC_DEV float ec_gelu(float x) {
    float c = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
    float t = ec_tanhf(__fmul_rn(0.7978845608028654f, __fadd_rn(x, c)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}

// Reference SiLU (src/gpt2.c:587-590).
EC_DEV float ec_silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, ec_expf(-x))); }
