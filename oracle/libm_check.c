/* libm_check.c -- TEST INFRASTRUCTURE.  The reference calls the host C
 * library's expf and tanhf (glibc 2.39 on its x86-64 build hosts); this
 * library's kernels use restatements of those published algorithms
 * (edgecore_b200/csrc/ec_common.cuh: ec_expf, ec_expm1f, ec_tanhf) so that
 * the GPU rounds exactly as the reference's CPU build.  This program restates
 * the same algorithms in C and compares them bit for bit with the host
 * library:
 *   expf  -- ARM optimized-routines (glibc sysdeps/ieee754/flt-32/e_expf.c):
 *            2^(k/32) from a 32-entry table times a cubic in double, with the
 *            fused multiply-adds of the FMA build glibc selects on AVX2/FMA
 *            hosts;
 *   tanhf -- fdlibm (s_tanhf.c) over fdlibm's expm1f (s_expm1f.c).
 *
 *   libm_check          every 64th float bit pattern (2^26 per function)
 *   libm_check --all    all 2^32 bit patterns
 * Exit status 0 when every compared value is identical (NaNs as NaNs).
 * Built by `make -C oracle` into oracle/_ref/libm_check. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

/* 2^(i/32) as the bits of the nearest double, minus i << 47. */
static const uint64_t T32[32] = {0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL, 0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL, 0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL, 0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL, 0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL, 0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL, 0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL, 0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL};

static inline double asd(uint64_t u) { double d; memcpy(&d, &u, 8); return d; }
static inline uint64_t asu(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }
static inline uint32_t fu(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float uf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static float myexpf(float x) {
    const double C0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32, C1 = 0x1.ebfce50fac4f3p-3 / 32 / 32,
                 C2 = 0x1.62e42ff0c52d6p-1 / 32, INVLN2N = 0x1.71547652b82fep+0 * 32, SHIFT = 0x1.8p+52;
    const uint32_t abstop = (fu(x) >> 20) & 0x7ff;
    if (abstop >= 0x42b) {
        if (fu(x) == 0xff800000u) return 0.0f;
        if (abstop >= 0x7f8) return x + x;
        if (x > 0x1.62e42ep6f) return INFINITY;
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double xd = (double)x;
    double z = INVLN2N * xd, kd = z + SHIFT;
    const uint64_t ki = asu(kd);
    kd -= SHIFT;
    const double r = fma(INVLN2N, xd, -kd);
    const double s = asd(T32[ki % 32] + (ki << 47));
    z = fma(C0, r, C1);
    const double r2 = r * r;
    double y = fma(C2, r, 1.0);
    y = fma(z, r2, y);
    return (float)(y * s);
}
static float my_expm1f(float x) {
    const float ln2_hi = 6.9313812256e-01f, ln2_lo = 9.0580006145e-06f, invln2 = 1.4426950216e+00f;
    const float Q1 = -3.3333335072e-02f, Q2 = 1.5873016091e-03f, Q3 = -7.9365076090e-05f,
                Q4 = 4.0082177293e-06f, Q5 = -2.0109921195e-07f;
    float y, hi, lo, c = 0.0f, t, e, hxs, hfx, r1;
    int32_t k;
    uint32_t hx = fu(x);
    const uint32_t xsb = hx & 0x80000000u;
    hx &= 0x7fffffffu;
    if (hx >= 0x4195b844u) {                       /* |x| >= 27 ln2 */
        if (hx >= 0x42b17218u) {
            if (hx > 0x7f800000u) return x + x;
            if (hx == 0x7f800000u) return xsb == 0 ? x : -1.0f;
            if (x > 8.8721679688e+01f) return INFINITY;
        }
        if (xsb != 0) return -1.0f;
    }
    if (hx > 0x3eb17218u) {                        /* |x| > 0.5 ln2 */
        if (hx < 0x3F851592u) {                    /* |x| < 1.5 ln2 */
            if (xsb == 0) { hi = x - ln2_hi; lo = ln2_lo; k = 1; }
            else { hi = x + ln2_hi; lo = -ln2_lo; k = -1; }
        } else {
            k = (int32_t)(invln2 * x + (xsb == 0 ? 0.5f : -0.5f));
            t = (float)k;
            hi = x - t * ln2_hi;
            lo = t * ln2_lo;
        }
        x = hi - lo;
        c = (hi - x) - lo;
    } else if (hx < 0x33000000u) {
        return x;
    } else {
        k = 0;
    }
    hfx = 0.5f * x;
    hxs = x * hfx;
    r1 = 1.0f + hxs * (Q1 + hxs * (Q2 + hxs * (Q3 + hxs * (Q4 + hxs * Q5))));
    t = 3.0f - r1 * hfx;
    e = hxs * ((r1 - t) / (6.0f - x * t));
    if (k == 0) return x - (x * e - hxs);
    e = (x * (e - c) - c);
    e -= hxs;
    if (k == -1) return 0.5f * (x - e) - 0.5f;
    if (k == 1) {
        if (x < -0.25f) return -2.0f * (e - (x + 0.5f));
        return 1.0f + 2.0f * (x - e);
    }
    if (k <= -2 || k > 56) {
        y = 1.0f - (e - x);
        if (k == 128) y = y * 2.0f * 0x1p127f;
        else y = uf(fu(y) + ((uint32_t)k << 23));
        return y - 1.0f;
    }
    if (k < 23) {
        t = uf(0x3f800000u - (0x1000000u >> k));
        y = t - (e - x);
        y = uf(fu(y) + ((uint32_t)k << 23));
    } else {
        t = uf((uint32_t)(0x7f - k) << 23);
        y = x - (e + t);
        y += 1.0f;
        y = uf(fu(y) + ((uint32_t)k << 23));
    }
    return y;
}
static float my_tanhf(float x) {
    const uint32_t jx = fu(x), ix = jx & 0x7fffffffu;
    float t, z;
    if (ix >= 0x7f800000u) return (int32_t)jx >= 0 ? 1.0f / x + 1.0f : 1.0f / x - 1.0f;
    if (ix < 0x41b00000u) {
        if (ix == 0) return x;
        if (ix < 0x24000000u) return x * (1.0f + x);
        if (ix >= 0x3f800000u) {
            t = my_expm1f(2.0f * fabsf(x));
            z = 1.0f - 2.0f / (t + 2.0f);
        } else {
            t = my_expm1f(-2.0f * fabsf(x));
            z = -t / (t + 2.0f);
        }
    } else {
        z = 1.0f - 1.0e-30f;
    }
    return (int32_t)jx >= 0 ? z : -z;
}

int main(int argc, char **argv)
{
    const uint64_t step = (argc > 1 && !strcmp(argv[1], "--all")) ? 1 : 64;
    uint64_t n = 0, be = 0, bt = 0;
    for (uint64_t u = 0; u < 0x100000000ull; u += step) {
        const float x = uf((uint32_t)u);
        const float a = expf(x), m = myexpf(x);
        if (fu(a) != fu(m) && !(isnan(a) && isnan(m))) {
            if (be < 4) printf("expf  x=%a host=%a restated=%a\n", x, a, m);
            be++;
        }
        const float ta = tanhf(x), tm = my_tanhf(x);
        if (fu(ta) != fu(tm) && !(isnan(ta) && isnan(tm))) {
            if (bt < 4) printf("tanhf x=%a host=%a restated=%a\n", x, ta, tm);
            bt++;
        }
        n++;
    }
    printf("libm_check: %llu inputs, expf %llu differ, tanhf %llu differ\n", (unsigned long long)n,
           (unsigned long long)be, (unsigned long long)bt);
    return (be || bt) ? 1 : 0;
}
