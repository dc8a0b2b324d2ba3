/*
 * Deterministic scalar arithmetic shared by the sm_100a kernels and the CPU oracle.
 *
 * Why this exists: tile keys, sort order and tile ranges must be bit-exact between the GPU path
 * and its CPU checker, and the rendered RGB must match to 1e-4.  Both depend on float decisions
 * (opacity cull, tile-overlap test, alpha threshold, transmittance stop) that a single ulp can
 * flip.  The contract is therefore:
 *   - every translation unit that includes this header is compiled WITHOUT implicit
 *     multiply-add contraction (nvcc -fmad=false, gcc -ffp-contract=off);
 *   - fused multiply-adds are written explicitly with fmaf() where wanted (FFMA on the GPU,
 *     correctly rounded fmaf on the host: identical results);
 *   - +,-,*,/ and sqrtf are IEEE round-to-nearest on both sides (nvcc's defaults
 *     -prec-div=true -prec-sqrt=true -ftz=false; never -use_fast_math);
 *   - exp and log are the functions below, written from the textbook methods named at each one,
 *     not taken from any vendor math library.  Both sides therefore compute the same bits.
 */
#ifndef GSX_DETMATH_H
#define GSX_DETMATH_H

#include <math.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define GSX_HD static __host__ __device__ __forceinline__
#else
#define GSX_HD static inline
#endif

GSX_HD float gsx_bits_to_float(uint32_t u)
{
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, sizeof(f));
    return f;
#endif
}

GSX_HD uint32_t gsx_float_to_bits(float f)
{
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, sizeof(u));
    return u;
#endif
}

/*
 * exp(x) by Cody-Waite range reduction and a degree-7 Taylor polynomial:
 *   x = n*ln2 + r, n = round(x/ln2), |r| <= ln2/2;  e^x = 2^n * P(r),
 *   P(r) = sum_{k=0..7} r^k/k!  (truncation error below 1e-8 relative on |r| <= 0.347).
 * ln2 is split into a 16-bit head (so n*head is exact for |n| <= 256) and a tail.
 * Results below 2^-126 (x < -87.33) are returned as 0; x > 88.72 returns +inf.
 * Measured against libm to within 2 ulp over the whole normal range (tests/test_oracle_pins.py, test_detmath_exp_log_within_two_ulp).
 */
GSX_HD float gsx_expf_inrange(float x);

GSX_HD float gsx_expf(float x)
{
    if(!(x == x)) {
        return x;
    }
    if(x > 88.72283935546875f) {
        return gsx_bits_to_float(0x7f800000u);
    }
    if(x < -87.33654022216797f) {
        return 0.0f;
    }
    return gsx_expf_inrange(x);
}

/* The same arithmetic as gsx_expf without the range checks: identical bits for
 * -87.33 <= x <= 88.72 (the blend kernels call it on x in [-5.6, 0]). */
GSX_HD float gsx_expf_inrange(float x)
{
    const float log2e = 1.44269502162933349609f;
    const float ln2_hi = 0.693145751953125f;
    const float ln2_lo = 1.42860682030941723212e-06f;
    const float n = rintf(x * log2e);
    float r = fmaf(-n, ln2_hi, x);
    r = fmaf(-n, ln2_lo, r);
    float p = 1.98412698412698412698e-04f;       /* 1/7! */
    p = fmaf(p, r, 1.38888888888888888889e-03f); /* 1/6! */
    p = fmaf(p, r, 8.33333333333333333333e-03f); /* 1/5! */
    p = fmaf(p, r, 4.16666666666666666667e-02f); /* 1/4! */
    p = fmaf(p, r, 1.66666666666666666667e-01f); /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    if(ni > 127) {
        p *= 2.0f;
        ni -= 1;
    }
    return p * gsx_bits_to_float((uint32_t)(ni + 127) << 23);
}

/*
 * log(x) for x > 0 by exponent/mantissa split and the atanh series:
 *   x = m * 2^e with m in [sqrt(1/2), sqrt(2)),  s = (m-1)/(m+1),
 *   log(m) = 2*atanh(s) = 2s * (1 + s^2/3 + s^4/5 + ... + s^10/11)   (|s| <= 0.1716).
 * x == 0 -> -inf, x < 0 -> NaN, +inf -> +inf; subnormals are pre-scaled by 2^23.
 */
GSX_HD float gsx_logf(float x)
{
    if(!(x == x) || x < 0.0f) {
        return gsx_bits_to_float(0x7fc00000u);
    }
    if(x == 0.0f) {
        return gsx_bits_to_float(0xff800000u);
    }
    uint32_t bits = gsx_float_to_bits(x);
    if(bits >= 0x7f800000u) {
        return x;
    }
    int e = 0;
    if(bits < 0x00800000u) {
        x *= 8388608.0f;
        bits = gsx_float_to_bits(x);
        e = -23;
    }
    e += (int)((bits >> 23) & 0xffu) - 127;
    float m = gsx_bits_to_float((bits & 0x007fffffu) | 0x3f800000u);
    if(m > 1.41421353816986083984f) {
        m *= 0.5f;
        e += 1;
    }
    const float s = (m - 1.0f) / (m + 1.0f);
    const float s2 = s * s;
    float q = 9.09090909090909090909e-02f;      /* 1/11 */
    q = fmaf(q, s2, 1.11111111111111111111e-01f); /* 1/9 */
    q = fmaf(q, s2, 1.42857142857142857143e-01f); /* 1/7 */
    q = fmaf(q, s2, 2.0e-01f);                    /* 1/5 */
    q = fmaf(q, s2, 3.33333333333333333333e-01f); /* 1/3 */
    const float two_s = s + s;
    const float log_m = fmaf(two_s * s2, q, two_s);
    const float ef = (float)e;
    const float ln2_hi = 0.693145751953125f;
    const float ln2_lo = 1.42860682030941723212e-06f;
    return fmaf(ef, ln2_hi, fmaf(ef, ln2_lo, log_m));
}

/* Logistic sigmoid in the two-branch form of fastgs/tinygs/common.hpp:36-47 (activate_opacity). */
GSX_HD float gsx_sigmoidf(float v)
{
    if(v >= 0.0f) {
        const float z = gsx_expf(-v);
        return 1.0f / (1.0f + z);
    }
    const float z = gsx_expf(v);
    return z / (1.0f + z);
}

/* __saturatef semantics: clamp to [0,1], NaN -> 0. */
GSX_HD float gsx_saturatef(float v)
{
    if(!(v > 0.0f)) {
        return 0.0f;
    }
    return v > 1.0f ? 1.0f : v;
}

#endif /* GSX_DETMATH_H */
