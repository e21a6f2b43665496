/* Deterministic fp32 helpers shared by host and device code.
 *
 * lq_expf: exp(x) by Cody-Waite reduction x = k*ln2 + r (ln2 split into a
 * 16-bit-exact high part and a low part, so k*ln2_hi is exact for |k| < 256)
 * and the degree-7 Taylor polynomial of exp(r) on |r| <= ln2/2 (truncation
 * error < 2e-9 relative), scaled by 2^k with exact power-of-two multiplies.
 * Only IEEE +, *, fma and rint are used, in a fixed order, so the CPU and the
 * GPU produce the same bits (build the device code with --fmad=false and the
 * host code with -ffp-contract=off).  Accuracy: within 2 ulp of the true
 * value (tests/test_math.py compares it with float64 exp over every 97th
 * float of [-104, 88.7]: at most 0.92 ulp).
 */
#ifndef LQ_MATH_H
#define LQ_MATH_H

#ifdef __CUDACC__
#define LQ_HD __host__ __device__ __forceinline__
#else
#include <math.h>
#include <string.h>
#define LQ_HD static inline
#endif

LQ_HD float lq_pow2i(int k) { /* 2^k for -126 <= k <= 127 */
#ifdef __CUDA_ARCH__
    return __int_as_float((k + 127) << 23);
#else
    unsigned u = (unsigned)(k + 127) << 23;
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}

LQ_HD float lq_expf(float x) {
    if (!(x > -104.0f)) return x != x ? x : 0.0f; /* NaN stays NaN; large negative -> 0 */
    if (x > 88.75f) return lq_pow2i(127) * 2.0f;  /* overflow -> +inf */
    const float k = rintf(x * 1.44269502f);
    float r = fmaf(k, -0.693145751953125f, x);
    r = fmaf(k, -1.42860677e-06f, r);
    float p = 1.98412698e-04f;          /* 1/5040 */
    p = fmaf(p, r, 1.38888889e-03f);    /* 1/720 */
    p = fmaf(p, r, 8.33333377e-03f);    /* 1/120 */
    p = fmaf(p, r, 4.16666679e-02f);    /* 1/24 */
    p = fmaf(p, r, 1.66666672e-01f);    /* 1/6 */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ki = (int)k;
    if (ki > 127) return p * lq_pow2i(127) * lq_pow2i(ki - 127);
    if (ki < -126) return p * lq_pow2i(ki + 64) * lq_pow2i(-64);
    return p * lq_pow2i(ki);
}

/* SwiGLU gate, v1-int8-vnni/runq.c:405-410: h1 * (1 / (1 + exp(-h1))) * h3 */
LQ_HD float lq_swiglu(float h1, float h3) {
    float v = h1 * (1.0f / (1.0f + lq_expf(-h1)));
    return v * h3;
}

#endif
