/* gdn_math.h -- scalar float functions for the decode kernel's elementwise
 * epilogues, written to agree with the host libm the reference is built
 * against (glibc expf is within a hair of correctly rounded) while staying
 * cheap on the GPU. Usable from host code (tests) and device code.
 *
 * gdn_expf  -- exp(x) by the table-driven method of P. T. P. Tang ("Table-
 *              driven implementation of the exponential function in IEEE
 *              floating-point arithmetic", ACM TOMS 15(2), 1989): x = (64k +
 *              j) ln2/64 + r with |r| <= ln2/128, exp(x) = 2^k * 2^(j/64) *
 *              exp(r); the reduction uses a three-part split of ln2/64 and
 *              the reconstruction runs in float-float arithmetic, so the
 *              result before the final rounding is within ~2^-39 of exp(x):
 *              it is the correctly rounded value except when exp(x) lies
 *              that close to a rounding boundary. The 64 table entries
 *              2^(j/64) = hi + lo are computed on the host in long double
 *              (gdn_exp_table_fill).
 * gdn_divf  -- a/b for normal, finite operands with a normal quotient (the
 *              sigmoid's ranges): Newton-refined reciprocal, then one
 *              correction step (P. Markstein, "Computation of elementary
 *              functions on the IBM RISC System/6000 processor", IBM J. Res.
 *              Dev. 34(1), 1990). On the host it is the IEEE division; the
 *              GPU tests compare the device form with the IEEE division.
 */
#ifndef GDN_MATH_H
#define GDN_MATH_H

#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define GDN_HD __host__ __device__ __forceinline__
#else
#define GDN_HD static inline
#endif

/* 64/ln2, and ln2/64 = L1 + L2 + L3 where L1 and L2 have 11 significant
 * bits, so n * L1 and n * L2 are exact for |n| < 2^13. */
#define GDN_EXP_INV_L 0x1.715476p+6f
#define GDN_EXP_L1 0x1.63p-7f
#define GDN_EXP_L2 (-0x1.bdp-19f)
#define GDN_EXP_L3 (-0x1.05c61p-35f)

/* table[j] = hi of 2^(j/64), table[64 + j] = 2^(j/64) - hi. */
static inline void gdn_exp_table_fill(float *table) {
    for (int j = 0; j < 64; ++j) {
        const long double v = exp2l((long double)j / 64.0L);
        const float hi = (float)v;
        table[j] = hi;
        table[64 + j] = (float)(v - (long double)hi);
    }
}

/* Single-rounding operations that the compiler may not fuse. */
#if defined(__CUDA_ARCH__)
#define GDN_ADD(a, b) __fadd_rn((a), (b))
#define GDN_SUB(a, b) __fsub_rn((a), (b))
#define GDN_MUL(a, b) __fmul_rn((a), (b))
#else
#define GDN_ADD(a, b) ((a) + (b))
#define GDN_SUB(a, b) ((a) - (b))
#define GDN_MUL(a, b) ((a) * (b))
#endif

GDN_HD float gdn_pow2f(int k) {
    const uint32_t b = (uint32_t)(k + 127) << 23;
#if defined(__CUDA_ARCH__)
    return __uint_as_float(b);
#else
    float f;
    memcpy(&f, &b, 4);
    return f;
#endif
}

/* exp(x); `table` = {hi[64], lo[64]} (see the header comment). Branch-free
 * (the special cases are selected at the end), so that independent calls
 * interleave. The final scaling by 2^k is split into two exact power-of-two
 * multiplies, 2^(k>>1) then 2^(k - (k>>1)): the first never leaves the normal
 * range, so the only rounding is the second one, and only when the result is
 * subnormal -- the single rounding ldexpf would do. */
GDN_HD float gdn_expf(float x, const float *table) {
    const float xc = fminf(fmaxf(x, -104.0f), 89.0f); /* keeps N in int range; NaN -> -104 */
    const float n = rintf(GDN_MUL(xc, GDN_EXP_INV_L));
    const int N = (int)n;
    /* r = x - n ln2/64 as rh + rl */
    const float r1 = fmaf(-n, GDN_EXP_L1, xc);         /* exact */
    const float p2 = GDN_MUL(n, GDN_EXP_L2);           /* exact */
    const float rh = GDN_SUB(r1, p2);
    const float bb = GDN_SUB(rh, r1);
    const float e2 = GDN_ADD(GDN_SUB(r1, GDN_SUB(rh, bb)), GDN_SUB(-p2, bb)); /* TwoSum error */
    const float rl = GDN_SUB(e2, GDN_MUL(n, GDN_EXP_L3));
    /* exp(rh + rl) - 1 = rh + q,  q = rl (1 + rh) + rh^2 (1/2 + rh (1/6 + rh/24)) */
    const float poly = GDN_ADD(0.5f, GDN_MUL(rh, GDN_ADD(0x1.555556p-3f, GDN_MUL(rh, 0x1.555556p-5f))));
    const float q = GDN_ADD(GDN_ADD(rl, GDN_MUL(rl, rh)), GDN_MUL(GDN_MUL(rh, rh), poly));
    const int j = N & 63;
    const int k = N >> 6; /* arithmetic shift: N = 64 k + j */
    const float th = table[j], tl = table[64 + j];
    /* T (1 + rh + q) = th + th*rh + (small terms), in float-float */
    const float a = GDN_MUL(th, rh);
    const float a_err = fmaf(th, rh, -a);              /* exact product error */
    const float s = GDN_ADD(th, a);
    const float s_err = GDN_SUB(a, GDN_SUB(s, th));    /* Fast2Sum, |th| >= |a| */
    const float tail = GDN_ADD(GDN_ADD(GDN_ADD(a_err, s_err), GDN_MUL(th, q)), GDN_MUL(tl, GDN_ADD(1.0f, rh)));
    const float m = GDN_ADD(s, tail);                  /* in [0.99, 1.99] */
    const int k1 = k >> 1;
    const float v = GDN_MUL(GDN_MUL(m, gdn_pow2f(k1)), gdn_pow2f(k - k1));
    float out = v;
    out = (x < -103.97208404541015625f) ? 0.0f : out;
    out = (x > 88.72283935546875f) ? INFINITY : out;
    out = (x != x) ? x : out;
    return out;
}

/* exp(x) as gdn_expf, and whether its rounding is in doubt. The float-float
 * value before the final rounding, s + tail, is within ~2^-39 of exp(x); its
 * rounding error err = (s + tail) - m is computed, and `zone` is set when the
 * value lies within GDN_EXP_ZONE ulp of a rounding boundary (the midpoint
 * between m and the float on err's side, half an ulp away -- a quarter of m's
 * ulp below a power of two), where a libm that is not correctly rounded may
 * round the other way. Results below the normal range (x < -87.33) are
 * always flagged: their final scaling rounds a second time. NaN and
 * overflowing inputs are not flagged. A flagged caller decides with a
 * more precise evaluation (the decode kernel's exact-exp path). */
#define GDN_EXP_ZONE 0.004f
GDN_HD float gdn_expf_zone(float x, const float *table, bool *zone) {
    const float xc = fminf(fmaxf(x, -104.0f), 89.0f);
    const float n = rintf(GDN_MUL(xc, GDN_EXP_INV_L));
    const int N = (int)n;
    const float r1 = fmaf(-n, GDN_EXP_L1, xc);
    const float p2 = GDN_MUL(n, GDN_EXP_L2);
    const float rh = GDN_SUB(r1, p2);
    const float bb = GDN_SUB(rh, r1);
    const float e2 = GDN_ADD(GDN_SUB(r1, GDN_SUB(rh, bb)), GDN_SUB(-p2, bb));
    const float rl = GDN_SUB(e2, GDN_MUL(n, GDN_EXP_L3));
    const float poly = GDN_ADD(0.5f, GDN_MUL(rh, GDN_ADD(0x1.555556p-3f, GDN_MUL(rh, 0x1.555556p-5f))));
    const float q = GDN_ADD(GDN_ADD(rl, GDN_MUL(rl, rh)), GDN_MUL(GDN_MUL(rh, rh), poly));
    const int j = N & 63;
    const int k = N >> 6;
    const float th = table[j], tl = table[64 + j];
    const float a = GDN_MUL(th, rh);
    const float a_err = fmaf(th, rh, -a);
    const float s = GDN_ADD(th, a);
    const float s_err = GDN_SUB(a, GDN_SUB(s, th));
    const float tail = GDN_ADD(GDN_ADD(GDN_ADD(a_err, s_err), GDN_MUL(th, q)), GDN_MUL(tl, GDN_ADD(1.0f, rh)));
    const float m = GDN_ADD(s, tail);
    /* rounding error of m: s - m is exact (Sterbenz), the sum rounds once */
    const float err = GDN_ADD(GDN_SUB(s, m), tail);
    /* ulp of m (m in [0.99, 1.99]); the gap below a power of two is half of it */
    const float u = (m >= 1.0f) ? 0x1p-23f : 0x1p-24f;
    const float gap = (err < 0.0f && (m == 1.0f)) ? GDN_MUL(0.5f, u) : u;
    const int k1 = k >> 1;
    const float v = GDN_MUL(GDN_MUL(m, gdn_pow2f(k1)), gdn_pow2f(k - k1));
    float out = v;
    out = (x < -103.97208404541015625f) ? 0.0f : out;
    out = (x > 88.72283935546875f) ? INFINITY : out;
    out = (x != x) ? x : out;
    const bool near = fabsf(err) >= GDN_MUL(GDN_SUB(0.5f, GDN_EXP_ZONE), gap);
    *zone = (x == x) && !(x > 88.72283935546875f) && (near || x < -87.33f);
    return out;
}

#if defined(__CUDA_ARCH__)
GDN_HD float gdn_divf(float a, float b) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
    y = fmaf(fmaf(-b, y, 1.0f), y, y);
    const float q = __fmul_rn(a, y);
    return fmaf(fmaf(-b, q, a), y, q);
}
#else
GDN_HD float gdn_divf(float a, float b) { return a / b; }
#endif

/* gdn_sigmoid (c_impl/gdn_model.cpp:1307-1316) on these primitives:
 * x >= 0: 1 / (1 + exp(-x)); x < 0: exp(x) / (1 + exp(x)); both are
 * num / (1 + z) with z = exp(-|x|), written without a branch. */
GDN_HD float gdn_sigmoidf(float x, const float *table) {
    const bool pos = x >= 0.0f;
    const float z = gdn_expf(pos ? -x : x, table);
    return gdn_divf(pos ? 1.0f : z, GDN_ADD(1.0f, z));
}

#endif
