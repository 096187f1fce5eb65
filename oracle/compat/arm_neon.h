/*
 * arm_neon.h (portable subset) -- TEST INFRASTRUCTURE for the oracle build.
 *
 * Lets the reference CPU attention path (kernel/attention.c, kernel/kv_cache.c,
 * kernel/ops.c of typhoon-ocr-server) compile unmodified on x86_64 with gcc, so
 * it can serve as the checker for the CUDA kernels.  It provides only the
 * AArch64 NEON intrinsics those three files use, each with the lane semantics
 * the Arm architecture documents:
 *
 *   vfmaq_f32(a,b,c) = a + b*c (fused, one rounding)     vfmsq_f32(a,b,c) = a - b*c (fused)
 *   vrndaq_f32       = round to nearest, ties away (roundf)
 *   vcvtq_s32_f32    = convert toward zero, saturating
 *   vaddvq_f32       = pairwise: (a0+a1) + (a2+a3)
 *   vrsqrteq_f32 / vrecpeq_f32 = estimates; here the exact value with the
 *                      mantissa cut to 8 bits (the estimate's precision), so
 *                      the two Newton steps the caller applies converge the
 *                      same way.  Bit-exactness with Apple silicon is not a
 *                      goal: parity is checked by tolerance.
 *   vrsqrtsq_f32(a,b) = (3 - a*b) / 2                     vrecpsq_f32(a,b) = 2 - a*b
 *
 * Nothing here is product code; only the oracle build includes it.
 */
#ifndef ORACLE_COMPAT_ARM_NEON_H
#define ORACLE_COMPAT_ARM_NEON_H

#include <math.h>
#include <stdint.h>
#include <string.h>

typedef float   float32x4_t __attribute__((vector_size(16)));
typedef int32_t int32x4_t   __attribute__((vector_size(16)));

#define NEON_INLINE static inline __attribute__((always_inline))

NEON_INLINE float32x4_t vld1q_f32(const float *p)
{
    float32x4_t r;
    memcpy(&r, p, sizeof r);
    return r;
}

NEON_INLINE void vst1q_f32(float *p, float32x4_t v) { memcpy(p, &v, sizeof v); }

NEON_INLINE float32x4_t vdupq_n_f32(float x) { float32x4_t r = {x, x, x, x}; return r; }
NEON_INLINE int32x4_t   vdupq_n_s32(int32_t x) { int32x4_t r = {x, x, x, x}; return r; }

NEON_INLINE float32x4_t vaddq_f32(float32x4_t a, float32x4_t b) { return a + b; }
NEON_INLINE float32x4_t vsubq_f32(float32x4_t a, float32x4_t b) { return a - b; }
NEON_INLINE float32x4_t vmulq_f32(float32x4_t a, float32x4_t b) { return a * b; }
NEON_INLINE float32x4_t vnegq_f32(float32x4_t a) { return -a; }
NEON_INLINE int32x4_t   vaddq_s32(int32x4_t a, int32x4_t b) { return a + b; }

NEON_INLINE float32x4_t vfmaq_f32(float32x4_t a, float32x4_t b, float32x4_t c)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = fmaf(b[i], c[i], a[i]);
    return r;
}

NEON_INLINE float32x4_t vfmsq_f32(float32x4_t a, float32x4_t b, float32x4_t c)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = fmaf(-b[i], c[i], a[i]);
    return r;
}

NEON_INLINE float32x4_t vmaxq_f32(float32x4_t a, float32x4_t b)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = a[i] > b[i] ? a[i] : b[i];
    return r;
}

NEON_INLINE float32x4_t vminq_f32(float32x4_t a, float32x4_t b)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = a[i] < b[i] ? a[i] : b[i];
    return r;
}

NEON_INLINE float32x4_t vrndaq_f32(float32x4_t a)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = roundf(a[i]);
    return r;
}

NEON_INLINE int32x4_t vcvtq_s32_f32(float32x4_t a)
{
    int32x4_t r;
    for (int i = 0; i < 4; i++) {
        float x = a[i];
        if (x != x)                 r[i] = 0;
        else if (x >= 2147483648.f) r[i] = INT32_MAX;
        else if (x < -2147483648.f) r[i] = INT32_MIN;
        else                        r[i] = (int32_t)x;   /* C truncates toward zero */
    }
    return r;
}

/* Shift by an immediate; a macro keeps the "constant n" contract of the intrinsic. */
#define vshlq_n_s32(a, n) ((int32x4_t)((a) << (n)))

NEON_INLINE float32x4_t vreinterpretq_f32_s32(int32x4_t a)
{
    float32x4_t r;
    memcpy(&r, &a, sizeof r);
    return r;
}

NEON_INLINE float vaddvq_f32(float32x4_t a) { return (a[0] + a[1]) + (a[2] + a[3]); }

#define vgetq_lane_f32(v, lane) ((float)((v)[(lane)]))

/* Keep the top 8 mantissa bits of x: the precision an Arm estimate delivers. */
NEON_INLINE float neon_compat_estimate_bits(float x)
{
    uint32_t u;
    memcpy(&u, &x, sizeof u);
    u &= 0xFFFF8000u;
    memcpy(&x, &u, sizeof u);
    return x;
}

NEON_INLINE float32x4_t vrsqrteq_f32(float32x4_t a)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = neon_compat_estimate_bits(1.0f / sqrtf(a[i]));
    return r;
}

NEON_INLINE float32x4_t vrecpeq_f32(float32x4_t a)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = neon_compat_estimate_bits(1.0f / a[i]);
    return r;
}

NEON_INLINE float32x4_t vrsqrtsq_f32(float32x4_t a, float32x4_t b)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = (3.0f - a[i] * b[i]) * 0.5f;
    return r;
}

NEON_INLINE float32x4_t vrecpsq_f32(float32x4_t a, float32x4_t b)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = 2.0f - a[i] * b[i];
    return r;
}

#endif /* ORACLE_COMPAT_ARM_NEON_H */
