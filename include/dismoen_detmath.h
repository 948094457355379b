/*
 * dismoen_detmath.h — arithmetic that must give the same bits on the host and on the GPU.
 *
 * The router selects the top-k experts on fp32 softmax probabilities with ties going to
 * the lower expert id (reference src/layers/topk.mojo:80-96).  Which of two nearly equal
 * experts wins therefore depends on the exact bits of exp(z - max), of the sum and of the
 * product by 1/sum (reference src/layers/router.mojo:140-183).  To make the device
 * selection bit-identical to a CPU restatement, the router uses this exp instead of the
 * platform's expf, with every rounding step spelled out as an explicit IEEE operation:
 *
 *   n = rint(x * log2(e))                       (x * log2e rounded once, then rint)
 *   r = (x - n * LN2_HI) - n * LN2_LO            (Cody-Waite reduction; LN2_HI has 15
 *                                                 significant bits so n * LN2_HI is exact)
 *   p = 1 + r + r^2/2! + ... + r^7/7!            (Taylor polynomial, Horner form with fma;
 *                                                 |r| <= ln2/2 gives truncation < 6e-9)
 *   exp(x) = p * 2^n                             (exact scaling by the exponent field)
 *
 * Results are within ~2 ulp of the true exponential for x in [-87, 88]; x < -87 returns
 * 0 (the softmax argument is always <= 0, so only underflow matters).
 *
 * DM_DET_FMA / DM_DET_MUL / DM_DET_ADD are single IEEE round-to-nearest operations on
 * both sides (never contracted or reassociated); host code that includes this header
 * must be compiled with -ffp-contract=off and without -ffast-math.
 */
#ifndef DISMOEN_DETMATH_H
#define DISMOEN_DETMATH_H

#include <stdint.h>

#if defined(__CUDACC__)
#define DM_DET_INLINE __host__ __device__ __forceinline__
#else
#define DM_DET_INLINE static inline
#include <math.h>
#include <string.h>
#endif

#if defined(__CUDA_ARCH__)
#define DM_DET_FMA(a, b, c) __fmaf_rn((a), (b), (c))
#define DM_DET_MUL(a, b) __fmul_rn((a), (b))
#define DM_DET_ADD(a, b) __fadd_rn((a), (b))
#define DM_DET_SUB(a, b) __fsub_rn((a), (b))
#define DM_DET_RINT(a) rintf(a)
#define DM_DET_DIV(a, b) __fdiv_rn((a), (b))
#define DM_DET_SQRT(a) __fsqrt_rn(a)
#else
#define DM_DET_FMA(a, b, c) fmaf((a), (b), (c))
#define DM_DET_MUL(a, b) ((a) * (b))
#define DM_DET_ADD(a, b) ((a) + (b))
#define DM_DET_SUB(a, b) ((a) - (b))
#define DM_DET_RINT(a) rintf(a)
#define DM_DET_DIV(a, b) ((a) / (b))
#define DM_DET_SQRT(a) sqrtf(a)
#endif

DM_DET_INLINE float dm_det_bits_to_float(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
#endif
}

/* Exponential for softmax arguments (see header comment). */
DM_DET_INLINE float dm_det_exp(float x) {
    const float LOG2E = 1.44269502162933349609375f;      /* log2(e) rounded to fp32   */
    const float LN2_HI = 0.693145751953125f;             /* 22713 / 32768             */
    const float LN2_LO = 1.428606765330187045e-06f;      /* ln2 - LN2_HI              */
    if (!(x >= -87.0f)) return (x != x) ? x : 0.0f;      /* NaN passes, underflow -> 0 */
    if (x > 88.0f) x = 88.0f;
    float n = DM_DET_RINT(DM_DET_MUL(x, LOG2E));
    float r = DM_DET_FMA(-n, LN2_HI, x);                 /* exact: n*LN2_HI is exact  */
    r = DM_DET_FMA(-n, LN2_LO, r);
    float p = 1.98412698412698412526e-04f;               /* 1/7! */
    p = DM_DET_FMA(p, r, 1.38888888888888894189e-03f);   /* 1/6! */
    p = DM_DET_FMA(p, r, 8.33333333333333321769e-03f);   /* 1/5! */
    p = DM_DET_FMA(p, r, 4.16666666666666643537e-02f);   /* 1/4! */
    p = DM_DET_FMA(p, r, 1.66666666666666657415e-01f);   /* 1/3! */
    p = DM_DET_FMA(p, r, 0.5f);
    p = DM_DET_FMA(p, r, 1.0f);
    p = DM_DET_FMA(p, r, 1.0f);
    int ni = (int)n;                                     /* in [-126, 127]            */
    float scale = dm_det_bits_to_float((uint32_t)(ni + 127) << 23);
    return DM_DET_MUL(p, scale);
}

#endif /* DISMOEN_DETMATH_H */
