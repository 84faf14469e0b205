/*
 * Portable stand-in for the handful of AArch64 NEON intrinsics that the
 * reference's CPU GEMVs use (src/ops/kernels.cpp:211-343), so that the
 * reference sources compile unmodified on x86-64 for use as a test oracle
 * and as the timed CPU baseline.
 *
 * This is test infrastructure only: it is included when the oracle build
 * compiles the reference's own files from their original location, and is
 * never part of the shipped CUDA library.
 *
 * Semantics follow the Arm intrinsics reference, lane by lane:
 *   vfmaq_f32(a,b,c)  fused a + b*c per lane (one rounding)  -> VFMADD (x86 FMA)
 *   vaddq_f32         per-lane add                            -> ADDPS
 *   vaddvq_f32(v)     across-vector add; AArch64 lowers it to two FADDP
 *                     steps, i.e. (v0+v1) + (v2+v3)
 *   vcvt_f32_f16      exact widening of 4 binary16 lanes      -> VCVTPH2PS (F16C)
 *   vcvt_f32_bf16     exact widening of 4 bfloat16 lanes: the 16 bits become
 *                     the upper half of the binary32 pattern  -> zero-extend + shift
 * Each x86 instruction applies the same IEEE operation to every lane as the
 * NEON one, so the rounding sequence is the one the reference gets on an
 * Apple M-series core, while the loops run at SIMD speed (one 128-bit
 * operation per NEON operation) instead of calling conversion routines per
 * element. Needs AVX2 + FMA + F16C (x86-64-v3).
 */
#pragma once
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifndef MF_NEON_COMPAT_TYPES
#define MF_NEON_COMPAT_TYPES
typedef float float32x4_t __attribute__((vector_size(16)));
typedef _Float16 float16_t;
typedef __bf16 bfloat16_t;
typedef struct { __m128i v; } float16x8_t;  /* 8 raw binary16 lanes */
typedef struct { __m128i v; } float16x4_t;  /* 4 raw binary16 lanes in the low 64 bits */
typedef struct { __m128i v; } bfloat16x8_t; /* 8 raw bfloat16 lanes */
typedef struct { __m128i v; } bfloat16x4_t; /* 4 raw bfloat16 lanes in the low 64 bits */
#endif

static inline float32x4_t vdupq_n_f32(float x) { return (float32x4_t)_mm_set1_ps(x); }

static inline float32x4_t vld1q_f32(const float* p) { return (float32x4_t)_mm_loadu_ps(p); }

static inline float32x4_t vfmaq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
    return (float32x4_t)_mm_fmadd_ps((__m128)b, (__m128)c, (__m128)a);
}

static inline float32x4_t vaddq_f32(float32x4_t a, float32x4_t b) {
    return (float32x4_t)_mm_add_ps((__m128)a, (__m128)b);
}

static inline float vaddvq_f32(float32x4_t v) {
    float lo = v[0] + v[1];
    float hi = v[2] + v[3];
    return lo + hi;
}

static inline float16x8_t vld1q_f16(const float16_t* p) {
    float16x8_t r = {_mm_loadu_si128((const __m128i*)p)};
    return r;
}

static inline float16x4_t vget_low_f16(float16x8_t a) {
    float16x4_t r = {a.v};
    return r;
}

static inline float16x4_t vget_high_f16(float16x8_t a) {
    float16x4_t r = {_mm_srli_si128(a.v, 8)};
    return r;
}

static inline float32x4_t vcvt_f32_f16(float16x4_t a) { return (float32x4_t)_mm_cvtph_ps(a.v); }

static inline bfloat16x8_t vld1q_bf16(const bfloat16_t* p) {
    bfloat16x8_t r = {_mm_loadu_si128((const __m128i*)p)};
    return r;
}

static inline bfloat16x4_t vget_low_bf16(bfloat16x8_t a) {
    bfloat16x4_t r = {a.v};
    return r;
}

static inline bfloat16x4_t vget_high_bf16(bfloat16x8_t a) {
    bfloat16x4_t r = {_mm_srli_si128(a.v, 8)};
    return r;
}

static inline float32x4_t vcvt_f32_bf16(bfloat16x4_t a) {
    return (float32x4_t)_mm_castsi128_ps(_mm_slli_epi32(_mm_cvtepu16_epi32(a.v), 16));
}
