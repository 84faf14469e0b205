/*
 * Portable stand-in for the handful of AArch64 NEON intrinsics that the
 * reference's CPU GEMVs use (src/ops/kernels.cpp:211-343), so that the
 * reference sources compile unmodified on x86-64 for use as a test oracle.
 *
 * This is test infrastructure only: it is included when the oracle build
 * compiles the reference's own files from their original location, and is
 * never part of the shipped CUDA library.
 *
 * Semantics follow the Arm intrinsics reference:
 *   vfmaq_f32(a,b,c)  lane-wise fused a + b*c (one rounding)      -> fmaf
 *   vaddvq_f32(v)     across-vector add; AArch64 lowers it to two FADDP
 *                     steps, i.e. (v0+v1) + (v2+v3)
 *   vcvt_f32_{f16,bf16} exact widening of 4 lanes
 * Every lane operation is written out so the rounding sequence is the one
 * the reference gets on an Apple M-series core.
 */
#pragma once
#include <math.h>
#include <stdint.h>

#ifndef MF_NEON_COMPAT_TYPES
#define MF_NEON_COMPAT_TYPES
typedef float float32x4_t __attribute__((vector_size(16)));
typedef _Float16 float16_t;
typedef __bf16 bfloat16_t;
typedef struct { float16_t v[8]; } float16x8_t;
typedef struct { float16_t v[4]; } float16x4_t;
typedef struct { bfloat16_t v[8]; } bfloat16x8_t;
typedef struct { bfloat16_t v[4]; } bfloat16x4_t;
#endif

static inline float32x4_t vdupq_n_f32(float x) {
    float32x4_t r = {x, x, x, x};
    return r;
}

static inline float32x4_t vld1q_f32(const float* p) {
    float32x4_t r = {p[0], p[1], p[2], p[3]};
    return r;
}

static inline float32x4_t vfmaq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
    float32x4_t r;
    r[0] = fmaf(b[0], c[0], a[0]);
    r[1] = fmaf(b[1], c[1], a[1]);
    r[2] = fmaf(b[2], c[2], a[2]);
    r[3] = fmaf(b[3], c[3], a[3]);
    return r;
}

static inline float32x4_t vaddq_f32(float32x4_t a, float32x4_t b) {
    float32x4_t r;
    r[0] = a[0] + b[0];
    r[1] = a[1] + b[1];
    r[2] = a[2] + b[2];
    r[3] = a[3] + b[3];
    return r;
}

static inline float vaddvq_f32(float32x4_t v) {
    float lo = v[0] + v[1];
    float hi = v[2] + v[3];
    return lo + hi;
}

static inline float16x8_t vld1q_f16(const float16_t* p) {
    float16x8_t r;
    for (int i = 0; i < 8; ++i) r.v[i] = p[i];
    return r;
}

static inline float16x4_t vget_low_f16(float16x8_t a) {
    float16x4_t r;
    for (int i = 0; i < 4; ++i) r.v[i] = a.v[i];
    return r;
}

static inline float16x4_t vget_high_f16(float16x8_t a) {
    float16x4_t r;
    for (int i = 0; i < 4; ++i) r.v[i] = a.v[4 + i];
    return r;
}

static inline float32x4_t vcvt_f32_f16(float16x4_t a) {
    float32x4_t r = {(float)a.v[0], (float)a.v[1], (float)a.v[2], (float)a.v[3]};
    return r;
}

static inline bfloat16x8_t vld1q_bf16(const bfloat16_t* p) {
    bfloat16x8_t r;
    for (int i = 0; i < 8; ++i) r.v[i] = p[i];
    return r;
}

static inline bfloat16x4_t vget_low_bf16(bfloat16x8_t a) {
    bfloat16x4_t r;
    for (int i = 0; i < 4; ++i) r.v[i] = a.v[i];
    return r;
}

static inline bfloat16x4_t vget_high_bf16(bfloat16x8_t a) {
    bfloat16x4_t r;
    for (int i = 0; i < 4; ++i) r.v[i] = a.v[4 + i];
    return r;
}

static inline float32x4_t vcvt_f32_bf16(bfloat16x4_t a) {
    float32x4_t r = {(float)a.v[0], (float)a.v[1], (float)a.v[2], (float)a.v[3]};
    return r;
}
