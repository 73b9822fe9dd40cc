/*
 * arm_neon.h -- portable scalar stand-in for the Arm NEON intrinsics the qma
 * reference engine uses, so the reference's own C sources build on x86_64
 * as a CPU oracle.  TEST INFRASTRUCTURE ONLY: nothing in the CUDA engine
 * includes or links this file.
 *
 * Each function is written from the public Arm C Language Extensions (ACLE)
 * description of the intrinsic of the same name, lane by lane:
 *   - vmlaq_f32 is an UNFUSED multiply then add (AArch64 lowers it to FMUL +
 *     FADD); vfmaq_n_f32 is FUSED (FMLA), written with fmaf().
 *   - vaddvq_f32 follows the AArch64 FADDP tree: (a0 + a1) + (a2 + a3).
 *   - vcvtaq_s32_f32 rounds to nearest with ties away from zero (FCVTAS),
 *     vcvtq_s32_f32 truncates toward zero (FCVTZS); both saturate.
 *   - vqmovn_* saturate to the narrower type.
 *   - vdotq_s32 (SDOT) adds, per 32-bit lane i, the four products of bytes
 *     4i..4i+3 to the accumulator lane.
 * Build the reference with -fno-strict-aliasing: it reinterprets arrays of
 * these vector structs as plain float arrays.
 */
#ifndef QMA_ORACLE_ARM_NEON_SHIM_H
#define QMA_ORACLE_ARM_NEON_SHIM_H

#include <stdint.h>
#include <math.h>

typedef struct { float    v[4];  } float32x4_t;
typedef struct { int32_t  v[4];  } int32x4_t;
typedef struct { uint32_t v[4];  } uint32x4_t;
typedef struct { int16_t  v[4];  } int16x4_t;
typedef struct { int16_t  v[8];  } int16x8_t;
typedef struct { uint16_t v[4];  } uint16x4_t;
typedef struct { uint16_t v[8];  } uint16x8_t;
typedef struct { int8_t   v[8];  } int8x8_t;
typedef struct { uint8_t  v[8];  } uint8x8_t;
typedef struct { int8_t   v[16]; } int8x16_t;
typedef struct { uint8_t  v[16]; } uint8x16_t;

#define QN_STATIC static inline

/* ---- saturation helpers ------------------------------------------------ */
QN_STATIC int32_t qn_sat_f32_s32(float x) {
    if (x != x) return 0;                       /* NaN -> 0 (FCVT*S) */
    if (x >= 2147483648.0f) return INT32_MAX;
    if (x < -2147483648.0f) return INT32_MIN;
    return (int32_t)x;
}
QN_STATIC int16_t qn_sat_s16(int32_t x) {
    return (int16_t)(x > INT16_MAX ? INT16_MAX : (x < INT16_MIN ? INT16_MIN : x));
}
QN_STATIC int8_t qn_sat_s8(int32_t x) {
    return (int8_t)(x > INT8_MAX ? INT8_MAX : (x < INT8_MIN ? INT8_MIN : x));
}

/* ---- duplicate / load / store ----------------------------------------- */
QN_STATIC float32x4_t vdupq_n_f32(float a) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a; return r; }
QN_STATIC int32x4_t  vdupq_n_s32(int32_t a) { int32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a; return r; }
QN_STATIC uint8x16_t vdupq_n_u8(uint8_t a) { uint8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = a; return r; }
QN_STATIC int8x16_t  vdupq_n_s8(int8_t a) { int8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = a; return r; }

QN_STATIC float32x4_t vld1q_f32(const float *p) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = p[i]; return r; }
QN_STATIC uint8x16_t  vld1q_u8(const uint8_t *p) { uint8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = p[i]; return r; }
QN_STATIC int8x16_t   vld1q_s8(const int8_t *p) { int8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = p[i]; return r; }
QN_STATIC void vst1q_f32(float *p, float32x4_t a) { for (int i = 0; i < 4; i++) p[i] = a.v[i]; }
QN_STATIC void vst1_s8(int8_t *p, int8x8_t a) { for (int i = 0; i < 8; i++) p[i] = a.v[i]; }

/* ---- float arithmetic -------------------------------------------------- */
QN_STATIC float32x4_t vabsq_f32(float32x4_t a) { for (int i = 0; i < 4; i++) a.v[i] = fabsf(a.v[i]); return a; }
QN_STATIC float32x4_t vmaxq_f32(float32x4_t a, float32x4_t b) {
    for (int i = 0; i < 4; i++) {
        float x = a.v[i], y = b.v[i];
        a.v[i] = (x != x || y != y) ? NAN : (x > y ? x : y);
    }
    return a;
}
QN_STATIC float vmaxvq_f32(float32x4_t a) {
    /* FMAXV: pairwise maximum tree */
    float m01 = a.v[0] > a.v[1] ? a.v[0] : a.v[1];
    float m23 = a.v[2] > a.v[3] ? a.v[2] : a.v[3];
    return m01 > m23 ? m01 : m23;
}
QN_STATIC float32x4_t vmulq_n_f32(float32x4_t a, float b) { for (int i = 0; i < 4; i++) a.v[i] = a.v[i] * b; return a; }
QN_STATIC float32x4_t vmlaq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
    for (int i = 0; i < 4; i++) { float p = b.v[i] * c.v[i]; a.v[i] = a.v[i] + p; }
    return a;
}
QN_STATIC float32x4_t vfmaq_n_f32(float32x4_t a, float32x4_t b, float n) {
    for (int i = 0; i < 4; i++) a.v[i] = fmaf(b.v[i], n, a.v[i]);
    return a;
}
QN_STATIC float vaddvq_f32(float32x4_t a) {
    float s01 = a.v[0] + a.v[1];
    float s23 = a.v[2] + a.v[3];
    return s01 + s23;
}

/* ---- conversions ------------------------------------------------------- */
QN_STATIC int32x4_t vcvtaq_s32_f32(float32x4_t a) {
    int32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = qn_sat_f32_s32(roundf(a.v[i])); return r;
}
QN_STATIC int32x4_t vcvtq_s32_f32(float32x4_t a) {
    int32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = qn_sat_f32_s32(truncf(a.v[i])); return r;
}
QN_STATIC float32x4_t vcvtq_f32_s32(int32x4_t a) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = (float)a.v[i]; return r; }
QN_STATIC float32x4_t vcvtq_f32_u32(uint32x4_t a) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = (float)a.v[i]; return r; }

/* ---- integer arithmetic ------------------------------------------------ */
QN_STATIC int32x4_t vminq_s32(int32x4_t a, int32x4_t b) { for (int i = 0; i < 4; i++) a.v[i] = a.v[i] < b.v[i] ? a.v[i] : b.v[i]; return a; }
QN_STATIC int32x4_t vmaxq_s32(int32x4_t a, int32x4_t b) { for (int i = 0; i < 4; i++) a.v[i] = a.v[i] > b.v[i] ? a.v[i] : b.v[i]; return a; }
QN_STATIC int32x4_t vmlaq_n_s32(int32x4_t a, int32x4_t b, int32_t n) {
    for (int i = 0; i < 4; i++) a.v[i] = (int32_t)((uint32_t)a.v[i] + (uint32_t)b.v[i] * (uint32_t)n);
    return a;
}
QN_STATIC int32_t vaddvq_s32(int32x4_t a) {
    return (int32_t)((uint32_t)a.v[0] + (uint32_t)a.v[1] + (uint32_t)a.v[2] + (uint32_t)a.v[3]);
}
QN_STATIC int16x8_t vaddq_s16(int16x8_t a, int16x8_t b) {
    for (int i = 0; i < 8; i++) a.v[i] = (int16_t)(uint16_t)((uint16_t)a.v[i] + (uint16_t)b.v[i]);
    return a;
}
QN_STATIC int16_t vaddvq_s16(int16x8_t a) {
    uint16_t s = 0; for (int i = 0; i < 8; i++) s = (uint16_t)(s + (uint16_t)a.v[i]);
    return (int16_t)s;
}
QN_STATIC int8x16_t vsubq_s8(int8x16_t a, int8x16_t b) {
    for (int i = 0; i < 16; i++) a.v[i] = (int8_t)(uint8_t)((uint8_t)a.v[i] - (uint8_t)b.v[i]);
    return a;
}
QN_STATIC int32x4_t vdotq_s32(int32x4_t acc, int8x16_t a, int8x16_t b) {
    for (int i = 0; i < 4; i++) {
        int32_t s = 0;
        for (int j = 0; j < 4; j++) s += (int32_t)a.v[4 * i + j] * (int32_t)b.v[4 * i + j];
        acc.v[i] = (int32_t)((uint32_t)acc.v[i] + (uint32_t)s);
    }
    return acc;
}

/* ---- narrowing / widening --------------------------------------------- */
QN_STATIC int16x4_t vqmovn_s32(int32x4_t a) { int16x4_t r; for (int i = 0; i < 4; i++) r.v[i] = qn_sat_s16(a.v[i]); return r; }
QN_STATIC int8x8_t  vqmovn_s16(int16x8_t a) { int8x8_t r; for (int i = 0; i < 8; i++) r.v[i] = qn_sat_s8(a.v[i]); return r; }
QN_STATIC int16x8_t vcombine_s16(int16x4_t lo, int16x4_t hi) {
    int16x8_t r; for (int i = 0; i < 4; i++) { r.v[i] = lo.v[i]; r.v[i + 4] = hi.v[i]; } return r;
}
QN_STATIC uint8x8_t vget_low_u8(uint8x16_t a)  { uint8x8_t r; for (int i = 0; i < 8; i++) r.v[i] = a.v[i]; return r; }
QN_STATIC uint8x8_t vget_high_u8(uint8x16_t a) { uint8x8_t r; for (int i = 0; i < 8; i++) r.v[i] = a.v[i + 8]; return r; }
QN_STATIC uint16x4_t vget_low_u16(uint16x8_t a)  { uint16x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a.v[i]; return r; }
QN_STATIC uint16x4_t vget_high_u16(uint16x8_t a) { uint16x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a.v[i + 4]; return r; }
QN_STATIC uint16x8_t vmovl_u8(uint8x8_t a)  { uint16x8_t r; for (int i = 0; i < 8; i++) r.v[i] = a.v[i]; return r; }
QN_STATIC uint32x4_t vmovl_u16(uint16x4_t a) { uint32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a.v[i]; return r; }

/* ---- bitwise / shifts / permutes -------------------------------------- */
QN_STATIC uint8x16_t vandq_u8(uint8x16_t a, uint8x16_t b) { for (int i = 0; i < 16; i++) a.v[i] &= b.v[i]; return a; }
QN_STATIC uint8x16_t vorrq_u8(uint8x16_t a, uint8x16_t b) { for (int i = 0; i < 16; i++) a.v[i] |= b.v[i]; return a; }
#define vshrq_n_u8(a, n) qn_shr_u8((a), (n))
#define vshlq_n_u8(a, n) qn_shl_u8((a), (n))
QN_STATIC uint8x16_t qn_shr_u8(uint8x16_t a, int n) { for (int i = 0; i < 16; i++) a.v[i] = (uint8_t)(a.v[i] >> n); return a; }
QN_STATIC uint8x16_t qn_shl_u8(uint8x16_t a, int n) { for (int i = 0; i < 16; i++) a.v[i] = (uint8_t)(a.v[i] << n); return a; }
QN_STATIC int8x16_t vreinterpretq_s8_u8(uint8x16_t a) { int8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = (int8_t)a.v[i]; return r; }
QN_STATIC uint8x16_t vzip1q_u8(uint8x16_t a, uint8x16_t b) {
    uint8x16_t r; for (int i = 0; i < 8; i++) { r.v[2 * i] = a.v[i]; r.v[2 * i + 1] = b.v[i]; } return r;
}
QN_STATIC uint8x16_t vzip2q_u8(uint8x16_t a, uint8x16_t b) {
    uint8x16_t r; for (int i = 0; i < 8; i++) { r.v[2 * i] = a.v[i + 8]; r.v[2 * i + 1] = b.v[i + 8]; } return r;
}

#endif /* QMA_ORACLE_ARM_NEON_SHIM_H */
