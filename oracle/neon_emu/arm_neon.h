/* arm_neon.h - a portable C model of the AArch64 Advanced SIMD intrinsics that phonon-2-c's csrc/blas.c,
 * csrc/tensor_ops.c and csrc/encoder.c use.
 * TEST INFRASTRUCTURE ONLY: oracle/Makefile puts this directory first on the include path when it compiles those
 * reference files for an x86 host with __aarch64__, __ARM_NEON and __ARM_FEATURE_DOTPROD defined, so that the
 * reference's NEON and int8 dot-product code paths (csrc/blas.c:76-149, 1068-1447; the NEON branches of
 * csrc/tensor_ops.c and csrc/encoder.c), which only an AArch64 toolchain compiles, run here and can be compared with
 * the C restatement (oracle/fv_oracle.c) and, through it, with the GPU kernels.
 *
 * Each function computes what the Arm architecture manual defines for the instruction behind the intrinsic (the
 * instruction is named beside each one), element by element, in plain C: integer lanes wrap or saturate as the
 * instruction says, FCVTNS rounds to nearest with ties to even and saturates, FMLA is fused (fmaf), FADDP adds
 * neighbouring pairs. Only the intrinsics those three files call are modelled. The vector types are GCC vector
 * types, so the reference's brace-initialised constants (csrc/blas.c:1192-1195) compile unchanged.
 */
#ifndef P2_ORACLE_NEON_EMU_ARM_NEON_H
#define P2_ORACLE_NEON_EMU_ARM_NEON_H

#include <math.h>
#include <stdint.h>
#include <string.h>

typedef int8_t   int8x8_t    __attribute__((vector_size(8)));
typedef int16_t  int16x4_t   __attribute__((vector_size(8)));
typedef int8_t   int8x16_t   __attribute__((vector_size(16)));
typedef uint8_t  uint8x16_t  __attribute__((vector_size(16)));
typedef int16_t  int16x8_t   __attribute__((vector_size(16)));
typedef uint16_t uint16x8_t  __attribute__((vector_size(16)));
typedef int32_t  int32x4_t   __attribute__((vector_size(16)));
typedef uint32_t uint32x4_t  __attribute__((vector_size(16)));
typedef float    float32x4_t __attribute__((vector_size(16)));
typedef struct { int8x16_t val[4]; } int8x16x4_t;

#define P2_NEON_EMU static inline __attribute__((always_inline))

/* ---- loads, stores, broadcasts (LD1, ST1, ST4, DUP) ---------------------------------------------------------- */
P2_NEON_EMU float32x4_t vld1q_f32(const float *p) { float32x4_t v; memcpy(&v, p, 16); return v; }
P2_NEON_EMU int8x16_t vld1q_s8(const int8_t *p) { int8x16_t v; memcpy(&v, p, 16); return v; }
P2_NEON_EMU void vst1q_f32(float *p, float32x4_t v) { memcpy(p, &v, 16); }
P2_NEON_EMU void vst1q_lane_s32(int32_t *p, int32x4_t v, int lane) { int32_t x = v[lane]; memcpy(p, &x, 4); }
/* ST4 {v0, v1, v2, v3}: element i of register j goes to byte 4 i + j. */
P2_NEON_EMU void vst4q_s8(int8_t *p, int8x16x4_t v)
{
    for (int i = 0; i < 16; i++)
        for (int j = 0; j < 4; j++) p[4 * i + j] = v.val[j][i];
}
P2_NEON_EMU float32x4_t vdupq_n_f32(float x) { float32x4_t v = {x, x, x, x}; return v; }
P2_NEON_EMU int32x4_t vdupq_n_s32(int32_t x) { int32x4_t v = {x, x, x, x}; return v; }
P2_NEON_EMU uint32x4_t vdupq_n_u32(uint32_t x) { uint32x4_t v = {x, x, x, x}; return v; }
P2_NEON_EMU uint16x8_t vdupq_n_u16(uint16_t x) { uint16x8_t v = {x, x, x, x, x, x, x, x}; return v; }
P2_NEON_EMU int8x16_t vdupq_n_s8(int8_t x)
{
    int8x16_t v;
    for (int i = 0; i < 16; i++) v[i] = x;
    return v;
}
P2_NEON_EMU uint8x16_t vdupq_n_u8(uint8_t x)
{
    uint8x16_t v;
    for (int i = 0; i < 16; i++) v[i] = x;
    return v;
}

/* ---- bit casts and halves (no instruction; INS/EXT views) ----------------------------------------------------- */
#define P2_NEON_CAST(name, to, from) \
    P2_NEON_EMU to name(from a) { to r; memcpy(&r, &a, sizeof(r)); return r; }
P2_NEON_CAST(vreinterpretq_s8_u8, int8x16_t, uint8x16_t)
P2_NEON_CAST(vreinterpretq_u8_u32, uint8x16_t, uint32x4_t)
P2_NEON_CAST(vreinterpretq_u8_u16, uint8x16_t, uint16x8_t)
P2_NEON_CAST(vreinterpretq_s32_s8, int32x4_t, int8x16_t)
P2_NEON_CAST(vreinterpretq_f32_s32, float32x4_t, int32x4_t)
#undef P2_NEON_CAST

P2_NEON_EMU int8x8_t vget_low_s8(int8x16_t a) { int8x8_t r; memcpy(&r, &a, 8); return r; }
P2_NEON_EMU int8x8_t vget_high_s8(int8x16_t a) { int8x8_t r; memcpy(&r, (const char *)&a + 8, 8); return r; }
P2_NEON_EMU int16x4_t vget_low_s16(int16x8_t a) { int16x4_t r; memcpy(&r, &a, 8); return r; }
P2_NEON_EMU int16x4_t vget_high_s16(int16x8_t a) { int16x4_t r; memcpy(&r, (const char *)&a + 8, 8); return r; }
P2_NEON_EMU int8x16_t vcombine_s8(int8x8_t lo, int8x8_t hi)
{
    int8x16_t r;
    memcpy(&r, &lo, 8); memcpy((char *)&r + 8, &hi, 8);
    return r;
}
P2_NEON_EMU int16x8_t vcombine_s16(int16x4_t lo, int16x4_t hi)
{
    int16x8_t r;
    memcpy(&r, &lo, 8); memcpy((char *)&r + 8, &hi, 8);
    return r;
}

/* ---- widening, narrowing, conversions (SXTL, SQXTN, SCVTF, FCVTNS) -------------------------------------------- */
P2_NEON_EMU int16x8_t vmovl_s8(int8x8_t a)
{
    int16x8_t r;
    for (int i = 0; i < 8; i++) r[i] = a[i];
    return r;
}
P2_NEON_EMU int32x4_t vmovl_s16(int16x4_t a)
{
    int32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = a[i];
    return r;
}
P2_NEON_EMU int16x4_t vqmovn_s32(int32x4_t a)
{
    int16x4_t r;
    for (int i = 0; i < 4; i++) r[i] = (int16_t)(a[i] > 32767 ? 32767 : a[i] < -32768 ? -32768 : a[i]);
    return r;
}
P2_NEON_EMU int8x8_t vqmovn_s16(int16x8_t a)
{
    int8x8_t r;
    for (int i = 0; i < 8; i++) r[i] = (int8_t)(a[i] > 127 ? 127 : a[i] < -128 ? -128 : a[i]);
    return r;
}
P2_NEON_EMU float32x4_t vcvtq_f32_s32(int32x4_t a)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = (float)a[i];   /* round to nearest even, as SCVTF under the default FPCR */
    return r;
}
/* FCVTNS: round to nearest, ties to even; NaN gives 0; out of range saturates. Integer arithmetic on the float's
 * bits, so no compiler flag and no rounding mode changes it. */
P2_NEON_EMU int32_t p2_neon_emu_fcvtns(float x)
{
    uint32_t u; memcpy(&u, &x, 4);
    const int neg = (int)(u >> 31);
    const int e = (int)((u >> 23) & 0xFF);
    uint32_t m = u & 0x7FFFFFu;
    if (e == 0xFF) return m ? 0 : (neg ? INT32_MIN : INT32_MAX);
    if (e < 126) return 0;                          /* |x| < 0.5 (zeros and denormals included) */
    m |= 0x800000u;                                 /* value = m · 2^(e − 150) */
    int64_t mag;
    if (e >= 150) {
        if (e - 150 > 31) mag = (int64_t)1 << 40;
        else mag = (int64_t)m << (e - 150);
    } else {
        const int sh = 150 - e;                     /* 1 .. 24 */
        const uint32_t q = m >> sh, rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
        mag = q + ((rem > half || (rem == half && (q & 1u))) ? 1 : 0);
    }
    const int64_t v = neg ? -mag : mag;
    return (int32_t)(v > INT32_MAX ? INT32_MAX : v < INT32_MIN ? INT32_MIN : v);
}
P2_NEON_EMU int32x4_t vcvtnq_s32_f32(float32x4_t a)
{
    int32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = p2_neon_emu_fcvtns(a[i]);
    return r;
}
/* FCVTZS: toward zero; NaN gives 0; out of range saturates. */
P2_NEON_EMU int32x4_t vcvtq_s32_f32(float32x4_t a)
{
    int32x4_t r;
    for (int i = 0; i < 4; i++) {
        const float x = a[i];
        r[i] = x != x ? 0 : x >= 2147483648.0f ? INT32_MAX : x <= -2147483648.0f ? INT32_MIN : (int32_t)x;
    }
    return r;
}

/* ---- fp32 arithmetic (FADD, FMUL, FSUB, FDIV, FNEG, FMLA, FABS, FMAX, FMIN, FMAXV, FADDP, FRINTN) --------------- */
P2_NEON_EMU float32x4_t vaddq_f32(float32x4_t a, float32x4_t b)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = a[i] + b[i];
    return r;
}
P2_NEON_EMU float32x4_t vdivq_f32(float32x4_t a, float32x4_t b)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = a[i] / b[i];
    return r;
}
/* FNEG flips the sign bit. */
P2_NEON_EMU float32x4_t vnegq_f32(float32x4_t a)
{
    uint32x4_t u; memcpy(&u, &a, 16);
    for (int i = 0; i < 4; i++) u[i] ^= 0x80000000u;
    float32x4_t r; memcpy(&r, &u, 16);
    return r;
}
/* FMLA by a scalar: a + b · s with one rounding. */
P2_NEON_EMU float32x4_t vfmaq_n_f32(float32x4_t a, float32x4_t b, float s)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = fmaf(b[i], s, a[i]);
    return r;
}
/* FRINTN: to an integral float, ties to even (the default rounding mode; nearbyintf raises no inexact flag). */
P2_NEON_EMU float32x4_t vrndnq_f32(float32x4_t a)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = nearbyintf(a[i]);
    return r;
}
P2_NEON_EMU float32x4_t vmulq_f32(float32x4_t a, float32x4_t b)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = a[i] * b[i];
    return r;
}
P2_NEON_EMU float32x4_t vmulq_n_f32(float32x4_t a, float b)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = a[i] * b;
    return r;
}
P2_NEON_EMU float32x4_t vsubq_f32(float32x4_t a, float32x4_t b)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = a[i] - b[i];
    return r;
}
/* FMLA: a + b · c with one rounding. */
P2_NEON_EMU float32x4_t vfmaq_f32(float32x4_t a, float32x4_t b, float32x4_t c)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = fmaf(b[i], c[i], a[i]);
    return r;
}
/* FABS clears the sign bit. */
P2_NEON_EMU float32x4_t vabsq_f32(float32x4_t a)
{
    uint32x4_t u; memcpy(&u, &a, 16);
    for (int i = 0; i < 4; i++) u[i] &= 0x7FFFFFFFu;
    float32x4_t r; memcpy(&r, &u, 16);
    return r;
}
/* FMAX: a NaN operand gives NaN; max(+0, −0) = +0. */
P2_NEON_EMU float p2_neon_emu_fmax(float a, float b)
{
    if (a != a) return a;
    if (b != b) return b;
    if (a == 0.0f && b == 0.0f) return signbit(a) ? b : a;
    return a > b ? a : b;
}
P2_NEON_EMU float32x4_t vmaxq_f32(float32x4_t a, float32x4_t b)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = p2_neon_emu_fmax(a[i], b[i]);
    return r;
}
/* FMIN: a NaN operand gives NaN; min(+0, −0) = −0. */
P2_NEON_EMU float p2_neon_emu_fmin(float a, float b)
{
    if (a != a) return a;
    if (b != b) return b;
    if (a == 0.0f && b == 0.0f) return signbit(a) ? a : b;
    return a < b ? a : b;
}
P2_NEON_EMU float32x4_t vminq_f32(float32x4_t a, float32x4_t b)
{
    float32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = p2_neon_emu_fmin(a[i], b[i]);
    return r;
}
/* FMAXV over four lanes: max(max(a0, a1), max(a2, a3)). */
P2_NEON_EMU float vmaxvq_f32(float32x4_t a)
{
    return p2_neon_emu_fmax(p2_neon_emu_fmax(a[0], a[1]), p2_neon_emu_fmax(a[2], a[3]));
}
/* FADDP twice: (a0 + a1) + (a2 + a3). The volatile temporaries keep a -ffast-math build from re-associating it. */
P2_NEON_EMU float vaddvq_f32(float32x4_t a)
{
    volatile float s01 = a[0] + a[1], s23 = a[2] + a[3];
    return s01 + s23;
}

/* ---- integer lane arithmetic and bit ops (ADD, SHL, SUB, NEG, MUL, AND, CMTST, BSL, USHL, TBL, SDOT) ------------ */
P2_NEON_EMU int32x4_t vaddq_s32(int32x4_t a, int32x4_t b)
{
    int32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = (int32_t)((uint32_t)a[i] + (uint32_t)b[i]);
    return r;
}
/* SHL by an immediate: the low bits shifted out, as an unsigned shift. */
P2_NEON_EMU int32x4_t vshlq_n_s32(int32x4_t a, int n)
{
    int32x4_t r;
    for (int i = 0; i < 4; i++) r[i] = (int32_t)((uint32_t)a[i] << n);
    return r;
}
P2_NEON_EMU int8x16_t vsubq_s8(int8x16_t a, int8x16_t b)
{
    int8x16_t r;
    for (int i = 0; i < 16; i++) r[i] = (int8_t)(uint8_t)((uint8_t)a[i] - (uint8_t)b[i]);
    return r;
}
P2_NEON_EMU int8x16_t vnegq_s8(int8x16_t a)
{
    int8x16_t r;
    for (int i = 0; i < 16; i++) r[i] = (int8_t)(uint8_t)(0u - (uint8_t)a[i]);
    return r;
}
P2_NEON_EMU int8x16_t vmulq_s8(int8x16_t a, int8x16_t b)
{
    int8x16_t r;
    for (int i = 0; i < 16; i++) r[i] = (int8_t)(uint8_t)((unsigned)(uint8_t)a[i] * (unsigned)(uint8_t)b[i]);
    return r;
}
P2_NEON_EMU uint8x16_t vandq_u8(uint8x16_t a, uint8x16_t b) { return a & b; }
P2_NEON_EMU int8x16_t vandq_s8(int8x16_t a, int8x16_t b) { return a & b; }
/* CMTST: all ones where a & b is nonzero. */
P2_NEON_EMU uint8x16_t vtstq_s8(int8x16_t a, int8x16_t b)
{
    uint8x16_t r;
    for (int i = 0; i < 16; i++) r[i] = (a[i] & b[i]) ? 0xFF : 0;
    return r;
}
/* BSL: bits of a where the mask is set, of b elsewhere. */
P2_NEON_EMU int8x16_t vbslq_s8(uint8x16_t mask, int8x16_t a, int8x16_t b)
{
    int8x16_t r;
    for (int i = 0; i < 16; i++) r[i] = (int8_t)((mask[i] & (uint8_t)a[i]) | (~mask[i] & (uint8_t)b[i]));
    return r;
}
/* USHL: shift each byte left by the signed count in the low byte of b; a negative count shifts right (logical);
 * counts of 8 or more either way give 0. */
P2_NEON_EMU uint8x16_t vshlq_u8(uint8x16_t a, int8x16_t b)
{
    uint8x16_t r;
    for (int i = 0; i < 16; i++) {
        const int s = b[i];
        r[i] = (s >= 8 || s <= -8) ? 0 : s >= 0 ? (uint8_t)(a[i] << s) : (uint8_t)(a[i] >> -s);
    }
    return r;
}
/* TBL with one table register: an index of 16 or more gives 0. */
P2_NEON_EMU uint8x16_t vqtbl1q_u8(uint8x16_t t, uint8x16_t idx)
{
    uint8x16_t r;
    for (int i = 0; i < 16; i++) r[i] = idx[i] < 16 ? t[idx[i]] : 0;
    return r;
}
/* SDOT (by element): lane i of acc gains the dot product of bytes 4i..4i+3 of a with bytes 4·lane..4·lane+3 of b. */
P2_NEON_EMU int32x4_t vdotq_laneq_s32(int32x4_t acc, int8x16_t a, int8x16_t b, int lane)
{
    int32x4_t r;
    for (int i = 0; i < 4; i++) {
        int32_t s = 0;
        for (int t = 0; t < 4; t++) s += (int32_t)a[4 * i + t] * (int32_t)b[4 * lane + t];
        r[i] = (int32_t)((uint32_t)acc[i] + (uint32_t)s);
    }
    return r;
}

#undef P2_NEON_EMU
#endif /* P2_ORACLE_NEON_EMU_ARM_NEON_H */
