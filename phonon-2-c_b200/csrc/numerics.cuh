// numerics.cuh - device helpers shared by the kernels that restate the reference's fp32 arithmetic.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace p2cu {

// One value of the reference's per-row int8 quantisation (csrc/blas.c:1123-1131): saturate(round_half_even(x * inv)).
// The conversion saturates and maps NaN to 0, as the reference's FCVTNS does when 1 / scale overflows to infinity.
__device__ __forceinline__ int8_t quant_one(float x, float inv) {
    int v = __float2int_rn(__fmul_rn(x, inv));
    v = v > 127 ? 127 : (v < -128 ? -128 : v);
    return static_cast<int8_t>(v);
}

// The row's scale and the reciprocal the 16-wide loop multiplies by. fm = 0: the reference's C source as written
// (csrc/blas.c:1120-1121, IEEE): scale = amax / 127, inv = 1 / scale. fm = 1: what its Makefile's build with
// -ffast-math computes (csrc/Makefile:2, measured on that build compiled here): scale = amax * (1/127) (the reciprocal
// of 127 rounded to fp32) and inv = 127 / amax (the compiler folds 1 / (amax / 127) into one division). Both are 1 for
// an all-zero row.
struct QuantRule { float scale, inv; };
// Host side: the rule every quantising kernel launched from now on follows (0 IEEE, 1 the -ffast-math build's; from
// P2CU_QUANT_FAST_MATH when first asked, p2cu_set_quant_fast_math after that). A captured graph keeps the rule its
// launches were captured with.
int quant_fast_math();
void set_quant_fast_math(int on);
__device__ __forceinline__ QuantRule quant_rule(float amax, int fm) {
    if (!(amax > 0.f)) return {1.0f, 1.0f};
    if (fm) return {__fmul_rn(amax, __int_as_float(0x3C010204)), __fdiv_rn(127.0f, amax)};
    const float scale = __fdiv_rn(amax, 127.0f);
    return {scale, __fdiv_rn(1.0f, scale)};
}

// The reference quantises the first K - K % 16 values of a row in its 16-wide loop (quant_one) and the last K % 16
// in a scalar tail, clamp(lrintf(x / scale), -127, 127) (csrc/blas.c:1139-1143): a division instead of the reciprocal,
// so a value near a half can round the other way. Its -ffast-math build (fm = 1) multiplies by inv there too, and a
// product that is not finite (inv overflowed: a row whose maximum is below about 1e-39) comes out of its lrintf and
// int conversion as 0.
__device__ __forceinline__ int8_t quant_tail(float x, float scale, float inv, int fm) {
    const float t = fm ? __fmul_rn(x, inv) : __fdiv_rn(x, scale);
    if (fm && !isfinite(t)) return 0;
    int v = __float2int_rn(t);
    v = v > 127 ? 127 : (v < -127 ? -127 : v);
    return static_cast<int8_t>(v);
}

// Value k of a quantised row of K values.
__device__ __forceinline__ int8_t quant_at(float x, const QuantRule& r, int k, int K, int fm) {
    return k < (K & ~15) ? quant_one(x, r.inv) : quant_tail(x, r.scale, r.inv, fm);
}

// exp(x) as the reference's AVX2 path evaluates it (csrc/tensor_ops.c:154-172): clamp to [-87, 87], k = round(x *
// log2 e), r = x - k * ln 2, a degree-5 Taylor polynomial in r by Horner's rule, times 2^k built in the exponent
// bits. The compiled reference fuses r into one fused multiply-subtract, as here.
//
// k is read off t + 1.5 * 2^23 (t = x log2 e, |t| <= 125.6): that sum lies in [2^23, 2^24), where the fp32 grid is
// the integers, so the addition rounds t half to even, exactly as rintf does, and the sum's bits are 0x4B400000 + k
// (checked for every fp32 |t| <= 126). It keeps the rounding and the conversion to an integer off the conversion
// unit, which runs at a quarter of the FMA rate. 2^k's bits (k + 127) << 23 are then (bits + 127) << 23: 0x4B400000
// shifted left by 23 leaves 32 bits.
__device__ __forceinline__ float exp_poly(float x) {
    x = fminf(fmaxf(x, -87.0f), 87.0f);
    const float sh = __fadd_rn(__fmul_rn(x, 1.44269504088896341f), 12582912.0f);
    const float kf = __fsub_rn(sh, 12582912.0f);
    const float r = __fmaf_rn(-kf, 0.69314718055994529f, x);
    float y = 1.0f / 120.0f;
    y = __fmaf_rn(y, r, 1.0f / 24.0f);
    y = __fmaf_rn(y, r, 1.0f / 6.0f);
    y = __fmaf_rn(y, r, 0.5f);
    y = __fmaf_rn(y, r, 1.0f);
    y = __fmaf_rn(y, r, 1.0f);
    return __fmul_rn(y, __int_as_float(static_cast<int>((__float_as_uint(sh) + 127u) << 23)));
}

// SiLU as the reference's vector loop computes it (csrc/tensor_ops.c:450-458): v * (1 / (1 + exp(0 - v))).
__device__ __forceinline__ float swish1(float v) {
    const float e = exp_poly(__fsub_rn(0.0f, v));
    return __fmul_rn(v, __frcp_rn(__fadd_rn(1.0f, e)));
}

// ---- two values per instruction: sm_100's packed fp32 arithmetic (PTX add / sub / mul / fma .rn.f32x2) ----------
//
// Each lane of a packed operation is the IEEE single-precision operation of its scalar form (round to nearest even,
// no flush to zero), so a formula written with them gives the scalar formula's bits lane by lane at half the issue
// slots for its adds, multiplies and FMAs - as long as no packed product whose rounding matters feeds a packed add
// (see exp_poly2).
__device__ __forceinline__ unsigned long long f2_pack(float2 v) {
    return (static_cast<unsigned long long>(__float_as_uint(v.y)) << 32) | __float_as_uint(v.x);
}
__device__ __forceinline__ float2 f2_unpack(unsigned long long u) {
    return make_float2(__uint_as_float(static_cast<unsigned>(u)), __uint_as_float(static_cast<unsigned>(u >> 32)));
}
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_pack(a)), "l"(f2_pack(b)), "l"(f2_pack(c)));
    return f2_unpack(d);
}
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_pack(a)), "l"(f2_pack(b)));
    return f2_unpack(d);
}
__device__ __forceinline__ float2 f2_sub(float2 a, float2 b) {
    unsigned long long d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_pack(a)), "l"(f2_pack(b)));
    return f2_unpack(d);
}
__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_pack(a)), "l"(f2_pack(b)));
    return f2_unpack(d);
}
__device__ __forceinline__ float2 f2_splat(float c) { return make_float2(c, c); }

// exp_poly on two values: the same operations in the same order (r = x - k ln 2 as fma(k, -ln 2, x), the same
// exactly rounded value as fma(-k, ln 2, x)). The products x log2 e stay scalar: a packed multiply whose result
// feeds a packed add can be contracted into one packed FMA (the .rn of the packed forms does not forbid it as it does
// for the scalar ones), which rounds x log2 e + 1.5 * 2^23 once and picks the other k wherever x log2 e lies within
// an ulp of a half (measured: 122 of the 2^32 inputs). y 2^k below is exact (a power of two, normal results), so its
// product may fuse into a following add without changing a bit.
__device__ __forceinline__ float2 exp_poly2(float2 x) {
    x.x = fminf(fmaxf(x.x, -87.0f), 87.0f);
    x.y = fminf(fmaxf(x.y, -87.0f), 87.0f);
    const float2 t = make_float2(__fmul_rn(x.x, 1.44269504088896341f), __fmul_rn(x.y, 1.44269504088896341f));
    const float2 sh = f2_add(t, f2_splat(12582912.0f));
    const float2 kf = f2_sub(sh, f2_splat(12582912.0f));
    const float2 r = f2_fma(kf, f2_splat(-0.69314718055994529f), x);
    float2 y = f2_splat(1.0f / 120.0f);
    y = f2_fma(y, r, f2_splat(1.0f / 24.0f));
    y = f2_fma(y, r, f2_splat(1.0f / 6.0f));
    y = f2_fma(y, r, f2_splat(0.5f));
    y = f2_fma(y, r, f2_splat(1.0f));
    y = f2_fma(y, r, f2_splat(1.0f));
    const float2 p2k = make_float2(__uint_as_float((__float_as_uint(sh.x) + 127u) << 23),
                                   __uint_as_float((__float_as_uint(sh.y) + 127u) << 23));
    return f2_mul(y, p2k);
}

// 1 / d, correctly rounded, for d in [1, 2^126), two values at a time; nd = -d. From the hardware estimate
// (rcp.approx, within an ulp) two steps of Markstein's correction y + y (1 - d y) (P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990): once y is within an ulp
// of 1 / d, 1 - d y is exact in one FMA and the last step rounds correctly. Checked against __frcp_rn for every fp32 d
// in the range; results are normal there (above 2^-126), so the estimate's flush to zero never applies.
__device__ __forceinline__ float2 rcp2_ge1(float2 d, float2 nd) {
    float2 y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y.x) : "f"(d.x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y.y) : "f"(d.y));
    float2 e = f2_fma(nd, y, f2_splat(1.0f));
    y = f2_fma(e, y, y);
    e = f2_fma(nd, y, f2_splat(1.0f));
    return f2_fma(e, y, y);
}

// swish1 on two values. 1 + e lies in [1, 2^126) (e <= exp_poly(87) = 0.71 * 2^126), the range of rcp2_ge1, and
// -1 - e is exactly -(1 + e).
__device__ __forceinline__ float2 swish2(float2 v) {
    const float2 e = exp_poly2(f2_sub(f2_splat(0.0f), v));
    return f2_mul(v, rcp2_ge1(f2_add(f2_splat(1.0f), e), f2_sub(f2_splat(-1.0f), e)));
}

// Sum of the eight lanes of an 8-lane group in the order of the reference's AVX2 horizontal sum
// (csrc/tensor_ops.c:182-190): ((v0 + v4) + (v2 + v6)) + ((v1 + v5) + (v3 + v7)); every lane of the group gets it.
__device__ __forceinline__ float hsum8(float v) {
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4, 8));
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2, 8));
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1, 8));
    return __shfl_sync(0xffffffffu, v, 0, 8);
}

__device__ __forceinline__ float max8(float v) {
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4, 8));
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2, 8));
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1, 8));
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// The window that row r belongs to: the largest w with off[w] <= r (off holds n + 1 prefix offsets).
__device__ __forceinline__ int find_window(const int* __restrict__ off, int n, int r) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (off[mid] <= r) lo = mid; else hi = mid - 1;
    }
    return lo;
}

}  // namespace p2cu
