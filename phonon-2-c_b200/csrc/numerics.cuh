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
__device__ __forceinline__ float exp_poly(float x) {
    x = fminf(fmaxf(x, -87.0f), 87.0f);
    const float kf = rintf(__fmul_rn(x, 1.44269504088896341f));
    const int ki = static_cast<int>(kf);
    const float r = __fmaf_rn(-kf, 0.69314718055994529f, x);
    float y = 1.0f / 120.0f;
    y = __fmaf_rn(y, r, 1.0f / 24.0f);
    y = __fmaf_rn(y, r, 1.0f / 6.0f);
    y = __fmaf_rn(y, r, 0.5f);
    y = __fmaf_rn(y, r, 1.0f);
    y = __fmaf_rn(y, r, 1.0f);
    return __fmul_rn(y, __int_as_float((ki + 127) << 23));
}

// SiLU as the reference's vector loop computes it (csrc/tensor_ops.c:450-458): v * (1 / (1 + exp(0 - v))).
__device__ __forceinline__ float swish1(float v) {
    const float e = exp_poly(__fsub_rn(0.0f, v));
    return __fmul_rn(v, __frcp_rn(__fadd_rn(1.0f, e)));
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
