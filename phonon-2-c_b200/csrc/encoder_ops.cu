// encoder_ops.cu - the FastConformer encoder's memory-bound ops on the device.
//
// Each kernel restates one of the reference's CPU loops (csrc/encoder.c, csrc/tensor_ops.c) in fp32 with the same
// operations in the same order where the result depends on it and the order can be reproduced: the polynomial exp of
// the vector loops, the FMA chains of the convolutions in tap order, the attention products as one FMA chain per
// output. Sums over a row (LayerNorm, softmax) are tree-ordered: the compiled reference's own results there depend on
// the host CPU (its -ffast-math build computes 1/sqrt with an approximate reciprocal square root refined by one Newton
// step, and calls a vectorised expf for short tails), so no order reproduces it bit for bit; these kernels agree with
// it to an ulp or two.
//
// Layout: activations are row-major [rows][features] and a batch of windows is stacked along the rows. Ops that
// look across rows (convolutions over time, attention) find a row's window in prefix tables of row offsets.
#include <cfloat>
#include <cstdint>
#include <cuda_runtime.h>
#include "encoder_ops.h"
#include "fv_gemm.h"
#include "kernels.h"
#include "numerics.cuh"

namespace p2cu {

namespace {

constexpr unsigned FULL = 0xffffffffu;

// ---- LayerNorm (csrc/tensor_ops.c:204-281): mean, variance, y = fma((x - mean) * inv_std, gamma, beta) ---------
//
// One warp per row with the row held in registers (one read of x, one write of y). The sums are tree-ordered; the
// reference sums in 8 lanes and takes 1/sqrt from an approximate reciprocal square root plus a Newton step, so the
// two agree to an ulp or two, not bit for bit, whatever order is used here.

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float4 ln_apply(float4 v, float mean, float inv, float4 g, float4 b) {
    return make_float4(__fmaf_rn(__fmul_rn(__fsub_rn(v.x, mean), inv), g.x, b.x),
                       __fmaf_rn(__fmul_rn(__fsub_rn(v.y, mean), inv), g.y, b.y),
                       __fmaf_rn(__fmul_rn(__fsub_rn(v.z, mean), inv), g.z, b.z),
                       __fmaf_rn(__fmul_rn(__fsub_rn(v.w, mean), inv), g.w, b.w));
}

__device__ __forceinline__ float amax4(float4 v) {
    return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

// quant_one on four values: the conversions as there, then two saturating packs (PTX cvt.pack.sat.s8.s32.b32 puts
// sat(b) in bits 0-7, sat(a) in bits 8-15 and c's low half above them), the clamp to [-128, 127] of quant_one.
__device__ __forceinline__ char4 quant4(float4 v, float inv) {
    const float2 t0 = f2_mul(make_float2(v.x, v.y), f2_splat(inv)), t1 = f2_mul(make_float2(v.z, v.w), f2_splat(inv));
    const int x = __float2int_rn(t0.x), y = __float2int_rn(t0.y), z = __float2int_rn(t1.x), w = __float2int_rn(t1.y);
    uint32_t zw, xyzw;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(zw) : "r"(w), "r"(z));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(xyzw) : "r"(y), "r"(x), "r"(zw));
    char4 c;
    *reinterpret_cast<uint32_t*>(&c) = xyzw;
    return c;
}

// LayerNorm of one row of D = 128 V held by a warp in registers (lane l: float4s l, l + 32, ...), in place; returns
// the row's largest magnitude after the norm.
template <int V>
__device__ __forceinline__ float ln_regs(float4 (&v)[V], const float* __restrict__ gamma,
                                         const float* __restrict__ beta, int lane) {
    constexpr int D = 128 * V;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) s = __fadd_rn(s, __fadd_rn(__fadd_rn(v[i].x, v[i].y), __fadd_rn(v[i].z, v[i].w)));
    const float mean = __fdiv_rn(warp_sum(s), static_cast<float>(D));
    float var = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const float a = __fsub_rn(v[i].x, mean), b = __fsub_rn(v[i].y, mean);
        const float c = __fsub_rn(v[i].z, mean), d = __fsub_rn(v[i].w, mean);
        var = __fmaf_rn(a, a, var); var = __fmaf_rn(b, b, var);
        var = __fmaf_rn(c, c, var); var = __fmaf_rn(d, d, var);
    }
    var = __fdiv_rn(warp_sum(var), static_cast<float>(D));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    const float4* b4 = reinterpret_cast<const float4*>(beta);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        v[i] = ln_apply(v[i], mean, inv, g4[lane + 32 * i], b4[lane + 32 * i]);
        amax = fmaxf(amax, amax4(v[i]));
    }
    return warp_max(amax);
}

// The normed row out: fp32 to out, or (QUANT) quantised to q / qscale.
template <int V, bool QUANT>
__device__ __forceinline__ void ln_store(const float4 (&v)[V], float amax, float* out, int ldo, int8_t* q,
                                         float* qscale, int row, int lane, int fm) {
    constexpr int D = 128 * V;
    if (!QUANT) {
        float4* orow = reinterpret_cast<float4*>(out + static_cast<size_t>(row) * ldo);
#pragma unroll
        for (int i = 0; i < V; ++i) orow[lane + 32 * i] = v[i];
        return;
    }
    const QuantRule qr = quant_rule(amax, fm);
    char4* qrow = reinterpret_cast<char4*>(q + static_cast<size_t>(row) * D);
#pragma unroll
    for (int i = 0; i < V; ++i) qrow[lane + 32 * i] = quant4(v[i], qr.inv);
    if (lane == 0) qscale[row] = qr.scale;
}

// The row completed by the K blocks of the GEMM that wrote it: v = fma(f_b, a_scale * alpha, v) block after block,
// the epilogue's fold (fv_combine_kernel with beta != 0) on the row in registers.
template <int V>
__device__ __forceinline__ void fold_regs(float4 (&v)[V], const KFold& fold, int row, int lane) {
    const float as = __fmul_rn(fold.a_scales[row], fold.alpha);
    for (int b = 0; b < fold.nblk; ++b) {
        const float4* fr = reinterpret_cast<const float4*>(fold.f + (static_cast<size_t>(b) * fold.m_pad + row) * 128 * V);
#pragma unroll
        for (int i = 0; i < V; ++i) {
            const float4 f = fr[lane + 32 * i];
            v[i] = make_float4(__fmaf_rn(f.x, as, v[i].x), __fmaf_rn(f.y, as, v[i].y), __fmaf_rn(f.z, as, v[i].z),
                               __fmaf_rn(f.w, as, v[i].w));
        }
    }
}

// D = 128 V; 8 rows per 256-thread block. FOLD: the row is first completed by a GEMM's K blocks and stored back.
template <int V, bool QUANT, bool FOLD>
__global__ void __launch_bounds__(256) ln_warp_kernel(float* x, int ldx, const float* __restrict__ gamma,
                                                      const float* __restrict__ beta, float* out, int ldo,
                                                      int8_t* __restrict__ q, float* __restrict__ qscale, int rows,
                                                      int fm, KFold fold) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= rows) return;
    float4* xr = reinterpret_cast<float4*>(x + static_cast<size_t>(row) * ldx);
    float4 v[V];
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = xr[lane + 32 * i];
    if (FOLD) {
        fold_regs<V>(v, fold, row, lane);
#pragma unroll
        for (int i = 0; i < V; ++i) xr[lane + 32 * i] = v[i];
    }
    const float amax = ln_regs<V>(v, gamma, beta, lane);
    ln_store<V, QUANT>(v, amax, out, ldo, q, qscale, row, lane, fm);
}

// The reference's per-row quantisation of rows of D = 128 V (D % 16 == 0, so no scalar tail), one warp per row held
// in registers: quant_rows_kernel's arithmetic for these rows, without its block-wide reduction and barrier.
template <int V>
__global__ void __launch_bounds__(256) quant_warp_kernel(const float* __restrict__ x, int8_t* __restrict__ q,
                                                         float* __restrict__ qscale, int rows, int fm) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * 128 * V);
    float4 v[V];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        v[i] = xr[lane + 32 * i];
        amax = fmaxf(amax, amax4(v[i]));
    }
    ln_store<V, true>(v, warp_max(amax), nullptr, 0, q, qscale, row, lane, fm);
}

// Two LayerNorms in a row (a block's closing norm, then the next block's first): x <- LN1(x) in place, then LN2 of
// the new row to out2 or quantised - the values LN2 would read back, straight from registers.
template <int V, bool QUANT, bool FOLD>
__global__ void __launch_bounds__(256) ln2_warp_kernel(float* x, int ldx, const float* __restrict__ g1,
                                                       const float* __restrict__ b1, const float* __restrict__ g2,
                                                       const float* __restrict__ b2, float* out2, int ldo,
                                                       int8_t* __restrict__ q, float* __restrict__ qscale, int rows,
                                                       int fm, KFold fold) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= rows) return;
    float4* xr = reinterpret_cast<float4*>(x + static_cast<size_t>(row) * ldx);
    float4 v[V];
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = xr[lane + 32 * i];
    if (FOLD) fold_regs<V>(v, fold, row, lane);
    ln_regs<V>(v, g1, b1, lane);
#pragma unroll
    for (int i = 0; i < V; ++i) xr[lane + 32 * i] = v[i];
    const float amax = ln_regs<V>(v, g2, b2, lane);
    ln_store<V, QUANT>(v, amax, out2, ldo, q, qscale, row, lane, fm);
}

// Any D and alignment: one 256-thread block per row, the row re-read from L1/L2 in each pass.
template <bool QUANT>
__global__ void __launch_bounds__(256) ln_rows_kernel(const float* __restrict__ x, int ldx,
                                                      const float* __restrict__ gamma, const float* __restrict__ beta,
                                                      float* out, int ldo, int8_t* __restrict__ q,
                                                      float* __restrict__ qscale, int D, int fm) {
    __shared__ float red[8];
    const int row = blockIdx.x;
    const float* xr = x + static_cast<size_t>(row) * ldx;
    auto block_sum = [&](float v) {
        v = warp_sum(v);
        __syncthreads();
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
        __syncthreads();
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) t = __fadd_rn(t, red[i]);
        return t;
    };
    float s = 0.f;
    for (int i = threadIdx.x; i < D; i += 256) s = __fadd_rn(s, xr[i]);
    const float mean = __fdiv_rn(block_sum(s), static_cast<float>(D));
    float var = 0.f;
    for (int i = threadIdx.x; i < D; i += 256) {
        const float d = __fsub_rn(xr[i], mean);
        var = __fmaf_rn(d, d, var);
    }
    var = __fdiv_rn(block_sum(var), static_cast<float>(D));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
    auto y = [&](int i) { return __fmaf_rn(__fmul_rn(__fsub_rn(xr[i], mean), inv), gamma[i], beta[i]); };
    if (!QUANT) {
        float* orow = out + static_cast<size_t>(row) * ldo;
        for (int i = threadIdx.x; i < D; i += 256) orow[i] = y(i);
        return;
    }
    float amax = 0.f;
    for (int i = threadIdx.x; i < D; i += 256) amax = fmaxf(amax, fabsf(y(i)));
    amax = warp_max(amax);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    float m = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) m = fmaxf(m, red[i]);
    const QuantRule qr = quant_rule(m, fm);
    const float scale = qr.scale;
    int8_t* qrow = q + static_cast<size_t>(row) * D;
    for (int i = threadIdx.x; i < D; i += 256) qrow[i] = quant_at(y(i), qr, i, D, fm);
    if (threadIdx.x == 0) qscale[row] = scale;
}

// ---- SiLU (csrc/tensor_ops.c:436-511) ------------------------------------------------------------------------------

__device__ __forceinline__ float block_max256(float v, float* red) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) m = fmaxf(m, red[i]);
    return m;
}

template <bool QUANT>
__global__ void __launch_bounds__(256) swish_rows_kernel(const float* __restrict__ h, int ldh, float* out, int ldo,
                                                         int8_t* __restrict__ q, float* __restrict__ qscale, int len,
                                                         int fm) {
    __shared__ float red[8];
    const int r = blockIdx.x;
    const float* hr = h + static_cast<size_t>(r) * ldh;
    if (!QUANT) {
        float* orow = out + static_cast<size_t>(r) * ldo;
        for (int i = threadIdx.x; i < len; i += 256) orow[i] = swish1(hr[i]);
        return;
    }
    float amax = 0.f;
    for (int i = threadIdx.x; i < len; i += 256) amax = fmaxf(amax, fabsf(swish1(hr[i])));
    amax = block_max256(amax, red);
    const QuantRule qr = quant_rule(amax, fm);
    const float scale = qr.scale;
    int8_t* qrow = q + static_cast<size_t>(r) * len;
    for (int i = threadIdx.x; i < len; i += 256) qrow[i] = quant_at(swish1(hr[i]), qr, i, len, fm);
    if (threadIdx.x == 0) qscale[r] = scale;
}

// len = 1024 V, one 256-thread block per row, the row in registers.
template <int V, bool QUANT>
__global__ void __launch_bounds__(256) swish_vec_kernel(const float* __restrict__ h, int ldh, float* out, int ldo,
                                                        int8_t* __restrict__ q, float* __restrict__ qscale, int fm) {
    __shared__ float red[8];
    constexpr int len = 1024 * V;
    const int r = blockIdx.x;
    const float4* hr = reinterpret_cast<const float4*>(h + static_cast<size_t>(r) * ldh);
    float4 v[V];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const float4 a = hr[threadIdx.x + 256 * i];
        const float2 s0 = swish2(make_float2(a.x, a.y)), s1 = swish2(make_float2(a.z, a.w));
        v[i] = make_float4(s0.x, s0.y, s1.x, s1.y);
        amax = fmaxf(amax, amax4(v[i]));
    }
    if (!QUANT) {
        float4* orow = reinterpret_cast<float4*>(out + static_cast<size_t>(r) * ldo);
#pragma unroll
        for (int i = 0; i < V; ++i) orow[threadIdx.x + 256 * i] = v[i];
        return;
    }
    amax = block_max256(amax, red);
    const QuantRule qr = quant_rule(amax, fm);
    const float scale = qr.scale, qinv = qr.inv;
    char4* qrow = reinterpret_cast<char4*>(q + static_cast<size_t>(r) * len);
#pragma unroll
    for (int i = 0; i < V; ++i) qrow[threadIdx.x + 256 * i] = quant4(v[i], qinv);
    if (threadIdx.x == 0) qscale[r] = scale;
}

__global__ void swish_kernel(float* x, size_t n) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) x[i] = swish1(x[i]);
}

// ---- softmax (csrc/tensor_ops.c:354-403, AVX2 branch), one warp per row ------------------------------------------
//
// max; e = exp(x - max) with the polynomial on the first 8 * floor(len / 8) values and expf on the tail; sum in the
// 8-lane order plus the tail in order; x = e * (1 / sum). `x` already holds the row's inputs.
__device__ __forceinline__ void softmax_row(float* x, int len, float mx) {
    const int lane = threadIdx.x & 31;
    const int nv = len & ~7;
    for (int j = lane; j < len; j += 32) {
        const float d = __fsub_rn(x[j], mx);
        x[j] = j < nv ? exp_poly(d) : expf(d);
    }
    __syncwarp();
    float s = 0.f;
    if (lane < 8)
        for (int j = lane; j < nv; j += 8) s = __fadd_rn(s, x[j]);
    s = hsum8(s);
    s = __shfl_sync(FULL, s, 0);
    for (int j = nv; j < len; ++j) s = __fadd_rn(s, x[j]);
    const float inv = __fdiv_rn(1.0f, s);
    __syncwarp();
    for (int j = lane; j < len; j += 32) x[j] = __fmul_rn(x[j], inv);
}

__global__ void __launch_bounds__(256) softmax_rows_kernel(float* x, int rows, int len) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;   // whole warps leave together
    float* xr = x + static_cast<size_t>(row) * len;
    float mx = -FLT_MAX;
    for (int j = threadIdx.x & 31; j < len; j += 32) mx = fmaxf(mx, xr[j]);
    mx = warp_max(mx);
    softmax_row(xr, len, mx);
}

// Attention scores (csrc/encoder.c:425-447): row (window w, head h, query i) of S_ac becomes
// softmax((ac[i][j] + bd[i][T - 1 - i + j]) * scale) over j = 0..T-1.
__global__ void __launch_bounds__(256) attn_softmax_kernel(float* s_ac, const float* __restrict__ s_bd,
                                                           const int* __restrict__ srow_off,
                                                           const long long* __restrict__ s_off,
                                                           const long long* __restrict__ b_off,
                                                           const int* __restrict__ Tw, int n_win, int rows,
                                                           float scale) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;
    const int w = find_window(srow_off, n_win, row);
    const int local = row - srow_off[w];
    const int T = Tw[w], L = 2 * T - 1;
    const int i = local % T;
    // score rows are stored with their lengths rounded up to a multiple of 4 floats (16-byte aligned rows)
    float* a = s_ac + s_off[w] + static_cast<long long>(local) * ((T + 3) & ~3);
    const float* b = s_bd + b_off[w] + static_cast<long long>(local) * ((L + 3) & ~3) + (T - 1 - i);
    float mx = -FLT_MAX;
    for (int j = threadIdx.x & 31; j < T; j += 32) {
        const float v = __fmul_rn(__fadd_rn(a[j], b[j]), scale);
        a[j] = v;
        mx = fmaxf(mx, v);
    }
    mx = warp_max(mx);
    __syncwarp();
    softmax_row(a, T, mx);
}

// ---- conv module: GLU, depthwise conv, SiLU (csrc/encoder.c:543-552, csrc/tensor_ops.c:559-649) -----------------

// gated = a / (1 + expneg(b)), expneg(b) = expf(b < -87 ? 87 : -b) (csrc/phonon2.h:38-41).
__device__ __forceinline__ float glu1(float a, float b) {
    return __fdiv_rn(a, __fadd_rn(1.0f, expf(b < -87.0f ? 87.0f : -b)));
}

// One block per row, four channels per thread (D % 4 == 0): no index division, 16-byte loads and stores.
__global__ void __launch_bounds__(256) glu_rows_kernel(const float* __restrict__ pw1, float* __restrict__ gated,
                                                       int D) {
    const float4* in = reinterpret_cast<const float4*>(pw1 + static_cast<size_t>(blockIdx.x) * 2 * D);
    float4* out = reinterpret_cast<float4*>(gated + static_cast<size_t>(blockIdx.x) * D);
    const int d4n = D / 4;
    for (int d4 = threadIdx.x; d4 < d4n; d4 += blockDim.x) {
        const float4 a = in[d4], b = in[d4n + d4];
        out[d4] = make_float4(glu1(a.x, b.x), glu1(a.y, b.y), glu1(a.z, b.z), glu1(a.w, b.w));
    }
}

// Any D: one thread per value.
__global__ void glu_any_kernel(const float* __restrict__ pw1, float* __restrict__ gated, int rows, int D) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(rows) * D) return;
    const size_t r = i / D, d = i % D;
    gated[i] = glu1(pw1[r * 2 * D + d], pw1[r * 2 * D + D + d]);
}

// DW_TR consecutive rows per CTA, 256 threads, four channels per thread: the DW_TR + 8 input rows the tile's taps
// reach are loaded once into registers (a CTA reads each input row three times from L2 instead of nine; four rows
// per CTA measured 9 % faster than eight, the smaller tiles' extra reads costing less than the CTAs they add). For
// each row (time step t of its window) and channel: bias + the 9 taps over t - 4 .. t + 4 that fall inside the
// window, as one FMA chain in tap order; then SiLU; then fp32 out or the row quantised. A tile whose taps all lie
// inside one window (every tile but those at a window's edges) skips the per-tap and per-row checks; DFIX = 1024
// (the model's width) makes the row stride a constant.
constexpr int DW_TR = 4;

template <bool SWISH, bool CHECK, int DFIX>
__device__ __forceinline__ void dw_taps(const float* __restrict__ gated, const float* __restrict__ w,
                                        const float* __restrict__ b, int g0, int rows, int D_, const int (&lo)[DW_TR],
                                        const int (&hi)[DW_TR], float (&v)[DW_TR][4]) {
    const int D = DFIX ? DFIX : D_;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int d = threadIdx.x + 256 * u;
        if (!DFIX && d >= D) {
#pragma unroll
            for (int i = 0; i < DW_TR; ++i) v[i][u] = 0.f;
            continue;
        }
        float x[DW_TR + 8];   // input rows g0 - 4 .. g0 + DW_TR + 3 of channel d
        const float* col = gated + d;
#pragma unroll
        for (int j = 0; j < DW_TR + 8; ++j) {
            const int g = g0 - 4 + j;
            x[j] = (!CHECK || (g >= 0 && g < rows)) ? __ldg(col + static_cast<ptrdiff_t>(g) * D) : 0.f;
        }
        float wk[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) wk[k] = __ldg(w + static_cast<size_t>(d) * 9 + k);
        const float bd = b ? __ldg(b + d) : 0.f;
#pragma unroll
        for (int i = 0; i < DW_TR; ++i) {
            float acc = bd;
#pragma unroll
            for (int k = 0; k < 9; ++k) {
                const int src = g0 + i - 4 + k;
                if (!CHECK || (src >= lo[i] && src < hi[i])) acc = __fmaf_rn(x[i + k], wk[k], acc);
            }
            v[i][u] = acc;
        }
    }
    if (SWISH) {   // channels d, d + 256 in the two lanes of the packed SiLU
#pragma unroll
        for (int i = 0; i < DW_TR; ++i)
#pragma unroll
            for (int u = 0; u < 4; u += 2) {
                const float2 r = swish2(make_float2(v[i][u], v[i][u + 1]));
                v[i][u] = r.x;
                v[i][u + 1] = r.y;
            }
    }
}

template <bool QUANT, bool SWISH, int DFIX>
__global__ void __launch_bounds__(256, 4) dwconv_swish_kernel(const float* __restrict__ gated, const float* __restrict__ w,
                                                           const float* __restrict__ b,
                                                           const int* __restrict__ row_off, int n_win,
                                                           float* __restrict__ out, int8_t* __restrict__ q,
                                                           float* __restrict__ qscale, int rows, int D_, int fm) {
    __shared__ float red[8][DW_TR];
    constexpr int PER = 4;   // channels per thread (D <= 1024)
    const int D = DFIX ? DFIX : D_;
    const int g0 = blockIdx.x * DW_TR;   // the tile's first row
    // the window bounds [lo, hi) of each of the tile's rows (without a window table the rows are one window)
    int lo[DW_TR], hi[DW_TR];
    {
        int win = row_off ? find_window(row_off, n_win, g0) : 0;
#pragma unroll
        for (int i = 0; i < DW_TR; ++i) {
            if (row_off) {
                while (win + 1 < n_win && g0 + i >= row_off[win + 1]) ++win;
                lo[i] = row_off[win];
                hi[i] = row_off[win + 1];
            } else {
                lo[i] = 0;
                hi[i] = rows;
            }
        }
    }
    // every tap of every row inside the first row's window (and so inside [0, rows))
    const bool inner = lo[DW_TR - 1] == lo[0] && g0 - 4 >= lo[0] && g0 + DW_TR + 3 < hi[0] && g0 - 4 >= 0 &&
                       g0 + DW_TR + 3 < rows;
    float v[DW_TR][PER];
    if (inner)
        dw_taps<SWISH, false, DFIX>(gated, w, b, g0, rows, D, lo, hi, v);
    else
        dw_taps<SWISH, true, DFIX>(gated, w, b, g0, rows, D, lo, hi, v);
    if constexpr (!QUANT) {
#pragma unroll
        for (int i = 0; i < DW_TR; ++i) {
            if (g0 + i >= rows) break;
#pragma unroll
            for (int u = 0; u < PER; ++u) {
                const int d = threadIdx.x + 256 * u;
                if (d < D) out[static_cast<size_t>(g0 + i) * D + d] = v[i][u];
            }
        }
        return;
    }
    if constexpr (QUANT) {
    // per row: the largest |value| over the 1024 channels (warp maxima in shared memory, then all eight)
#pragma unroll
    for (int i = 0; i < DW_TR; ++i) {
        float a = 0.f;
#pragma unroll
        for (int u = 0; u < PER; ++u) a = fmaxf(a, fabsf(v[i][u]));
        a = warp_max(a);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5][i] = a;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < DW_TR; ++i) {
        const int r = g0 + i;
        if (r >= rows) break;
        float amax = red[0][i];
#pragma unroll
        for (int k = 1; k < 8; ++k) amax = fmaxf(amax, red[k][i]);
        const QuantRule qr = quant_rule(amax, fm);
#pragma unroll
        for (int u = 0; u < PER; ++u) {
            const int d = threadIdx.x + 256 * u;
            if (d < D) q[static_cast<size_t>(r) * D + d] = quant_at(v[i][u], qr, d, D, fm);
        }
        if (threadIdx.x == 0) qscale[r] = qr.scale;
    }
    }
}

// ---- convolutional subsampling (csrc/encoder.c:98-225) ------------------------------------------------------------

__device__ __forceinline__ int conv_out(int n) { return (n + 2 - 3) / 2 + 1; }

// Conv2d(1 -> C, 3x3, stride 2, pad 1) + ReLU, then the depthwise Conv2d(C, 3x3, stride 2, pad 1) + bias that
// follows it, per window: mel [frames][W_IN] -> [rows2][W2][C], C fastest. The first convolution's outputs are
// computed where the second needs them instead of stored (each about twice; stored they are 6.3 GB at config 3):
// one block per output row, the 7 mel rows the row reaches in shared memory, a thread per four channels and eight
// output columns (each mel value read from shared memory feeds the four channels' FMAs). Every
// first-convolution output is bias, then its in-range taps in (kh, kw) order as one FMA chain, then ReLU; every
// output is bias, then the in-range first-convolution outputs in (kh, kw) order as one FMA chain - the two layers'
// own chains (csrc/encoder.c:103-153, 185-194), so the result is that of the two layers run one after the other.
template <int W_IN>
__global__ void __launch_bounds__(256) sub_conv0_dw_kernel(const float* __restrict__ mel,
                                                           const int* __restrict__ mel_off,
                                                           const int* __restrict__ h1_off,
                                                           const int* __restrict__ h2_off, int n_win,
                                                           const float* __restrict__ w0, const float* __restrict__ b0,
                                                           const float* __restrict__ w2, const float* __restrict__ b2,
                                                           float* __restrict__ out, int C) {
    constexpr int W1 = (W_IN - 1) / 2 + 1, W2 = (W1 - 1) / 2 + 1;
    constexpr int CPT = 4, OPT = 8;              // channels and output columns per thread
    constexpr int NJ = 2 * OPT + 1;              // first-convolution columns the thread's outputs reach
    static_assert(W2 % OPT == 0 && (W2 / OPT) * 64 == 256, "four column groups of 64 threads");
    __shared__ float xs[7][W_IN];   // mel rows 4 oh2 - 3 .. 4 oh2 + 3 of the window (zeros outside it)
    const int r2 = blockIdx.x;
    const int win = find_window(h2_off, n_win, r2);
    const int oh2 = r2 - h2_off[win];
    const int H1 = h1_off[win + 1] - h1_off[win];
    const int H = mel_off[win + 1] - mel_off[win];
    const float* x = mel + static_cast<size_t>(mel_off[win]) * W_IN;
    for (int e = threadIdx.x; e < 7 * W_IN; e += blockDim.x) {
        const int jr = e / W_IN, col = e % W_IN, ih = 4 * oh2 - 3 + jr;
        xs[jr][col] = (ih >= 0 && ih < H) ? x[static_cast<size_t>(ih) * W_IN + col] : 0.f;
    }
    __syncthreads();
    const int cg = threadIdx.x & 63, wg = threadIdx.x >> 6;   // channels 4 cg .. + 3, outputs 8 wg .. 8 wg + 7
    const int ow0 = OPT * wg, iw0 = 2 * ow0 - 1;              // the thread's first first-convolution column
    for (int c0 = CPT * cg; c0 < C; c0 += CPT * 64) {
        float w0c[CPT][9], w2c[CPT][9], b0c[CPT], acc[CPT][OPT];
#pragma unroll
        for (int u = 0; u < CPT; ++u) {
#pragma unroll
            for (int k = 0; k < 9; ++k) {
                w0c[u][k] = w0[(c0 + u) * 9 + k];
                w2c[u][k] = w2[(c0 + u) * 9 + k];
            }
            b0c[u] = b0[c0 + u];
#pragma unroll
            for (int o = 0; o < OPT; ++o) acc[u][o] = b2[c0 + u];
        }
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {   // the second convolution's row taps: first-convolution row ih1
            const int ih1 = 2 * oh2 - 1 + kh;
            if (ih1 < 0 || ih1 >= H1) continue;
            float cv[CPT][NJ];   // first-convolution columns iw0 .. iw0 + 16 of row ih1, four channels
#pragma unroll
            for (int u = 0; u < CPT; ++u)
#pragma unroll
                for (int jc = 0; jc < NJ; ++jc) cv[u][jc] = b0c[u];
#pragma unroll
            for (int kh0 = 0; kh0 < 3; ++kh0) {   // each column's taps in (kh0, kw0) order, one mel value per 4 FMAs
                const int ih = 2 * ih1 - 1 + kh0;   // mel row 4 oh2 - 3 + 2 kh + kh0
                if (ih < 0 || ih >= H) continue;
                const float* xr = xs[2 * kh + kh0];
#pragma unroll
                for (int jc = 0; jc < NJ; ++jc) {
#pragma unroll
                    for (int kw0 = 0; kw0 < 3; ++kw0) {
                        const int iw = 2 * (iw0 + jc) - 1 + kw0;
                        if (iw >= 0 && iw < W_IN) {
                            const float xv = xr[iw];
#pragma unroll
                            for (int u = 0; u < CPT; ++u) cv[u][jc] = __fmaf_rn(xv, w0c[u][kh0 * 3 + kw0], cv[u][jc]);
                        }
                    }
                }
            }
#pragma unroll
            for (int o = 0; o < OPT; ++o)
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) {
                    const int jc = 2 * o + kw, iw1 = iw0 + jc;
                    if (iw1 >= 0 && iw1 < W1) {
#pragma unroll
                        for (int u = 0; u < CPT; ++u) {
                            const float a = cv[u][jc] > 0.f ? cv[u][jc] : 0.f;   // ReLU of the first convolution
                            acc[u][o] = __fmaf_rn(a, w2c[u][kh * 3 + kw], acc[u][o]);
                        }
                    }
                }
        }
#pragma unroll
        for (int o = 0; o < OPT; ++o)
            *reinterpret_cast<float4*>(out + (static_cast<size_t>(r2) * W2 + ow0 + o) * C + c0) =
                make_float4(acc[0][o], acc[1][o], acc[2][o], acc[3][o]);
    }
}

constexpr int SUB_OW = 16;   // output columns per block of the depthwise subsampling convolution

// Depthwise Conv2d(C, 3x3, stride 2, pad 1) + bias (no activation), per window: [rows_in][W_in][C] ->
// [rows_out][W_out][C]. One block per output row and 16 output columns, one thread per channel (loads coalesced
// across channels).
__global__ void __launch_bounds__(256) sub_dwconv_kernel(const float* __restrict__ in, const int* __restrict__ in_off,
                                                         const int* __restrict__ out_off, int n_win,
                                                         const float* __restrict__ w, const float* __restrict__ b,
                                                         float* __restrict__ out, int W_in, int C) {
    const int W_out = conv_out(W_in);
    const int ro = blockIdx.x, ow0 = blockIdx.y * SUB_OW;
    const int win = find_window(out_off, n_win, ro);
    const int oh = ro - out_off[win];
    const int H = in_off[win + 1] - in_off[win];
    const float* x = in + static_cast<size_t>(in_off[win]) * W_in * C;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float wc[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) wc[k] = w[c * 9 + k];
        const float bc = b[c];
        for (int ow = ow0; ow < ow0 + SUB_OW && ow < W_out; ++ow) {
            float acc = bc;
#pragma unroll
            for (int kh = 0; kh < 3; ++kh) {
                const int ih = 2 * oh - 1 + kh;
                if (ih < 0 || ih >= H) continue;
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) {
                    const int iw = 2 * ow - 1 + kw;
                    if (iw >= 0 && iw < W_in)
                        acc = __fmaf_rn(x[(static_cast<size_t>(ih) * W_in + iw) * C + c], wc[kh * 3 + kw], acc);
                }
            }
            out[(static_cast<size_t>(ro) * W_out + ow) * C + c] = acc;
        }
    }
}

// One block per frame, W = 16 and C = 256: the frame's [16][256] values through shared memory, read along the channels
// and written 16 consecutive values (one channel's W positions) per thread.
__global__ void __launch_bounds__(256) sub_flatten16_kernel(const float* __restrict__ in, float* __restrict__ out) {
    __shared__ float tile[16][256];
    const float* src = in + static_cast<size_t>(blockIdx.x) * 16 * 256;
#pragma unroll
    for (int wv = 0; wv < 16; ++wv) tile[wv][threadIdx.x] = src[wv * 256 + threadIdx.x];
    __syncthreads();
    float4* dst = reinterpret_cast<float4*>(out + (static_cast<size_t>(blockIdx.x) * 256 + threadIdx.x) * 16);
#pragma unroll
    for (int q = 0; q < 4; ++q)
        dst[q] = make_float4(tile[4 * q][threadIdx.x], tile[4 * q + 1][threadIdx.x], tile[4 * q + 2][threadIdx.x],
                             tile[4 * q + 3][threadIdx.x]);
}

__global__ void sub_flatten_kernel(const float* __restrict__ in, float* __restrict__ out, int rows, int W, int C) {
    const size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t per = static_cast<size_t>(W) * C;
    if (idx >= static_cast<size_t>(rows) * per) return;
    const size_t r = idx / per;
    const int j = static_cast<int>(idx % per), c = j / W, wv = j % W;
    out[idx] = in[(r * W + wv) * C + c];
}

__global__ void gather_rows_kernel(float* __restrict__ dst, const float* __restrict__ src,
                                   const int* __restrict__ map, int rows, int cols) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(rows) * cols) return;
    const size_t r = i / cols, c = i % cols;
    dst[i] = src[static_cast<size_t>(map[r]) * cols + c];
}

// V of every (window, head) transposed: vt[block + d * ldT + j] = qkv[(r0 + j) * 3072 + 2048 + h * 128 + d], ldT = T
// rounded up to a multiple of 4; block = vt_off[w] + h * 128 * ldT. One block per 32 rows x 32 columns of one head.
__global__ void __launch_bounds__(256) v_transpose_kernel(const float* __restrict__ qkv, float* __restrict__ vt,
                                                          const int* __restrict__ row_off,
                                                          const long long* __restrict__ vt_off, int n_win, int rows) {
    __shared__ float tile[32][33];
    const int r0 = blockIdx.x * 32, h = blockIdx.y >> 2, d0 = (blockIdx.y & 3) * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 x 8
    for (int j = ty; j < 32; j += 8) {
        const int r = r0 + j;
        tile[j][tx] = r < rows ? qkv[static_cast<size_t>(r) * 3072 + 2048 + h * 128 + d0 + tx] : 0.f;
    }
    __syncthreads();
    const int r = r0 + tx;
    if (r >= rows) return;
    const int w = find_window(row_off, n_win, r);
    const int T = row_off[w + 1] - row_off[w], ldT = (T + 3) & ~3, j = r - row_off[w];
    float* blk = vt + vt_off[w] + static_cast<long long>(h) * 128 * ldT;
    for (int d = ty; d < 32; d += 8) blk[static_cast<size_t>(d0 + d) * ldT + j] = tile[tx][d];
}

__global__ void bias_rows_kernel(float* x, const float* __restrict__ b, size_t total, int N) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < total) x[i] = __fadd_rn(x[i], b[i % N]);
}

// One block per row, four values per thread (N % 4 == 0, 16-byte aligned rows).
__global__ void __launch_bounds__(256) bias_rows4_kernel(float* x, const float* __restrict__ b, int N) {
    float4* row = reinterpret_cast<float4*>(x + static_cast<size_t>(blockIdx.x) * N);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    for (int i = threadIdx.x; i < N / 4; i += blockDim.x) {
        const float4 v = row[i], c = b4[i];
        row[i] = make_float4(__fadd_rn(v.x, c.x), __fadd_rn(v.y, c.y), __fadd_rn(v.z, c.z), __fadd_rn(v.w, c.w));
    }
}

// ---- grouped SIMT fp32 GEMM (the attention products, csrc/encoder.c:282-316, 505-519) ---------------------------
//
// One CTA per 64 x 128 output tile of one group; every thread owns 4 x 8 outputs and runs one FMA chain per output
// over k in order from 0, as the reference's sgemm does (csrc/blas.c:155-181).
constexpr int GM = 64, GN = 128, GK = 16;

__global__ void __launch_bounds__(256) group_gemm_kernel(const GemmGroup* __restrict__ groups, int n_groups,
                                                         const float* __restrict__ A, const float* __restrict__ B,
                                                         float* __restrict__ C, const float* __restrict__ a_bias,
                                                         int transB) {
    __shared__ __align__(16) float As[GK][GM + 4];
    __shared__ __align__(16) float Bs[GK][GN];
    const int tile = blockIdx.x;
    int lo = 0, hi = n_groups - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (groups[mid].tile0 <= tile) lo = mid; else hi = mid - 1;
    }
    const GemmGroup g = groups[lo];
    const int tn = (g.N + GN - 1) / GN;
    const int tl = tile - g.tile0;
    const int m0 = (tl / tn) * GM, n0 = (tl % tn) * GN;
    const float* Ag = A + g.a_off;
    const float* Bg = B + g.b_off;
    float* Cg = C + g.c_off;
    const float* ab = (a_bias && g.bias_off >= 0) ? a_bias + g.bias_off : nullptr;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;

    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

    for (int k0 = 0; k0 < g.K; k0 += GK) {
        __syncthreads();
        {   // A: 64 rows x 16 k; thread t loads row t / 4, k quad t % 4
            const int r = tid >> 2, kq = (tid & 3) * 4, m = m0 + r;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int k = k0 + kq + i;
                float a = 0.f;
                if (m < g.M && k < g.K) {
                    a = Ag[static_cast<size_t>(m) * g.lda + k];
                    if (ab) a = __fadd_rn(a, ab[k]);
                }
                As[kq + i][r] = a;
            }
        }
        if (!transB) {   // B [k][n]: thread t loads k row t / 16, columns 8 (t % 16) .. + 7
            const int kr = tid >> 4, c8 = (tid & 15) * 8, k = k0 + kr;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int n = n0 + c8 + j;
                Bs[kr][c8 + j] = (k < g.K && n < g.N) ? Bg[static_cast<size_t>(k) * g.ldb + n] : 0.f;
            }
        } else {         // B [n][k]: thread t loads column t / 2, k 8 (t % 2) .. + 7
            const int nc = tid >> 1, kh = (tid & 1) * 8, n = n0 + nc;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int k = k0 + kh + j;
                Bs[kh + j][nc] = (k < g.K && n < g.N) ? Bg[static_cast<size_t>(n) * g.ldb + k] : 0.f;
            }
        }
        __syncthreads();
        const int kend = g.K - k0 < GK ? g.K - k0 : GK;   // never add a term beyond K
        if (kend == GK) {
#pragma unroll
            for (int kk = 0; kk < GK; ++kk) {
                const float4 a = *reinterpret_cast<const float4*>(&As[kk][4 * ty]);
                const float4 b0 = *reinterpret_cast<const float4*>(&Bs[kk][4 * tx]);
                const float4 b1 = *reinterpret_cast<const float4*>(&Bs[kk][64 + 4 * tx]);
                const float av[4] = {a.x, a.y, a.z, a.w};
                const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
            }
        } else {
            for (int kk = 0; kk < kend; ++kk) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        acc[i][j] = __fmaf_rn(As[kk][4 * ty + i], Bs[kk][j < 4 ? 4 * tx + j : 64 + 4 * tx + j - 4],
                                              acc[i][j]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + 4 * ty + i;
        if (m >= g.M) continue;
        float* crow = Cg + static_cast<size_t>(m) * g.ldc;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int na = n0 + 4 * tx + j, nb = n0 + 64 + 4 * tx + j;
            if (na < g.N) crow[na] = acc[i][j];
            if (nb < g.N) crow[nb] = acc[i][4 + j];
        }
    }
}

// ---- fused relative-position attention for windows of up to ATT_MAXT frames (csrc/encoder.c:470-528) -----------
//
// One CTA per (32 queries of one window, head). Phase 1 computes the score rows
//     s[i][j] = ((Q_i + bias_u) . K_j + (Q_i + bias_v) . P_{T-1-i+j}) * scale
// each dot product one FMA chain over d = 0..127 in order, added after both chains as the reference adds ac and
// the shifted bd; only the band of positions a query tile needs is loaded (the reference computes all 2T - 1).
// Phase 2 is the softmax of each row in shared memory, phase 3 the context rows sum_j s[i][j] V_j, one FMA chain
// over j in order per output, written straight into the concatenated-heads layout [row][h * 128 + d].
constexpr int AQ = 32, AK = 64, AD = 32, AP = 96;

__global__ void __launch_bounds__(128) attn_fused_kernel(const float* __restrict__ qkv, const float* __restrict__ P,
                                                         const float* __restrict__ bias_u,
                                                         const float* __restrict__ bias_v,
                                                         const int* __restrict__ row_off,
                                                         const int2* __restrict__ tiles, int Tmax, int SS,
                                                         float scale, float* __restrict__ attn) {
    extern __shared__ __align__(16) float smem[];
    float* S = smem;                   // [AQ][SS] score rows
    float* buf = smem + AQ * SS;       // phase 1: Qu [AD][AQ], Qv [AD][AQ], K [AD][AK], P [AD][AP]; phase 3: V [32][128]
    float* Qu_s = buf;
    float* Qv_s = Qu_s + AD * AQ;
    float* K_s = Qv_s + AD * AQ;
    float* P_s = K_s + AD * AK;
    const int2 tile = tiles[blockIdx.x];
    const int w = tile.x, q0 = tile.y, h = blockIdx.y;
    const int r0 = row_off[w], T = row_off[w + 1] - r0;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const float* Qb = qkv + static_cast<size_t>(r0) * 3 * 1024 + h * 128;
    const float* Kb = Qb + 1024;
    const float* Vb = Qb + 2048;
    const float* bu = bias_u + h * 128;
    const float* bv = bias_v + h * 128;
    const float* Pw = P + static_cast<size_t>(Tmax - T) * 1024 + h * 128;   // row p = this window's position p

    for (int j0 = 0; j0 < T; j0 += AK) {
        float ac[4][4], bd[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) ac[a][b] = bd[a][b] = 0.f;
        const int pbase = T - 1 - q0 - (AQ - 1) + j0;   // the position at band index 0
        for (int dc = 0; dc < 128; dc += AD) {
            __syncthreads();
            for (int e = tid; e < AQ * AD; e += 128) {
                const int qi = e / AD, dd = e % AD, i = q0 + qi;
                float u = 0.f, v = 0.f;
                if (i < T) {
                    const float qv = Qb[static_cast<size_t>(i) * 3072 + dc + dd];
                    u = __fadd_rn(qv, bu[dc + dd]);
                    v = __fadd_rn(qv, bv[dc + dd]);
                }
                Qu_s[dd * AQ + qi] = u;
                Qv_s[dd * AQ + qi] = v;
            }
            for (int e = tid; e < AK * AD; e += 128) {
                const int jj = e / AD, dd = e % AD, j = j0 + jj;
                K_s[dd * AK + jj] = j < T ? Kb[static_cast<size_t>(j) * 3072 + dc + dd] : 0.f;
            }
            for (int e = tid; e < AP * AD; e += 128) {
                const int pl = e / AD, dd = e % AD, p = pbase + pl;
                P_s[dd * AP + pl] = (p >= 0 && p < 2 * T - 1) ? Pw[static_cast<size_t>(p) * 1024 + dc + dd] : 0.f;
            }
            __syncthreads();
            const int pl0 = (AQ - 4) - 4 * ty + 4 * tx;   // band index of (row 4ty + 3, column 4tx)
#pragma unroll 8
            for (int dd = 0; dd < AD; ++dd) {
                const float4 qu = *reinterpret_cast<const float4*>(&Qu_s[dd * AQ + 4 * ty]);
                const float4 qv = *reinterpret_cast<const float4*>(&Qv_s[dd * AQ + 4 * ty]);
                const float4 k = *reinterpret_cast<const float4*>(&K_s[dd * AK + 4 * tx]);
                const float4 p0 = *reinterpret_cast<const float4*>(&P_s[dd * AP + pl0]);
                const float4 p1 = *reinterpret_cast<const float4*>(&P_s[dd * AP + pl0 + 4]);
                const float uq[4] = {qu.x, qu.y, qu.z, qu.w}, vq[4] = {qv.x, qv.y, qv.z, qv.w};
                const float kk[4] = {k.x, k.y, k.z, k.w};
                const float pp[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
                for (int a = 0; a < 4; ++a)
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        ac[a][b] = __fmaf_rn(uq[a], kk[b], ac[a][b]);
                        bd[a][b] = __fmaf_rn(vq[a], pp[3 - a + b], bd[a][b]);
                    }
            }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int j = j0 + 4 * tx + b;
                if (j < T) S[(4 * ty + a) * SS + j] = __fmul_rn(__fadd_rn(ac[a][b], bd[a][b]), scale);
            }
    }
    __syncthreads();

    // phase 2: softmax of each valid row (max; the polynomial exp on the first 8 * floor(T / 8), expf on the tail,
    // as the reference's vector loop and scalar tail; e * (1 / sum))
    const int lane = tid & 31, warp = tid >> 5;
    const int nv = T & ~7;
    for (int r = warp; r < AQ; r += 4) {
        if (q0 + r >= T) break;
        float* Sr = S + r * SS;
        float mx = -FLT_MAX;
        for (int j = lane; j < T; j += 32) mx = fmaxf(mx, Sr[j]);
        mx = warp_max(mx);
        float sum = 0.f;
        for (int j = lane; j < T; j += 32) {
            const float d = __fsub_rn(Sr[j], mx);
            const float e = j < nv ? exp_poly(d) : expf(d);
            Sr[j] = e;
            sum = __fadd_rn(sum, e);
        }
        const float inv = __fdiv_rn(1.0f, warp_sum(sum));
        for (int j = lane; j < T; j += 32) Sr[j] = __fmul_rn(Sr[j], inv);
    }

    // phase 3: context rows; thread (ty, tx) owns rows 4ty..4ty+3 and columns 4tx..+3, 64+4tx..+3
    float o[4][8];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 8; ++b) o[a][b] = 0.f;
    float* V_s = buf;   // [32 keys][128]
    for (int k0 = 0; k0 < T; k0 += 32) {
        __syncthreads();
        for (int e = tid; e < 32 * 32; e += 128) {
            const int jj = e >> 5, c4 = e & 31, j = k0 + jj;
            const float4 v = j < T ? *reinterpret_cast<const float4*>(Vb + static_cast<size_t>(j) * 3072 + 4 * c4)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(&V_s[jj * 128 + 4 * c4]) = v;
        }
        __syncthreads();
        const int kend = T - k0 < 32 ? T - k0 : 32;
        for (int jj = 0; jj < kend; ++jj) {
            const float4 v0 = *reinterpret_cast<const float4*>(&V_s[jj * 128 + 4 * tx]);
            const float4 v1 = *reinterpret_cast<const float4*>(&V_s[jj * 128 + 64 + 4 * tx]);
            const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                const float sa = S[(4 * ty + a) * SS + k0 + jj];
#pragma unroll
                for (int b = 0; b < 8; ++b) o[a][b] = __fmaf_rn(sa, vv[b], o[a][b]);
            }
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int i = q0 + 4 * ty + a;
        if (i >= T) continue;
        float* dst = attn + static_cast<size_t>(r0 + i) * 1024 + h * 128;
        *reinterpret_cast<float4*>(dst + 4 * tx) = make_float4(o[a][0], o[a][1], o[a][2], o[a][3]);
        *reinterpret_cast<float4*>(dst + 64 + 4 * tx) = make_float4(o[a][4], o[a][5], o[a][6], o[a][7]);
    }
}

unsigned blocks_for(size_t n, int threads) { return static_cast<unsigned>((n + threads - 1) / threads); }

}  // namespace

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

cudaError_t quant_rows_dense_launch(const float* x, int8_t* q, float* qscale, int rows, int D, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    if (D != 1024 || !al16(x) || !al16(q)) return quant_rows_launch(x, rows, D, D, q, qscale, s);
    quant_warp_kernel<8><<<static_cast<unsigned>((rows + 7) / 8), 256, 0, s>>>(x, q, qscale, rows, quant_fast_math());
    return cudaGetLastError();
}

cudaError_t ln_rows_launch(const float* x, int ldx, const float* gamma, const float* beta, float* out, int ldo,
                           int8_t* q, float* qscale, int rows, int D, cudaStream_t s, const KFold* fold) {
    if (rows <= 0) return cudaSuccess;
    const int fm = quant_fast_math();
    const bool vec = (D == 1024 || D == 512 || D == 256 || D == 128) && ldx % 4 == 0 && al16(x) && al16(gamma) &&
                     al16(beta) && (q ? al16(q) : (ldo % 4 == 0 && al16(out)));
    float* xw = const_cast<float*>(x);   // written only when folding, which the caller asks for on its own rows
    if (fold && fold->nblk > 0) {
        if (D == 1024 && ldx == D && vec) {
            const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
            if (q) ln_warp_kernel<8, true, true><<<grid, 256, 0, s>>>(xw, ldx, gamma, beta, out, ldo, q, qscale, rows,
                                                                     fm, *fold);
            else ln_warp_kernel<8, false, true><<<grid, 256, 0, s>>>(xw, ldx, gamma, beta, out, ldo, q, qscale, rows,
                                                                    fm, *fold);
            return cudaGetLastError();
        }
        cudaError_t e = fv_combine_launch(fold->f, fold->m_pad, fold->nblk, fold->a_scales, fold->alpha, 0, xw, rows,
                                          D, ldx, s);
        if (e != cudaSuccess) return e;
    }
    const KFold none{};
    if (vec) {
        const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
#define P2CU_LN(V)                                                                                                   \
        if (q) ln_warp_kernel<V, true, false><<<grid, 256, 0, s>>>(xw, ldx, gamma, beta, out, ldo, q, qscale, rows,   \
                                                                   fm, none);                                        \
        else ln_warp_kernel<V, false, false><<<grid, 256, 0, s>>>(xw, ldx, gamma, beta, out, ldo, q, qscale, rows,    \
                                                                  fm, none);
        switch (D) {
        case 1024: P2CU_LN(8) break;
        case 512: P2CU_LN(4) break;
        case 256: P2CU_LN(2) break;
        default: P2CU_LN(1) break;
        }
#undef P2CU_LN
        return cudaGetLastError();
    }
    if (q) ln_rows_kernel<true><<<rows, 256, 0, s>>>(x, ldx, gamma, beta, out, ldo, q, qscale, D, fm);
    else ln_rows_kernel<false><<<rows, 256, 0, s>>>(x, ldx, gamma, beta, out, ldo, q, qscale, D, fm);
    return cudaGetLastError();
}

cudaError_t ln2_rows_launch(float* x, int ldx, const float* g1, const float* b1, const float* g2, const float* b2,
                            float* out2, int ldo, int8_t* q, float* qscale, int rows, int D, cudaStream_t s,
                            const KFold* fold) {
    if (rows <= 0) return cudaSuccess;
    const bool vec = D == 1024 && ldx % 4 == 0 && al16(x) && al16(g1) && al16(b1) && al16(g2) && al16(b2) &&
                     (q ? al16(q) : (ldo % 4 == 0 && al16(out2)));
    const bool folding = fold && fold->nblk > 0;
    if (!vec || (folding && ldx != D)) {   // two passes (the first folds)
        cudaError_t e = ln_rows_launch(x, ldx, g1, b1, x, ldx, nullptr, nullptr, rows, D, s, fold);
        return e != cudaSuccess ? e : ln_rows_launch(x, ldx, g2, b2, out2, ldo, q, qscale, rows, D, s);
    }
    const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
    const int fm = quant_fast_math();
    const KFold f = folding ? *fold : KFold{};
    if (folding) {
        if (q) ln2_warp_kernel<8, true, true><<<grid, 256, 0, s>>>(x, ldx, g1, b1, g2, b2, out2, ldo, q, qscale, rows,
                                                                  fm, f);
        else ln2_warp_kernel<8, false, true><<<grid, 256, 0, s>>>(x, ldx, g1, b1, g2, b2, out2, ldo, q, qscale, rows,
                                                                 fm, f);
    } else {
        if (q) ln2_warp_kernel<8, true, false><<<grid, 256, 0, s>>>(x, ldx, g1, b1, g2, b2, out2, ldo, q, qscale,
                                                                   rows, fm, f);
        else ln2_warp_kernel<8, false, false><<<grid, 256, 0, s>>>(x, ldx, g1, b1, g2, b2, out2, ldo, q, qscale,
                                                                  rows, fm, f);
    }
    return cudaGetLastError();
}

cudaError_t swish_rows_launch(const float* h, int ldh, float* out, int ldo, int8_t* q, float* qscale, int rows,
                              int len, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    const int fm = quant_fast_math();
    const bool vec = (len == 4096 || len == 2048 || len == 1024) && ldh % 4 == 0 && al16(h) &&
                     (q ? al16(q) : (ldo % 4 == 0 && al16(out)));
    if (vec) {
#define P2CU_SW(V)                                                                                                   \
        if (q) swish_vec_kernel<V, true><<<rows, 256, 0, s>>>(h, ldh, out, ldo, q, qscale, fm);                          \
        else swish_vec_kernel<V, false><<<rows, 256, 0, s>>>(h, ldh, out, ldo, q, qscale, fm);
        switch (len) {
        case 4096: P2CU_SW(4) break;
        case 2048: P2CU_SW(2) break;
        default: P2CU_SW(1) break;
        }
#undef P2CU_SW
        return cudaGetLastError();
    }
    if (q) swish_rows_kernel<true><<<rows, 256, 0, s>>>(h, ldh, out, ldo, q, qscale, len, fm);
    else swish_rows_kernel<false><<<rows, 256, 0, s>>>(h, ldh, out, ldo, q, qscale, len, fm);
    return cudaGetLastError();
}

cudaError_t swish_launch(float* x, size_t n, cudaStream_t s) {
    if (!n) return cudaSuccess;
    swish_kernel<<<blocks_for(n, 256), 256, 0, s>>>(x, n);
    return cudaGetLastError();
}

cudaError_t softmax_rows_launch(float* x, int rows, int len, cudaStream_t s) {
    if (rows <= 0 || len <= 0) return cudaSuccess;
    softmax_rows_kernel<<<blocks_for(static_cast<size_t>(rows) * 32, 256), 256, 0, s>>>(x, rows, len);
    return cudaGetLastError();
}

cudaError_t glu_rows_launch(const float* pw1, float* gated, int rows, int D, cudaStream_t s) {
    const size_t n = static_cast<size_t>(rows) * D;
    if (!n) return cudaSuccess;
    if (D % 4 == 0 && al16(pw1) && al16(gated))
        glu_rows_kernel<<<rows, 256, 0, s>>>(pw1, gated, D);
    else
        glu_any_kernel<<<blocks_for(n, 256), 256, 0, s>>>(pw1, gated, rows, D);
    return cudaGetLastError();
}

cudaError_t dwconv_swish_launch(const float* gated, const float* w, const float* b, const int* row_off, int n_win,
                                float* out, int8_t* q, float* qscale, int rows, int D, cudaStream_t s, bool swish) {
    if (rows <= 0) return cudaSuccess;
    if (D > 1024) return cudaErrorInvalidValue;
    auto* k = D == 1024
                  ? (q ? (swish ? dwconv_swish_kernel<true, true, 1024> : dwconv_swish_kernel<true, false, 1024>)
                       : (swish ? dwconv_swish_kernel<false, true, 1024> : dwconv_swish_kernel<false, false, 1024>))
                  : (q ? (swish ? dwconv_swish_kernel<true, true, 0> : dwconv_swish_kernel<true, false, 0>)
                       : (swish ? dwconv_swish_kernel<false, true, 0> : dwconv_swish_kernel<false, false, 0>));
    k<<<(rows + DW_TR - 1) / DW_TR, 256, 0, s>>>(gated, w, b, row_off, n_win, out, q, qscale, rows, D,
                                                 quant_fast_math());
    return cudaGetLastError();
}

cudaError_t gather_rows_launch(float* dst, const float* src, const int* map, int rows, int cols, cudaStream_t s) {
    const size_t n = static_cast<size_t>(rows) * cols;
    if (!n) return cudaSuccess;
    gather_rows_kernel<<<blocks_for(n, 256), 256, 0, s>>>(dst, src, map, rows, cols);
    return cudaGetLastError();
}

cudaError_t sub_conv0_dw_launch(const float* mel, const int* mel_off, const int* h1_off, const int* h2_off, int n_win,
                                const float* w0, const float* b0, const float* w2, const float* b2, float* out,
                                int rows2, int W_in, int C, cudaStream_t s) {
    if (rows2 <= 0) return cudaSuccess;
    if (W_in != 128 || C % 4) return cudaErrorInvalidValue;   // the model's 128 mel bins, channels in fours
    sub_conv0_dw_kernel<128><<<rows2, 256, 0, s>>>(mel, mel_off, h1_off, h2_off, n_win, w0, b0, w2, b2, out, C);
    return cudaGetLastError();
}

cudaError_t sub_dwconv_launch(const float* in, const int* in_off, const int* out_off, int n_win, const float* w,
                              const float* b, float* out, int rows_out, int W_in, int C, cudaStream_t s) {
    const int W_out = (W_in - 1) / 2 + 1;
    if (rows_out <= 0 || W_out <= 0) return cudaSuccess;
    sub_dwconv_kernel<<<dim3(rows_out, (W_out + SUB_OW - 1) / SUB_OW), 256, 0, s>>>(in, in_off, out_off, n_win, w, b,
                                                                                   out, W_in, C);
    return cudaGetLastError();
}

cudaError_t sub_flatten_launch(const float* in, float* out, int rows, int W, int C, cudaStream_t s) {
    const size_t n = static_cast<size_t>(rows) * W * C;
    if (!n) return cudaSuccess;
    if (W == 16 && C == 256 && al16(out))
        sub_flatten16_kernel<<<rows, 256, 0, s>>>(in, out);
    else
        sub_flatten_kernel<<<blocks_for(n, 256), 256, 0, s>>>(in, out, rows, W, C);
    return cudaGetLastError();
}

cudaError_t v_transpose_launch(const float* qkv, float* vt, const int* row_off, const long long* vt_off, int n_win,
                               int rows, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    v_transpose_kernel<<<dim3((rows + 31) / 32, 32), 256, 0, s>>>(qkv, vt, row_off, vt_off, n_win, rows);
    return cudaGetLastError();
}

cudaError_t bias_rows_launch(float* x, const float* b, int rows, int N, cudaStream_t s) {
    const size_t n = static_cast<size_t>(rows) * N;
    if (!n) return cudaSuccess;
    if (N % 4 == 0 && al16(x) && al16(b))
        bias_rows4_kernel<<<rows, 256, 0, s>>>(x, b, N);
    else
        bias_rows_kernel<<<blocks_for(n, 256), 256, 0, s>>>(x, b, n, N);
    return cudaGetLastError();
}

int group_gemm_tiles(int M, int N) { return ((M + GM - 1) / GM) * ((N + GN - 1) / GN); }

cudaError_t group_gemm_launch(const GemmGroup* groups, int n_groups, int total_tiles, const float* A, const float* B,
                              float* C, const float* a_bias, int transB, cudaStream_t s) {
    if (total_tiles <= 0 || n_groups <= 0) return cudaSuccess;
    group_gemm_kernel<<<total_tiles, 256, 0, s>>>(groups, n_groups, A, B, C, a_bias, transB);
    return cudaGetLastError();
}

cudaError_t attn_softmax_launch(float* s_ac, const float* s_bd, const int* srow_off, const long long* s_off,
                                const long long* b_off, const int* Tw, int n_win, int H, int rows, float scale,
                                cudaStream_t s) {
    (void)H;
    if (rows <= 0) return cudaSuccess;
    attn_softmax_kernel<<<blocks_for(static_cast<size_t>(rows) * 32, 256), 256, 0, s>>>(s_ac, s_bd, srow_off, s_off,
                                                                                       b_off, Tw, n_win, rows, scale);
    return cudaGetLastError();
}

}  // namespace p2cu

namespace p2cu {

int attn_fused_smem_bytes(int Tmax) {
    const int SS = (Tmax + 3) / 4 * 4 + 4;
    const int buf = (2 * AD * AQ + AD * AK + AD * AP) > 32 * 128 ? (2 * AD * AQ + AD * AK + AD * AP) : 32 * 128;
    return static_cast<int>((AQ * SS + buf) * sizeof(float));
}

cudaError_t attn_fused_launch(const float* qkv, const float* P, const float* bias_u, const float* bias_v,
                              const int* row_off, const int2* tiles, int n_tiles, int Tmax, float scale, float* attn,
                              cudaStream_t s) {
    if (n_tiles <= 0) return cudaSuccess;
    if (Tmax > ATT_MAXT) return cudaErrorInvalidValue;
    const int bytes = attn_fused_smem_bytes(Tmax);
    if (bytes > 48 * 1024) {   // a per-device attribute: set on every launch that needs it (cheap, host only)
        cudaError_t e = cudaFuncSetAttribute(attn_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess) return e;
    }
    const int SS = (Tmax + 3) / 4 * 4 + 4;
    attn_fused_kernel<<<dim3(n_tiles, 8), 128, bytes, s>>>(qkv, P, bias_u, bias_v, row_off, tiles, Tmax, SS, scale,
                                                           attn);
    return cudaGetLastError();
}

}  // namespace p2cu
