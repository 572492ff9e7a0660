// encoder_ops.cu - the FastConformer encoder's memory-bound ops on the device.
//
// Each kernel restates one of the reference's CPU loops (csrc/encoder.c, csrc/tensor_ops.c) in fp32 with the same
// order of operations where that order is fixed by the source: LayerNorm's 8-lane sums and horizontal-sum tree, the
// polynomial exp of the vector loops, the FMA chains of the convolutions in tap order. Where the compiled reference
// depends on the host CPU (its -ffast-math build computes 1/sqrt with an approximate reciprocal square root refined
// by one Newton step, and calls a vectorised expf for short tails) these kernels use IEEE operations instead, so
// they agree with the reference to a few ulp, not bit for bit.
//
// Layout: activations are row-major [rows][features] and a batch of windows is stacked along the rows. Ops that
// look across rows (convolutions over time, attention) find a row's window in prefix tables of row offsets.
#include <cfloat>
#include <cstdint>
#include <cuda_runtime.h>
#include "encoder_ops.h"
#include "numerics.cuh"

namespace p2cu {

namespace {

constexpr unsigned FULL = 0xffffffffu;

// ---- LayerNorm (csrc/tensor_ops.c:204-281, AVX2 branch): 8 lanes per row -----------------------------------------
//
// sum: per lane l, x[l] + x[l + 8] + ... in order, then the horizontal-sum tree, then the D % 8 tail in order;
// mean = sum / D; var = (same shape over fma(d, d, .)) / D; y = fma((x - mean) * inv_std, gamma, beta).
template <bool QUANT>
__global__ void __launch_bounds__(256) ln_rows_kernel(const float* __restrict__ x, int ldx,
                                                      const float* __restrict__ gamma, const float* __restrict__ beta,
                                                      float* out, int ldo, int8_t* __restrict__ q,
                                                      float* __restrict__ qscale, int rows, int D) {
    const int vl = threadIdx.x & 7;
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 3;
    const bool active = row < rows;
    const float* xr = x + static_cast<size_t>(active ? row : 0) * ldx;
    const int nv = D & ~7;

    float s = 0.f;
    if (active)
        for (int i = vl; i < nv; i += 8) s = __fadd_rn(s, xr[i]);
    s = hsum8(s);
    if (active)
        for (int i = nv; i < D; ++i) s = __fadd_rn(s, xr[i]);
    const float mean = __fdiv_rn(s, static_cast<float>(D));

    float v = 0.f;
    if (active)
        for (int i = vl; i < nv; i += 8) {
            const float d = __fsub_rn(xr[i], mean);
            v = __fmaf_rn(d, d, v);
        }
    v = hsum8(v);
    if (active)
        for (int i = nv; i < D; ++i) {
            const float d = __fsub_rn(xr[i], mean);
            v = __fmaf_rn(d, d, v);
        }
    const float var = __fdiv_rn(v, static_cast<float>(D));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));

    if (!QUANT) {
        if (!active) return;
        float* orow = out + static_cast<size_t>(row) * ldo;
        for (int i = vl; i < D; i += 8)
            orow[i] = __fmaf_rn(__fmul_rn(__fsub_rn(xr[i], mean), inv), gamma[i], beta[i]);
        return;
    }
    // Quantised output: the normalised row is computed twice (once for its maximum, once to quantise), never stored.
    float amax = 0.f;
    if (active)
        for (int i = vl; i < D; i += 8)
            amax = fmaxf(amax, fabsf(__fmaf_rn(__fmul_rn(__fsub_rn(xr[i], mean), inv), gamma[i], beta[i])));
    amax = max8(amax);
    if (!active) return;
    const float scale = quant_scale(amax);
    const float qinv = __fdiv_rn(1.0f, scale);
    int8_t* qrow = q + static_cast<size_t>(row) * D;
    for (int i = vl; i < D; i += 8)
        qrow[i] = quant_one(__fmaf_rn(__fmul_rn(__fsub_rn(xr[i], mean), inv), gamma[i], beta[i]), qinv);
    if (vl == 0) qscale[row] = scale;
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
                                                         int8_t* __restrict__ q, float* __restrict__ qscale, int len) {
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
    const float scale = quant_scale(amax);
    const float qinv = __fdiv_rn(1.0f, scale);
    int8_t* qrow = q + static_cast<size_t>(r) * len;
    for (int i = threadIdx.x; i < len; i += 256) qrow[i] = quant_one(swish1(hr[i]), qinv);
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
    float* a = s_ac + s_off[w] + static_cast<long long>(local) * T;
    const float* b = s_bd + b_off[w] + static_cast<long long>(local) * L + (T - 1 - i);
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
__global__ void glu_rows_kernel(const float* __restrict__ pw1, float* __restrict__ gated, int rows, int D) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(rows) * D) return;
    const size_t r = i / D, d = i % D;
    const float a = pw1[r * 2 * D + d], b = pw1[r * 2 * D + D + d];
    gated[i] = __fdiv_rn(a, __fadd_rn(1.0f, expf(b < -87.0f ? 87.0f : -b)));
}

// One CTA per row (time step t of its window): for each channel, bias + the 9 taps over t - 4 .. t + 4 that fall
// inside the window, as one FMA chain in tap order; then SiLU; then fp32 out or the row quantised.
template <bool QUANT, bool SWISH>
__global__ void __launch_bounds__(256) dwconv_swish_kernel(const float* __restrict__ gated, const float* __restrict__ w,
                                                           const float* __restrict__ b,
                                                           const int* __restrict__ row_off, int n_win,
                                                           float* __restrict__ out, int8_t* __restrict__ q,
                                                           float* __restrict__ qscale, int rows, int D) {
    __shared__ float red[8];
    constexpr int PER = 4;   // channels per thread (D <= 1024)
    const int r = blockIdx.x;
    // without a window table the rows are one window
    const int win = row_off ? find_window(row_off, n_win, r) : 0;
    const int r0 = row_off ? row_off[win] : 0, T = row_off ? row_off[win + 1] - r0 : rows, t = r - r0;
    float v[PER];
    float amax = 0.f;
#pragma unroll
    for (int u = 0; u < PER; ++u) {
        const int d = threadIdx.x + 256 * u;
        v[u] = 0.f;
        if (d < D) {
            float acc = b ? b[d] : 0.f;
            const float* wd = w + static_cast<size_t>(d) * 9;
#pragma unroll
            for (int k = 0; k < 9; ++k) {
                const int src = t - 4 + k;
                if (src >= 0 && src < T) acc = __fmaf_rn(gated[static_cast<size_t>(r0 + src) * D + d], wd[k], acc);
            }
            v[u] = SWISH ? swish1(acc) : acc;
            amax = fmaxf(amax, fabsf(v[u]));
        }
    }
    if (!QUANT) {
#pragma unroll
        for (int u = 0; u < PER; ++u) {
            const int d = threadIdx.x + 256 * u;
            if (d < D) out[static_cast<size_t>(r) * D + d] = v[u];
        }
        return;
    }
    amax = block_max256(amax, red);
    const float scale = quant_scale(amax);
    const float qinv = __fdiv_rn(1.0f, scale);
#pragma unroll
    for (int u = 0; u < PER; ++u) {
        const int d = threadIdx.x + 256 * u;
        if (d < D) q[static_cast<size_t>(r) * D + d] = quant_one(v[u], qinv);
    }
    if (threadIdx.x == 0) qscale[r] = scale;
}

// ---- convolutional subsampling (csrc/encoder.c:98-225) ------------------------------------------------------------

__device__ __forceinline__ int conv_out(int n) { return (n + 2 - 3) / 2 + 1; }

// Conv2d(1 -> C, 3x3, stride 2, pad 1) + ReLU; out [rows1][W1][C], C fastest.
__global__ void sub_conv0_kernel(const float* __restrict__ mel, const int* __restrict__ mel_off,
                                 const int* __restrict__ h1_off, int n_win, const float* __restrict__ w,
                                 const float* __restrict__ b, float* __restrict__ out, int rows1, int W_in, int C) {
    const int W1 = conv_out(W_in);
    const size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<size_t>(rows1) * W1 * C) return;
    const int c = static_cast<int>(idx % C);
    const size_t rest = idx / C;
    const int ow = static_cast<int>(rest % W1), r1 = static_cast<int>(rest / W1);
    const int win = find_window(h1_off, n_win, r1);
    const int oh = r1 - h1_off[win];
    const int H = mel_off[win + 1] - mel_off[win];
    const float* x = mel + static_cast<size_t>(mel_off[win]) * W_in;
    const float* wc = w + c * 9;
    float acc = b[c];
#pragma unroll
    for (int kh = 0; kh < 3; ++kh) {
        const int ih = 2 * oh - 1 + kh;
        if (ih < 0 || ih >= H) continue;
#pragma unroll
        for (int kw = 0; kw < 3; ++kw) {
            const int iw = 2 * ow - 1 + kw;
            if (iw >= 0 && iw < W_in) acc = __fmaf_rn(x[static_cast<size_t>(ih) * W_in + iw], wc[kh * 3 + kw], acc);
        }
    }
    out[idx] = acc > 0.f ? acc : 0.f;
}

// Depthwise Conv2d(C, 3x3, stride 2, pad 1) + bias (no activation), per window.
__global__ void sub_dwconv_kernel(const float* __restrict__ in, const int* __restrict__ in_off,
                                  const int* __restrict__ out_off, int n_win, const float* __restrict__ w,
                                  const float* __restrict__ b, float* __restrict__ out, int rows_out, int W_in,
                                  int C) {
    const int W_out = conv_out(W_in);
    const size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<size_t>(rows_out) * W_out * C) return;
    const int c = static_cast<int>(idx % C);
    const size_t rest = idx / C;
    const int ow = static_cast<int>(rest % W_out), ro = static_cast<int>(rest / W_out);
    const int win = find_window(out_off, n_win, ro);
    const int oh = ro - out_off[win];
    const int H = in_off[win + 1] - in_off[win];
    const float* x = in + static_cast<size_t>(in_off[win]) * W_in * C + c;
    const float* wc = w + c * 9;
    float acc = b[c];
#pragma unroll
    for (int kh = 0; kh < 3; ++kh) {
        const int ih = 2 * oh - 1 + kh;
        if (ih < 0 || ih >= H) continue;
#pragma unroll
        for (int kw = 0; kw < 3; ++kw) {
            const int iw = 2 * ow - 1 + kw;
            if (iw >= 0 && iw < W_in)
                acc = __fmaf_rn(x[(static_cast<size_t>(ih) * W_in + iw) * C], wc[kh * 3 + kw], acc);
        }
    }
    out[idx] = acc;
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

__global__ void bias_rows_kernel(float* x, const float* __restrict__ b, size_t total, int N) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < total) x[i] = __fadd_rn(x[i], b[i % N]);
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

unsigned blocks_for(size_t n, int threads) { return static_cast<unsigned>((n + threads - 1) / threads); }

}  // namespace

cudaError_t ln_rows_launch(const float* x, int ldx, const float* gamma, const float* beta, float* out, int ldo,
                           int8_t* q, float* qscale, int rows, int D, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    const unsigned grid = blocks_for(static_cast<size_t>(rows) * 8, 256);
    if (q) ln_rows_kernel<true><<<grid, 256, 0, s>>>(x, ldx, gamma, beta, out, ldo, q, qscale, rows, D);
    else ln_rows_kernel<false><<<grid, 256, 0, s>>>(x, ldx, gamma, beta, out, ldo, q, qscale, rows, D);
    return cudaGetLastError();
}

cudaError_t swish_rows_launch(const float* h, int ldh, float* out, int ldo, int8_t* q, float* qscale, int rows,
                              int len, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    if (q) swish_rows_kernel<true><<<rows, 256, 0, s>>>(h, ldh, out, ldo, q, qscale, len);
    else swish_rows_kernel<false><<<rows, 256, 0, s>>>(h, ldh, out, ldo, q, qscale, len);
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
    glu_rows_kernel<<<blocks_for(n, 256), 256, 0, s>>>(pw1, gated, rows, D);
    return cudaGetLastError();
}

cudaError_t dwconv_swish_launch(const float* gated, const float* w, const float* b, const int* row_off, int n_win,
                                float* out, int8_t* q, float* qscale, int rows, int D, cudaStream_t s, bool swish) {
    if (rows <= 0) return cudaSuccess;
    if (D > 1024) return cudaErrorInvalidValue;
    auto* k = q ? (swish ? dwconv_swish_kernel<true, true> : dwconv_swish_kernel<true, false>)
                : (swish ? dwconv_swish_kernel<false, true> : dwconv_swish_kernel<false, false>);
    k<<<rows, 256, 0, s>>>(gated, w, b, row_off, n_win, out, q, qscale, rows, D);
    return cudaGetLastError();
}

cudaError_t gather_rows_launch(float* dst, const float* src, const int* map, int rows, int cols, cudaStream_t s) {
    const size_t n = static_cast<size_t>(rows) * cols;
    if (!n) return cudaSuccess;
    gather_rows_kernel<<<blocks_for(n, 256), 256, 0, s>>>(dst, src, map, rows, cols);
    return cudaGetLastError();
}

cudaError_t sub_conv0_launch(const float* mel, const int* mel_off, const int* h1_off, int n_win, const float* w,
                             const float* b, float* out, int rows1, int W_in, int C, cudaStream_t s) {
    const size_t n = static_cast<size_t>(rows1) * ((W_in - 1) / 2 + 1) * C;
    if (!n) return cudaSuccess;
    sub_conv0_kernel<<<blocks_for(n, 256), 256, 0, s>>>(mel, mel_off, h1_off, n_win, w, b, out, rows1, W_in, C);
    return cudaGetLastError();
}

cudaError_t sub_dwconv_launch(const float* in, const int* in_off, const int* out_off, int n_win, const float* w,
                              const float* b, float* out, int rows_out, int W_in, int C, cudaStream_t s) {
    const size_t n = static_cast<size_t>(rows_out) * ((W_in - 1) / 2 + 1) * C;
    if (!n) return cudaSuccess;
    sub_dwconv_kernel<<<blocks_for(n, 256), 256, 0, s>>>(in, in_off, out_off, n_win, w, b, out, rows_out, W_in, C);
    return cudaGetLastError();
}

cudaError_t sub_flatten_launch(const float* in, float* out, int rows, int W, int C, cudaStream_t s) {
    const size_t n = static_cast<size_t>(rows) * W * C;
    if (!n) return cudaSuccess;
    sub_flatten_kernel<<<blocks_for(n, 256), 256, 0, s>>>(in, out, rows, W, C);
    return cudaGetLastError();
}

cudaError_t bias_rows_launch(float* x, const float* b, int rows, int N, cudaStream_t s) {
    const size_t n = static_cast<size_t>(rows) * N;
    if (!n) return cudaSuccess;
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
