// exact.cu - the exact (fp32 expansion) GEMM, bit for bit the reference's arithmetic.
//
// The reference's exact path (csrc/blas.c:60-70, 155-181, 841-910, 931-987) scales C by beta, expands B to fp32 in
// its pack step and runs register-blocked FMA micro-kernels that load C, run c = fma(alpha * a[m][k], w[k][n], c)
// over a K block in order and store C, block after block: per output, one sequential FMA chain over k = 0..K-1.
// Here every thread owns 4 x 8 outputs and runs exactly that chain, so results are identical to the reference's.
// B is one of: five-value planes (w = s * fma(f, hi - lo, lo), blas.c:895-896), an int8 table (w = q * scale[n],
// blas.c:826-829) or an fp32 matrix (p2_sgemm NN, blas.c:748-763).
#include <cstdint>
#include <cuda_runtime.h>
#include "kernels.h"

namespace p2cu {

constexpr int XM = 64, XN = 128, XK = 16, XPAD = 4;

template <int BKIND>
__global__ void __launch_bounds__(256) exact_gemm_kernel(ExactParams p) {
    __shared__ __align__(16) float As[XK][XM + XPAD];   // alpha * A, transposed: As[k][m]
    __shared__ __align__(16) float Bs[XK][XN];          // the expanded weights
    __shared__ float s_lo[XN], s_d[XN], s_sc[XN];

    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * XM, n0 = blockIdx.x * XN;

    if (tid < XN) {
        const int n = n0 + tid;
        if (BKIND == BK_FIVE && n < p.N) {
            s_lo[tid] = p.lo[n];
            s_d[tid] = __fsub_rn(p.hi[n], p.lo[n]);
        } else if (BKIND == BK_TABLE && n < p.N) {
            s_sc[tid] = p.scales[n];
        }
    }

    // Accumulators start from beta * C (scale_c: 0 when beta == 0, C when beta == 1, C * beta otherwise).
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + 4 * ty + i;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int n = n0 + (j < 4 ? 4 * tx + j : 64 + 4 * tx + (j - 4));
            float c = 0.f;
            if (p.beta != 0.f && m < p.M && n < p.N) {
                c = p.C[static_cast<size_t>(m) * p.ldc + n];
                if (p.beta != 1.f) c = __fmul_rn(c, p.beta);
            }
            acc[i][j] = c;
        }
    }

    for (int k0 = 0; k0 < p.K; k0 += XK) {
        __syncthreads();
        {   // A tile: 64 rows x 16 k, thread t loads row t / 4, k quad t % 4
            const int r = tid >> 2, kq = (tid & 3) * 4, m = m0 + r;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int k = k0 + kq + i;
                float a = 0.f;
                if (m < p.M && k < p.K)
                    a = p.transA ? p.A[static_cast<size_t>(k) * p.lda + m] : p.A[static_cast<size_t>(m) * p.lda + k];
                As[kq + i][r] = __fmul_rn(p.alpha, a);
            }
        }
        {   // B tile: 16 k x 128 columns, thread t expands row t / 16, columns 8 (t % 16) .. + 7
            const int kr = tid >> 4, c8 = (tid & 15) * 8, k = k0 + kr;
            float w[8];
            if (BKIND == BK_F32) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int n = n0 + c8 + j;
                    w[j] = (k < p.K && n < p.N) ? (p.transB ? p.Bf[static_cast<size_t>(n) * p.ldb + k]
                                                            : p.Bf[static_cast<size_t>(k) * p.ldb + n]) : 0.f;
                }
            } else if (k < p.K && n0 + c8 < p.N) {   // N % 16 == 0 for the quantised operands
                if (BKIND == BK_FIVE) {
                    const int n = n0 + c8;
                    const uint32_t sb = *reinterpret_cast<const uint16_t*>(p.signs + static_cast<size_t>(k) * (p.N / 4) + n / 4);
                    const uint32_t fb = p.flags[static_cast<size_t>(k) * (p.N / 8) + n / 8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float s = static_cast<float>(static_cast<int>((sb >> (2 * j)) & 3u) - 1);
                        const float f = static_cast<float>((fb >> j) & 1u);
                        w[j] = __fmul_rn(s, __fmaf_rn(f, s_d[c8 + j], s_lo[c8 + j]));
                    }
                } else if (BKIND == BK_TABLE) {
                    const int8_t* src = p.q8 + static_cast<size_t>(k) * p.ldb + n0 + c8;
#pragma unroll
                    for (int j = 0; j < 8; ++j) w[j] = __fmul_rn(static_cast<float>(src[j]), s_sc[c8 + j]);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) w[j] = 0.f;
            }
            *reinterpret_cast<float4*>(&Bs[kr][c8]) = make_float4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<float4*>(&Bs[kr][c8 + 4]) = make_float4(w[4], w[5], w[6], w[7]);
        }
        __syncthreads();
        const int kend = p.K - k0 < XK ? p.K - k0 : XK;   // never add a term beyond K
        if (kend == XK) {
#pragma unroll
            for (int kk = 0; kk < XK; ++kk) {
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
        if (m >= p.M) continue;
        float* crow = p.C + static_cast<size_t>(m) * p.ldc;
        const int na = n0 + 4 * tx, nb = n0 + 64 + 4 * tx;
        if (p.bias || p.relu || p.residual) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int n = j < 4 ? na + j : nb + j - 4;
                if (n >= p.N) continue;
                float v = acc[i][j];
                if (p.bias) v = __fadd_rn(v, p.bias[n]);
                if (p.relu) v = v > 0.f ? v : 0.f;
                if (p.residual) v = __fmaf_rn(v, p.res_alpha, crow[n]);
                acc[i][j] = v;
            }
        }
        if (p.vec_store) {   // N % 4 == 0, ldc % 4 == 0 and C 16-byte aligned
            if (na < p.N) *reinterpret_cast<float4*>(crow + na) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
            if (nb < p.N) *reinterpret_cast<float4*>(crow + nb) = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (na + j < p.N) crow[na + j] = acc[i][j];
                if (nb + j < p.N) crow[nb + j] = acc[i][4 + j];
            }
        }
    }
}

cudaError_t exact_gemm_launch(const ExactParams& p, cudaStream_t stream) {
    dim3 grid((p.N + XN - 1) / XN, (p.M + XM - 1) / XM);
    switch (p.bkind) {
    case BK_FIVE:  exact_gemm_kernel<BK_FIVE><<<grid, 256, 0, stream>>>(p); break;
    case BK_TABLE: exact_gemm_kernel<BK_TABLE><<<grid, 256, 0, stream>>>(p); break;
    default:       exact_gemm_kernel<BK_F32><<<grid, 256, 0, stream>>>(p); break;
    }
    return cudaGetLastError();
}

}  // namespace p2cu
