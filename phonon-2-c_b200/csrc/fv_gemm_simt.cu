// fv_gemm_simt.cu - the five-value / int8-table GEMM on quantised rows for the shapes the tensor-core kernels do not
// take: N not a multiple of 128 or K not a multiple of 16 (the reference accepts any N % 16 == 0 and K % 4 == 0 in its
// int8 modes, csrc/blas.c:989-995, 1404-1437), or C not 16-byte aligned. Same arithmetic as the tensor-core path and
// the reference (csrc/blas.c:1257-1366): exact int32 sums restarting every 1024 rows of K, then per block, in K order,
// f = (float)accS * c1 [+ (float)accT * c2 fused], C = (first block and beta == 0) ? f * as : fma(f, as, C) with
// as = a_scale[m] * alpha. One thread per output; these shapes are rare and small, so the kernel is plain SIMT: a
// warp shares one row of A (broadcast loads) and reads 32 neighbouring columns of the weight.
#include <cstdint>
#include <cuda_runtime.h>
#include "fv_gemm.h"
#include "fv_common.cuh"

namespace p2cu {

constexpr int SIMT_COLS = 32, SIMT_ROWS = 8, SIMT_KBLK = 1024;

__global__ void __launch_bounds__(SIMT_COLS * SIMT_ROWS)
fv_gemm_simt_kernel(const int8_t* __restrict__ q, const uint8_t* __restrict__ signs,
                    const uint8_t* __restrict__ flags, const int8_t* __restrict__ table, int ldb, FvGemmParams p) {
    const int n = blockIdx.x * SIMT_COLS + (threadIdx.x % SIMT_COLS);
    if (n >= p.N) return;
    const int N = p.N, K = p.K;
    // per-column factors (csrc/blas.c:1316-1336)
    float c1, c2 = 0.f;
    int clo = 0;
    if (p.cmode == CM_Q8B) {
        c1 = p.scales[n];
    } else if (p.cmode == CM_INT8) {
        c1 = p.lo[n];
        c2 = __fsub_rn(p.hi[n], p.lo[n]);
    } else {   // int8w: codes sign * (flag ? 127 : clo), f = (float)acc * (hi * (1 / 127))
        c1 = __fmul_rn(p.hi[n], 1.0f / 127.0f);
        clo = clo_of(p.lo[n], p.hi[n]);
    }
    const bool two = p.cmode == CM_INT8;
    for (int m = blockIdx.y * SIMT_ROWS + static_cast<int>(threadIdx.x / SIMT_COLS); m < p.M;
         m += gridDim.y * SIMT_ROWS) {
        const int8_t* qr = q + static_cast<size_t>(m) * K;
        const float as = __fmul_rn(p.a_scales[m], p.alpha);
        float* cp = p.C + static_cast<size_t>(m) * p.ldc + n;
        float c = p.beta_zero ? 0.f : *cp;
        for (int k0 = 0; k0 < K; k0 += SIMT_KBLK) {
            const int k1 = K - k0 < SIMT_KBLK ? K : k0 + SIMT_KBLK;
            int accS = 0, accT = 0;
            for (int k = k0; k < k1; ++k) {
                const int a = qr[k];
                if (table) {
                    accS += a * static_cast<int>(table[static_cast<size_t>(k) * ldb + n]);
                } else {
                    const int s = static_cast<int>((signs[static_cast<size_t>(k) * (N / 4) + (n >> 2)] >>
                                                    (2 * (n & 3))) & 3u) - 1;
                    const int f = (flags[static_cast<size_t>(k) * (N / 8) + (n >> 3)] >> (n & 7)) & 1;
                    if (two) {
                        accS += a * s;
                        accT += f ? a * s : 0;
                    } else {
                        accS += a * s * (f ? 127 : clo);
                    }
                }
            }
            float fv = __fmul_rn(__int2float_rn(accS), c1);
            if (two) fv = __fmaf_rn(__int2float_rn(accT), c2, fv);
            c = (k0 == 0 && p.beta_zero) ? __fmul_rn(fv, as) : __fmaf_rn(fv, as, c);
        }
        *cp = c;
    }
}

cudaError_t fv_gemm_simt_launch(const int8_t* q, const uint8_t* signs, const uint8_t* flags, const int8_t* table,
                                int ldb, const FvGemmParams& p, cudaStream_t stream) {
    const unsigned gx = static_cast<unsigned>((p.N + SIMT_COLS - 1) / SIMT_COLS);
    const int rows = (p.M + SIMT_ROWS - 1) / SIMT_ROWS;
    const unsigned gy = static_cast<unsigned>(rows < 65535 ? rows : 65535);
    fv_gemm_simt_kernel<<<dim3(gx, gy), SIMT_COLS * SIMT_ROWS, 0, stream>>>(q, signs, flags, table, ldb, p);
    return cudaGetLastError();
}

}  // namespace p2cu
