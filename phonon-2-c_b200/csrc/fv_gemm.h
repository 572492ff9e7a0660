// fv_gemm.h - launch interface of the tcgen05 five-value / int8-table GEMM (fv_gemm.cu). Internal to the library.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace p2cu {

// How the epilogue turns int32 sums into fp32 (the reference's GEMM modes, csrc/blas.c:1316-1336).
enum : int { CM_INT8 = 0, CM_INT8W = 2, CM_Q8B = 8 };

struct FvGemmParams {
    int M, N, K;
    float alpha;
    int beta_zero;            // 1: the first 1024-row K block stores into C; 0: every block accumulates into C
    int cmode;                // CM_*
    const float* a_scales;    // [M] per-row scales of the quantised A
    const float* lo;          // [N] five-value magnitudes (CM_INT8, CM_INT8W)
    const float* hi;          // [N]
    const float* scales;      // [N] int8-table column scales (CM_Q8B)
    float* C;
    int ldc;
    uint32_t* err;            // device error word (timeouts), first error wins
};

// Five-value planes: A [M, K] int8 (128 x 128 boxes, 128-byte swizzle), signs [K, N/4] (32 x 128 boxes) and
// flags [K, N/8] (16 x 128 boxes). Requires N % 128 == 0 and K % 16 == 0.
cudaError_t fv_gemm_launch_planes(const CUtensorMap& a, const CUtensorMap& signs, const CUtensorMap& flags,
                                  const FvGemmParams& p, cudaStream_t stream);

// int8 table [K, N] (128 x 128 boxes, 128-byte swizzle): the int8-table weights, or cached int8w codes.
cudaError_t fv_gemm_launch_table(const CUtensorMap& a, const CUtensorMap& table, const FvGemmParams& p,
                                 cudaStream_t stream);

}  // namespace p2cu
