// kernels.h - launch interfaces of the SIMT kernels (quant.cu, exact.cu). Internal to the library.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace p2cu {

// The B operand of the exact GEMM.
enum : int { BK_FIVE = 0, BK_TABLE = 1, BK_F32 = 2 };

struct ExactParams {
    int M, N, K;
    float alpha, beta;
    const float* A; int lda; int transA;
    int bkind;
    const uint8_t* signs; const uint8_t* flags; const float* lo; const float* hi;   // BK_FIVE
    const int8_t* q8; const float* scales;                                          // BK_TABLE
    const float* Bf; int transB;                                                    // BK_F32
    int ldb;
    float* C; int ldc;
    int vec_store;
    // Epilogue, in this order: + bias[n] (a separate rounded add, as the reference's bias loops), ReLU, then
    // C = fma(result, res_alpha, C) (the reference's residual axpy, csrc/encoder.c:252-275); beta must be 0 with it.
    const float* bias;
    int relu;
    int residual;
    float res_alpha;
};

cudaError_t quant_rows_launch(const float* A, int M, int K, int lda, int8_t* q, float* scales, cudaStream_t stream);
cudaError_t fv_codes_launch(const uint8_t* signs, const uint8_t* flags, const float* lo, const float* hi, int K, int N,
                            int8_t* codes, cudaStream_t stream);
cudaError_t exact_gemm_launch(const ExactParams& p, cudaStream_t stream);

}  // namespace p2cu
