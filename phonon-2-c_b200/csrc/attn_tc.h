// attn_tc.h - grouped fp32-accurate GEMMs on the tensor cores (attn_tc.cu), for the attention products. Internal.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace p2cu {

// One problem: C[m][n] = sum_k (A[m][k] + bias[k]) * op(B)[k][n] for m < M, n < N, k < K, with A rows lda apart
// (K-major), B either [n][k] rows ldb apart or [k][n] rows ldb apart (per launch), C rows ldc
// apart. Offsets are in elements from the chosen bases; tile0 is the group's first 128 x 128 tile in the launch.
struct TcGroup {
    int M, N, K, tile0;
    long long a_off, b_off, c_off;
    int lda, ldb, ldc;
    int a_src, b_src, c_dst;
    int bias_sel;   // -1: no bias; else the index into TcArgs::bias
    int bias_off;
};

// Base pointers of one launch; a group picks its operands among them. With no group table the launch computes
// `single` alone.
struct TcArgs {
    const float* src[2];    // operand bases
    float* dst[2];          // result bases
    const float* bias[2];   // per-K vectors added to A on load
    uint32_t* err;          // device error word for bounded waits
    TcGroup single;
    const float* out_bias = nullptr;   // per-column vector added to every result (nullptr: none)
    int out_relu = 0;                  // results below zero become zero (after the bias)
};

int tc_gemm_tiles(int M, int N);

// All groups of one launch; b_kn selects the [k][n] layout of B for every group.
cudaError_t attn_tc_launch(const TcGroup* groups, int n_groups, int total_tiles, const TcArgs& args, bool b_kn,
                           cudaStream_t s);

}  // namespace p2cu
