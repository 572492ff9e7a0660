// gemm.h - the GEMM entry points and error helpers api.cu offers the library's other translation units.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include "p2cuda.h"

namespace p2cu {

// A 2-D tiled tensor map over `base` ([outer][inner] elements of `esize` bytes, rows `stride` bytes apart), boxes
// box_in x box_out, swizzle 128 / 64 / 32 bytes or 0; P2CU_EINVAL with a message when the driver refuses it.
int make_tile_map(CUtensorMap* map, const void* base, int esize, uint64_t inner, uint64_t outer, uint64_t stride,
                  uint32_t box_in, uint32_t box_out, int swizzle, const char* what);

// Optional epilogue of the exact (fp32) GEMM: + bias[n], then ReLU, then C = fma(result, res_alpha, C).
struct Epilogue {
    const float* bias = nullptr;
    int relu = 0;
    int residual = 0;
    float res_alpha = 1.0f;
};

// Set p2cu_last_error()'s text for this thread and return `code`.
int fail_fmt(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);
void set_error_message(int code, const char* msg);
uint32_t* device_error_word();

// Bytes of K-block slices the tensor-core GEMM needs for K > 1024 (0 otherwise).
size_t gemm_split_bytes(int M, int N, int K);

// The per-block values of a GEMM with K > 1024 still to be folded into its C, C = fma(f_b, a_scale * alpha, C) block
// after block (what fv_combine_kernel does with beta != 0): the workspace slices f [nblk][m_pad][N] (N = the row
// length of C), the A rows' scales and alpha. nblk = 0: nothing to fold.
struct KFold {
    const float* f = nullptr;
    int m_pad = 0, nblk = 0;
    const float* a_scales = nullptr;
    float alpha = 1.0f;
};

// The tensor-core GEMM on quantised rows q / a_scales; B five-value (planes or cached codes) or q8 / scales an int8
// table. mode P2CU_INT8 or P2CU_INT8W for five-value weights. With `defer` (and beta 1, K > 1024) the fold of the
// K blocks into C is left to the caller's next kernel and described in *defer (nblk 0 when there is none); the
// workspace must then stay untouched until that kernel has run.
int gemm_i8(int M, int N, int K, float alpha, const int8_t* q, const float* a_scales, const P2cuFiveValue* B,
            const int8_t* q8, const float* scales, int ldb, int mode, float beta, float* C, int ldc, void* ws,
            size_t ws_bytes, cudaStream_t s, const char* who, KFold* defer = nullptr);

// The exact fp32 GEMM (one FMA chain per output) on B five-value, an int8 table or an fp32 matrix.
int gemm_exact(int M, int N, int K, float alpha, const float* A, int lda, int transA, const P2cuFiveValue* B,
               const int8_t* q8, const float* scales, const float* Bf, int ldb, int transB, float beta, float* C,
               int ldc, const Epilogue* epi, cudaStream_t s, const char* who);

}  // namespace p2cu
