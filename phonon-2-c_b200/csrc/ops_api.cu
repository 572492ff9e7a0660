// ops_api.cu - the encoder's row ops on device rows (include/p2cuda.h), each one launch of an encoder_ops kernel.
#include <cstdint>
#include <cuda_runtime.h>
#include "p2cuda.h"
#include "gemm.h"
#include "encoder_ops.h"
#include "attn_tc.h"

namespace {

int done(cudaError_t e, const char* who) { return e == cudaSuccess ? P2CU_OK : p2cu::cuda_error(e, who); }

int rows_ok(const void* a, const void* b, int rows, int cols, const char* who) {
    if (rows < 0 || cols <= 0) return p2cu::fail_fmt(P2CU_EINVAL, "%s: shape [%d, %d]", who, rows, cols);
    if (rows && (!a || !b)) return p2cu::fail_fmt(P2CU_EINVAL, "%s: NULL pointer", who);
    return P2CU_OK;
}

}  // namespace

extern "C" {

int p2cu_layer_norm_rows(const float* x, const float* gamma, const float* beta, float* out, int n_rows, int D,
                         void* stream) {
    if (int rc = rows_ok(x, out, n_rows, D, "p2cu_layer_norm_rows")) return rc;
    if (n_rows && (!gamma || !beta)) return p2cu::fail_fmt(P2CU_EINVAL, "p2cu_layer_norm_rows: NULL gamma / beta");
    return done(p2cu::ln_rows_launch(x, D, gamma, beta, out, D, nullptr, nullptr, n_rows, D,
                                     static_cast<cudaStream_t>(stream)),
                "p2cu_layer_norm_rows");
}

int p2cu_layer_norm_quant_rows(const float* x, const float* gamma, const float* beta, signed char* q, float* scales,
                               int n_rows, int D, void* stream) {
    if (int rc = rows_ok(x, q, n_rows, D, "p2cu_layer_norm_quant_rows")) return rc;
    if (n_rows && (!gamma || !beta || !scales))
        return p2cu::fail_fmt(P2CU_EINVAL, "p2cu_layer_norm_quant_rows: NULL pointer");
    return done(p2cu::ln_rows_launch(x, D, gamma, beta, nullptr, 0, reinterpret_cast<int8_t*>(q), scales, n_rows, D,
                                     static_cast<cudaStream_t>(stream)),
                "p2cu_layer_norm_quant_rows");
}

int p2cu_swish(float* x, size_t n, void* stream) {
    if (n && !x) return p2cu::fail_fmt(P2CU_EINVAL, "p2cu_swish: NULL pointer");
    return done(p2cu::swish_launch(x, n, static_cast<cudaStream_t>(stream)), "p2cu_swish");
}

int p2cu_swish_quant_rows(const float* h, signed char* q, float* scales, int n_rows, int len, void* stream) {
    if (int rc = rows_ok(h, q, n_rows, len, "p2cu_swish_quant_rows")) return rc;
    if (n_rows && !scales) return p2cu::fail_fmt(P2CU_EINVAL, "p2cu_swish_quant_rows: NULL scales");
    return done(p2cu::swish_rows_launch(h, len, nullptr, 0, reinterpret_cast<int8_t*>(q), scales, n_rows, len,
                                        static_cast<cudaStream_t>(stream)),
                "p2cu_swish_quant_rows");
}

int p2cu_softmax_rows(float* x, int n_rows, int len, void* stream) {
    if (int rc = rows_ok(x, x, n_rows, len, "p2cu_softmax_rows")) return rc;
    return done(p2cu::softmax_rows_launch(x, n_rows, len, static_cast<cudaStream_t>(stream)), "p2cu_softmax_rows");
}

int p2cu_depthwise_conv1d_rows(const float* x, const float* w, const float* b, float* out, int C, int T,
                               void* stream) {
    if (int rc = rows_ok(x, out, T, C, "p2cu_depthwise_conv1d_rows")) return rc;
    if (T && !w) return p2cu::fail_fmt(P2CU_EINVAL, "p2cu_depthwise_conv1d_rows: NULL weights");
    if (C > 1024) return p2cu::fail_fmt(P2CU_EUNSUPPORTED, "p2cu_depthwise_conv1d_rows: C = %d > 1024", C);
    if (T == 0) return P2CU_OK;
    // one window of T rows; a NULL bias is a zero bias, as in the reference (csrc/tensor_ops.c:631)
    return done(p2cu::dwconv_swish_launch(x, w, b, nullptr, 1, out, nullptr, nullptr, T, C,
                                          static_cast<cudaStream_t>(stream), false),
                "p2cu_depthwise_conv1d_rows");
}

int p2cu_sgemm_tf32x3(int transB, int M, int N, int K, const float* A, int lda, const float* B, int ldb, float* C,
                      int ldc, void* stream) {
    if (M < 0 || N < 0 || K < 0) return p2cu::fail_fmt(P2CU_EINVAL, "p2cu_sgemm_tf32x3: shape M=%d N=%d K=%d", M, N, K);
    if (M == 0 || N == 0) return P2CU_OK;
    if (K == 0) return p2cu::fail_fmt(P2CU_EUNSUPPORTED, "p2cu_sgemm_tf32x3: K = 0");
    if (!A || !B || !C) return p2cu::fail_fmt(P2CU_EINVAL, "p2cu_sgemm_tf32x3: NULL pointer");
    if (lda < K || ldc < N || ldb < (transB ? K : N))
        return p2cu::fail_fmt(P2CU_EINVAL, "p2cu_sgemm_tf32x3: leading dimensions lda=%d ldb=%d ldc=%d", lda, ldb, ldc);
    p2cu::TcArgs a{};
    a.src[0] = A; a.src[1] = B;
    a.dst[0] = C; a.dst[1] = C;
    a.err = p2cu::device_error_word();
    p2cu::TcGroup& g = a.single;
    g.M = M; g.N = N; g.K = K; g.tile0 = 0;
    g.a_src = 0; g.b_src = 1; g.c_dst = 0; g.lda = lda; g.ldb = ldb; g.ldc = ldc; g.bias_sel = -1;
    return done(p2cu::attn_tc_launch(nullptr, 0, p2cu::tc_gemm_tiles(M, N), a, !transB,
                                     static_cast<cudaStream_t>(stream)),
                "p2cu_sgemm_tf32x3");
}

}  // extern "C"
