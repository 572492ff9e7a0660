// ops_api.cu - the encoder's row ops on device rows (include/p2cuda.h), each one launch of an encoder_ops kernel.
#include <cstdint>
#include <cuda_runtime.h>
#include "p2cuda.h"
#include "gemm.h"
#include "encoder_ops.h"

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

}  // extern "C"
