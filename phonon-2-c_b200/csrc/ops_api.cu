// ops_api.cu - the encoder's row ops on device rows (include/p2cuda.h), each one launch of an encoder_ops kernel.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
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

namespace {

// The scratch of p2cu_rel_attention: the windows' row offsets, the launch's tiles, then (when its keys are split) the
// merge counters and the split parts.
struct RelAttnLayout {
    std::vector<p2cu::AttnTile> tiles;
    int n_groups = 0;
    bool split = false;
    size_t tiles_off = 0, counters_off = 0, parts_off = 0, bytes = 0;
};

int sm_count() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                  cudaSuccess) {
        (void)cudaGetLastError();
        return 148;
    }
    return sms;
}

RelAttnLayout rel_attention_layout(int n_win, const int* T) {
    RelAttnLayout l;
    const int n = p2cu::attn_rel_tc_plan(T, n_win, sm_count(), l.tiles, &l.n_groups);
    for (const p2cu::AttnTile& t : l.tiles) l.split = l.split || t.nsplit > 1;
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    l.tiles_off = up(static_cast<size_t>(n_win + 1) * sizeof(int));
    l.counters_off = up(l.tiles_off + static_cast<size_t>(n) * sizeof(p2cu::AttnTile));
    l.parts_off = up(l.counters_off + (l.split ? static_cast<size_t>(l.n_groups) * 8 * sizeof(int) : 0));
    l.bytes = l.parts_off + (l.split ? p2cu::attn_rel_tc_part_bytes(n) : 0);
    return l;
}

}  // namespace

size_t p2cu_rel_attention_ws_bytes(int n_win, const int* T) {
    if (n_win <= 0 || !T) return 0;
    for (int w = 0; w < n_win; ++w)
        if (T[w] <= 0) return 0;
    return rel_attention_layout(n_win, T).bytes;
}

int p2cu_rel_attention(const float* qkv, const float* P, const float* bias_u, const float* bias_v, const int* T,
                       int n_win, int Tmax, float* attn, void* ws, size_t ws_bytes, void* stream) {
    const char* who = "p2cu_rel_attention";
    if (n_win < 0) return p2cu::fail_fmt(P2CU_EINVAL, "%s: n_win = %d", who, n_win);
    if (n_win == 0) return P2CU_OK;
    if (!qkv || !P || !bias_u || !bias_v || !T || !attn || !ws)
        return p2cu::fail_fmt(P2CU_EINVAL, "%s: NULL pointer", who);
    if (Tmax <= 0 || Tmax > p2cu::ATT_MAXT)
        return p2cu::fail_fmt(P2CU_EUNSUPPORTED, "%s: Tmax = %d (1 .. %d)", who, Tmax, p2cu::ATT_MAXT);
    for (int w = 0; w < n_win; ++w)
        if (T[w] <= 0 || T[w] > Tmax)
            return p2cu::fail_fmt(P2CU_EINVAL, "%s: T[%d] = %d, Tmax = %d", who, w, T[w], Tmax);
    if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(P) | reinterpret_cast<uintptr_t>(bias_u) |
         reinterpret_cast<uintptr_t>(bias_v) | reinterpret_cast<uintptr_t>(attn) |
         reinterpret_cast<uintptr_t>(ws)) & 15)
        return p2cu::fail_fmt(P2CU_EINVAL, "%s: pointers must be 16-byte aligned", who);
    const RelAttnLayout l = rel_attention_layout(n_win, T);
    if (ws_bytes < l.bytes) return p2cu::fail_fmt(P2CU_EINVAL, "%s: ws_bytes %zu < %zu", who, ws_bytes, l.bytes);
    std::vector<uint8_t> host(l.counters_off, 0);
    int* off = reinterpret_cast<int*>(host.data());
    off[0] = 0;
    for (int w = 0; w < n_win; ++w) off[w + 1] = off[w] + T[w];
    std::memcpy(host.data() + l.tiles_off, l.tiles.data(), l.tiles.size() * sizeof(p2cu::AttnTile));
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    // from pageable memory: the call returns once the bytes are staged, so `host` may go out of scope
    cudaError_t e = cudaMemcpyAsync(ws, host.data(), host.size(), cudaMemcpyHostToDevice, s);
    uint8_t* wsb = static_cast<uint8_t*>(ws);
    if (e == cudaSuccess && l.split)
        e = cudaMemsetAsync(wsb + l.counters_off, 0, static_cast<size_t>(l.n_groups) * 8 * sizeof(int), s);
    if (e != cudaSuccess) return p2cu::cuda_error(e, who);
    return p2cu::attn_rel_tc_launch(qkv, off[n_win], P, bias_u, bias_v, reinterpret_cast<const int*>(wsb),
                                    reinterpret_cast<const p2cu::AttnTile*>(wsb + l.tiles_off),
                                    static_cast<int>(l.tiles.size()), Tmax, 1.0f / sqrtf(128.0f), attn,
                                    l.split ? wsb + l.parts_off : nullptr,
                                    l.split ? reinterpret_cast<int*>(wsb + l.counters_off) : nullptr,
                                    p2cu::device_error_word(), s);
}

}  // extern "C"
