// api.cu - the device-pointer C ABI (include/p2cuda.h): argument checks, TMA descriptors, kernel selection.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <mutex>
#include <cuda.h>
#include <cuda_runtime.h>
#include "p2cuda.h"
#include "fv_gemm.h"
#include "kernels.h"
#include "numerics.cuh"
#include "gemm.h"

namespace {

thread_local char g_msg[512] = "";

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(P2CU_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

// The device error word the kernels report bounded-wait timeouts in; one per device (a __device__ variable exists
// once per device the module is loaded on), its address looked up per device.
__device__ uint32_t g_dev_err;

uint32_t* dev_err_ptr() {
    static uint32_t* ptrs[64] = {};
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!ptrs[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_dev_err) != cudaSuccess) return nullptr;
        ptrs[dev] = static_cast<uint32_t*>(p);
    }
    return ptrs[dev];
}

#ifdef P2CU_TRACE
// Diagnostic builds: pipeline timestamps of one CTA per GEMM launch (see fv_gemm.cu).
__device__ long long g_trace[512];
long long* trace_ptr() {
    void* p = nullptr;
    cudaGetSymbolAddress(&p, g_trace);
    return static_cast<long long*>(p);
}
#endif

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time dependency on libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// A 2-D tensor map: `inner` elements per row of `esize` bytes, `outer` rows `stride` bytes apart, boxes box_in x
// box_out elements, swizzle 0 / 64 / 128 (bytes).
int make_map(CUtensorMap* map, const void* base, int esize, uint64_t inner, uint64_t outer, uint64_t stride,
             uint32_t box_in, uint32_t box_out, int swizzle, const char* what) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(P2CU_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
    if (reinterpret_cast<uintptr_t>(base) % 16) return fail(P2CU_EINVAL, "%s: base address not 16-byte aligned", what);
    if (stride % 16) return fail(P2CU_EINVAL, "%s: row stride %llu not a multiple of 16 bytes", what,
                                 static_cast<unsigned long long>(stride));
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {stride};
    const cuuint32_t box[2] = {box_in, box_out};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapSwizzle sw = swizzle == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE;
    CUresult r = enc(map, esize == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                     const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(P2CU_ECUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
    return P2CU_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// SMs of the current device (looked up once per device).
int sm_count() {
    static int counts[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!counts[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        counts[dev] = n;
    }
    return counts[dev];
}

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

__global__ void scale_c_kernel(float* C, int M, int N, int ldc, float beta) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(M) * N) return;
    const int m = static_cast<int>(i / N), n = static_cast<int>(i % N);
    float* c = C + static_cast<size_t>(m) * ldc + n;
    *c = beta == 0.f ? 0.f : __fmul_rn(*c, beta);
}

// C = beta * C as the reference's scale_c (csrc/blas.c:60-70): nothing for beta == 1, zeros for beta == 0.
int scale_c(float* C, int M, int N, int ldc, float beta, cudaStream_t s) {
    if (beta == 1.f || M == 0 || N == 0) return P2CU_OK;
    const size_t total = static_cast<size_t>(M) * N;
    scale_c_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(C, M, N, ldc, beta);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? P2CU_OK : cuda_fail(e, "scale_c");
}

int check_gemm_common(int M, int N, int K, const void* C, int ldc, const char* who) {
    if (M < 0 || N < 0 || K < 0) return fail(P2CU_EINVAL, "%s: negative shape M=%d N=%d K=%d", who, M, N, K);
    if (!C && M && N) return fail(P2CU_EINVAL, "%s: C is NULL", who);
    if (ldc < N) return fail(P2CU_EINVAL, "%s: ldc=%d < N=%d", who, ldc, N);
    return P2CU_OK;
}

// Tile width for the tensor-core GEMM: the widest tile (128 for the two int8-mode planes, else 256) that still gives
// about half the SMs a CTA, else 64. P2CU_TILE_N=64|128|256 forces one (where the operand kind allows it).
// An on / off override from the environment: 1 forces, 0 forbids, -1 (unset or anything else) leaves the choice to
// the shape. Read once per variable (callers keep the result in a function-local static, initialised thread-safely).
int env_switch(const char* name) {
    const char* e = getenv(name);
    return e && e[0] == '1' ? 1 : e && e[0] == '0' ? 0 : -1;
}

int choose_bn(int M, int N, int nblk, int kind) {
    static const int forced = [] {
        const char* e = getenv("P2CU_TILE_N");
        const int v = e ? atoi(e) : 0;
        return (v == 64 || v == 128 || v == 256) ? v : 0;
    }();
    const int widest = kind == p2cu::KIND_ST ? 128 : 256;
    if (forced) return forced > widest ? widest : forced;
    const long mt = (M + 127) / 128;
    for (int bn = widest; bn > 64; bn /= 2)
        if (N % bn == 0 && static_cast<long>(N / bn) * mt * nblk >= 74) return bn;
    return 64;
}

size_t split_bytes(int M, int N, int K) {
    const int nblk = (K + 1023) / 1024;
    if (nblk <= 1) return 0;
    const size_t m_pad = (static_cast<size_t>(M) + 127) / 128 * 128;
    return round256(static_cast<size_t>(nblk) * m_pad * N * sizeof(float));
}

// The int8w GEMM with the weights expanded into tensor memory (fv_gemm_t.cu) for few rows, when B carries the
// value-index plane: N % 128 == 0, K % 16 == 0, M <= 1024 (P2CU_TGEMM=0 forbids it, 1 takes it up to M = 4096).
// Returns RUN_T_DECLINED for shapes it does not take, so the caller picks another kernel.
constexpr int RUN_T_DECLINED = 1;

// K > 1024: fold the per-block slices into C now, or (with `defer`, beta 1 and a dense C) describe them in *defer for
// the caller's next kernel to fold.
cudaError_t fold_or_defer(const void* ws, int m_pad, int nblk, const float* a_scales, float alpha, int beta_zero,
                          float* C, int M, int N, int ldc, cudaStream_t s, p2cu::KFold* defer) {
    if (defer && !beta_zero && ldc == N) {
        defer->f = static_cast<const float*>(ws);
        defer->m_pad = m_pad;
        defer->nblk = nblk;
        defer->a_scales = a_scales;
        defer->alpha = alpha;
        return cudaSuccess;
    }
    return p2cu::fv_combine_launch(static_cast<const float*>(ws), m_pad, nblk, a_scales, alpha, beta_zero, C, M, N,
                                   ldc, s);
}

int run_t(int M, int N, int K, float alpha, const int8_t* q, const float* a_scales, const P2cuFiveValue* B,
          float beta, float* C, int ldc, void* ws, size_t ws_bytes, cudaStream_t s, const char* who,
          p2cu::KFold* defer) {
    static const int t_env = env_switch("P2CU_TGEMM");
    if (t_env == 0 || N % 128 || K % 16 || M > (t_env == 1 ? 4096 : 1024)) return RUN_T_DECLINED;
    if (!B->lo || !B->hi) return fail(P2CU_EINVAL, "%s: lo / hi are NULL", who);
    if (B->K != K || B->N != N)
        return fail(P2CU_EINVAL, "%s: weight is [%d, %d], GEMM wants [%d, %d]", who, B->K, B->N, K, N);
    const int nblk = (K + 1023) / 1024;
    const size_t need = split_bytes(M, N, K);
    if (need && (!ws || ws_bytes < need || !aligned16(ws)))
        return fail(P2CU_EINVAL, "%s: K = %d needs %zu bytes of 16-byte aligned workspace, %zu given", who, K, need,
                    ws ? ws_bytes : 0);
    int rc;
    if (beta != 0.f && beta != 1.f) {
        if ((rc = scale_c(C, M, N, ldc, beta, s))) return rc;
        beta = 1.f;
    }
    p2cu::FvGemmTParams p{};
    p.M = M; p.N = N; p.K = K; p.alpha = alpha; p.beta_zero = beta == 0.f;
    p.a_scales = a_scales; p.lo = B->lo; p.hi = B->hi; p.C = C; p.ldc = ldc;
    p.vindex = B->vindex; p.kchunks = (K + 31) / 32;
    p.ws = static_cast<float*>(ws); p.ksplit = nblk; p.m_pad = (M + 127) / 128 * 128; p.err = dev_err_ptr();
#ifdef P2CU_TRACE
    static int t_launches = 0;
    p.trace_slot = t_launches++;
#endif
    const int mt = p2cu::fv_gemm_t_rows(M, N, nblk, sm_count());
    if (!aligned16(B->vindex)) return fail(P2CU_EINVAL, "%s: value-index plane not 16-byte aligned", who);
    CUtensorMap ta;
    if ((rc = make_map(&ta, q, 1, K, M, K, 128, mt, 128, "A"))) return rc;
    cudaError_t e = p2cu::fv_gemm_t_launch(mt, ta, p, s);
    if (e == cudaSuccess && nblk > 1)
        e = fold_or_defer(ws, p.m_pad, nblk, a_scales, alpha, p.beta_zero, C, M, N, ldc, s, defer);
    return e == cudaSuccess ? P2CU_OK : cuda_fail(e, who);
}

// The tcgen05 GEMM on quantised rows. `B` five-value (planes or cached codes) or `q8`/`scales` an int8 table.
// `ws` holds the per-block slices when K > 1024 (split_bytes).
int run_i8(int M, int N, int K, float alpha, const int8_t* q, const float* a_scales, const P2cuFiveValue* B,
           const int8_t* q8, const float* scales, int ldb, int mode, float beta, float* C, int ldc, void* ws,
           size_t ws_bytes, cudaStream_t s, const char* who, p2cu::KFold* defer = nullptr) {
    if (defer) defer->nblk = 0;
    int rc = check_gemm_common(M, N, K, C, ldc, who);
    if (rc) return rc;
    if (N % 16) return fail(P2CU_EINVAL, "%s: N = %d is not a multiple of 16", who, N);
    if (M == 0 || N == 0) return P2CU_OK;
    if (alpha == 0.f || K == 0) return scale_c(C, M, N, ldc, beta, s);   // no products: C = beta * C
    if (!q || !a_scales) return fail(P2CU_EINVAL, "%s: quantised A is NULL", who);
    if (B && mode == P2CU_INT8W && B->vindex) {
        rc = run_t(M, N, K, alpha, q, a_scales, B, beta, C, ldc, ws, ws_bytes, s, who, defer);
        if (rc != RUN_T_DECLINED) return rc;
    }
    if (N % 128 || K % 16 || !aligned16(C) || ldc % 4) {
        // shapes the tensor-core kernels do not take (the reference's int8 path takes any N % 16 == 0): the SIMT
        // kernel, same sums and epilogue (fv_gemm_simt.cu)
        p2cu::FvGemmParams p{};
        p.M = M; p.N = N; p.K = K; p.alpha = alpha; p.a_scales = a_scales; p.C = C; p.ldc = ldc;
        const int8_t* table = nullptr;
        const uint8_t *signs = nullptr, *flags = nullptr;
        int tld = 0;
        if (B) {
            if (!B->lo || !B->hi) return fail(P2CU_EINVAL, "%s: lo / hi are NULL", who);
            if (B->K != K || B->N != N)
                return fail(P2CU_EINVAL, "%s: weight is [%d, %d], GEMM wants [%d, %d]", who, B->K, B->N, K, N);
            p.lo = B->lo; p.hi = B->hi;
            p.cmode = mode == P2CU_INT8W ? p2cu::CM_INT8W : p2cu::CM_INT8;
            if (mode == P2CU_INT8W && B->codes) {
                table = B->codes; tld = N;
            } else {
                if (!B->signs || !B->flags) return fail(P2CU_EINVAL, "%s: planes are NULL", who);
                signs = B->signs; flags = B->flags;
            }
        } else {
            if (!q8 || !scales) return fail(P2CU_EINVAL, "%s: int8 table is NULL", who);
            if (ldb < N) return fail(P2CU_EINVAL, "%s: ldb=%d < N=%d", who, ldb, N);
            p.cmode = p2cu::CM_Q8B; p.scales = scales;
            table = q8; tld = ldb;
        }
        if (beta != 0.f && beta != 1.f) {
            if ((rc = scale_c(C, M, N, ldc, beta, s))) return rc;
            beta = 1.f;
        }
        p.beta_zero = beta == 0.f;
        cudaError_t e = p2cu::fv_gemm_simt_launch(q, signs, flags, table, tld, p, s);
        return e == cudaSuccess ? P2CU_OK : cuda_fail(e, who);
    }
    const int nblk = (K + 1023) / 1024;
    const size_t need = split_bytes(M, N, K);
    if (need && (!ws || ws_bytes < need || !aligned16(ws)))
        return fail(P2CU_EINVAL, "%s: K = %d needs %zu bytes of 16-byte aligned workspace, %zu given", who, K, need,
                    ws ? ws_bytes : 0);
    if (beta != 0.f && beta != 1.f) {
        if ((rc = scale_c(C, M, N, ldc, beta, s))) return rc;
        beta = 1.f;
    }
    p2cu::FvGemmParams p{};
    p.M = M; p.N = N; p.K = K; p.alpha = alpha; p.beta_zero = beta == 0.f;
    p.a_scales = a_scales; p.C = C; p.ldc = ldc; p.err = dev_err_ptr();
    p.ksplit = nblk;
    p.m_pad = (M + 127) / 128 * 128;
#ifdef P2CU_TRACE
    p.trace = trace_ptr();
#endif
    const bool planes = B && !(mode == P2CU_INT8W && B->codes);
    const int kind = !planes ? p2cu::KIND_TABLE : mode == P2CU_INT8W ? p2cu::KIND_CODES : p2cu::KIND_ST;
    // CTA pairs (256 x 256 tiles, fv_gemm_2sm.cu) for int8w / int8-table products with at least as many pair tiles
    // as the GPU has SM pairs (large M: batched windows); P2CU_PAIR=1 forces them where they apply, 0 forbids them.
    static const int pair_env = env_switch("P2CU_PAIR");
    const bool vec_ok = aligned16(B ? B->lo : nullptr) && aligned16(B ? B->hi : nullptr) && aligned16(scales);
    const bool pair_ok = vec_ok && kind != p2cu::KIND_ST && N % 256 == 0;
    const bool use_pair = pair_ok && (pair_env == 1 ||
                                      (pair_env == -1 &&
                                       2 * p2cu::fv_gemm_2sm_tiles(M, N, nblk) >= p2cu::fv_gemm_p_min_tiles()));
    const int bn = use_pair ? 128 : choose_bn(M, N, nblk, kind);
    const int atom = bn > 128 ? 128 : bn;   // an int8 table is loaded in boxes one swizzle atom wide
    CUtensorMap ta, tb0, tb1, tout;
    if ((rc = make_map(&ta, q, 1, K, M, K, 128, 128, 128, "A"))) return rc;
    // output box: 32 columns x 128 rows (one CTA's chunk), or x 32 rows for the pair kernel (one warp's block)
    const uint32_t out_rows = use_pair ? 32 : 128;
    if (nblk > 1)
        rc = make_map(&tout, ws, 4, N, static_cast<uint64_t>(nblk) * p.m_pad, static_cast<uint64_t>(N) * 4, 32,
                      out_rows, 128, "workspace");
    else
        rc = make_map(&tout, C, 4, N, M, static_cast<uint64_t>(ldc) * 4, 32, out_rows, 128, "C");
    if (rc) return rc;
    if (B) {
        if (!B->lo || !B->hi) return fail(P2CU_EINVAL, "%s: lo / hi are NULL", who);
        if (B->K != K || B->N != N) return fail(P2CU_EINVAL, "%s: weight is [%d, %d], GEMM wants [%d, %d]", who, B->K,
                                                B->N, K, N);
        p.lo = B->lo; p.hi = B->hi;
        p.cmode = mode == P2CU_INT8W ? p2cu::CM_INT8W : p2cu::CM_INT8;
        if (!planes) {   // int8w from the cached codes: one plane, f = (float)acc * (hi / 127)
            if ((rc = make_map(&tb0, B->codes, 1, N, K, N, atom, 128, atom, "codes"))) return rc;
            tb1 = tb0;
        } else {
            if (!B->signs || !B->flags) return fail(P2CU_EINVAL, "%s: planes are NULL", who);
            if ((rc = make_map(&tb0, B->signs, 1, N / 4, K, N / 4, bn / 4, 128, 0, "signs"))) return rc;
            if ((rc = make_map(&tb1, B->flags, 1, N / 8, K, N / 8, bn / 8 < 16 ? 16 : bn / 8, 128, 0, "flags")))
                return rc;
        }
    } else {
        if (!q8 || !scales) return fail(P2CU_EINVAL, "%s: int8 table is NULL", who);
        if (ldb < N) return fail(P2CU_EINVAL, "%s: ldb=%d < N=%d", who, ldb, N);
        p.cmode = p2cu::CM_Q8B;
        p.scales = scales;
        if ((rc = make_map(&tb0, q8, 1, N, K, ldb, atom, 128, atom, "B"))) return rc;
        tb1 = tb0;
    }
    // Many tiles (large M): the persistent kernel, where it measured faster - expanded planes, or more than one
    // 1024-row K block (with one K block from an int8 table or the code cache the one-tile-per-CTA kernel streams as
    // fast). P2CU_PERSIST=1 forces it, 0 forbids it. Its epilogue reads the per-column constants as 16-byte vectors.
    static const int persist_env = env_switch("P2CU_PERSIST");
    const bool many = p2cu::fv_gemm_p_tiles(M, N, bn, nblk) > p2cu::fv_gemm_p_min_tiles();
    const bool persist = vec_ok && (persist_env == 1 ||
                                    (persist_env == -1 && many && (kind != p2cu::KIND_TABLE || nblk > 1)));
    cudaError_t e = use_pair  ? p2cu::fv_gemm_2sm_launch(kind, ta, tb0, tb1, tout, p, s)
                    : persist ? p2cu::fv_gemm_p_launch(bn, kind, ta, tb0, tb1, tout, p, s)
                              : p2cu::fv_gemm_launch(bn, kind, ta, tb0, tb1, tout, p, s);
    if (e == cudaSuccess && nblk > 1)
        e = fold_or_defer(ws, p.m_pad, nblk, a_scales, alpha, p.beta_zero, C, M, N, ldc, s, defer);
    return e == cudaSuccess ? P2CU_OK : cuda_fail(e, who);
}

int run_exact(int M, int N, int K, float alpha, const float* A, int lda, int transA, const P2cuFiveValue* B,
              const int8_t* q8, const float* scales, const float* Bf, int ldb, int transB, float beta, float* C,
              int ldc, cudaStream_t s, const char* who, const p2cu::Epilogue* epi = nullptr) {
    int rc = check_gemm_common(M, N, K, C, ldc, who);
    if (rc) return rc;
    if (M == 0 || N == 0) return P2CU_OK;
    if (alpha == 0.f) return scale_c(C, M, N, ldc, beta, s);
    if (!A) return fail(P2CU_EINVAL, "%s: A is NULL", who);
    p2cu::ExactParams p{};
    p.M = M; p.N = N; p.K = K; p.alpha = alpha; p.beta = beta;
    p.A = A; p.lda = lda; p.transA = transA; p.ldb = ldb; p.transB = transB; p.C = C; p.ldc = ldc;
    p.vec_store = (N % 4 == 0) && (ldc % 4 == 0) && aligned16(C);
    if (epi) {
        if (epi->residual && beta != 0.f) return fail(P2CU_EINVAL, "%s: a residual epilogue needs beta == 0", who);
        if (epi->residual && alpha == 0.f) return fail(P2CU_EINVAL, "%s: a residual epilogue needs alpha != 0", who);
        p.bias = epi->bias; p.relu = epi->relu; p.residual = epi->residual; p.res_alpha = epi->res_alpha;
    }
    if (B) {
        if (N % 16) return fail(P2CU_EINVAL, "%s: N = %d is not a multiple of 16", who, N);
        if (B->K != K || B->N != N) return fail(P2CU_EINVAL, "%s: weight is [%d, %d], GEMM wants [%d, %d]", who, B->K,
                                                B->N, K, N);
        if (!B->signs || !B->flags || !B->lo || !B->hi) return fail(P2CU_EINVAL, "%s: planes are NULL", who);
        p.bkind = p2cu::BK_FIVE;
        p.signs = B->signs; p.flags = B->flags; p.lo = B->lo; p.hi = B->hi;
    } else if (q8) {
        if (N % 16) return fail(P2CU_EINVAL, "%s: N = %d is not a multiple of 16", who, N);
        if (!scales) return fail(P2CU_EINVAL, "%s: scales are NULL", who);
        p.bkind = p2cu::BK_TABLE;
        p.q8 = q8; p.scales = scales;
    } else {
        if (!Bf) return fail(P2CU_EINVAL, "%s: B is NULL", who);
        p.bkind = p2cu::BK_F32;
        p.Bf = Bf;
    }
    cudaError_t e = p2cu::exact_gemm_launch(p, s);
    return e == cudaSuccess ? P2CU_OK : cuda_fail(e, who);
}

}  // namespace

namespace p2cu {
// For the library's other translation units: set the text p2cu_last_error() returns on this thread.
void set_error_message(int code, const char* msg) { fail(code, "%s", msg); }

int fail_fmt(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_error(cudaError_t e, const char* what) { return cuda_fail(e, what); }

uint32_t* device_error_word() { return dev_err_ptr(); }

size_t gemm_split_bytes(int M, int N, int K) { return split_bytes(M, N, K); }

int make_tile_map(CUtensorMap* map, const void* base, int esize, uint64_t inner, uint64_t outer, uint64_t stride,
                  uint32_t box_in, uint32_t box_out, int swizzle, const char* what) {
    return make_map(map, base, esize, inner, outer, stride, box_in, box_out, swizzle, what);
}

int gemm_i8(int M, int N, int K, float alpha, const int8_t* q, const float* a_scales, const P2cuFiveValue* B,
            const int8_t* q8, const float* scales, int ldb, int mode, float beta, float* C, int ldc, void* ws,
            size_t ws_bytes, cudaStream_t s, const char* who, KFold* defer) {
    return run_i8(M, N, K, alpha, q, a_scales, B, q8, scales, ldb, mode, beta, C, ldc, ws, ws_bytes, s, who, defer);
}

int gemm_exact(int M, int N, int K, float alpha, const float* A, int lda, int transA, const P2cuFiveValue* B,
               const int8_t* q8, const float* scales, const float* Bf, int ldb, int transB, float beta, float* C,
               int ldc, const Epilogue* epi, cudaStream_t s, const char* who) {
    return run_exact(M, N, K, alpha, A, lda, transA, B, q8, scales, Bf, ldb, transB, beta, C, ldc, s, who, epi);
}
}  // namespace p2cu

extern "C" {

#ifdef P2CU_TRACE
__attribute__((visibility("default"))) int p2cu_debug_trace(long long* out, int n) {
    return cudaMemcpyFromSymbol(out, g_trace, sizeof(long long) * (n < 512 ? n : 512)) == cudaSuccess ? 0 : -1;
}
#endif

const char* p2cu_last_error(void) { return g_msg; }

int p2cu_check_device(void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The error word comes back on the stream itself, into a page-locked word of the calling thread, so that one
    // synchronisation covers the work and the read (each host thread keeps its word for the process's life).
    static thread_local uint32_t* word = nullptr;
    if (!word && cudaMallocHost(&word, sizeof(uint32_t)) != cudaSuccess) {
        cudaGetLastError();
        word = nullptr;
    }
    cudaError_t e = cudaSuccess;
    uint32_t v = 0, zero = 0;
    if (word) {
        e = cudaMemcpyFromSymbolAsync(word, g_dev_err, sizeof(uint32_t), 0, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return cuda_fail(e, "stream");
        v = *word;
    } else {
        if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_fail(e, "stream");
        if ((e = cudaMemcpyFromSymbol(&v, g_dev_err, sizeof(v))) != cudaSuccess) return cuda_fail(e, "error word");
    }
    if (v) {
        cudaMemcpyToSymbol(g_dev_err, &zero, sizeof(zero));
        return fail(P2CU_EDEVICE, "a kernel stopped early and reported device error code %u", v);
    }
    return P2CU_OK;
}

int p2cu_set_quant_fast_math(int on) {
    const int prev = p2cu::quant_fast_math();
    p2cu::set_quant_fast_math(on);
    return prev;
}

int p2cu_quant_fast_math(void) { return p2cu::quant_fast_math(); }

int p2cu_quant_rows(const float* A, int M, int K, int lda, signed char* q, float* scales, void* stream) {
    if (M < 0 || K < 0 || lda < K) return fail(P2CU_EINVAL, "p2cu_quant_rows: bad shape M=%d K=%d lda=%d", M, K, lda);
    if (M == 0 || K == 0) return P2CU_OK;
    if (!A || !q || !scales) return fail(P2CU_EINVAL, "p2cu_quant_rows: NULL pointer");
    cudaError_t e = p2cu::quant_rows_launch(A, M, K, lda, reinterpret_cast<int8_t*>(q), scales,
                                            static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? P2CU_OK : cuda_fail(e, "p2cu_quant_rows");
}

int p2cu_sgemm_fvb_q8a(int M, int N, int K, float alpha, const signed char* q, const float* a_scales,
                       const P2cuFiveValue* B, int mode, float beta, float* C, int ldc, void* workspace,
                       size_t workspace_bytes, void* stream) {
    if (!B) return fail(P2CU_EINVAL, "p2cu_sgemm_fvb_q8a: B is NULL");
    if (mode != P2CU_INT8 && mode != P2CU_INT8W) return fail(P2CU_EINVAL, "p2cu_sgemm_fvb_q8a: mode %d", mode);
    return run_i8(M, N, K, alpha, reinterpret_cast<const int8_t*>(q), a_scales, B, nullptr, nullptr, 0, mode, beta,
                  C, ldc, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), "p2cu_sgemm_fvb_q8a");
}

int p2cu_sgemm_q8b_q8a(int M, int N, int K, float alpha, const signed char* q, const float* a_scales,
                       const signed char* B, const float* scales, int ldb, float beta, float* C, int ldc,
                       void* workspace, size_t workspace_bytes, void* stream) {
    return run_i8(M, N, K, alpha, reinterpret_cast<const int8_t*>(q), a_scales, nullptr,
                  reinterpret_cast<const int8_t*>(B), scales, ldb, P2CU_INT8, beta, C, ldc, workspace,
                  workspace_bytes, static_cast<cudaStream_t>(stream), "p2cu_sgemm_q8b_q8a");
}

size_t p2cu_q8a_workspace_bytes(int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    return split_bytes(M, N, K);
}

size_t p2cu_gemm_workspace_bytes(int M, int N, int K, int mode) {
    if (mode == P2CU_EXACT || K % 4 || M <= 0 || K <= 0 || N <= 0) return 0;   // K % 4 != 0 runs the exact path
    return round256(static_cast<size_t>(M) * K) + round256(static_cast<size_t>(M) * sizeof(float)) +
           split_bytes(M, N, K);
}

// Quantise A into the head of the workspace; the rest (if any) is handed to the GEMM for its K-block slices.
static int quantise_into(const float* A, int M, int N, int K, int lda, void* ws, size_t ws_bytes, int8_t** q,
                         float** sc, void** rest, size_t* rest_bytes, cudaStream_t s, const char* who) {
    const size_t need = p2cu_gemm_workspace_bytes(M, N, K, P2CU_INT8);
    if (!ws || ws_bytes < need) return fail(P2CU_EINVAL, "%s: workspace of %zu bytes, %zu needed", who, ws_bytes, need);
    if (!aligned16(ws)) return fail(P2CU_EINVAL, "%s: workspace not 16-byte aligned", who);
    if (!A) return fail(P2CU_EINVAL, "%s: A is NULL", who);
    const size_t head = round256(static_cast<size_t>(M) * K) + round256(static_cast<size_t>(M) * sizeof(float));
    *q = static_cast<int8_t*>(ws);
    *sc = reinterpret_cast<float*>(static_cast<char*>(ws) + round256(static_cast<size_t>(M) * K));
    *rest = static_cast<char*>(ws) + head;
    *rest_bytes = ws_bytes - head;
    cudaError_t e = p2cu::quant_rows_launch(A, M, K, lda, *q, *sc, s);
    return e == cudaSuccess ? P2CU_OK : cuda_fail(e, who);
}

int p2cu_sgemm_fvb(int M, int N, int K, float alpha, const float* A, int lda, const P2cuFiveValue* B, int mode,
                   float beta, float* C, int ldc, void* workspace, size_t workspace_bytes, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!B) return fail(P2CU_EINVAL, "p2cu_sgemm_fvb: B is NULL");
    if (mode == P2CU_EXACT)
        return run_exact(M, N, K, alpha, A, lda, 0, B, nullptr, nullptr, nullptr, 0, 0, beta, C, ldc, s,
                         "p2cu_sgemm_fvb");
    if (mode != P2CU_INT8 && mode != P2CU_INT8W) return fail(P2CU_EINVAL, "p2cu_sgemm_fvb: mode %d", mode);
    if (K % 4)   // the reference quantises only whole quads; other K take its exact path (csrc/blas.c:1490-1495)
        return run_exact(M, N, K, alpha, A, lda, 0, B, nullptr, nullptr, nullptr, 0, 0, beta, C, ldc, s,
                         "p2cu_sgemm_fvb");
    int rc = check_gemm_common(M, N, K, C, ldc, "p2cu_sgemm_fvb");
    if (rc) return rc;
    if (M == 0 || N == 0) return P2CU_OK;
    if (alpha == 0.f || K == 0) return scale_c(C, M, N, ldc, beta, s);
    int8_t* q;
    float* sc;
    void* rest;
    size_t rest_bytes;
    if ((rc = quantise_into(A, M, N, K, lda, workspace, workspace_bytes, &q, &sc, &rest, &rest_bytes, s,
                            "p2cu_sgemm_fvb")))
        return rc;
    return run_i8(M, N, K, alpha, q, sc, B, nullptr, nullptr, 0, mode, beta, C, ldc, rest, rest_bytes, s,
                  "p2cu_sgemm_fvb");
}

int p2cu_sgemm_q8b(int M, int N, int K, float alpha, const float* A, int lda, const signed char* B,
                   const float* scales, int ldb, int mode, float beta, float* C, int ldc, void* workspace,
                   size_t workspace_bytes, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (mode == P2CU_EXACT || K % 4)   // K % 4 != 0: the reference's exact path (csrc/blas.c:1470-1478)
        return run_exact(M, N, K, alpha, A, lda, 0, nullptr, reinterpret_cast<const int8_t*>(B), scales, nullptr, ldb,
                         0, beta, C, ldc, s, "p2cu_sgemm_q8b");
    int rc = check_gemm_common(M, N, K, C, ldc, "p2cu_sgemm_q8b");
    if (rc) return rc;
    if (M == 0 || N == 0) return P2CU_OK;
    if (alpha == 0.f || K == 0) return scale_c(C, M, N, ldc, beta, s);
    int8_t* q;
    float* sc;
    void* rest;
    size_t rest_bytes;
    if ((rc = quantise_into(A, M, N, K, lda, workspace, workspace_bytes, &q, &sc, &rest, &rest_bytes, s,
                            "p2cu_sgemm_q8b")))
        return rc;
    return run_i8(M, N, K, alpha, q, sc, nullptr, reinterpret_cast<const int8_t*>(B), scales, ldb, P2CU_INT8, beta, C,
                  ldc, rest, rest_bytes, s, "p2cu_sgemm_q8b");
}

int p2cu_sgemm(int transA, int transB, int M, int N, int K, float alpha, const float* A, int lda, const float* B,
               int ldb, float beta, float* C, int ldc, void* stream) {
    return run_exact(M, N, K, alpha, A, lda, transA ? 1 : 0, nullptr, nullptr, nullptr, B, ldb, transB ? 1 : 0, beta,
                     C, ldc, static_cast<cudaStream_t>(stream), "p2cu_sgemm");
}

size_t p2cu_fv_vindex_bytes(int K, int N) {
    if (K <= 0 || N <= 0) return 0;
    return static_cast<size_t>((K + 31) / 32) * N * 16;
}

int p2cu_fv_pack_vindex(const P2cuFiveValue* B, unsigned int* vindex, void* stream) {
    if (!B || !vindex || !B->signs || !B->flags) return fail(P2CU_EINVAL, "p2cu_fv_pack_vindex: NULL pointer");
    if (B->K <= 0 || B->N <= 0 || B->N % 16)
        return fail(P2CU_EINVAL, "p2cu_fv_pack_vindex: shape [%d, %d]", B->K, B->N);
    if (!aligned16(vindex)) return fail(P2CU_EINVAL, "p2cu_fv_pack_vindex: output not 16-byte aligned");
    cudaError_t e = p2cu::fv_vindex_launch(B->signs, B->flags, B->K, B->N, vindex, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? P2CU_OK : cuda_fail(e, "p2cu_fv_pack_vindex");
}

int p2cu_fv_pack_codes(const P2cuFiveValue* B, signed char* codes, void* stream) {
    if (!B || !codes || !B->signs || !B->flags || !B->lo || !B->hi)
        return fail(P2CU_EINVAL, "p2cu_fv_pack_codes: NULL pointer");
    if (B->K <= 0 || B->N <= 0 || B->N % 16) return fail(P2CU_EINVAL, "p2cu_fv_pack_codes: shape [%d, %d]", B->K, B->N);
    cudaError_t e = p2cu::fv_codes_launch(B->signs, B->flags, B->lo, B->hi, B->K, B->N,
                                          reinterpret_cast<int8_t*>(codes), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? P2CU_OK : cuda_fail(e, "p2cu_fv_pack_codes");
}

}  // extern "C"
