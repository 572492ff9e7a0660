/*  blas.h - phonon-2-c's GEMM layer ABI (its csrc/blas.h, v0.1.0), implemented on B200 by libphonon2_b200.so.
 *
 *  Same names, argument lists, types and contracts as the reference, so that the reference's callers (its
 *  tensor_ops.c, encoder.c, weights.c, bench_gemm.c, the Python bindings) link against this library unchanged.
 *  All pointers here are HOST pointers, as in the reference. Behind each call:
 *    - five-value and int8-table weights are uploaded to the GPU once, on first use, and found again by their host
 *      address (weights are read-only for a model's life, as the reference's mmap'd planes are);
 *    - A (and C when beta != 0) are copied to the device, the GEMM runs on the calling thread's CUDA stream, and C
 *      is copied back before the call returns, so the calls stay synchronous like the reference's;
 *    - P2_GEMM = int8 | int8w | exact (and P2_EXACT = 1) select the mode as in the reference (csrc/blas.c:1027-1047);
 *      the int8 modes run on the tensor cores on every host, the default is int8w.
 *  Contract violations abort() with a message, as the reference's do (csrc/blas.c:989-995).
 */
#ifndef P2_BLAS_H
#define P2_BLAS_H

#include "phonon2.h"

#ifdef __cplusplus
extern "C" {
#endif

/* csrc/blas.h:19-22 */
typedef enum {
    P2_NO_TRANS = 111,
    P2_TRANS    = 112
} P2Trans;

/* fp32 C = alpha * op(A) * op(B) + beta * C, row-major with leading dimensions (csrc/blas.h:24-29). */
P2_API void p2_sgemm(P2Trans transA, P2Trans transB, int M, int N, int K, float alpha, const float *A, int lda,
                     const float *B, int ldb, float beta, float *C, int ldc);

/* The reference's variant for use inside its pool workers (csrc/blas.h:31-36); here the same call as p2_sgemm. */
P2_API void p2_sgemm_st(P2Trans transA, P2Trans transB, int M, int N, int K, float alpha, const float *A, int lda,
                        const float *B, int ldb, float beta, float *C, int ldc);

/* Five-value B [K, N] (csrc/blas.h:38-45): w[k][n] = sign * (flag ? hi[n] : lo[n]). */
typedef struct {
    const unsigned char *signs;   /* [K][N/4]: code 0 -> -1, 1 -> 0, 2 -> +1 at bits 2*(n & 3) */
    const unsigned char *flags;   /* [K][N/8]: bit (n & 7) set -> |w| = hi[n] */
    const float         *lo;      /* [N] */
    const float         *hi;      /* [N] */
    const signed char   *codes;   /* optional: the buffer p2_fv_pack_codes returned for this weight, or NULL */
} FiveValueB;

/* The int8w codes sign * (flag ? 127 : round(127 lo / hi)) of a whole weight (csrc/blas.h:51). The returned buffer
 * (K * N bytes, malloc'd, the caller frees it) holds them row-major [K][N]; passing it back in FiveValueB.codes makes
 * the int8w GEMM stream these codes (kept on the GPU) instead of expanding the planes. NULL on a bad shape. */
P2_API signed char *p2_fv_pack_codes(const FiveValueB *b, int K, int N);

/* C = alpha * A * B + beta * C with B an int8 table [K, N] (ldb bytes per row), one scale per column; N % 16 == 0
 * (csrc/blas.h:54-57). */
P2_API void p2_sgemm_q8b(int M, int N, int K, float alpha, const float *A, int lda, const signed char *B,
                         const float *scales, int ldb, float beta, float *C, int ldc);

/* C = alpha * A * B + beta * C with B five-value [K, N]; N % 16 == 0 (csrc/blas.h:60-63). */
P2_API void p2_sgemm_fvb(int M, int N, int K, float alpha, const float *A, int lda, const FiveValueB *B, float beta,
                         float *C, int ldc);

/* The GEMM mode in words, and whether it is the exact one (csrc/blas.h:67-68). */
P2_API const char *p2_gemm_mode(void);
P2_API int p2_gemm_exact(void);

/* Prepare a QuantA of M rows of K for the int8 GEMMs; -1 in exact mode (the caller then takes the fp32 route).
 * The buffer belongs to the calling thread and is reused by its next prepare (csrc/blas.h:72-73). */
P2_API int  p2_quant_prepare(QuantA *qa, int M, int K);
P2_API void p2_quant_row(const QuantA *qa, int m, const float *row);   /* any thread may call it */

/* The int8 GEMMs on a prepared QuantA; beta 0 stores, 1 accumulates (csrc/blas.h:76-79). */
P2_API void p2_sgemm_fvb_q8a(int M, int N, int K, float alpha, const QuantA *A, const FiveValueB *B, float beta,
                             float *C, int ldc);
P2_API void p2_sgemm_q8b_q8a(int M, int N, int K, float alpha, const QuantA *A, const signed char *B,
                             const float *scales, int ldb, float beta, float *C, int ldc);

/* ---- additions of this build (no counterpart in the reference) --------------------------------------------------- */

/* The GPU the calling thread's GEMMs run on (the analogue of the reference's per-thread p2_set_pool,
 * csrc/threadpool.h:42-46). Default: the CUDA device current when the thread first calls in. Returns 0 or -1. */
P2_API int p2_b200_set_device(int device);

/* Drop every weight uploaded so far on every device (call before freeing or reusing host weight memory). */
P2_API void p2_b200_release_weights(void);

#ifdef __cplusplus
}
#endif

#endif /* P2_BLAS_H */
