/*  ref_int8_blas.c - the int8 GEMM entry points of phonon-2-c's blas.h, restated, for an x86 build of the
 *  reference's own encoder.
 *
 *  TEST INFRASTRUCTURE ONLY. oracle/Makefile links this file with phonon-2-c's encoder.c, tensor_ops.c, threadpool.c
 *  (and the rest of its library) compiled unchanged from the reference's sources, plus its blas.c compiled with the
 *  int8 entry points renamed (refx_*). The result, _ref/libphonon2_ref_i8.so, runs the reference encoder's int8
 *  control flow (csrc/encoder.c:319-612: LayerNorm / SiLU / head-concat / depthwise-conv rows quantised as they are
 *  produced, residuals added in the GEMM epilogue) on x86, where the reference's own int8 kernels do not compile
 *  (they need AArch64 dot products, csrc/blas.c:1021-1023). The int8 arithmetic is fv_oracle.c's restatement of
 *  csrc/blas.c:1114-1370; everything else is the reference's code. Only tests/ load this library.
 *
 *  Mode (orc_shim_set_mode): 0 = int8 (two planes), 2 = int8w (codes), 1 = exact (every call forwards to the
 *  reference's own fp32 path, p2_quant_prepare declines as on x86).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include "phonon2.h"
#include "blas.h"

/* the reference's own blas.c definitions, renamed when that file is compiled for this library */
void refx_sgemm_fvb(int M, int N, int K, float alpha, const float *A, int lda, const FiveValueB *B, float beta,
                    float *C, int ldc);
void refx_sgemm_q8b(int M, int N, int K, float alpha, const float *A, int lda, const signed char *B,
                    const float *scales, int ldb, float beta, float *C, int ldc);

/* fv_oracle.c */
void orc_quant_row(const float *row, int K, int8_t *q, float *scale_out);
void orc_gemm_i8(int M, int N, int K, float alpha, const int8_t *q, const float *a_scales, int mode,
                 const uint8_t *signs, const uint8_t *flags, const float *lo, const float *hi,
                 const int8_t *q8, const float *scales, int ldb, float beta, float *C, int ldc);
void orc_sgemm_i8(int M, int N, int K, float alpha, const float *A, int lda, int mode,
                  const uint8_t *signs, const uint8_t *flags, const float *lo, const float *hi,
                  const int8_t *q8, const float *scales, int ldb, float beta, float *C, int ldc);

enum { SHIM_INT8 = 0, SHIM_EXACT = 1, SHIM_INT8W = 2, ORC_Q8B = 8 };
static int g_mode = SHIM_INT8W;

__attribute__((visibility("default"))) void orc_shim_set_mode(int mode) { g_mode = mode; }

static int fv_mode(void) { return g_mode == SHIM_INT8 ? 0 : 2; }

/* The calling thread's QuantA buffer, reused by the next prepare as in the reference (csrc/phonon2.h:429-431). */
static __thread signed char *t_q;
static __thread float *t_s;
static __thread size_t t_capq, t_caps;

int p2_quant_prepare(QuantA *qa, int M, int K)
{
    if (g_mode == SHIM_EXACT || M <= 0 || K <= 0 || K % 4) return -1;
    size_t nq = (size_t)M * K, ns = (size_t)M;
    if (nq > t_capq) { free(t_q); t_q = (signed char *)malloc(nq); t_capq = t_q ? nq : 0; }
    if (ns > t_caps) { free(t_s); t_s = (float *)malloc(ns * sizeof(float)); t_caps = t_s ? ns : 0; }
    if (!t_q || !t_s) return -1;
    qa->q = t_q; qa->scales = t_s; qa->M = M; qa->K = K;
    return 0;
}

void p2_quant_row(const QuantA *qa, int m, const float *row)
{
    orc_quant_row(row, qa->K, (int8_t *)qa->q + (size_t)m * qa->K, qa->scales + m);
}

void p2_sgemm_fvb_q8a(int M, int N, int K, float alpha, const QuantA *A, const FiveValueB *B, float beta, float *C,
                      int ldc)
{
    orc_gemm_i8(M, N, K, alpha, (const int8_t *)A->q, A->scales, fv_mode(), B->signs, B->flags, B->lo, B->hi, NULL,
                NULL, 0, beta, C, ldc);
}

void p2_sgemm_q8b_q8a(int M, int N, int K, float alpha, const QuantA *A, const signed char *B, const float *scales,
                      int ldb, float beta, float *C, int ldc)
{
    orc_gemm_i8(M, N, K, alpha, (const int8_t *)A->q, A->scales, ORC_Q8B, NULL, NULL, NULL, NULL,
                (const int8_t *)B, scales, ldb, beta, C, ldc);
}

void p2_sgemm_fvb(int M, int N, int K, float alpha, const float *A, int lda, const FiveValueB *B, float beta,
                  float *C, int ldc)
{
    if (g_mode == SHIM_EXACT || K % 4) { refx_sgemm_fvb(M, N, K, alpha, A, lda, B, beta, C, ldc); return; }
    orc_sgemm_i8(M, N, K, alpha, A, lda, fv_mode(), B->signs, B->flags, B->lo, B->hi, NULL, NULL, 0, beta, C, ldc);
}

void p2_sgemm_q8b(int M, int N, int K, float alpha, const float *A, int lda, const signed char *B,
                  const float *scales, int ldb, float beta, float *C, int ldc)
{
    if (g_mode == SHIM_EXACT || K % 4) { refx_sgemm_q8b(M, N, K, alpha, A, lda, B, scales, ldb, beta, C, ldc); return; }
    orc_sgemm_i8(M, N, K, alpha, A, lda, ORC_Q8B, NULL, NULL, NULL, NULL, (const int8_t *)B, scales, ldb, beta, C,
                 ldc);
}

signed char *p2_fv_pack_codes(const FiveValueB *b, int K, int N)
{
    (void)b; (void)K; (void)N;
    return NULL;   /* no code cache in this checker: the planes are expanded every call */
}

int p2_gemm_exact(void) { return g_mode == SHIM_EXACT; }

const char *p2_gemm_mode(void)
{
    return g_mode == SHIM_EXACT ? "exact (reference)" : g_mode == SHIM_INT8 ? "int8 (restated)" : "int8w (restated)";
}
