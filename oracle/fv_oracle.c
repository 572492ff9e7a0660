/*  fv_oracle.c - CPU restatement of phonon-2-c's five-value GEMM arithmetic.
 *
 *  TEST INFRASTRUCTURE ONLY. This file is the checker the GPU kernels are compared against; only tests/,
 *  __graft_entry__.smoke() and bench.py's cpu_baseline leg load it. Nothing in the product links it.
 *
 *  What it restates (reference paths are relative to the phonon-2-c project root):
 *    - per-row symmetric int8 quantisation of A ............. csrc/blas.c:1114-1144 (quant_pack_row)
 *    - the two int8 planes S = sign, T = sign * flag ........ csrc/blas.c:1190-1220 (fv_row16_i8, pack_fv_panel)
 *    - the int8w code plane sign * (flag ? 127 : clo) ....... csrc/blas.c:1222-1240, clo at 1316-1328
 *    - int32 sums restarted every 1024 rows of K ............ csrc/blas.c:1025, 1257-1282, 1339-1353
 *    - the fp32 epilogue per K block, in the reference order  csrc/blas.c:1316-1366
 *    - the exact (fp32 expansion) path as one FMA chain ...... csrc/blas.c:60-70 (scale_c), 155-181, 841-910, 931-987
 *    - the int8-table operand (q8b) ......................... csrc/blas.c:806-836, 1243-1254, 1462-1479
 *
 *  Parity status. The exact path is pinned: tests compare it bit for bit with the reference's own blas.c compiled
 *  from source (oracle/Makefile -> oracle/_ref/). The int8 / int8w paths of the reference only compile on AArch64 with
 *  the dot-product extension (blas.c:1021-1023); no such compiler exists here, so their bit-level parity is UNPINNED
 *  by the reference itself. They are cross-checked against the pinned exact path on activations the quantiser maps
 *  exactly (integer-valued rows whose max is 127), where both must agree up to fp32 rounding.
 *
 *  Numerics choices (documented ambiguity): the reference is built with -ffast-math, which lets the compiler turn
 *  amax / 127.0f and 127.0f * lo / hi into multiplications by reciprocals. This restatement uses IEEE division for
 *  both, as the C source is written. All FMAs are explicit fmaf() and the file is compiled with -ffp-contract=off.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_KBLK 1024   /* K rows per int32 block in the reference's int8 kernels (blas.c:1025, KC_I8) */

/* ---- quantisation ---------------------------------------------------------------------------------------- */

/* Round half to even with saturation, as the NEON vcvtnq_s32_f32 (FCVTNS) the reference uses (blas.c:1124-1127):
 * NaN gives 0 and values beyond the int32 range give its ends. Both occur when 1 / scale overflows to infinity (a row
 * whose largest magnitude is below about 3.7e-37): x * inf is +-inf, and 0 * inf is NaN. */
static int32_t round_even(float x)
{
    if (x != x) return 0;
    if (x >= 2147483648.0f) return INT32_MAX;
    if (x <= -2147483648.0f) return INT32_MIN;
    return (int32_t)nearbyintf(x);   /* default rounding mode is to-nearest-even */
}

static int8_t sat8(int32_t v)         /* vqmovn_s32 then vqmovn_s16: saturate to [-128, 127] */
{
    return (int8_t)(v > 127 ? 127 : v < -128 ? -128 : v);
}

/* One row: amax over |x|, scale = amax / 127 (1 when the row is all zero). The first K - K % 16 values take the
 * reference's 16-wide loop, q = sat(rne(x * (1 / scale))) (blas.c:1122-1138); the last K % 16 its scalar tail,
 * q = clamp(lrintf(x / scale), -127, 127) (blas.c:1139-1143): a division rather than the reciprocal, so a value can
 * round to the other side of a half. */
void orc_quant_row(const float *row, int K, int8_t *q, float *scale_out)
{
    float amax = 0.0f;
    for (int k = 0; k < K; k++) {
        float v = fabsf(row[k]);
        if (v > amax) amax = v;
    }
    float scale = amax > 0.0f ? amax / 127.0f : 1.0f;
    float inv = 1.0f / scale;
    const int k16 = K & ~15;
    for (int k = 0; k < k16; k++) q[k] = sat8(round_even(row[k] * inv));
    for (int k = k16; k < K; k++) {
        int32_t v = round_even(row[k] / scale);
        q[k] = (int8_t)(v > 127 ? 127 : v < -127 ? -127 : v);
    }
    *scale_out = scale;
}

void orc_quant_rows(const float *A, int M, int K, int lda, int8_t *q, float *scales)
{
    #pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) orc_quant_row(A + (size_t)m * lda, K, q + (size_t)m * K, scales + m);
}

/* The same row as the reference's Makefile builds it (-O3 -ffast-math, csrc/Makefile:2), which its compiler derives
 * from the same source: amax / 127.0f becomes amax * (1/127) (the reciprocal rounded to fp32), 1 / scale folds into
 * 127 / amax (one division), and the tail's x / scale becomes x times that reciprocal; the tail's lrintf of a product
 * that is not finite (the reciprocal overflowed: a row whose largest magnitude is below about 1e-39) comes out of the
 * int conversion as 0. Pinned against that build of the reference compiled here (tests/test_ref_neon.py). */
void orc_quant_row_fast_math(const float *row, int K, int8_t *q, float *scale_out)
{
    float amax = 0.0f;
    for (int k = 0; k < K; k++) {
        float v = fabsf(row[k]);
        if (v > amax) amax = v;
    }
    const float recip127 = 1.0f / 127.0f;
    const float scale = amax > 0.0f ? amax * recip127 : 1.0f;
    const float inv = amax > 0.0f ? 127.0f / amax : 1.0f;
    const int k16 = K & ~15;
    for (int k = 0; k < k16; k++) q[k] = sat8(round_even(row[k] * inv));
    for (int k = k16; k < K; k++) {
        const float t = row[k] * inv;
        const int32_t v = isfinite(t) ? round_even(t) : 0;
        q[k] = (int8_t)(v > 127 ? 127 : v < -127 ? -127 : v);
    }
    *scale_out = scale;
}

void orc_quant_rows_fast_math(const float *A, int M, int K, int lda, int8_t *q, float *scales)
{
    #pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) orc_quant_row_fast_math(A + (size_t)m * lda, K, q + (size_t)m * K, scales + m);
}

/* ---- five-value planes ----------------------------------------------------------------------------------- */

/* sign of w[k][n] in {-1, 0, +1}: 2-bit code at bits 2*(n&3) of signs[k*N/4 + n/4], code - 1 (blas.h:38-45). */
static inline int fv_sign(const uint8_t *signs, int N, int k, int n)
{
    return (int)((signs[(size_t)k * (N / 4) + (n >> 2)] >> (2 * (n & 3))) & 3) - 1;
}

static inline int fv_flag(const uint8_t *flags, int N, int k, int n)
{
    return (flags[(size_t)k * (N / 8) + (n >> 3)] >> (n & 7)) & 1;
}

/* clo[n] = clamp(lrintf(127 * lo / hi), 0, 127), 0 when hi <= 0 (blas.c:1319-1324). */
int orc_clo(float lo, float hi)
{
    int c = hi > 0.0f ? (int)lrintf(127.0f * lo / hi) : 0;
    return c < 0 ? 0 : c > 127 ? 127 : c;
}

/* The int8w codes of a whole weight as a plain row-major [K][N] int8 plane (blas.c:1222-1240 values; the
 * reference's panel layout is a CPU cache layout and plays no part in the values). */
void orc_fv_codes(const uint8_t *signs, const uint8_t *flags, const float *lo, const float *hi, int K, int N,
                  int8_t *codes)
{
    #pragma omp parallel for schedule(static)
    for (int k = 0; k < K; k++)
        for (int n = 0; n < N; n++) {
            int s = fv_sign(signs, N, k, n);
            int mag = fv_flag(flags, N, k, n) ? 127 : orc_clo(lo[n], hi[n]);
            codes[(size_t)k * N + n] = (int8_t)(s * mag);
        }
}

/* The exact fp32 weight: s * fma(f, hi - lo, lo), i.e. one of {0, +-lo, +-hi} bit for bit (blas.c:838-840, 895). */
static inline float fv_weight(const uint8_t *signs, const uint8_t *flags, const float *lo, const float *hi,
                              int N, int k, int n)
{
    float s = (float)fv_sign(signs, N, k, n), f = (float)fv_flag(flags, N, k, n);
    return s * fmaf(f, hi[n] - lo[n], lo[n]);
}

/* ---- int32 accumulators per K block ---------------------------------------------------------------------- */

/* mode 0 = int8 (two planes: accS = sum q*S, accT = sum q*T), mode 2 = int8w (accS = sum q*code, accT unused),
 * mode 8 = int8 table (accS = sum q*B). Outputs are [nblk][M][N], nblk = ceil(K / 1024). */
enum { ORC_INT8 = 0, ORC_INT8W = 2, ORC_Q8B = 8 };

void orc_acc_blocks(int M, int N, int K, const int8_t *q, int mode,
                    const uint8_t *signs, const uint8_t *flags, const float *lo, const float *hi,
                    const int8_t *q8, int ldb, int32_t *accS, int32_t *accT)
{
    int nblk = (K + ORC_KBLK - 1) / ORC_KBLK;
    int8_t *clo = (int8_t *)malloc((size_t)N);
    if (mode == ORC_INT8W)
        for (int n = 0; n < N; n++) clo[n] = (int8_t)orc_clo(lo[n], hi[n]);
    /* Per block, the B operand(s) of every column as a contiguous int8 row over the block's k: P = the int8w codes,
     * the int8 table, or S (sign); Q = T (sign * flag) in int8 mode. Then plain integer dot products. */
    int8_t *P = (int8_t *)malloc((size_t)N * ORC_KBLK), *Q = (int8_t *)malloc((size_t)N * ORC_KBLK);
    for (int b = 0; b < nblk; b++) {
        int k0 = b * ORC_KBLK, kb = (k0 + ORC_KBLK < K ? ORC_KBLK : K - k0);
        #pragma omp parallel for schedule(static)
        for (int n = 0; n < N; n++)
            for (int i = 0; i < kb; i++) {
                int k = k0 + i;
                int8_t pv, qv = 0;
                if (mode == ORC_Q8B) pv = q8[(size_t)k * ldb + n];
                else {
                    int s = fv_sign(signs, N, k, n), f = fv_flag(flags, N, k, n);
                    if (mode == ORC_INT8W) pv = (int8_t)(s * (f ? 127 : clo[n]));
                    else { pv = (int8_t)s; qv = (int8_t)(s * f); }
                }
                P[(size_t)n * ORC_KBLK + i] = pv;
                Q[(size_t)n * ORC_KBLK + i] = qv;
            }
        #pragma omp parallel for schedule(dynamic, 4)
        for (int m = 0; m < M; m++) {
            const int8_t *qr = q + (size_t)m * K + k0;
            int32_t *s_out = accS + ((size_t)b * M + m) * N;
            int32_t *t_out = accT ? accT + ((size_t)b * M + m) * N : NULL;
            for (int n = 0; n < N; n++) {
                const int8_t *pr = P + (size_t)n * ORC_KBLK, *tr = Q + (size_t)n * ORC_KBLK;
                int32_t sS = 0, sT = 0;
                for (int i = 0; i < kb; i++) sS += (int32_t)qr[i] * pr[i];
                if (t_out) {
                    for (int i = 0; i < kb; i++) sT += (int32_t)qr[i] * tr[i];
                    t_out[n] = sT;
                }
                s_out[n] = sS;
            }
        }
    }
    free(P);
    free(Q);
    free(clo);
}

/* ---- the int8 GEMM with the reference epilogue ----------------------------------------------------------- */

/* scale_c (blas.c:60-70): C = beta * C, zeros for beta == 0, nothing for beta == 1. */
static void scale_rows(float *C, int M, int N, int ldc, float beta)
{
    if (beta == 1.0f) return;
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) C[(size_t)m * ldc + n] = beta == 0.0f ? 0.0f : C[(size_t)m * ldc + n] * beta;
}

/* C = alpha * A * B + beta * C on pre-quantised A (q row-major [M][K], one scale per row), as p2_sgemm_fvb_q8a and
 * p2_sgemm_q8b_q8a run it (blas.c:1430-1446): alpha == 0 only scales C; other beta than 0 and 1 scale C first (scale_c,
 * blas.c:60-70) and then accumulate. Per K block b and element:
 *   int8w: f = (float)acc * (hi * (1/127))            int8: f = fma((float)accT, hi - lo, (float)accS * lo)
 *   q8b:   f = (float)acc * scale[n]
 *   as = a_scale[m] * alpha;  C = (beta == 0 && b == 0) ? f * as : fma(f, as, C)      (blas.c:1316-1366) */
void orc_gemm_i8(int M, int N, int K, float alpha, const int8_t *q, const float *a_scales, int mode,
                 const uint8_t *signs, const uint8_t *flags, const float *lo, const float *hi,
                 const int8_t *q8, const float *scales, int ldb, float beta, float *C, int ldc)
{
    if (alpha == 0.0f) { scale_rows(C, M, N, ldc, beta); return; }
    if (beta != 0.0f && beta != 1.0f) { scale_rows(C, M, N, ldc, beta); beta = 1.0f; }
    int nblk = (K + ORC_KBLK - 1) / ORC_KBLK;
    size_t plane = (size_t)nblk * M * N;
    int32_t *accS = (int32_t *)malloc(plane * sizeof(int32_t));
    int32_t *accT = mode == ORC_INT8 ? (int32_t *)malloc(plane * sizeof(int32_t)) : NULL;
    orc_acc_blocks(M, N, K, q, mode, signs, flags, lo, hi, q8, ldb, accS, accT);
    const float inv127 = 1.0f / 127.0f;
    #pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        float as = a_scales[m] * alpha;
        float *crow = C + (size_t)m * ldc;
        for (int b = 0; b < nblk; b++) {
            const int32_t *sS = accS + ((size_t)b * M + m) * N;
            const int32_t *sT = accT ? accT + ((size_t)b * M + m) * N : NULL;
            int store = (beta == 0.0f && b == 0);
            for (int n = 0; n < N; n++) {
                float f;
                if (mode == ORC_INT8W)     f = (float)sS[n] * (hi[n] * inv127);
                else if (mode == ORC_Q8B)  f = (float)sS[n] * scales[n];
                else                       f = fmaf((float)sT[n], hi[n] - lo[n], (float)sS[n] * lo[n]);
                crow[n] = store ? f * as : fmaf(f, as, crow[n]);
            }
        }
    }
    free(accS);
    free(accT);
}

/* ---- the exact path: one FMA chain per output ------------------------------------------------------------ */

/* The exact path: scale_c (blas.c:60-70), then for every output c = fma(alpha * a[m][k], w[k][n], c) over
 * k = 0..K-1 in order: the micro-kernels load C, run the chain over a KC block and store C, block after block
 * (blas.c:155-181, 960-985). */

void orc_gemm_exact(int M, int N, int K, float alpha, const float *A, int lda,
                    const uint8_t *signs, const uint8_t *flags, const float *lo, const float *hi,
                    const int8_t *q8, const float *scales, int ldb, float beta, float *C, int ldc)
{
    scale_rows(C, M, N, ldc, beta);
    if (alpha == 0.0f) return;
    float *W = (float *)malloc((size_t)K * N * sizeof(float));
    #pragma omp parallel for schedule(static)
    for (int k = 0; k < K; k++)
        for (int n = 0; n < N; n++)
            W[(size_t)k * N + n] = q8 ? (float)q8[(size_t)k * ldb + n] * scales[n]   /* pack_B_panel_q8c */
                                      : fv_weight(signs, flags, lo, hi, N, k, n);
    #pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        float *crow = C + (size_t)m * ldc;
        const float *arow = A + (size_t)m * lda;
        for (int k = 0; k < K; k++) {
            float a = alpha * arow[k];
            const float *w = W + (size_t)k * N;
            for (int n = 0; n < N; n++) crow[n] = fmaf(a, w[n], crow[n]);
        }
    }
    free(W);
}

/* The full int8 entry as p2_sgemm_fvb runs it when the int8 path is on (blas.c:1481-1495): quantise A, then the
 * GEMM on the quantised rows. */
void orc_sgemm_i8(int M, int N, int K, float alpha, const float *A, int lda, int mode,
                  const uint8_t *signs, const uint8_t *flags, const float *lo, const float *hi,
                  const int8_t *q8, const float *scales, int ldb, float beta, float *C, int ldc)
{
    if (alpha == 0.0f) { scale_rows(C, M, N, ldc, beta); return; }
    int8_t *q = (int8_t *)malloc((size_t)M * K);
    float *sc = (float *)malloc((size_t)M * sizeof(float));
    orc_quant_rows(A, M, K, lda, q, sc);
    if (beta != 0.0f && beta != 1.0f) { scale_rows(C, M, N, ldc, beta); beta = 1.0f; }
    orc_gemm_i8(M, N, K, alpha, q, sc, mode, signs, flags, lo, hi, q8, scales, ldb, beta, C, ldc);
    free(q);
    free(sc);
}
