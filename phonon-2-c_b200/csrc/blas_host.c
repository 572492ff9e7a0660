/*  blas_host.c - phonon-2-c's host-pointer GEMM ABI (include/blas.h) on top of the device ABI (include/p2cuda.h).
 *
 *  The reference's blas.c (csrc/blas.c) runs these calls on a CPU thread pool. Here each calling thread gets a
 *  CUDA stream and grow-only device buffers (the analogue of the reference's per-thread I8Bufs and B_pack,
 *  csrc/blas.c:529-557, 1070-1110); weights are uploaded once and found again by their host address; activations
 *  and results cross PCIe on every call, and the call returns once C is back in host memory. No arithmetic runs on
 *  the host: quantisation, the fp32 expansion and all products happen in the library's kernels.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <cuda_runtime_api.h>
#include "blas.h"
#include "p2cuda.h"

/* ---- failure: the reference aborts on contract violations and out-of-memory (csrc/blas.c:989-995, 1309) ---- */

static void die(const char *who, const char *what)
{
    fprintf(stderr, "%s: %s\n", who, what);
    abort();
}

static void check_cuda(cudaError_t e, const char *who)
{
    if (e != cudaSuccess) die(who, cudaGetErrorString(e));
}

static void check_p2(int rc, const char *who)
{
    if (rc != P2CU_OK) die(who, p2cu_last_error());
}

static void require_panel_aligned(int N, const char *who)
{
    if (N % 16 != 0) {
        fprintf(stderr, "%s: N = %d is not a multiple of 16\n", who, N);
        abort();
    }
}

/* ---- GEMM mode: P2_GEMM / P2_EXACT, read once (csrc/blas.c:1027-1047) ---- */

static int g_mode = -1;
static pthread_once_t g_mode_once = PTHREAD_ONCE_INIT;

static void mode_init(void)
{
    const char *g = getenv("P2_GEMM"), *e = getenv("P2_EXACT");
    int mode = P2CU_INT8W;
    if (g && strcmp(g, "exact") == 0) mode = P2CU_EXACT;
    else if (g && strcmp(g, "int8") == 0) mode = P2CU_INT8;
    else if (g && strcmp(g, "int8w") == 0) mode = P2CU_INT8W;
    if (e && e[0] && e[0] != '0') mode = P2CU_EXACT;
    g_mode = mode;
}

static int gemm_mode(void)
{
    pthread_once(&g_mode_once, mode_init);
    return g_mode;
}

const char *p2_gemm_mode(void)
{
    switch (gemm_mode()) {
    case P2CU_INT8:  return "int8 tensor-core products, exact weights (sm_100a)";
    case P2CU_INT8W: return "int8 tensor-core products, int8 weights (sm_100a)";
    default:         return "fp32 expansion (exact, sm_100a)";
    }
}

int p2_gemm_exact(void) { return gemm_mode() == P2CU_EXACT; }

/* For the library's encoder entry points (host_entry.cu): the mode in P2CU_* numbering. Not exported. */
int p2b_gemm_mode(void) { return gemm_mode(); }

/* ---- per-thread context ---- */

typedef struct {
    int          device;
    cudaStream_t stream;
    void        *dA;  size_t capA;    /* fp32 A, dense */
    void        *dB;  size_t capB;    /* fp32 B (p2_sgemm only), dense */
    void        *dC;  size_t capC;    /* fp32 C, dense */
    void        *ws;  size_t capW;    /* quantised A */
    float       *hq;  size_t capQ;    /* pinned host rows of the current QuantA */
} Ctx;

static pthread_key_t  g_ctx_key;
static pthread_once_t g_ctx_once = PTHREAD_ONCE_INIT;
static __thread int   t_device = -1;   /* set by p2_b200_set_device */

static void ctx_destroy(void *p)
{
    Ctx *c = (Ctx *)p;
    if (!c) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    cudaFree(c->dA); cudaFree(c->dB); cudaFree(c->dC); cudaFree(c->ws);
    cudaFreeHost(c->hq);
    cudaStreamDestroy(c->stream);
    cudaSetDevice(prev);
    free(c);
}

static void ctx_key_init(void) { pthread_key_create(&g_ctx_key, ctx_destroy); }

static Ctx *ctx_get(const char *who)
{
    pthread_once(&g_ctx_once, ctx_key_init);
    Ctx *c = (Ctx *)pthread_getspecific(g_ctx_key);
    int want = t_device;
    if (want < 0) check_cuda(cudaGetDevice(&want), who);
    if (c && c->device != want) {   /* the thread moved to another GPU: start over there */
        ctx_destroy(c);
        pthread_setspecific(g_ctx_key, NULL);
        c = NULL;
    }
    if (!c) {
        c = (Ctx *)calloc(1, sizeof(*c));
        if (!c) die(who, "out of memory");
        c->device = want;
        check_cuda(cudaSetDevice(want), who);
        check_cuda(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), who);
        pthread_setspecific(g_ctx_key, c);
    }
    check_cuda(cudaSetDevice(c->device), who);
    return c;
}

static void *grow(void **p, size_t *cap, size_t need, const char *who)
{
    if (need <= *cap) return *p;
    if (*p) cudaFree(*p);
    *p = NULL;
    *cap = 0;
    size_t n = need + need / 4;
    check_cuda(cudaMalloc(p, n), who);
    *cap = n;
    return *p;
}

/* The GPU the calling thread's calls run on (p2_b200_set_device, else the current device). Not exported. */
int p2b_thread_device(void)
{
    int d = t_device;
    if (d < 0 && cudaGetDevice(&d) != cudaSuccess) d = 0;
    return d;
}

int p2_b200_set_device(int device)
{
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return -1;
    t_device = device;
    return 0;
}

/* ---- weight registry: device copies found by host address and device ---- */

enum { W_FIVE = 1, W_TABLE = 2 };

typedef struct Entry {
    const void   *key;
    int           kind, device, K, N, ldb;
    uint64_t      print;          /* fingerprint of the host weight, to notice reused addresses */
    void         *block;          /* one device allocation holding every copy */
    P2cuFiveValue fv;             /* W_FIVE: device planes (+ codes once packed) */
    void         *codes;          /* W_FIVE: device int8w codes, or NULL */
    const signed char *q8;        /* W_TABLE: device table (dense, N bytes per row) */
    const float  *scales;         /* W_TABLE */
    struct Entry *next;
} Entry;

#define REG_BUCKETS 1024
static Entry          *g_reg[REG_BUCKETS];
static pthread_mutex_t g_reg_mu = PTHREAD_MUTEX_INITIALIZER;

static uint64_t mix(uint64_t h, uint64_t v)
{
    h ^= v + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    return h;
}

static uint64_t bytes_print(uint64_t h, const void *p, size_t n)
{
    const unsigned char *b = (const unsigned char *)p;
    size_t take = n < 64 ? n : 64;
    for (size_t i = 0; i < take; i++) h = mix(h, b[i]);
    for (size_t i = n - take; i < n; i++) h = mix(h, b[i]);
    return h;
}

static uint64_t five_print(const FiveValueB *b, int K, int N)
{
    uint64_t h = mix(mix((uint64_t)K, (uint64_t)N), (uint64_t)(uintptr_t)b->flags);
    h = mix(mix(h, (uint64_t)(uintptr_t)b->lo), (uint64_t)(uintptr_t)b->hi);
    h = bytes_print(h, b->signs, (size_t)K * N / 4);
    h = bytes_print(h, b->flags, (size_t)K * N / 8);
    h = bytes_print(h, b->lo, (size_t)N * sizeof(float));
    return bytes_print(h, b->hi, (size_t)N * sizeof(float));
}

static unsigned bucket(const void *key, int device)
{
    uint64_t v = (uint64_t)(uintptr_t)key * 0x9e3779b97f4a7c15ull + (uint64_t)device;
    return (unsigned)(v >> 40) % REG_BUCKETS;
}

static Entry *reg_find(const void *key, int kind, int device, uint64_t print)
{
    for (Entry *e = g_reg[bucket(key, device)]; e; e = e->next)
        if (e->key == key && e->kind == kind && e->device == device && e->print == print) return e;
    return NULL;
}

static void reg_insert(Entry *e)
{
    unsigned b = bucket(e->key, e->device);
    e->next = g_reg[b];
    g_reg[b] = e;
}

static size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

/* The device copy of a five-value weight (uploaded on first sight). Caller holds g_reg_mu. */
static Entry *five_entry(const FiveValueB *b, int K, int N, Ctx *c, const char *who)
{
    if (!b || !b->signs || !b->flags || !b->lo || !b->hi) die(who, "five-value weight with NULL planes");
    uint64_t print = five_print(b, K, N);
    Entry *e = reg_find(b->signs, W_FIVE, c->device, print);
    if (e) return e;
    size_t s_b = (size_t)K * N / 4, f_b = (size_t)K * N / 8, v_b = (size_t)N * sizeof(float);
    size_t o_f = al256(s_b), o_lo = o_f + al256(f_b), o_hi = o_lo + al256(v_b), o_vi = o_hi + al256(v_b);
    size_t total = o_vi + al256(p2cu_fv_vindex_bytes(K, N));
    e = (Entry *)calloc(1, sizeof(*e));
    if (!e) die(who, "out of memory");
    check_cuda(cudaMalloc(&e->block, total), who);
    char *d = (char *)e->block;
    check_cuda(cudaMemcpy(d, b->signs, s_b, cudaMemcpyHostToDevice), who);
    check_cuda(cudaMemcpy(d + o_f, b->flags, f_b, cudaMemcpyHostToDevice), who);
    check_cuda(cudaMemcpy(d + o_lo, b->lo, v_b, cudaMemcpyHostToDevice), who);
    check_cuda(cudaMemcpy(d + o_hi, b->hi, v_b, cudaMemcpyHostToDevice), who);
    e->key = b->signs; e->kind = W_FIVE; e->device = c->device; e->K = K; e->N = N; e->print = print;
    e->fv.signs = (const unsigned char *)d;
    e->fv.flags = (const unsigned char *)(d + o_f);
    e->fv.lo = (const float *)(d + o_lo);
    e->fv.hi = (const float *)(d + o_hi);
    e->fv.codes = NULL;
    e->fv.K = K; e->fv.N = N;
    /* the value-index plane, read by the int8w GEMMs of few rows (include/p2cuda.h p2cu_fv_pack_vindex) */
    check_p2(p2cu_fv_pack_vindex(&e->fv, (unsigned int *)(d + o_vi), c->stream), who);
    check_cuda(cudaStreamSynchronize(c->stream), who);
    e->fv.vindex = (const unsigned int *)(d + o_vi);
    reg_insert(e);
    return e;
}

/* Device int8w codes of a registered five-value weight, packed on the GPU on first request. */
static void ensure_codes(Entry *e, Ctx *c, const char *who)
{
    if (e->codes) return;
    check_cuda(cudaMalloc(&e->codes, (size_t)e->K * e->N), who);
    check_p2(p2cu_fv_pack_codes(&e->fv, (signed char *)e->codes, c->stream), who);
    check_cuda(cudaStreamSynchronize(c->stream), who);
    e->fv.codes = (const signed char *)e->codes;
}

static Entry *table_entry(const signed char *B, const float *scales, int K, int N, int ldb, Ctx *c, const char *who)
{
    if (!B || !scales) die(who, "int8 table with NULL data");
    uint64_t print = mix(mix(mix((uint64_t)K, (uint64_t)N), (uint64_t)ldb), (uint64_t)(uintptr_t)scales);
    print = bytes_print(print, B, (size_t)(K - 1) * ldb + N);
    print = bytes_print(print, scales, (size_t)N * sizeof(float));
    Entry *e = reg_find(B, W_TABLE, c->device, print);
    if (e) return e;
    size_t q_b = (size_t)K * N, o_s = al256(q_b), total = o_s + al256((size_t)N * sizeof(float));
    e = (Entry *)calloc(1, sizeof(*e));
    if (!e) die(who, "out of memory");
    check_cuda(cudaMalloc(&e->block, total), who);
    char *d = (char *)e->block;
    check_cuda(cudaMemcpy2D(d, (size_t)N, B, (size_t)ldb, (size_t)N, (size_t)K, cudaMemcpyHostToDevice), who);
    check_cuda(cudaMemcpy(d + o_s, scales, (size_t)N * sizeof(float), cudaMemcpyHostToDevice), who);
    e->key = B; e->kind = W_TABLE; e->device = c->device; e->K = K; e->N = N; e->ldb = ldb; e->print = print;
    e->q8 = (const signed char *)d;
    e->scales = (const float *)(d + o_s);
    reg_insert(e);
    return e;
}

void p2b_release_encoder_models(void);   /* host_entry.cu */

void p2_b200_release_weights(void)
{
    p2b_release_encoder_models();
    pthread_mutex_lock(&g_reg_mu);
    int prev = 0;
    cudaGetDevice(&prev);
    for (int i = 0; i < REG_BUCKETS; i++) {
        Entry *e = g_reg[i];
        while (e) {
            Entry *n = e->next;
            cudaSetDevice(e->device);
            cudaDeviceSynchronize();
            cudaFree(e->block);
            cudaFree(e->codes);
            free(e);
            e = n;
        }
        g_reg[i] = NULL;
    }
    cudaSetDevice(prev);
    pthread_mutex_unlock(&g_reg_mu);
}

/* ---- moving activations ---- */

/* rows x cols floats from host (row pitch ld floats) into dense device memory. */
static void put_rows(Ctx *c, void *dst, const float *src, int rows, int cols, int ld, const char *who)
{
    if (rows <= 0 || cols <= 0) return;
    check_cuda(cudaMemcpy2DAsync(dst, (size_t)cols * sizeof(float), src, (size_t)ld * sizeof(float),
                                 (size_t)cols * sizeof(float), (size_t)rows, cudaMemcpyHostToDevice, c->stream), who);
}

static void get_rows(Ctx *c, float *dst, const void *src, int rows, int cols, int ld, const char *who)
{
    if (rows <= 0 || cols <= 0) return;
    check_cuda(cudaMemcpy2DAsync(dst, (size_t)ld * sizeof(float), src, (size_t)cols * sizeof(float),
                                 (size_t)cols * sizeof(float), (size_t)rows, cudaMemcpyDeviceToHost, c->stream), who);
}

static void finish(Ctx *c, const char *who)
{
    check_p2(p2cu_check_device(c->stream), who);   /* synchronises, then reads the device error word */
}

/* ---- the ABI ---- */

void p2_sgemm(P2Trans transA, P2Trans transB, int M, int N, int K, float alpha, const float *A, int lda,
              const float *B, int ldb, float beta, float *C, int ldc)
{
    const char *who = "p2_sgemm";
    if (M <= 0 || N <= 0) return;
    Ctx *c = ctx_get(who);
    int tA = transA == P2_TRANS, tB = transB == P2_TRANS;
    int a_rows = tA ? K : M, a_cols = tA ? M : K, b_rows = tB ? N : K, b_cols = tB ? K : N;
    void *dA = grow(&c->dA, &c->capA, (size_t)M * K * sizeof(float) + 16, who);
    void *dB = grow(&c->dB, &c->capB, (size_t)K * N * sizeof(float) + 16, who);
    void *dC = grow(&c->dC, &c->capC, (size_t)M * N * sizeof(float) + 16, who);
    if (alpha != 0.0f && K > 0) {
        put_rows(c, dA, A, a_rows, a_cols, lda, who);
        put_rows(c, dB, B, b_rows, b_cols, ldb, who);
    }
    if (beta != 0.0f) put_rows(c, dC, C, M, N, ldc, who);
    check_p2(p2cu_sgemm(tA, tB, M, N, K, alpha, (const float *)dA, a_cols, (const float *)dB, b_cols, beta,
                        (float *)dC, N, c->stream), who);
    get_rows(c, C, dC, M, N, ldc, who);
    finish(c, who);
}

void p2_sgemm_st(P2Trans transA, P2Trans transB, int M, int N, int K, float alpha, const float *A, int lda,
                 const float *B, int ldb, float beta, float *C, int ldc)
{
    p2_sgemm(transA, transB, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

static void run_fvb(int M, int N, int K, float alpha, const float *A, int lda, const FiveValueB *B, float beta,
                    float *C, int ldc, const char *who)
{
    require_panel_aligned(N, who);
    if (M <= 0 || N <= 0) return;
    Ctx *c = ctx_get(who);
    int mode = gemm_mode();
    pthread_mutex_lock(&g_reg_mu);
    Entry *e = five_entry(B, K, N, c, who);
    if (mode == P2CU_INT8W && B->codes) ensure_codes(e, c, who);
    P2cuFiveValue fv = e->fv;
    pthread_mutex_unlock(&g_reg_mu);
    if (mode != P2CU_INT8W || !B->codes) fv.codes = NULL;
    size_t wsb = p2cu_gemm_workspace_bytes(M, N, K, mode);
    void *dA = grow(&c->dA, &c->capA, (size_t)M * K * sizeof(float) + 16, who);
    void *dC = grow(&c->dC, &c->capC, (size_t)M * N * sizeof(float) + 16, who);
    void *ws = grow(&c->ws, &c->capW, wsb + 256, who);
    if (alpha != 0.0f && K > 0) put_rows(c, dA, A, M, K, lda, who);
    if (beta != 0.0f) put_rows(c, dC, C, M, N, ldc, who);
    check_p2(p2cu_sgemm_fvb(M, N, K, alpha, (const float *)dA, K, &fv, mode, beta, (float *)dC, N, ws, c->capW,
                            c->stream), who);
    get_rows(c, C, dC, M, N, ldc, who);
    finish(c, who);
}

void p2_sgemm_fvb(int M, int N, int K, float alpha, const float *A, int lda, const FiveValueB *B, float beta,
                  float *C, int ldc)
{
    run_fvb(M, N, K, alpha, A, lda, B, beta, C, ldc, "p2_sgemm_fvb");
}

static void run_q8b(int M, int N, int K, float alpha, const float *A, int lda, const signed char *B,
                    const float *scales, int ldb, float beta, float *C, int ldc, int mode, const char *who)
{
    require_panel_aligned(N, who);
    if (M <= 0 || N <= 0) return;
    Ctx *c = ctx_get(who);
    pthread_mutex_lock(&g_reg_mu);
    Entry *e = table_entry(B, scales, K, N, ldb, c, who);
    const signed char *q8 = e->q8;
    const float *sc = e->scales;
    pthread_mutex_unlock(&g_reg_mu);
    size_t wsb = p2cu_gemm_workspace_bytes(M, N, K, mode);
    void *dA = grow(&c->dA, &c->capA, (size_t)M * K * sizeof(float) + 16, who);
    void *dC = grow(&c->dC, &c->capC, (size_t)M * N * sizeof(float) + 16, who);
    void *ws = grow(&c->ws, &c->capW, wsb + 256, who);
    if (alpha != 0.0f && K > 0) put_rows(c, dA, A, M, K, lda, who);
    if (beta != 0.0f) put_rows(c, dC, C, M, N, ldc, who);
    check_p2(p2cu_sgemm_q8b(M, N, K, alpha, (const float *)dA, K, q8, sc, N, mode, beta, (float *)dC, N, ws,
                            c->capW, c->stream), who);
    get_rows(c, C, dC, M, N, ldc, who);
    finish(c, who);
}

void p2_sgemm_q8b(int M, int N, int K, float alpha, const float *A, int lda, const signed char *B,
                  const float *scales, int ldb, float beta, float *C, int ldc)
{
    /* An int8 table has one plane: int8 and int8w are the same GEMM for it (csrc/blas.c:1243-1254). */
    int mode = gemm_mode() == P2CU_EXACT ? P2CU_EXACT : P2CU_INT8;
    run_q8b(M, N, K, alpha, A, lda, B, scales, ldb, beta, C, ldc, mode, "p2_sgemm_q8b");
}

signed char *p2_fv_pack_codes(const FiveValueB *b, int K, int N)
{
    const char *who = "p2_fv_pack_codes";
    if (K % 4 != 0 || N % 16 != 0 || K <= 0) return NULL;
    Ctx *c = ctx_get(who);
    signed char *host = (signed char *)malloc((size_t)K * N);
    if (!host) return NULL;
    pthread_mutex_lock(&g_reg_mu);
    Entry *e = five_entry(b, K, N, c, who);
    ensure_codes(e, c, who);
    check_cuda(cudaMemcpy(host, e->codes, (size_t)K * N, cudaMemcpyDeviceToHost), who);
    pthread_mutex_unlock(&g_reg_mu);
    return host;
}

/* ---- QuantA: the rows are kept as fp32 in pinned memory and quantised on the GPU inside the GEMM ---- */

int p2_quant_prepare(QuantA *qa, int M, int K)
{
    const char *who = "p2_quant_prepare";
    if (gemm_mode() == P2CU_EXACT || K % 4 != 0 || M <= 0 || K <= 0) return -1;
    Ctx *c = ctx_get(who);
    size_t need = (size_t)M * K * sizeof(float);
    if (need > c->capQ) {
        cudaFreeHost(c->hq);
        c->hq = NULL;
        c->capQ = 0;
        if (cudaMallocHost((void **)&c->hq, need) != cudaSuccess) return -1;
        c->capQ = need;
    }
    qa->q = (signed char *)c->hq;
    qa->scales = NULL;
    qa->M = M;
    qa->K = K;
    return 0;
}

void p2_quant_row(const QuantA *qa, int m, const float *row)
{
    memcpy((float *)qa->q + (size_t)m * qa->K, row, (size_t)qa->K * sizeof(float));
}

void p2_sgemm_fvb_q8a(int M, int N, int K, float alpha, const QuantA *A, const FiveValueB *B, float beta,
                      float *C, int ldc)
{
    if (!A || !A->q || A->K != K || A->M < M) die("p2_sgemm_fvb_q8a", "QuantA does not match the GEMM");
    run_fvb(M, N, K, alpha, (const float *)A->q, K, B, beta, C, ldc, "p2_sgemm_fvb_q8a");
}

void p2_sgemm_q8b_q8a(int M, int N, int K, float alpha, const QuantA *A, const signed char *B, const float *scales,
                      int ldb, float beta, float *C, int ldc)
{
    if (!A || !A->q || A->K != K || A->M < M) die("p2_sgemm_q8b_q8a", "QuantA does not match the GEMM");
    run_q8b(M, N, K, alpha, (const float *)A->q, K, B, scales, ldb, beta, C, ldc, P2CU_INT8, "p2_sgemm_q8b_q8a");
}
