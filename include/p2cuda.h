/*  p2cuda.h - device-pointer entry points of the B200 five-value GEMM library (libphonon2_b200.so).
 *
 *  The reference-facing ABI is blas.h (the same names and arguments as phonon-2-c's csrc/blas.h, host pointers).
 *  This header is the layer beneath it: every pointer here is device memory, every call is asynchronous on the
 *  CUDA stream given (a cudaStream_t passed as void *, NULL = the legacy default stream), and nothing here
 *  allocates: scratch memory is passed in by the caller. All functions return P2CU_OK (0) or a negative P2CU_E*
 *  code, with a message in p2cu_last_error().
 *
 *  Layouts follow the reference's weight format (csrc/blas.h:38-45, csrc/phonon2.h:110-126):
 *    five-value B [K, N]: signs [K][N/4] (2-bit code sign+1 of column n at bits 2*(n&3)), flags [K][N/8]
 *                         (bit n&7 set -> |w| = hi[n]), lo / hi [N] fp32 holding fp16 values;
 *    int8 table B [K, N]: int8 rows of ldb bytes, one fp32 scale per column;
 *    A, C: fp32 row-major with leading dimensions lda / ldc (in elements).
 *  Quantised activations are row-major int8 [M][K] (K bytes per row) with one fp32 scale per row.
 */
#ifndef P2CUDA_H
#define P2CUDA_H

#include <stddef.h>
#include "phonon2.h"

#if defined(__GNUC__)
#define P2CU_API __attribute__((visibility("default")))
#else
#define P2CU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    P2CU_OK = 0,
    P2CU_EINVAL = -1,        /* a contract violation: shapes, alignment, NULL pointers */
    P2CU_ECUDA = -2,         /* a CUDA runtime / driver error */
    P2CU_EDEVICE = -3,       /* a kernel gave up waiting (bounded waits) and reported it */
    P2CU_EUNSUPPORTED = -4   /* a shape this build does not cover */
};

/* GEMM modes, numbered as the reference's internal enum (csrc/blas.c:1027): int8 = A quantised, two exact weight
 * planes; exact = fp32 expansion; int8w = A quantised, one int8 code plane. */
enum { P2CU_INT8 = 0, P2CU_EXACT = 1, P2CU_INT8W = 2 };

/* A five-value weight resident on the device. `codes` optionally points at the weight's int8w codes as a row-major
 * [K][N] int8 plane (p2cu_fv_pack_codes); with it the int8w GEMM streams the codes instead of expanding planes.
 * `vindex` optionally points at the weight's value-index plane (p2cu_fv_pack_vindex, 4 bits per weight); with it
 * int8w GEMMs of few rows (M up to about a thousand) expand the weights straight into tensor memory. */
typedef struct {
    const unsigned char *signs;
    const unsigned char *flags;
    const float         *lo;
    const float         *hi;
    const signed char   *codes;
    int                  K, N;
    const unsigned int  *vindex;
} P2cuFiveValue;

/* The message of the last failed call on this host thread ("" when none). */
P2CU_API const char *p2cu_last_error(void);

/* Synchronise `stream`, then read and clear the device's error word: P2CU_EDEVICE when a kernel reported a wait that
 * ran out, P2CU_ECUDA on a CUDA error, else P2CU_OK. */
P2CU_API int p2cu_check_device(void *stream);

/* The quantisation rule of every int8 path (p2cu_quant_rows, the int8 GEMM entry points, the encoder's quantising
 * row ops). 0 (the default): the reference's C source as written, IEEE division - scale = amax / 127,
 * 1 / scale, and x / scale in the scalar tail (csrc/blas.c:1114-1144). 1: the arithmetic of the reference as its
 * Makefile builds it (csrc/Makefile:2, -ffast-math), which that compiler derives from the same source:
 * scale = amax * (1/127), the reciprocal 127 / amax, x times it in the tail (a non-finite product there gives 0).
 * The environment variable P2CU_QUANT_FAST_MATH=1 selects 1 before the first call. Kernels follow the rule in force
 * when they are launched (a captured graph: when it was captured). p2cu_set_quant_fast_math returns the previous
 * rule. No counterpart in the reference, which has one rule per build. */
P2CU_API int p2cu_set_quant_fast_math(int on);
P2CU_API int p2cu_quant_fast_math(void);

/* Per-row int8 quantisation (csrc/blas.c:1114-1144): q [M][K] int8, scales [M]. */
P2CU_API int p2cu_quant_rows(const float *A, int M, int K, int lda, signed char *q, float *scales, void *stream);

/* C = alpha * A * B + beta * C on quantised A (csrc/blas.c:1430-1437). mode P2CU_INT8 or P2CU_INT8W. N % 16 == 0;
 * the tcgen05 kernels take N % 128 == 0, K % 16 == 0 and C 16-byte aligned with ldc % 4 == 0, other shapes a SIMT
 * kernel with the same arithmetic. beta: 0 stores, 1 accumulates, other values scale C first. When K > 1024 the GEMM
 * keeps one fp32 value per output and 1024-row block of K in `workspace` (p2cu_q8a_workspace_bytes; 0 otherwise)
 * and folds them into C in block order, as the reference's blockwise epilogue does. */
P2CU_API int p2cu_sgemm_fvb_q8a(int M, int N, int K, float alpha, const signed char *q, const float *a_scales,
                                const P2cuFiveValue *B, int mode, float beta, float *C, int ldc, void *workspace,
                                size_t workspace_bytes, void *stream);

/* The same with an int8 table B [K, N] (row stride ldb bytes) and one scale per column (csrc/blas.c:1439-1446). */
P2CU_API int p2cu_sgemm_q8b_q8a(int M, int N, int K, float alpha, const signed char *q, const float *a_scales,
                                const signed char *B, const float *scales, int ldb, float beta, float *C, int ldc,
                                void *workspace, size_t workspace_bytes, void *stream);

/* Workspace bytes of the q8a GEMMs (K-block slices when K > 1024, else 0). */
P2CU_API size_t p2cu_q8a_workspace_bytes(int M, int N, int K);

/* Workspace bytes of p2cu_sgemm_fvb / p2cu_sgemm_q8b: the quantised activations plus the K-block slices
 * (0 in exact mode, and when K % 4 != 0, which runs the exact path). */
P2CU_API size_t p2cu_gemm_workspace_bytes(int M, int N, int K, int mode);

/* C = alpha * A * B + beta * C from fp32 A (csrc/blas.c:1481-1499 / 1462-1479): in the int8 modes A is quantised
 * into `workspace` first (K % 4 != 0 takes the exact path instead, as in the reference); in P2CU_EXACT the weights
 * are expanded to fp32 and every output is the reference's FMA chain, bit for bit. */
P2CU_API int p2cu_sgemm_fvb(int M, int N, int K, float alpha, const float *A, int lda, const P2cuFiveValue *B, int mode,
                   float beta, float *C, int ldc, void *workspace, size_t workspace_bytes, void *stream);
P2CU_API int p2cu_sgemm_q8b(int M, int N, int K, float alpha, const float *A, int lda, const signed char *B,
                   const float *scales, int ldb, int mode, float beta, float *C, int ldc, void *workspace,
                   size_t workspace_bytes, void *stream);

/* fp32 C = alpha * op(A) * op(B) + beta * C (csrc/blas.c:748-763); trans flags 0 / 1. NN is the reference's FMA chain
 * bit for bit; the transposed forms run one sequential chain per output. */
P2CU_API int p2cu_sgemm(int transA, int transB, int M, int N, int K, float alpha, const float *A, int lda, const float *B,
               int ldb, float beta, float *C, int ldc, void *stream);

/* The int8w codes of B as a row-major [K][N] int8 plane (csrc/blas.c:1391-1400 values): codes has K * N bytes. */
P2CU_API int p2cu_fv_pack_codes(const P2cuFiveValue *B, signed char *codes, void *stream);

/* The value-index plane of B, a device-side form of the reference's sign and magnitude planes (csrc/blas.h:38-45,
 * written by convert_weights.py:114-125) for the small-M int8w GEMM: one 4-bit index per weight into the column's
 * int8w codes (0: zero, 1: +clo, 2: -clo, 3: +127, 4: -127, 5 and 6: the unused 2-bit code 3 with flag 0 / 1, which
 * the reference multiplies in as sign +2, csrc/blas.c:1197-1238), 32 consecutive K rows of one column in 16 bytes:
 * vindex[(kc * N + n) * 4 + v] holds rows 32 kc + 8 v + t of column n at bits 4 t .. 4 t + 3 (rows past K: 0).
 * vindex has p2cu_fv_vindex_bytes(K, N) = 16 * ceil(K / 32) * N bytes, 16-byte aligned. Set B->vindex to it
 * afterwards. No counterpart in the reference (its int8w path re-expands the planes per panel, csrc/blas.c:1224-1240,
 * or keeps an 8-bit code cache). */
P2CU_API size_t p2cu_fv_vindex_bytes(int K, int N);
P2CU_API int p2cu_fv_pack_vindex(const P2cuFiveValue *B, unsigned int *vindex, void *stream);

/* Bytes of the fixed device array behind p2cu_sgemm_fvb_noalloc (16 MiB), held on every device that loads the
 * library until the process exits. */
#define P2CU_NOALLOC_SCRATCH_BYTES (16u << 20)

/* p2cu_sgemm_fvb without a workspace argument, for callers that cannot allocate device memory: a real-time thread
 * (cudaMalloc may block and synchronise the device) or a host that grants a fixed memory budget. No counterpart in the reference (its GEMMs use per-thread host buffers).
 * The scratch - quantised activations and, for K > 1024, the per-block partials; p2cu_gemm_workspace_bytes(M, N, K,
 * mode) bytes - lives in one fixed array of P2CU_NOALLOC_SCRATCH_BYTES per device; larger shapes are refused with
 * P2CU_EINVAL and a message. This function calls no cudaMalloc, cudaFree or other allocating routine. Its first call
 * on a device looks up the array's device address (cudaGetSymbolAddress, that device current): make that first call
 * before any stream capture. Every call on a device shares the array, so calls whose kernels overlap on the GPU (on
 * different streams, or from different threads) race on it and must be serialised by the caller; nothing in it
 * needs to start at zero. The address looked up on the first call belongs to the device's context: after
 * cudaDeviceReset on a device, this entry point must not be called on that device again in the process. */
P2CU_API int p2cu_sgemm_fvb_noalloc(int M, int N, int K, float alpha, const float *A, int lda, const P2cuFiveValue *B,
                                    int mode, float beta, float *C, int ldc, void *stream);

/* ---- The encoder's row ops on device rows (the reference's ops ABI, csrc/phonon2.h:424-465) ----------------------
 * Every array is row-major fp32 [rows][features] in device memory; quantised rows are int8 [rows][features] with one
 * fp32 scale per row, as p2cu_quant_rows writes them. */

/* LayerNorm, eps 1e-5 (p2_layer_norm_rows, csrc/tensor_ops.c:204-303); out may be x (p2_layer_norm_rows_inplace). */
P2CU_API int p2cu_layer_norm_rows(const float *x, const float *gamma, const float *beta, float *out, int n_rows, int D,
                                  void *stream);
/* LayerNorm straight into quantised rows (p2_layer_norm_quant_rows, csrc/tensor_ops.c:329-350). */
P2CU_API int p2cu_layer_norm_quant_rows(const float *x, const float *gamma, const float *beta, signed char *q,
                                        float *scales, int n_rows, int D, void *stream);
/* x * sigmoid(x) in place (p2_swish, csrc/tensor_ops.c:436-490). */
P2CU_API int p2cu_swish(float *x, size_t n, void *stream);
/* SiLU of each row straight into quantised rows (p2_swish_quant_rows, csrc/tensor_ops.c:492-511). */
P2CU_API int p2cu_swish_quant_rows(const float *h, signed char *q, float *scales, int n_rows, int len, void *stream);
/* Softmax of each row in place (p2_softmax_rows, csrc/tensor_ops.c:354-428). */
P2CU_API int p2cu_softmax_rows(float *x, int n_rows, int len, void *stream);
/* Depthwise convolution over time with kernel 9 and padding 4 (p2_depthwise_conv1d with K = 9, csrc/tensor_ops.c:
 * 559-649), on time-major rows: x and out are [T][C], w is [C][9], b is [C] or NULL. */
P2CU_API int p2cu_depthwise_conv1d_rows(const float *x, const float *w, const float *b, float *out, int C, int T,
                                        void *stream);

/* C = A op(B) in fp32 on the tensor cores: A [M][K] (rows lda apart), op(B) = B^T with B [N][K] (transB != 0) or
 * B [K][N] (rows ldb apart), C [M][N] (rows ldc apart), overwritten. Each operand value is split into two tf32 parts
 * and three tcgen05 products are summed (hi*hi + hi*lo + lo*hi), which keeps fp32 accuracy (relative error about
 * 2^-21 per product); the summation order is the tensor core's, not one FMA chain. No counterpart in the reference,
 * which runs its fp32 attention products on the CPU (csrc/encoder.c:282-316); the encoder uses this kernel for them. */
P2CU_API int p2cu_sgemm_tf32x3(int transB, int M, int N, int K, const float *A, int lda, const float *B, int ldb,
                               float *C, int ldc, void *stream);

/* Relative-position self-attention of one encoder layer (self_attention's core, csrc/encoder.c:471-528) for n_win
 * windows on device rows, as the encoder runs it: qkv [R][3072] holds each window's Q | K | V rows (window w's T[w]
 * rows follow window w - 1's), P [2 Tmax - 1][1024] the projected positions of a window of Tmax frames (a window of
 * T frames uses rows Tmax - T .. Tmax + T - 2), bias_u and bias_v [1024]. attn [R][1024] receives, per head h and
 * window, softmax(((Q_h + bias_u) K_h^T + shift((Q_h + bias_v) P_h^T)) / sqrt(128)) V_h, the heads concatenated
 * (csrc/encoder.c:425-447 for the shift). T: the windows' lengths in host memory, each <= Tmax <= 512. One kernel on
 * the tensor cores, the products in the three-part tf32 split (fp32 accuracy, the summation order the tensor core's),
 * the scores never in device memory. ws: device scratch of p2cu_rel_attention_ws_bytes(n_win, T) bytes, 16-byte
 * aligned; every pointer 16-byte aligned. */
P2CU_API size_t p2cu_rel_attention_ws_bytes(int n_win, const int *T);
P2CU_API int p2cu_rel_attention(const float *qkv, const float *P, const float *bias_u, const float *bias_v,
                                const int *T, int n_win, int Tmax, float *attn, void *ws, size_t ws_bytes,
                                void *stream);

/* ---- The encoder on the device (csrc/encoder.c) ------------------------------------------------------------------
 * Unlike the calls above these allocate device memory, once: p2cu_model_upload copies a model's weights to the
 * current device, p2cu_encoder_create makes a plan with every buffer of one batch of windows and captures its forward
 * pass in a CUDA graph; p2cu_encoder_run then launches that graph and allocates nothing. */
typedef struct P2cuModel P2cuModel;
typedef struct P2cuEncoder P2cuEncoder;

/* Copy the encoder weights of `m` (host pointers, as phonon-2-c's loader maps them) into one allocation on the current
 * device, and the decoder's fp32 tables too when m->dec.embed_w is set. codes != 0 also builds the int8w code plane of every five-value weight there (the reference's
 * P2_CACHE_CODES, K * N bytes each), which the int8w GEMMs then stream instead of expanding the planes. */
P2CU_API int p2cu_model_upload(const P2Model *m, int codes, P2cuModel **out);
P2CU_API void p2cu_model_free(P2cuModel *m);
P2CU_API size_t p2cu_model_bytes(const P2cuModel *m);

/* A plan for `n_windows` windows of n_frames[w] mel frames each, in mode P2CU_INT8, P2CU_INT8W or P2CU_EXACT, on the
 * model's device. chunk_frames > 0 encodes each window's frames in chunks of that many frames with chunk_overlap
 * frames of context on each side (p2_encoder_chunked); 0 encodes every window in one pass. */
P2CU_API int p2cu_encoder_create(const P2cuModel *m, const int *n_frames, int n_windows, int mode, int chunk_frames,
                                 int chunk_overlap, P2cuEncoder **out);
P2CU_API void p2cu_encoder_destroy(P2cuEncoder *e);
/* Encoder frames of window w (three stride-2 halvings of its mel frames), or of all windows together for w < 0. */
P2CU_API int p2cu_encoder_frames(const P2cuEncoder *e, int window);
/* The plan's input: the windows' mel frames stacked, [sum n_frames][128] fp32, written by the caller before a run. */
P2CU_API float *p2cu_encoder_mel(P2cuEncoder *e);
/* The plan's output: the windows' encoder frames stacked, [sum frames][640] fp32, valid after a run completes. */
P2CU_API float *p2cu_encoder_out(P2cuEncoder *e);
/* One forward pass over the plan's input on `stream` (one graph launch). Runs on one plan must not overlap. */
P2CU_API int p2cu_encoder_run(P2cuEncoder *e, void *stream);

/* ---- The greedy TDT decoder on the device (csrc/decoder.c) ------------------------------------------------------
 * p2cu_decoder_create allocates the state and token buffers of up to max_windows windows (at most 512) of up to
 * max_frames encoder frames together; the calls after it allocate nothing. The model must have been uploaded with its
 * decoder tables. The decoder's kernel is one cooperative launch with one CTA on each SM. */
typedef struct P2cuDecoder P2cuDecoder;
P2CU_API int p2cu_decoder_create(const P2cuModel *m, int max_windows, int max_frames, P2cuDecoder **out);
P2CU_API void p2cu_decoder_destroy(P2cuDecoder *d);
/* Greedy decoding (csrc/decoder.c:100-141) of n_windows windows whose encoder frames are stacked in `enc` (device,
 * [sum n_frames][640], 16-byte aligned); n_frames is a host array. Asynchronous on `stream`. */
P2CU_API int p2cu_decode(P2cuDecoder *d, const float *enc, const int *n_frames, int n_windows, void *stream);
/* After p2cu_decode: synchronises `stream`, writes offsets[0..n_windows] (window w's tokens are
 * [offsets[w], offsets[w + 1]) of the decode's list) and copies the first min(cap, total) tokens into `tokens`.
 * Returns the total token count, or a negative P2CU_E* code. */
P2CU_API int p2cu_decoder_read(P2cuDecoder *d, int *offsets, P2Token *tokens, int cap, void *stream);
/* The same lists on the device: tokens as [total][3] ints (id, frame, duration), offsets [n_windows + 1]. */
P2CU_API const int *p2cu_decoder_tokens(const P2cuDecoder *d);
P2CU_API const int *p2cu_decoder_offsets(const P2cuDecoder *d);
/* One prediction-network step (csrc/decoder.c:62-74) on device pointers: state is an LSTMState (h[2][640] then
 * c[2][640]) updated in place, dec_out [640]. Asynchronous on `stream`. */
P2CU_API int p2cu_decoder_step(P2cuDecoder *d, int token_id, float *state, float *dec_out, void *stream);
/* The joint network (csrc/decoder.c:78-88) on device pointers: logits [8198]. Asynchronous on `stream`. */
P2CU_API int p2cu_joint(P2cuDecoder *d, const float *enc_t, const float *dec_out, float *logits, void *stream);

/* ---- The log-mel front end on the device (csrc/mel.c) ---------------------------------------------------------------
 * p2cu_mel_create allocates the plan's tables for up to max_windows windows of max_samples samples together; runs
 * allocate nothing. p2cu_mel_run computes, for each window of n_samples[w] samples (16 kHz, host array) stacked in
 * `audio` (device), n_samples[w] / 160 frames of normalised log-mel features into `mel` (device, [sum frames][128],
 * windows stacked) on `stream`; it waits for its small host-to-device table copies before returning. A window needs at
 * least 320 samples (two frames), as in the reference. */
typedef struct P2cuMel P2cuMel;
P2CU_API int p2cu_mel_create(int max_windows, long long max_samples, P2cuMel **out);
P2CU_API void p2cu_mel_destroy(P2cuMel *plan);
P2CU_API int p2cu_mel_frames(long long n_samples);
P2CU_API int p2cu_mel_run(P2cuMel *plan, const float *audio, const long long *n_samples, int n_windows, float *mel,
                          void *stream);

/* ---- The segmenter's energy measures (csrc/segment.c) --------------------------------------------------------------
 * p2cu_block_rms: for each window w of device `audio` ([starts[w], starts[w] + lens[w]); host arrays), the RMS of
 * its blocks of 50 ms aligned to its start, the last one zero-padded (csrc/segment.c:36-48), into `rms` (device), the
 * windows' ceil(lens[w] / block) values one after another. Asynchronous on `stream`.
 * The p2cu_seg_* functions are host code: the decisions csrc/segment.c and csrc/engine.c:213-251 take from block RMS
 * values (`rms`, n_blocks of them, over n_samples samples), restated exactly. */
P2CU_API int p2cu_block_rms(const float *audio, const long long *starts, const int *lens, int n_windows,
                            int sample_rate, float *rms, void *stream);
P2CU_API int p2cu_seg_block(int sample_rate);
P2CU_API int p2cu_seg_blocks(int n_samples, int sample_rate);
P2CU_API int p2cu_seg_window_max_samples(int sample_rate);
/* p2_first_cut (csrc/segment.c:90-118): rms covers the first window-max samples. */
P2CU_API int p2cu_seg_first_cut(const float *rms, int n_blocks, int n_samples, int sample_rate);
/* p2_split_point (csrc/segment.c:142-151): rms covers the window. */
P2CU_API int p2cu_seg_split_point(const float *rms, int n_blocks, int n_samples, int sample_rate);
P2CU_API float p2cu_seg_speech_gate(const float *rms, int n_blocks);
P2CU_API float p2cu_seg_speech_share(const float *rms, int n_blocks, int sample_rate, int from, int to, float gate);
/* Whether a decoded window has a stretch of 2 s or more without a token (no RMS needed), and the full dropout test
 * of csrc/engine.c:224-251 at 16 kHz (the first quiet stretch's samples and speech share to the optional outputs). */
P2CU_API int p2cu_seg_long_gap(const P2Token *toks, int n_toks, int n_samples);
P2CU_API int p2cu_seg_dropped_out(const float *rms, int n_blocks, int n_samples, const P2Token *toks, int n_toks,
                                  int *gap_from, int *gap_to, float *speech);

/* p2cu_probe_wait_timeout: the kernels' bounded-wait path, exercised without a fault - one warp waits on an mbarrier
 * phase that nothing completes, gives up after `limit` polls (1 .. 2^20), records code 1 in the device error word and
 * returns; `seconds` is the launch's duration. Returns what p2cu_check_device then returns: P2CU_EDEVICE (the word is
 * cleared, the context stays usable). No counterpart in the reference (its CPU loops have no waits to bound). */
P2CU_API int p2cu_probe_wait_timeout(unsigned limit, double *seconds);

#ifdef __cplusplus
}
#endif

#endif /* P2CUDA_H */
