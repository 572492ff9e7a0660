/*  phonon2.h - the phonon-2-c types and constants this library's ABI uses, laid out exactly as phonon-2-c's own
 *  csrc/phonon2.h lays them out (v0.1.0), so that objects compiled against either header interoperate.
 *
 *  Only declarations this library implements live here (the weight and model structs, QuantA, the model
 *  constants, the encoder entry points). phonon-2-c's engine, audio front end, decoder and tokenizer keep their own
 *  header and sources; a build that links them with libphonon2_b200.so gets the GEMM layer and the encoder from the
 *  GPU.
 *  Each type cites the reference declaration it mirrors (csrc/phonon2.h line numbers).
 */
#ifndef PHONON2_H
#define PHONON2_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define P2_API __attribute__((visibility("default")))
#else
#define P2_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* The model's dimensions (csrc/phonon2.h:73-105). */
#define P2_D_MODEL      1024
#define P2_N_HEADS      8
#define P2_HEAD_DIM     128
#define P2_FF_DIM       4096
#define P2_N_BLOCKS     24
#define P2_CONV_KERNEL  9
#define P2_N_MELS       128
#define P2_SUB_CHANNELS 256
#define P2_SUB_FACTOR   8
#define P2_LSTM_HIDDEN  640
#define P2_LSTM_LAYERS  2
#define P2_EMBED_DIM    640
#define P2_JOINT_DIM    640
#define P2_VOCAB        8193
#define P2_BLANK        8192
#define P2_N_DURATIONS  5
#define P2_N_LOGITS     (P2_VOCAB + P2_N_DURATIONS)

/* Audio front end (csrc/phonon2.h:99-105) */
#define P2_SAMPLE_RATE  16000
#define P2_HOP_LEN      160
#define P2_FRAME_SECONDS ((float)(P2_SUB_FACTOR * P2_HOP_LEN) / (float)P2_SAMPLE_RATE)   /* 0.08 s per encoder frame */

/* A GEMM weight op(B) = [K, N] in one of three storage kinds (csrc/phonon2.h:109-126). */
typedef enum {
    P2_W_F32 = 0,   /* fp32 [K, N] */
    P2_W_I8  = 8,   /* int8 [K, N], one fp32 scale per column */
    P2_W_FV  = 5    /* five-value: per column n the values {0, +-lo[n], +-hi[n]} as sign and magnitude planes */
} P2WeightKind;

typedef struct {
    P2WeightKind kind;
    int K, N;
    const float         *f32;
    const signed char   *q8;
    const float         *scales;
    const unsigned char *signs;    /* [K][N/4], the 2-bit code (sign + 1) of column n at bits 2*(n & 3) */
    const unsigned char *flags;    /* [K][N/8], bit (n & 7) set when |w| = hi[n] */
    const float         *lo, *hi;  /* [N] */
    signed char         *codes;    /* optional pre-expanded int8w codes (p2_fv_pack_codes), else NULL */
} Weight;

/* csrc/phonon2.h:128-137: the 8x convolutional subsampling. */
typedef struct {
    const float *conv0_w, *conv0_b;   /* Conv2d 1 -> 256, 3x3, stride 2 */
    const float *conv2_w, *conv2_b;   /* depthwise 3x3, stride 2 */
    const float *conv3_w, *conv3_b;   /* pointwise 256 -> 256 */
    const float *conv5_w, *conv5_b;   /* depthwise 3x3, stride 2 */
    const float *conv6_w, *conv6_b;   /* pointwise 256 -> 256 */
    Weight       linear_w;            /* [4096, 1024] int8 table */
    const float *linear_b;
} SubsamplingWeights;

/* csrc/phonon2.h:139-142 */
typedef struct {
    Weight linear1_w;   /* [1024, 4096] */
    Weight linear2_w;   /* [4096, 1024] */
} FFWeights;

/* csrc/phonon2.h:144-150 */
typedef struct {
    Weight       qkv_w;    /* [1024, 3072]: Q | K | V */
    Weight       pos_w;    /* [1024, 1024] */
    Weight       out_w;    /* [1024, 1024] */
    const float *bias_u;   /* [8 x 128] */
    const float *bias_v;
} MHAWeights;

/* csrc/phonon2.h:152-157 */
typedef struct {
    Weight       pw1_w;    /* [1024, 2048], followed by a GLU */
    const float *dw_w;     /* [1024 x 9] depthwise, BatchNorm folded in */
    const float *dw_b;     /* [1024] */
    Weight       pw2_w;    /* [1024, 1024] */
} ConvModWeights;

/* csrc/phonon2.h:159-169 */
typedef struct {
    const float *norm_ff1_w, *norm_ff1_b;
    FFWeights    ff1;
    const float *norm_sa_w, *norm_sa_b;
    MHAWeights   mha;
    const float *norm_conv_w, *norm_conv_b;
    ConvModWeights conv;
    const float *norm_ff2_w, *norm_ff2_b;
    FFWeights    ff2;
    const float *norm_out_w, *norm_out_b;
} ConformerBlock;

/* csrc/phonon2.h:177-182 */
typedef struct {
    SubsamplingWeights subsampling;
    ConformerBlock     blocks[P2_N_BLOCKS];
    Weight             projector_w;   /* [1024, 640] int8 table */
    const float       *projector_b;
} EncoderWeights;

#define P2_DEC_OWNED 8

/* csrc/phonon2.h:189-199 */
typedef struct {
    const float *embed_w;
    const float *lstm_w_ih[P2_LSTM_LAYERS];
    const float *lstm_w_hh[P2_LSTM_LAYERS];
    const float *lstm_b_ih[P2_LSTM_LAYERS];
    const float *lstm_b_hh[P2_LSTM_LAYERS];
    const float *proj_w, *proj_b;
    const float *head_w, *head_b;
    float       *owned[P2_DEC_OWNED];
    int          n_owned;
} DecoderWeights;

/* csrc/phonon2.h:201-206 */
typedef struct {
    EncoderWeights enc;
    DecoderWeights dec;
    void          *map;
    size_t         map_len;
} P2Model;

/* csrc/phonon2.h:210-220 */
typedef struct {
    float h[P2_LSTM_LAYERS][P2_LSTM_HIDDEN];
    float c[P2_LSTM_LAYERS][P2_LSTM_HIDDEN];
} LSTMState;

typedef struct {
    int id;        /* token id, never blank */
    int frame;     /* encoder frame it was emitted at */
    int duration;  /* frames the decoder then advanced, 0..4 */
} P2Token;

/* Activations prepared for the int8 GEMMs (csrc/phonon2.h:432-436). In this build the rows given to p2_quant_row
 * are kept as fp32 in `q` (a buffer of the calling thread) and quantised on the GPU inside the GEMM, with the
 * reference's rounding; `scales` is NULL. Callers that only pass a QuantA from prepare to the GEMM see no
 * difference. */
typedef struct {
    signed char *q;
    float       *scales;
    int          M, K;
} QuantA;

/* Encoder progress on stderr in the reference (csrc/phonon2.h:224); this build prints nothing per block but keeps
 * the variable, which the reference's engine and CLI set. */
P2_API extern int p2_verbose;

/* The encoder, mel [n_frames x 128] -> projected frames [T' x 640], T' = three stride-2 halvings of n_frames; the
 * caller frees *out (csrc/phonon2.h:394-395). Runs on the GPU of the calling thread (p2_b200_set_device): the
 * model's weights are uploaded there on first use (found again by the P2Model's address) and the whole forward pass
 * runs as one CUDA graph. The mode is the GEMM layer's (P2_GEMM / P2_EXACT); beyond 500 frames of T' (or as P2_CHUNK
 * says) the sequence is encoded in chunks of P2_CHUNK_SIZE (400) frames with P2_CHUNK_OVERLAP (8) frames of context,
 * as the reference does. Returns 0, or -1 with a message on stderr. */
P2_API int p2_encoder(const P2Model *m, const float *mel, int n_frames, float **out, int *out_len);

/* The chunked encoder regardless of length (csrc/phonon2.h:397-398). Same contract. */
P2_API int p2_encoder_chunked(const P2Model *m, const float *mel, int n_frames, float **out, int *out_len);

/* The encoder over a batch of windows spread across GPUs. No counterpart in the reference, whose engine encodes the
 * windows of long audio one after another (csrc/engine.c:311-357). Window w has n_frames[w] mel frames; `mel` holds
 * the windows' frames one after another ([sum n_frames][128]) and `out` receives their encoder frames the same way
 * ([sum T'_w][640], T'_w three stride-2 halvings of n_frames[w]). The windows go to the `n_devices` GPUs listed
 * (all visible GPUs when n_devices is 0), longest first to the GPU with the fewest frames so far; each GPU encodes
 * its share as one batch from one host thread, with no collective. Results equal p2_encoder's window by window.
 * Each GPU keeps its last two plans (window sets) for reuse. Returns 0, or -1 with a message on stderr. */
P2_API int p2_b200_encode_windows(const P2Model *m, const float *mel, const int *n_frames, int n_windows,
                                  const int *devices, int n_devices, float *out);

/* The prediction network's step (csrc/phonon2.h:400-401, csrc/decoder.c:62-74): embedding row of token_id, two LSTM
 * layers updating *state, decoder projector into dec_out [640]. Host pointers; runs on the calling thread's GPU with
 * the model's decoder tables uploaded there on first use. */
P2_API void p2_decoder_step(const P2Model *m, int token_id, LSTMState *state, float *dec_out);

/* The joint network (csrc/phonon2.h:403-404, csrc/decoder.c:78-88): logits [8198] = head . relu(enc_t + dec_out) +
 * bias, 8193 token logits then 5 duration logits. Host pointers, calling thread's GPU. */
P2_API void p2_joint(const P2Model *m, const float *enc_t, const float *dec_out, float *logits);

/* Greedy TDT decoding of T encoder frames [T x 640] (csrc/phonon2.h:406-407, csrc/decoder.c:100-141): the whole
 * loop runs as one launch on the calling thread's GPU. *out_tokens is malloc'd (the caller frees it) and the token
 * count returned, or -1 with a message on stderr. */
P2_API int p2_greedy_decode(const P2Model *m, const float *enc_out, int T, P2Token **out_tokens);

/* Log-mel features of 16 kHz audio (csrc/phonon2.h:391-392, csrc/mel.c): n_samples / 160 frames of 128 normalised
 * log-mel values, computed on the calling thread's GPU; *out_mel is malloc'd (the caller frees it). Returns 0, or -1
 * with a message on stderr (fewer than 320 samples: "audio too short", as the reference). */
P2_API int p2_mel_spectrogram(const float *audio, int n_samples, float **out_mel, int *out_frames);

/* The whole path from audio: log-mel, encoder and greedy decoder per window on the device, windows spread across GPUs
 * as p2_b200_encode_windows spreads them. Window w has n_samples[w] samples (16 kHz), the windows one after another in
 * `audio`; tokens / n_tokens as p2_b200_transcribe_windows. No counterpart in the reference, whose engine runs
 * p2_mel_spectrogram, p2_encoder and p2_greedy_decode window after window (csrc/engine.c:256-292). */
P2_API int p2_b200_transcribe_audio_windows(const P2Model *m, const float *audio, const long long *n_samples,
                                            int n_windows, const int *devices, int n_devices, P2Token **tokens,
                                            int *n_tokens);

/* Encoder and greedy decoder over a batch of windows spread across GPUs, the encoder frames staying on the device. No
 * counterpart in the reference, whose engine runs p2_encoder then p2_greedy_decode window after window
 * (csrc/engine.c:100-125, 311-357). Windows, mel layout and GPU placement as p2_b200_encode_windows. tokens[w] receives
 * a malloc'd array of window w's tokens (NULL when it has none; the caller frees each) and n_tokens[w] their count.
 * Returns 0, or -1 with a message on stderr. */
P2_API int p2_b200_transcribe_windows(const P2Model *m, const float *mel, const int *n_frames, int n_windows,
                                      const int *devices, int n_devices, P2Token **tokens, int *n_tokens);

/* ---- Long audio (csrc/segment.c, csrc/engine.c:253-357) ----------------------------------------------------------- */

/* A window of samples [start, end) of long audio (csrc/phonon2.h:359). */
typedef struct { int start, end; } P2Window;

/* p2_plan_windows (csrc/phonon2.h:360-366) with the block RMS computed on the calling thread's GPU: audio longer than
 * the maximum window (35 s, or P2_WINDOW_MAX) cut at the longest pause of the 10 s before each maximum. 16 kHz audio
 * only. Returns the number of windows in the malloc'd *out (freed by the caller), 0 for no audio or on failure. */
P2_API int p2_b200_plan_windows(const float *audio, int n_samples, int sample_rate, P2Window **out);
/* p2_split_point (csrc/phonon2.h:367-368) likewise: the middle of the longest pause in the middle third. */
P2_API int p2_b200_split_point(const float *audio, int n_samples, int sample_rate);

/* p2_b200_transcribe_long, p2_b200_windows_free: phonon2_b200.h (included here; an edited engine.c that keeps the
 * reference's phonon2.h includes it after that header). */
#include "phonon2_b200.h"

#ifdef __cplusplus
}
#endif

#endif /* PHONON2_H */
