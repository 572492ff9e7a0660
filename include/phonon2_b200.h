/* phonon2_b200.h - the batched long-audio entry points of libphonon2_b200, in a header of their own so that the
 * reference's engine, edited to call them and still compiled against the reference's own phonon2.h
 * (phonon-2-c_b200/integration/engine_gpu_windows.patch), can include it after that header. include/phonon2.h includes
 * it too. Needs P2Model and P2Token from phonon2.h (either one) first. No counterpart in the reference, whose engine
 * decodes a recording's windows one after another (csrc/engine.c:331-353). */
#ifndef PHONON2_B200_H
#define PHONON2_B200_H

#ifndef P2_API
#if defined(__GNUC__)
#define P2_API __attribute__((visibility("default")))
#else
#define P2_API
#endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* One decoded window of p2_b200_transcribe_long. */
typedef struct {
    int      start, end;      /* samples [start, end) of the audio given */
    int      depth;           /* re-decode splits that made it: 0 for a planned window */
    int      encoder_frames;  /* its encoder frames (80 ms each) */
    P2Token *tokens;          /* its tokens, frames relative to `start` (malloc'd; NULL when n_tokens is 0) */
    int      n_tokens;
} P2B200Window;

/* Long 16 kHz audio as p2_transcribe decodes it (csrc/engine.c:293-357) - pause-aligned windows over 35 s, a window
 * that went quiet over speech re-decoded as two halves, at most two levels deep; P2_SEGMENT, P2_REDECODE and
 * P2_WINDOW_MAX keep their meaning - with each split depth's windows decoded as one batch spread over the GPUs
 * (`devices`, or all GPUs when n_devices is 0). Non-finite samples count as zeros. *out receives the final windows in
 * the order the reference appends them as segments (by start), freed with p2_b200_windows_free; *encoder_frames (if
 * not NULL) the encoder frames of every decode, split windows included (P2Result.encoder_frames). Returns 0, or -1
 * with a message on stderr. */
P2_API int p2_b200_transcribe_long(const P2Model *m, const float *audio, int n_samples, const int *devices,
                                   int n_devices, P2B200Window **out, int *n_out, long long *encoder_frames);
P2_API void p2_b200_windows_free(P2B200Window *windows, int n);

#ifdef __cplusplus
}
#endif

#endif /* PHONON2_B200_H */
