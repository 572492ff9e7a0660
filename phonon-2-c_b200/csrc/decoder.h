// decoder.h - the batched greedy TDT decoder kernel (decoder.cu). Internal to the library.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

// Tokens a window may emit at one frame before its pointer is forced on (csrc/phonon2.h:92); a window of T frames
// emits at most this many times T tokens.
#define P2CU_DEC_MAX_SYMBOLS 10

namespace p2cu {

// What a launch does: the whole greedy decode of every window; one prediction-network step on first_token from the
// given state (p2_decoder_step); or the joint logits of one frame (p2_joint).
enum : int { DEC_DECODE = 0, DEC_STEP = 1, DEC_JOINT = 2 };

// Everything one cooperative decode launch reads and writes (device pointers).
struct DecParams {
    int mode;              // DEC_*
    int first_token;       // the token of the first step (the blank for a decode)
    float* logits;         // DEC_JOINT: [8198] out
    // the prediction and joint networks, fp32 (csrc/phonon2.h:189-199)
    const float *embed, *wih0, *whh0, *bih0, *bhh0, *wih1, *whh1, *bih1, *bhh1, *proj, *projb, *head, *headb;
    const float* enc;      // [sum T][640] encoder frames of the windows, stacked
    const int* win_off;    // [B + 1] prefix frame offsets
    int B;
    int max_iters;         // a bound on loop iterations (11 T + 1 covers every window)
    // state: h and c zeroed by the host before a decode
    float* h;              // [2 sides][2 layers][B][640]
    float* c;              // [2 layers][B][640]
    float* dec;            // [B][640] decoder projector output
    float* cand;           // [2][grid][B] (value, row) token candidates of each CTA, double-buffered by iteration
    float* dur;            // [2][B][5] duration logits
    int* tokens;           // [10 sum T][3] per-window token lists, window b's at 10 win_off[b]
    // output
    int* tok_out;          // [sum of counts][3] id, frame, duration, window after window
    int* tok_off;          // [B + 1] prefix offsets into tok_out
    int* count;            // [B] tokens emitted
    // grid barrier's arrival count (zeroed by the host before each launch) and error word
    unsigned* bar_count;
    uint32_t* err;
};

int decoder_smem_bytes(int grid);
int decoder_max_windows();
int decoder_max_units();
int decoder_max_grid(int device);   // one CTA per SM when it fits, else 0
cudaError_t tdt_decode_launch(const DecParams& p, int grid, cudaStream_t s);

}  // namespace p2cu
