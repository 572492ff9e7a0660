// model.h - a model's weights on the device (P2cuModel, filled by p2cu_model_upload in encoder.cu). Internal to the
// library: the encoder plans and the decoder read the same arena.
#pragma once
#include <cstddef>
#include <cstdint>
#include "p2cuda.h"

namespace p2cu {

// A GEMM weight on the device.
struct DWeight {
    int kind = -1;   // P2_W_FV, P2_W_I8, P2_W_F32
    int K = 0, N = 0;
    P2cuFiveValue fv{};
    const int8_t* q8 = nullptr;
    const float* scales = nullptr;
    const float* f32 = nullptr;
};

// One conformer block's tables.
struct DBlock {
    const float *n_ff1_w, *n_ff1_b, *n_sa_w, *n_sa_b, *n_conv_w, *n_conv_b, *n_ff2_w, *n_ff2_b, *n_out_w, *n_out_b;
    const float *bias_u, *bias_v, *dw_w, *dw_b;
    DWeight ff1a, ff1b, qkv, pos, out, pw1, pw2, ff2a, ff2b;
};

}  // namespace p2cu

struct P2cuModel {
    int device = 0;
    char* arena = nullptr;
    size_t bytes = 0;
    int codes = 0;
    const float *c0w, *c0b, *c2w, *c2b, *c3w, *c3b, *c5w, *c5b, *c6w, *c6b, *lin_b, *proj_b;
    p2cu::DWeight lin, proj;
    p2cu::DBlock blk[P2_N_BLOCKS];
    // the prediction and joint networks (fp32, csrc/phonon2.h:189-199); all null when the model has no decoder
    int has_dec = 0;
    const float *embed = nullptr, *wih[2] = {}, *whh[2] = {}, *bih[2] = {}, *bhh[2] = {};
    const float *dproj = nullptr, *dproj_b = nullptr, *head = nullptr, *head_b = nullptr;
};
