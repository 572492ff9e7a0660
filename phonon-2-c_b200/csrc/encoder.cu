// encoder.cu - the FastConformer encoder on the device (csrc/encoder.c of phonon-2-c, run without host round trips).
//
// A P2cuModel is the reference's P2Model (host pointers, as weights.c maps them) copied once into one device arena.
// A P2cuEncoder is a plan for one batch of windows: the windows' mel frames are stacked along the rows, every GEMM
// runs once over all windows' rows (M = sum of frames), and the ops that look across rows (the subsampling
// convolutions, attention, the depthwise convolution) stop at window edges. All buffers are allocated when the plan
// is made; the forward pass (subsampling, 24 conformer blocks, projector) is captured once into a CUDA graph and
// each run is one graph launch.
//
// The sequence of operations and their arithmetic follow the reference per mode (csrc/encoder.c:184-225, 319-624,
// 725-751): in the int8 modes the normalised and activated rows are quantised as they are produced and the
// residuals are added in the GEMM epilogues (β = 1); in exact mode every GEMM is the fp32 FMA chain and the
// residuals are separate axpys, here fused into the exact GEMM's epilogue with the same rounding.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>
#include <cuda_runtime.h>
#include "p2cuda.h"
#include "gemm.h"
#include "encoder_ops.h"
#include "attn_tc.h"
#include "kernels.h"
#include "fv_gemm.h"
#include "model.h"

namespace {

using p2cu::fail_fmt;

constexpr int D = P2_D_MODEL, H = P2_N_HEADS, DH = P2_HEAD_DIM, FF = P2_FF_DIM, NB = P2_N_BLOCKS;
constexpr int SUBC = P2_SUB_CHANNELS, NMEL = P2_N_MELS;

int conv_out(int n) { return (n + 2 - 3) / 2 + 1; }   // csrc/encoder.c:174

using p2cu::DWeight;
using p2cu::DBlock;

}  // namespace

namespace {

// Collects host arrays, lays them out 256-byte aligned in one arena and copies them.
struct Uploader {
    struct Item { const void* host; size_t bytes; const void** slot; size_t off; };
    std::vector<Item> items;
    size_t total = 0;
    int bad = 0;
    char what[160] = "";

    void add(const void* host, size_t bytes, const void** slot, const char* name) {
        if (!host) {
            if (!bad) snprintf(what, sizeof(what), "%s is NULL", name);
            bad = 1;
            return;
        }
        items.push_back({host, bytes, slot, total});
        total += (bytes + 255) & ~size_t(255);
    }
    void f32(const float* h, size_t n, const float** slot, const char* name) {
        add(h, n * sizeof(float), reinterpret_cast<const void**>(slot), name);
    }
    void weight(const Weight& w, int K, int N, DWeight* d, const char* name) {
        if (w.K != K || w.N != N) {
            if (!bad) snprintf(what, sizeof(what), "%s is [%d, %d], [%d, %d] expected", name, w.K, w.N, K, N);
            bad = 1;
            return;
        }
        d->kind = w.kind; d->K = K; d->N = N;
        const size_t kn = static_cast<size_t>(K) * N;
        switch (w.kind) {
        case P2_W_FV:
            d->fv.K = K; d->fv.N = N;
            add(w.signs, kn / 4, reinterpret_cast<const void**>(&d->fv.signs), name);
            add(w.flags, kn / 8, reinterpret_cast<const void**>(&d->fv.flags), name);
            add(w.lo, N * sizeof(float), reinterpret_cast<const void**>(&d->fv.lo), name);
            add(w.hi, N * sizeof(float), reinterpret_cast<const void**>(&d->fv.hi), name);
            break;
        case P2_W_I8:
            add(w.q8, kn, reinterpret_cast<const void**>(&d->q8), name);
            add(w.scales, N * sizeof(float), reinterpret_cast<const void**>(&d->scales), name);
            break;
        case P2_W_F32:
            add(w.f32, kn * sizeof(float), reinterpret_cast<const void**>(&d->f32), name);
            break;
        default:
            if (!bad) snprintf(what, sizeof(what), "%s has weight kind %d", name, static_cast<int>(w.kind));
            bad = 1;
        }
    }
};

int upload_model(const P2Model* m, int codes, P2cuModel** out) {
    if (!m || !out) return fail_fmt(P2CU_EINVAL, "p2cu_model_upload: NULL argument");
    auto* d = new P2cuModel();
    cudaGetDevice(&d->device);
    Uploader u;
    const SubsamplingWeights& s = m->enc.subsampling;
    u.f32(s.conv0_w, SUBC * 9, &d->c0w, "subsampling.conv.0.weight");
    u.f32(s.conv0_b, SUBC, &d->c0b, "subsampling.conv.0.bias");
    u.f32(s.conv2_w, SUBC * 9, &d->c2w, "subsampling.conv.2.weight");
    u.f32(s.conv2_b, SUBC, &d->c2b, "subsampling.conv.2.bias");
    u.f32(s.conv3_w, SUBC * SUBC, &d->c3w, "subsampling.conv.3.weight");
    u.f32(s.conv3_b, SUBC, &d->c3b, "subsampling.conv.3.bias");
    u.f32(s.conv5_w, SUBC * 9, &d->c5w, "subsampling.conv.5.weight");
    u.f32(s.conv5_b, SUBC, &d->c5b, "subsampling.conv.5.bias");
    u.f32(s.conv6_w, SUBC * SUBC, &d->c6w, "subsampling.conv.6.weight");
    u.f32(s.conv6_b, SUBC, &d->c6b, "subsampling.conv.6.bias");
    u.weight(s.linear_w, SUBC * (NMEL / P2_SUB_FACTOR), D, &d->lin, "subsampling.linear.weight");
    u.f32(s.linear_b, D, &d->lin_b, "subsampling.linear.bias");
    for (int i = 0; i < NB; ++i) {
        const ConformerBlock& b = m->enc.blocks[i];
        DBlock& o = d->blk[i];
        char name[96];
#define BF(field, src, n) snprintf(name, sizeof(name), "layers.%d." #src, i); u.f32(b.src, n, &o.field, name)
#define BW(field, src, K, N) snprintf(name, sizeof(name), "layers.%d." #src, i); u.weight(b.src, K, N, &o.field, name)
        BF(n_ff1_w, norm_ff1_w, D); BF(n_ff1_b, norm_ff1_b, D);
        BW(ff1a, ff1.linear1_w, D, FF); BW(ff1b, ff1.linear2_w, FF, D);
        BF(n_sa_w, norm_sa_w, D); BF(n_sa_b, norm_sa_b, D);
        BW(qkv, mha.qkv_w, D, 3 * D); BW(pos, mha.pos_w, D, D); BW(out, mha.out_w, D, D);
        BF(bias_u, mha.bias_u, D); BF(bias_v, mha.bias_v, D);
        BF(n_conv_w, norm_conv_w, D); BF(n_conv_b, norm_conv_b, D);
        BW(pw1, conv.pw1_w, D, 2 * D); BF(dw_w, conv.dw_w, D * P2_CONV_KERNEL); BF(dw_b, conv.dw_b, D);
        BW(pw2, conv.pw2_w, D, D);
        BF(n_ff2_w, norm_ff2_w, D); BF(n_ff2_b, norm_ff2_b, D);
        BW(ff2a, ff2.linear1_w, D, FF); BW(ff2b, ff2.linear2_w, FF, D);
        BF(n_out_w, norm_out_w, D); BF(n_out_b, norm_out_b, D);
#undef BF
#undef BW
    }
    u.weight(m->enc.projector_w, D, P2_JOINT_DIM, &d->proj, "encoder_projector.weight");
    u.f32(m->enc.projector_b, P2_JOINT_DIM, &d->proj_b, "encoder_projector.bias");
    const DecoderWeights& dw = m->dec;
    if (dw.embed_w) {   // a model without decoder tables uploads the encoder alone
        constexpr size_t HID = P2_LSTM_HIDDEN, G4 = 4 * HID;
        d->has_dec = 1;
        u.f32(dw.embed_w, static_cast<size_t>(P2_VOCAB) * P2_EMBED_DIM, &d->embed, "decoder.embedding");
        for (int l = 0; l < 2; ++l) {
            u.f32(dw.lstm_w_ih[l], G4 * (l ? HID : P2_EMBED_DIM), &d->wih[l], "decoder.lstm.weight_ih");
            u.f32(dw.lstm_w_hh[l], G4 * HID, &d->whh[l], "decoder.lstm.weight_hh");
            u.f32(dw.lstm_b_ih[l], G4, &d->bih[l], "decoder.lstm.bias_ih");
            u.f32(dw.lstm_b_hh[l], G4, &d->bhh[l], "decoder.lstm.bias_hh");
        }
        u.f32(dw.proj_w, static_cast<size_t>(P2_JOINT_DIM) * HID, &d->dproj, "decoder_projector.weight");
        u.f32(dw.proj_b, P2_JOINT_DIM, &d->dproj_b, "decoder_projector.bias");
        u.f32(dw.head_w, static_cast<size_t>(P2_N_LOGITS) * P2_JOINT_DIM, &d->head, "joint.head.weight");
        u.f32(dw.head_b, P2_N_LOGITS, &d->head_b, "joint.head.bias");
    }
    if (u.bad) {
        delete d;
        return fail_fmt(P2CU_EINVAL, "p2cu_model_upload: %s", u.what);
    }
    // Every five-value weight also gets its value-index plane (p2cu_fv_pack_vindex, 4 bits per weight: the int8w GEMMs
    // of one window read it), and with `codes` the int8w code plane (the reference's P2_CACHE_CODES,
    // csrc/weights.c:381-395: K x N bytes).
    size_t codes_bytes = 0, vindex_bytes = 0;
    std::vector<DWeight*> fvs;
    for (int i = 0; i < NB; ++i) {
        DBlock& o = d->blk[i];
        for (DWeight* w : {&o.ff1a, &o.ff1b, &o.qkv, &o.pos, &o.out, &o.pw1, &o.pw2, &o.ff2a, &o.ff2b})
            if (w->kind == P2_W_FV) {
                fvs.push_back(w);
                vindex_bytes += (p2cu_fv_vindex_bytes(w->K, w->N) + 255) & ~size_t(255);
                if (codes) codes_bytes += (static_cast<size_t>(w->K) * w->N + 255) & ~size_t(255);
            }
    }
    cudaError_t e = cudaMalloc(&d->arena, u.total + vindex_bytes + codes_bytes);
    if (e != cudaSuccess) {
        delete d;
        return p2cu::cuda_error(e, "p2cu_model_upload: cudaMalloc");
    }
    d->bytes = u.total + vindex_bytes + codes_bytes;
    for (const auto& it : u.items) {
        e = cudaMemcpy(d->arena + it.off, it.host, it.bytes, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) break;
        *it.slot = d->arena + it.off;
    }
    if (e == cudaSuccess) {
        size_t off = u.total;
        for (DWeight* w : fvs) {
            uint32_t* vi = reinterpret_cast<uint32_t*>(d->arena + off);
            e = p2cu::fv_vindex_launch(w->fv.signs, w->fv.flags, w->K, w->N, vi, 0);
            if (e != cudaSuccess) break;
            w->fv.vindex = vi;
            off += (p2cu_fv_vindex_bytes(w->K, w->N) + 255) & ~size_t(255);
        }
        for (DWeight* w : fvs) {
            if (!codes || e != cudaSuccess) break;
            int8_t* c = reinterpret_cast<int8_t*>(d->arena + off);
            e = p2cu::fv_codes_launch(w->fv.signs, w->fv.flags, w->fv.lo, w->fv.hi, w->K, w->N, c, 0);
            if (e != cudaSuccess) break;
            w->fv.codes = reinterpret_cast<const signed char*>(c);
            off += (static_cast<size_t>(w->K) * w->N + 255) & ~size_t(255);
        }
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        d->codes = codes ? 1 : 0;
    }
    if (e != cudaSuccess) {
        cudaFree(d->arena);
        delete d;
        return p2cu::cuda_error(e, "p2cu_model_upload: copy");
    }
    *out = d;
    return P2CU_OK;
}

}  // namespace

struct P2cuEncoder {
    const P2cuModel* m = nullptr;
    int device = 0, mode = P2CU_INT8W;
    // Subsampling level: one entry per mel window (prefix offsets have n_mel_win + 1 entries).
    int n_mel_win = 0;
    std::vector<int> n_mel, Tp, mel_off, h1_off, h2_off, sub_off;
    // Block level: the windows the conformer blocks see - the mel windows themselves, or their chunks when the plan
    // chunks long windows (csrc/encoder.c:663-710).
    int n_win = 0;
    std::vector<int> T, row_off;
    bool chunked = false;
    int mel_rows = 0, rows1 = 0, rows2 = 0, R_sub = 0, R = 0, Tmax = 0, L = 0;
    long long s_total = 0, b_total = 0, vt_total = 0;
    int srows = 0;
    float scale = 0.f;

    char* arena = nullptr;
    // device buffers
    float *mel, *s1, *s2dw, *s2, *s3dw, *s3, *flat, *x_sub, *x, *big, *lnbuf, *gated, *attn, *pe, *P, *s_ac, *s_bd,
        *vt, *out;
    int8_t *q, *pe_q;
    float *qs, *pe_s;
    void* ws = nullptr;
    size_t ws_bytes = 0;
    int *d_mel_off, *d_h1_off, *d_h2_off, *d_sub_off, *d_row_off, *d_srow_off, *d_T, *d_gather, *d_scatter;
    long long *d_s_off, *d_b_off, *d_vt_off;
    p2cu::GemmGroup *g_ac, *g_bd, *g_av;
    int ng = 0, t_ac = 0, t_bd = 0, t_av = 0;
    int2* att_tiles = nullptr;   // fused SIMT attention (windows <= ATT_MAXT frames): (window, first query) per tile
    int n_att_tiles = 0;
    p2cu::AttnTile* tc_tiles = nullptr;   // fused tensor-core attention: the launch's tiles (attn_rel_tc_plan)
    int n_tc_tiles = 0;
    void* att_parts = nullptr;            // its split parts and merge counters, when a tile's keys are split
    int* att_counters = nullptr;
    // Attention path: 3 = one tensor-core kernel per layer, scores in TMEM (windows of at most ATT_MAXT frames; the
    // default), 0 = tensor-core products as grouped split-tf32 GEMMs with the scores in HBM (the default for longer
    // windows), 1 = SIMT grouped GEMMs, 2 = SIMT fused kernel (short windows). P2CU_ATTN=tc_fused|tc|simt|fused.
    int attn_path = 0;
    // The K blocks of the last int8 GEMM into x still to be folded (its workspace slices): the LayerNorm that reads
    // x next folds them in the same launch. No GEMM runs while one is pending (it would reuse the workspace).
    p2cu::KFold pending;
    p2cu::TcGroup *tc_scores = nullptr, *tc_context = nullptr;
    int n_tc = 0, t_tc_scores = 0, t_tc_context = 0;

    cudaStream_t stream = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    // A lazy plan runs its first pass eagerly on the caller's stream and is captured into a graph on its second run:
    // window sets that are seen once (each split depth of long audio, each length of the reference engine's
    // window-by-window calls) then cost one pass instead of an eager check pass, a capture and the run.
    bool lazy = false;
    bool capture_failed = false;
    int eager_runs = 0;
};

namespace {

// p2_wmatmul (csrc/tensor_ops.c:30-46) on fp32 rows A: C = alpha * A @ W + beta * C.
int wmatmul(P2cuEncoder& e, const float* A, int M, const DWeight& W, float* C, float alpha, float beta,
            const p2cu::Epilogue* epi, cudaStream_t s, const char* who) {
    const int K = W.K, N = W.N;
    if (W.kind == P2_W_F32 || e.mode == P2CU_EXACT)
        return p2cu::gemm_exact(M, N, K, alpha, A, K, 0, W.kind == P2_W_FV ? &W.fv : nullptr, W.q8, W.scales, W.f32,
                                N, 0, beta, C, N, epi, s, who);
    if (epi) return fail_fmt(P2CU_EINVAL, "%s: epilogue on the int8 path", who);
    cudaError_t ce = p2cu::quant_rows_launch(A, M, K, K, e.q, e.qs, s);
    if (ce != cudaSuccess) return p2cu::cuda_error(ce, who);
    return p2cu::gemm_i8(M, N, K, alpha, e.q, e.qs, W.kind == P2_W_FV ? &W.fv : nullptr, W.q8, W.scales, N,
                         W.kind == P2_W_FV ? e.mode : P2CU_INT8, beta, C, N, e.ws, e.ws_bytes, s, who);
}

// p2_wmatmul_q8a (csrc/tensor_ops.c:48-63) on rows already quantised into e.q / e.qs.
// defer: leave the K-block fold of a K > 1024 product into C (beta 1) to the next LayerNorm (e.pending).
int wmatmul_q8a(P2cuEncoder& e, int M, const DWeight& W, float* C, float alpha, float beta, cudaStream_t s,
                const char* who, bool defer = false) {
    if (W.kind == P2_W_F32) return fail_fmt(P2CU_EINVAL, "%s: fp32 weight has no int8 path", who);
    if (e.pending.nblk) return fail_fmt(P2CU_EINVAL, "%s: a K-block fold is still pending", who);
    return p2cu::gemm_i8(M, W.N, W.K, alpha, e.q, e.qs, W.kind == P2_W_FV ? &W.fv : nullptr, W.q8, W.scales, W.N,
                         W.kind == P2_W_FV ? e.mode : P2CU_INT8, beta, C, W.N, e.ws, e.ws_bytes, s, who,
                         defer ? &e.pending : nullptr);
}

// The pending fold for the LayerNorm about to read x, and no fold pending after it.
const p2cu::KFold* take_fold(P2cuEncoder& e, p2cu::KFold& hold) {
    hold = e.pending;
    e.pending.nblk = 0;
    return &hold;
}

#define TRY(x) do { int rc_ = (x); if (rc_ != P2CU_OK) return rc_; } while (0)
#define TRYC(x, what) do { cudaError_t ce_ = (x); if (ce_ != cudaSuccess) return p2cu::cuda_error(ce_, what); } while (0)

// A 1x1 convolution over channel rows (csrc/encoder.c:192-196, 203-208): out[m] = relu(W in[m] + b), W [256 out][256
// in], on the tensor cores with the split-tf32 products of the attention (fp32 accuracy; the reference's fp32 FMA
// chain differs by an ulp or two).
int conv1x1_tc(const float* in, int rows, const float* w, const float* b, float* out, cudaStream_t s,
               const char* what) {
    p2cu::TcArgs a{};
    a.src[0] = in; a.src[1] = w;
    a.dst[0] = out; a.dst[1] = out;
    a.err = p2cu::device_error_word();
    a.out_bias = b;
    a.out_relu = 1;
    p2cu::TcGroup& g = a.single;
    g.M = rows; g.N = SUBC; g.K = SUBC; g.tile0 = 0;
    g.a_src = 0; g.b_src = 1; g.c_dst = 0; g.lda = SUBC; g.ldb = SUBC; g.ldc = SUBC; g.bias_sel = -1;
    TRYC(p2cu::attn_tc_launch(nullptr, 0, p2cu::tc_gemm_tiles(rows, SUBC), a, false, s), what);
    return P2CU_OK;
}

// csrc/encoder.c:184-225: three stride-2 convolutions, flatten, linear 4096 -> 1024 + bias.
int subsampling(P2cuEncoder& e, cudaStream_t s) {
    const P2cuModel& m = *e.m;
    const int W1 = conv_out(NMEL), W2 = conv_out(W1), W3 = conv_out(W2);
    const int nw = e.n_mel_win;
    TRYC(p2cu::sub_conv0_dw_launch(e.mel, e.d_mel_off, e.d_h1_off, e.d_h2_off, nw, m.c0w, m.c0b, m.c2w, m.c2b, e.s2dw,
                                   e.rows2, NMEL, SUBC, s),
         "subsampling conv0 + conv2");
    TRY(conv1x1_tc(e.s2dw, e.rows2 * W2, m.c3w, m.c3b, e.s2, s, "subsampling conv3"));
    TRYC(p2cu::sub_dwconv_launch(e.s2, e.d_h2_off, e.d_sub_off, nw, m.c5w, m.c5b, e.s3dw, e.R_sub, W2, SUBC, s),
         "subsampling conv5");
    TRY(conv1x1_tc(e.s3dw, e.R_sub * W3, m.c6w, m.c6b, e.s3, s, "subsampling conv6"));
    TRYC(p2cu::sub_flatten_launch(e.s3, e.flat, e.R_sub, W3, SUBC, s), "subsampling flatten");
    TRY(wmatmul(e, e.flat, e.R_sub, m.lin, e.x_sub, 1.f, 0.f, nullptr, s, "subsampling linear"));
    TRYC(p2cu::bias_rows_launch(e.x_sub, m.lin_b, e.R_sub, D, s), "subsampling bias");
    return P2CU_OK;
}

// csrc/encoder.c:319-348.
// prev_w / prev_b: the previous block's closing norm (norm_out), applied to x first in the same launch, or null.
int feed_forward(P2cuEncoder& e, const float* nw, const float* nb, const DWeight& w1, const DWeight& w2,
                 cudaStream_t s, const float* prev_w = nullptr, const float* prev_b = nullptr) {
    if (e.mode != P2CU_EXACT) {
        p2cu::KFold hold;
        if (prev_w)
            TRYC(p2cu::ln2_rows_launch(e.x, D, prev_w, prev_b, nw, nb, nullptr, 0, e.q, e.qs, e.R, D, s,
                                       take_fold(e, hold)),
                 "norm_out + ff layernorm");
        else
            TRYC(p2cu::ln_rows_launch(e.x, D, nw, nb, nullptr, 0, e.q, e.qs, e.R, D, s, take_fold(e, hold)),
                 "ff layernorm");
        TRY(wmatmul_q8a(e, e.R, w1, e.big, 1.f, 0.f, s, "ff linear1"));
        TRYC(p2cu::swish_rows_launch(e.big, FF, nullptr, 0, e.q, e.qs, e.R, FF, s), "ff swish");
        // x += ½ · ff(x); with K = 4096 the fold of its K blocks goes with the next LayerNorm
        return wmatmul_q8a(e, e.R, w2, e.x, 0.5f, 1.f, s, "ff linear2", true);
    }
    if (prev_w)
        TRYC(p2cu::ln2_rows_launch(e.x, D, prev_w, prev_b, nw, nb, e.lnbuf, D, nullptr, nullptr, e.R, D, s),
             "norm_out + ff layernorm");
    else
        TRYC(p2cu::ln_rows_launch(e.x, D, nw, nb, e.lnbuf, D, nullptr, nullptr, e.R, D, s), "ff layernorm");
    TRY(wmatmul(e, e.lnbuf, e.R, w1, e.big, 1.f, 0.f, nullptr, s, "ff linear1"));
    TRYC(p2cu::swish_rows_launch(e.big, FF, e.big, FF, nullptr, nullptr, e.R, FF, s), "ff swish");
    p2cu::Epilogue res;
    res.residual = 1;
    res.res_alpha = 0.5f;
    return wmatmul(e, e.big, e.R, w2, e.x, 1.f, 0.f, &res, s, "ff linear2");
}

// csrc/encoder.c:470-528.
int self_attention(P2cuEncoder& e, const DBlock& b, cudaStream_t s) {
    const bool i8 = e.mode != P2CU_EXACT;
    if (i8) {
        p2cu::KFold hold;
        TRYC(p2cu::ln_rows_launch(e.x, D, b.n_sa_w, b.n_sa_b, nullptr, 0, e.q, e.qs, e.R, D, s, take_fold(e, hold)),
             "mhsa layernorm");
        TRY(wmatmul_q8a(e, e.R, b.qkv, e.big, 1.f, 0.f, s, "qkv"));
        // pe rows were quantised when the plan was made: the same rows every layer (csrc/encoder.c:500)
        TRY(p2cu::gemm_i8(e.L, D, D, 1.f, e.pe_q, e.pe_s, b.pos.kind == P2_W_FV ? &b.pos.fv : nullptr, b.pos.q8,
                          b.pos.scales, D, b.pos.kind == P2_W_FV ? e.mode : P2CU_INT8, 0.f, e.P, D, e.ws, e.ws_bytes,
                          s, "pos"));
    } else {
        TRYC(p2cu::ln_rows_launch(e.x, D, b.n_sa_w, b.n_sa_b, e.lnbuf, D, nullptr, nullptr, e.R, D, s),
             "mhsa layernorm");
        TRY(wmatmul(e, e.lnbuf, e.R, b.qkv, e.big, 1.f, 0.f, nullptr, s, "qkv"));
        TRY(wmatmul(e, e.pe, e.L, b.pos, e.P, 1.f, 0.f, nullptr, s, "pos"));
    }
    if (e.attn_path == 0) {   // tensor cores: AC and BD in one launch, softmax, then the context
        p2cu::TcArgs a{};
        a.src[0] = e.big; a.src[1] = e.P;
        a.dst[0] = e.s_ac; a.dst[1] = e.s_bd;
        a.bias[0] = b.bias_u; a.bias[1] = b.bias_v;
        a.err = p2cu::device_error_word();
        TRYC(p2cu::attn_tc_launch(e.tc_scores, 2 * e.n_tc, e.t_tc_scores, a, false, s), "attention scores");
        TRYC(p2cu::attn_softmax_launch(e.s_ac, e.s_bd, e.d_srow_off, e.d_s_off, e.d_b_off, e.d_T, e.n_win, H,
                                       e.srows, e.scale, s),
             "attention softmax");
        TRYC(p2cu::v_transpose_launch(e.big, e.vt, e.d_row_off, e.d_vt_off, e.n_win, e.R, s), "attention v^T");
        p2cu::TcArgs c{};
        c.src[0] = e.s_ac; c.src[1] = e.vt;
        c.dst[0] = e.attn; c.dst[1] = e.attn;
        c.err = a.err;
        TRYC(p2cu::attn_tc_launch(e.tc_context, e.n_tc, e.t_tc_context, c, false, s), "attention context");
    } else if (e.attn_path == 3) {
        TRY(p2cu::attn_rel_tc_launch(e.big, e.R, e.P, b.bias_u, b.bias_v, e.d_row_off, e.tc_tiles, e.n_tc_tiles,
                                     e.Tmax, e.scale, e.attn, e.att_parts, e.att_counters, p2cu::device_error_word(),
                                     s));
    } else if (e.n_att_tiles) {
        TRYC(p2cu::attn_fused_launch(e.big, e.P, b.bias_u, b.bias_v, e.d_row_off, e.att_tiles, e.n_att_tiles, e.Tmax,
                                     e.scale, e.attn, s),
             "attention");
    } else {   // windows longer than the fused kernel holds: the products as grouped GEMMs, scores in HBM
        TRYC(p2cu::group_gemm_launch(e.g_ac, e.ng, e.t_ac, e.big, e.big, e.s_ac, b.bias_u, 1, s), "attention ac");
        TRYC(p2cu::group_gemm_launch(e.g_bd, e.ng, e.t_bd, e.big, e.P, e.s_bd, b.bias_v, 1, s), "attention bd");
        TRYC(p2cu::attn_softmax_launch(e.s_ac, e.s_bd, e.d_srow_off, e.d_s_off, e.d_b_off, e.d_T, e.n_win, H,
                                       e.srows, e.scale, s),
             "attention softmax");
        TRYC(p2cu::group_gemm_launch(e.g_av, e.ng, e.t_av, e.s_ac, e.big, e.attn, nullptr, 0, s), "attention av");
    }
    if (i8) {
        TRYC(p2cu::quant_rows_dense_launch(e.attn, e.q, e.qs, e.R, D, s), "attention quant");
        return wmatmul_q8a(e, e.R, b.out, e.x, 1.f, 1.f, s, "out");   // x += attn @ W_o
    }
    p2cu::Epilogue res;
    res.residual = 1;
    return wmatmul(e, e.attn, e.R, b.out, e.x, 1.f, 0.f, &res, s, "out");
}

// csrc/encoder.c:573-612.
int conv_module(P2cuEncoder& e, const DBlock& b, cudaStream_t s) {
    const bool i8 = e.mode != P2CU_EXACT;
    if (i8) {
        TRYC(p2cu::ln_rows_launch(e.x, D, b.n_conv_w, b.n_conv_b, nullptr, 0, e.q, e.qs, e.R, D, s),
             "conv layernorm");
        TRY(wmatmul_q8a(e, e.R, b.pw1, e.big, 1.f, 0.f, s, "pw1"));
    } else {
        TRYC(p2cu::ln_rows_launch(e.x, D, b.n_conv_w, b.n_conv_b, e.lnbuf, D, nullptr, nullptr, e.R, D, s),
             "conv layernorm");
        TRY(wmatmul(e, e.lnbuf, e.R, b.pw1, e.big, 1.f, 0.f, nullptr, s, "pw1"));
    }
    TRYC(p2cu::glu_rows_launch(e.big, e.gated, e.R, D, s), "glu");
    if (i8) {
        TRYC(p2cu::dwconv_swish_launch(e.gated, b.dw_w, b.dw_b, e.d_row_off, e.n_win, nullptr, e.q, e.qs, e.R, D, s),
             "depthwise conv");
        return wmatmul_q8a(e, e.R, b.pw2, e.x, 1.f, 1.f, s, "pw2");   // x += conv(x)
    }
    TRYC(p2cu::dwconv_swish_launch(e.gated, b.dw_w, b.dw_b, e.d_row_off, e.n_win, e.lnbuf, nullptr, nullptr, e.R, D,
                                   s),
         "depthwise conv");
    p2cu::Epilogue res;
    res.residual = 1;
    return wmatmul(e, e.lnbuf, e.R, b.pw2, e.x, 1.f, 0.f, &res, s, "pw2");
}

// The whole forward pass on stream s (csrc/encoder.c:617-624, 725-751).
int forward(P2cuEncoder& e, cudaStream_t s) {
    e.pending.nblk = 0;   // a pass that failed part way leaves nothing for this one
    TRY(subsampling(e, s));
    if (e.chunked)   // each chunk's frames, with their overlap context, as a window of its own
        TRYC(p2cu::gather_rows_launch(e.x, e.x_sub, e.d_gather, e.R, D, s), "chunk gather");
    for (int i = 0; i < NB; ++i) {
        const DBlock& b = e.m->blk[i];
        // block i - 1's closing norm goes with this block's first LayerNorm (one launch, csrc/encoder.c:617-624)
        const DBlock* pb = i > 0 ? &e.m->blk[i - 1] : nullptr;
        TRY(feed_forward(e, b.n_ff1_w, b.n_ff1_b, b.ff1a, b.ff1b, s, pb ? pb->n_out_w : nullptr,
                         pb ? pb->n_out_b : nullptr));
        TRY(self_attention(e, b, s));
        TRY(conv_module(e, b, s));
        TRY(feed_forward(e, b.n_ff2_w, b.n_ff2_b, b.ff2a, b.ff2b, s));
        p2cu::KFold hold;
        if (i == NB - 1)
            TRYC(p2cu::ln_rows_launch(e.x, D, b.n_out_w, b.n_out_b, e.x, D, nullptr, nullptr, e.R, D, s,
                                      take_fold(e, hold)),
                 "norm_out");
    }
    const float* fin = e.x;
    if (e.chunked) {   // every frame from the chunk that owns it, without the overlap (csrc/encoder.c:704)
        TRYC(p2cu::gather_rows_launch(e.x_sub, e.x, e.d_scatter, e.R_sub, D, s), "chunk scatter");
        fin = e.x_sub;
    }
    TRY(wmatmul(e, fin, e.R_sub, e.m->proj, e.out, 1.f, 0.f, nullptr, s, "projector"));
    TRYC(p2cu::bias_rows_launch(e.out, e.m->proj_b, e.R_sub, P2_JOINT_DIM, s), "projector bias");
    return P2CU_OK;
}

// [2T-1 x D] relative positions T-1 .. -(T-1), even columns sin, odd cos (csrc/encoder.c:79-96), computed on the
// host with the C library's powf / sinf / cosf in float, as the reference does.
std::vector<float> rel_pos_encoding(int T) {
    const int L = 2 * T - 1;
    std::vector<float> pe(static_cast<size_t>(L) * D);
    std::vector<float> inv(D / 2);
    for (int i = 0; i < D / 2; ++i) inv[i] = 1.0f / powf(10000.0f, static_cast<float>(2 * i) / static_cast<float>(D));
    for (int j = 0; j < L; ++j) {
        const float pos = static_cast<float>(T - 1 - j);
        float* row = pe.data() + static_cast<size_t>(j) * D;
        for (int i = 0; i < D / 2; ++i) {
            const float f = inv[i] * pos;
            row[2 * i] = sinf(f);
            row[2 * i + 1] = cosf(f);
        }
    }
    return pe;
}

void destroy_plan(P2cuEncoder* e) {
    if (!e) return;
    if (e->exec) cudaGraphExecDestroy(e->exec);
    if (e->graph) cudaGraphDestroy(e->graph);
    if (e->stream) cudaStreamDestroy(e->stream);
    if (e->arena) cudaFree(e->arena);
    delete e;
}

size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

int create_plan(const P2cuModel* m, const int* n_frames, int n_mel_win, int mode, int chunk, int overlap,
                P2cuEncoder** out, bool lazy) {
    if (!m || !n_frames || !out || n_mel_win <= 0) return fail_fmt(P2CU_EINVAL, "p2cu_encoder_create: bad arguments");
    if (chunk > 0 && overlap < 0) return fail_fmt(P2CU_EINVAL, "p2cu_encoder_create: overlap %d", overlap);
    if (mode != P2CU_INT8 && mode != P2CU_INT8W && mode != P2CU_EXACT)
        return fail_fmt(P2CU_EINVAL, "p2cu_encoder_create: mode %d", mode);
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != m->device)
        return fail_fmt(P2CU_EINVAL, "p2cu_encoder_create: the model lives on device %d, device %d is current",
                        m->device, dev);
    auto* e = new P2cuEncoder();
    e->m = m; e->device = dev; e->mode = mode; e->n_mel_win = n_mel_win;
    e->mel_off.push_back(0); e->h1_off.push_back(0); e->h2_off.push_back(0); e->sub_off.push_back(0);
    e->row_off.push_back(0);
    std::vector<int> gather, scatter;
    for (int w = 0; w < n_mel_win; ++w) {
        if (n_frames[w] < 1) {
            destroy_plan(e);
            return fail_fmt(P2CU_EINVAL, "p2cu_encoder_create: window %d has %d mel frames", w, n_frames[w]);
        }
        const int h1 = conv_out(n_frames[w]), h2 = conv_out(h1), tp = conv_out(h2);
        const int base = e->sub_off.back();
        e->n_mel.push_back(n_frames[w]);
        e->Tp.push_back(tp);
        e->mel_off.push_back(e->mel_off.back() + n_frames[w]);
        e->h1_off.push_back(e->h1_off.back() + h1);
        e->h2_off.push_back(e->h2_off.back() + h2);
        e->sub_off.push_back(base + tp);
        scatter.resize(base + tp);
        // the block windows of this mel window: itself, or chunks of `chunk` frames with `overlap` frames of context
        // on each side (csrc/encoder.c:663-710)
        const int n_chunks = chunk > 0 ? (tp + chunk - 1) / chunk : 1;
        for (int ci = 0; ci < n_chunks; ++ci) {
            const int out_start = chunk > 0 ? ci * chunk : 0;
            const int out_end = chunk > 0 ? std::min(out_start + chunk, tp) : tp;
            const int in_start = chunk > 0 ? std::max(out_start - overlap, 0) : 0;
            const int in_end = chunk > 0 ? std::min(out_end + overlap, tp) : tp;
            const int t = in_end - in_start, r0 = e->row_off.back();
            for (int j = 0; j < t; ++j) gather.push_back(base + in_start + j);
            for (int f = out_start; f < out_end; ++f) scatter[base + f] = r0 + (out_start - in_start) + (f - out_start);
            e->T.push_back(t);
            e->row_off.push_back(r0 + t);
            e->Tmax = t > e->Tmax ? t : e->Tmax;
        }
    }
    e->n_win = static_cast<int>(e->T.size());
    const int n_win = e->n_win;
    e->mel_rows = e->mel_off.back(); e->rows1 = e->h1_off.back(); e->rows2 = e->h2_off.back();
    e->R_sub = e->sub_off.back(); e->R = e->row_off.back();
    e->chunked = chunk > 0 && e->R != e->R_sub;
    if (chunk > 0 && !e->chunked)   // one chunk per window covering all of it: the full-length pass
        for (int r = 0; r < e->R; ++r) e->chunked |= gather[r] != r;
    e->L = 2 * e->Tmax - 1;
    e->scale = 1.0f / sqrtf(static_cast<float>(DH));

    // attention tables and GEMM groups (one group per window and head)
    std::vector<int> srow_off{0};
    std::vector<long long> s_off, b_off, vt_off;
    std::vector<p2cu::GemmGroup> gac, gbd, gav;
    int tac = 0, tbd = 0, tav = 0;
    for (int w = 0; w < n_win; ++w) {
        const int t = e->T[w], Lw = 2 * t - 1, r0 = e->row_off[w];
        s_off.push_back(e->s_total);
        b_off.push_back(e->b_total);
        const int ldS = (t + 3) & ~3, ldB = (Lw + 3) & ~3;   // 16-byte aligned score rows
        for (int h = 0; h < H; ++h) {
            const long long sac = e->s_total + static_cast<long long>(h) * t * ldS;
            const long long sbd = e->b_total + static_cast<long long>(h) * t * ldB;
            p2cu::GemmGroup g{};
            // AC = (Q + bias_u) K^T: A = Q columns of QKV, B = K columns (transposed), C = S_ac
            g.M = t; g.N = t; g.K = DH; g.tile0 = tac;
            g.a_off = static_cast<long long>(r0) * 3 * D + h * DH; g.lda = 3 * D;
            g.b_off = static_cast<long long>(r0) * 3 * D + D + h * DH; g.ldb = 3 * D;
            g.c_off = sac; g.ldc = ldS; g.bias_off = h * DH;
            gac.push_back(g); tac += p2cu::group_gemm_tiles(g.M, g.N);
            // BD = (Q + bias_v) P^T over this window's 2T-1 positions, rows Tmax-T .. Tmax+T-2 of P (the positions
            // T-1 .. -(T-1) of a window of T frames)
            g.N = Lw; g.tile0 = tbd;
            g.b_off = static_cast<long long>(e->Tmax - t) * D + h * DH; g.ldb = D;
            g.c_off = sbd; g.ldc = ldB;
            gbd.push_back(g); tbd += p2cu::group_gemm_tiles(g.M, g.N);
            // AV = S V into the concatenated heads [R][D]
            g.M = t; g.N = DH; g.K = t; g.tile0 = tav;
            g.a_off = sac; g.lda = ldS;
            g.b_off = static_cast<long long>(r0) * 3 * D + 2 * D + h * DH; g.ldb = 3 * D;
            g.c_off = static_cast<long long>(r0) * D + h * DH; g.ldc = D; g.bias_off = -1;
            gav.push_back(g); tav += p2cu::group_gemm_tiles(g.M, g.N);
        }
        vt_off.push_back(e->vt_total);
        e->vt_total += static_cast<long long>(H) * DH * ldS;
        e->s_total += static_cast<long long>(H) * t * ldS;
        e->b_total += static_cast<long long>(H) * t * ldB;
        srow_off.push_back(srow_off.back() + H * t);
    }
    e->srows = srow_off.back();
    {
        const char* ap = getenv("P2CU_ATTN");
        const bool fits = e->Tmax <= p2cu::ATT_MAXT;
        if (ap && strcmp(ap, "simt") == 0) e->attn_path = 1;
        else if (ap && strcmp(ap, "fused") == 0) e->attn_path = 2;
        else if (ap && strcmp(ap, "tc") == 0) e->attn_path = 0;
        else e->attn_path = fits ? 3 : 0;
    }
    // tensor-core groups: scores (AC then BD groups, one launch) and context (one launch)
    std::vector<p2cu::TcGroup> tcs, tcc;
    {
        int ts = 0, tc = 0;
        for (int pass = 0; pass < 2; ++pass)
            for (int w = 0; w < n_win; ++w) {
                const int t = e->T[w], Lw = 2 * t - 1, r0 = e->row_off[w];
                for (int h = 0; h < H; ++h) {
                    p2cu::TcGroup g{};
                    g.M = t; g.K = DH; g.tile0 = ts;
                    g.a_off = static_cast<long long>(r0) * 3 * D + h * DH; g.lda = 3 * D;
                    g.a_src = 0;
                    g.bias_off = h * DH;
                    if (pass == 0) {   // AC = (Q + bias_u) K^T
                        g.N = t;
                        g.b_src = 0; g.b_off = static_cast<long long>(r0) * 3 * D + D + h * DH; g.ldb = 3 * D;
                        g.c_dst = 0; g.c_off = gac[w * H + h].c_off; g.ldc = gac[w * H + h].ldc;
                        g.bias_sel = 0;
                    } else {           // BD = (Q + bias_v) P^T over the window's 2T - 1 positions
                        g.N = Lw;
                        g.b_src = 1; g.b_off = static_cast<long long>(e->Tmax - t) * D + h * DH; g.ldb = D;
                        g.c_dst = 1; g.c_off = gbd[w * H + h].c_off; g.ldc = gbd[w * H + h].ldc;
                        g.bias_sel = 1;
                    }
                    tcs.push_back(g);
                    ts += p2cu::tc_gemm_tiles(g.M, g.N);
                    if (pass == 0) {   // context = S V into the concatenated heads, V^T (K-major) from vt
                        p2cu::TcGroup c{};
                        const int ldS = gac[w * H + h].ldc;
                        c.M = t; c.N = DH; c.K = t; c.tile0 = tc;
                        c.a_src = 0; c.a_off = gac[w * H + h].c_off; c.lda = ldS;
                        c.b_src = 1; c.b_off = vt_off[w] + static_cast<long long>(h) * DH * ldS; c.ldb = ldS;
                        c.c_dst = 0; c.c_off = static_cast<long long>(r0) * D + h * DH; c.ldc = D;
                        c.bias_sel = -1;
                        tcc.push_back(c);
                        tc += p2cu::tc_gemm_tiles(c.M, c.N);
                    }
                }
            }
        e->n_tc = static_cast<int>(tcc.size());
        e->t_tc_scores = ts;
        e->t_tc_context = tc;
    }
    const bool fused = (e->attn_path == 2 || e->attn_path == 3) && e->Tmax <= p2cu::ATT_MAXT;
    std::vector<int2> att_tiles;
    std::vector<p2cu::AttnTile> tc_tiles;
    int tc_groups = 0;
    bool tc_split = false;
    if (fused) {
        if (e->attn_path == 3) {   // 128-query tiles, the keys split over CTAs when there are few tiles
            int dev = 0, sms = 148;
            if (cudaGetDevice(&dev) != cudaSuccess ||
                cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
                sms = 148;
            e->n_tc_tiles = p2cu::attn_rel_tc_plan(e->T.data(), n_win, sms, tc_tiles, &tc_groups);
            for (const p2cu::AttnTile& t : tc_tiles) tc_split = tc_split || t.nsplit > 1;
        } else {                   // (window, first query) of every 32-query tile
            for (int w = 0; w < n_win; ++w)
                for (int q0 = 0; q0 < e->T[w]; q0 += 32) att_tiles.push_back(make_int2(w, q0));
            e->n_att_tiles = static_cast<int>(att_tiles.size());
        }
        e->s_total = e->b_total = 0;   // no score matrices in HBM
    }
    e->ng = static_cast<int>(gac.size());
    e->t_ac = tac; e->t_bd = tbd; e->t_av = tav;

    // one arena for every buffer
    const int R = e->R, L = e->L, Rs = e->R_sub;
    const int W1 = conv_out(NMEL), W2 = conv_out(W1), W3 = conv_out(W2);
    const size_t f = sizeof(float);
    e->ws_bytes = p2cu::gemm_split_bytes(std::max(R, Rs), D, FF);
    struct Slot { void** p; size_t bytes; };
    const size_t s1_bytes = static_cast<size_t>(Rs) * FF * f;   // the flattened frames (the first convolution's
                                                                // outputs are not stored)
    const size_t q_bytes = static_cast<size_t>(std::max(R, Rs)) * FF;
    std::vector<Slot> slots = {
        {reinterpret_cast<void**>(&e->mel), static_cast<size_t>(e->mel_rows) * NMEL * f},
        {reinterpret_cast<void**>(&e->s1), s1_bytes},
        {reinterpret_cast<void**>(&e->s2dw), static_cast<size_t>(e->rows2) * W2 * SUBC * f},
        {reinterpret_cast<void**>(&e->s2), static_cast<size_t>(e->rows2) * W2 * SUBC * f},
        {reinterpret_cast<void**>(&e->s3dw), static_cast<size_t>(Rs) * W3 * SUBC * f},
        {reinterpret_cast<void**>(&e->s3), static_cast<size_t>(Rs) * W3 * SUBC * f},
        {reinterpret_cast<void**>(&e->x_sub), e->chunked ? static_cast<size_t>(Rs) * D * f : 0},
        {reinterpret_cast<void**>(&e->x), static_cast<size_t>(R) * D * f},
        {reinterpret_cast<void**>(&e->big), static_cast<size_t>(R) * FF * f},
        {reinterpret_cast<void**>(&e->lnbuf), static_cast<size_t>(R) * D * f},
        {reinterpret_cast<void**>(&e->gated), static_cast<size_t>(R) * D * f},
        {reinterpret_cast<void**>(&e->attn), static_cast<size_t>(R) * D * f},
        {reinterpret_cast<void**>(&e->q), q_bytes},
        {reinterpret_cast<void**>(&e->qs), static_cast<size_t>(std::max(R, Rs)) * f},
        {reinterpret_cast<void**>(&e->pe), static_cast<size_t>(L) * D * f},
        {reinterpret_cast<void**>(&e->pe_q), static_cast<size_t>(L) * D},
        {reinterpret_cast<void**>(&e->pe_s), static_cast<size_t>(L) * f},
        {reinterpret_cast<void**>(&e->P), static_cast<size_t>(L) * D * f},
        {reinterpret_cast<void**>(&e->s_ac), static_cast<size_t>(e->s_total) * f},
        {reinterpret_cast<void**>(&e->s_bd), static_cast<size_t>(e->b_total) * f},
        {reinterpret_cast<void**>(&e->vt), e->attn_path == 0 ? static_cast<size_t>(e->vt_total) * f : 0},
        {reinterpret_cast<void**>(&e->d_vt_off), n_win * sizeof(long long)},
        {reinterpret_cast<void**>(&e->out), static_cast<size_t>(Rs) * P2_JOINT_DIM * f},
        {&e->ws, e->ws_bytes},
        {reinterpret_cast<void**>(&e->d_mel_off), (n_mel_win + 1) * sizeof(int)},
        {reinterpret_cast<void**>(&e->d_h1_off), (n_mel_win + 1) * sizeof(int)},
        {reinterpret_cast<void**>(&e->d_h2_off), (n_mel_win + 1) * sizeof(int)},
        {reinterpret_cast<void**>(&e->d_sub_off), (n_mel_win + 1) * sizeof(int)},
        {reinterpret_cast<void**>(&e->d_gather), static_cast<size_t>(R) * sizeof(int)},
        {reinterpret_cast<void**>(&e->d_scatter), static_cast<size_t>(Rs) * sizeof(int)},
        {reinterpret_cast<void**>(&e->d_row_off), (n_win + 1) * sizeof(int)},
        {reinterpret_cast<void**>(&e->d_srow_off), (n_win + 1) * sizeof(int)},
        {reinterpret_cast<void**>(&e->d_T), n_win * sizeof(int)},
        {reinterpret_cast<void**>(&e->d_s_off), n_win * sizeof(long long)},
        {reinterpret_cast<void**>(&e->d_b_off), n_win * sizeof(long long)},
        {reinterpret_cast<void**>(&e->g_ac), gac.size() * sizeof(p2cu::GemmGroup)},
        {reinterpret_cast<void**>(&e->g_bd), gbd.size() * sizeof(p2cu::GemmGroup)},
        {reinterpret_cast<void**>(&e->g_av), gav.size() * sizeof(p2cu::GemmGroup)},
        {reinterpret_cast<void**>(&e->att_tiles), att_tiles.size() * sizeof(int2)},
        {reinterpret_cast<void**>(&e->tc_tiles), tc_tiles.size() * sizeof(p2cu::AttnTile)},
        {&e->att_parts, tc_split ? p2cu::attn_rel_tc_part_bytes(e->n_tc_tiles) : 0},
        {reinterpret_cast<void**>(&e->att_counters), tc_split ? static_cast<size_t>(tc_groups) * 8 * sizeof(int) : 0},
        {reinterpret_cast<void**>(&e->tc_scores), tcs.size() * sizeof(p2cu::TcGroup)},
        {reinterpret_cast<void**>(&e->tc_context), tcc.size() * sizeof(p2cu::TcGroup)},
    };
    size_t total = 0;
    for (const Slot& sl : slots) total += al256(sl.bytes ? sl.bytes : 1);
    cudaError_t ce = cudaMalloc(&e->arena, total);
    if (ce != cudaSuccess) {
        destroy_plan(e);
        return p2cu::cuda_error(ce, "p2cu_encoder_create: cudaMalloc");
    }
    size_t off = 0;
    for (const Slot& sl : slots) {
        *sl.p = e->arena + off;
        off += al256(sl.bytes ? sl.bytes : 1);
    }
    if (!e->ws_bytes) e->ws = nullptr;
    e->flat = e->s1;   // the flattened frames reuse the first convolution's buffer
    if (!e->chunked) e->x_sub = e->x;
    const std::vector<float> pe = rel_pos_encoding(e->Tmax);
    std::vector<int> Tw(e->T);
    struct Copy { void* dst; const void* src; size_t bytes; };
    const Copy copies[] = {
        {e->pe, pe.data(), pe.size() * f},
        {e->d_mel_off, e->mel_off.data(), (n_mel_win + 1) * sizeof(int)},
        {e->d_h1_off, e->h1_off.data(), (n_mel_win + 1) * sizeof(int)},
        {e->d_h2_off, e->h2_off.data(), (n_mel_win + 1) * sizeof(int)},
        {e->d_sub_off, e->sub_off.data(), (n_mel_win + 1) * sizeof(int)},
        {e->d_gather, gather.data(), static_cast<size_t>(R) * sizeof(int)},
        {e->d_scatter, scatter.data(), static_cast<size_t>(Rs) * sizeof(int)},
        {e->d_row_off, e->row_off.data(), (n_win + 1) * sizeof(int)},
        {e->d_srow_off, srow_off.data(), (n_win + 1) * sizeof(int)},
        {e->d_T, Tw.data(), n_win * sizeof(int)},
        {e->d_s_off, s_off.data(), n_win * sizeof(long long)},
        {e->d_b_off, b_off.data(), n_win * sizeof(long long)},
        {e->d_vt_off, vt_off.data(), n_win * sizeof(long long)},
        {e->g_ac, gac.data(), gac.size() * sizeof(p2cu::GemmGroup)},
        {e->g_bd, gbd.data(), gbd.size() * sizeof(p2cu::GemmGroup)},
        {e->g_av, gav.data(), gav.size() * sizeof(p2cu::GemmGroup)},
        {e->att_tiles, att_tiles.data(), att_tiles.size() * sizeof(int2)},
        {e->tc_tiles, tc_tiles.data(), tc_tiles.size() * sizeof(p2cu::AttnTile)},
        {e->tc_scores, tcs.data(), tcs.size() * sizeof(p2cu::TcGroup)},
        {e->tc_context, tcc.data(), tcc.size() * sizeof(p2cu::TcGroup)},
    };
    for (const Copy& c : copies)
        if (c.bytes && (ce = cudaMemcpy(c.dst, c.src, c.bytes, cudaMemcpyHostToDevice)) != cudaSuccess) break;
    if (ce == cudaSuccess) ce = cudaMemset(e->mel, 0, static_cast<size_t>(e->mel_rows) * NMEL * f);
    if (ce == cudaSuccess && e->attn_path == 0)   // V^T's padding columns stay zero
        ce = cudaMemset(e->vt, 0, static_cast<size_t>(e->vt_total) * f);
    if (ce == cudaSuccess && tc_split)   // the split attention's merge counters start at zero
        ce = cudaMemset(e->att_counters, 0, static_cast<size_t>(tc_groups) * 8 * sizeof(int));
    if (!tc_split) e->att_parts = nullptr, e->att_counters = nullptr;
    if (ce == cudaSuccess) ce = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
    if (ce == cudaSuccess && mode != P2CU_EXACT)
        ce = p2cu::quant_rows_launch(e->pe, L, D, D, e->pe_q, e->pe_s, e->stream);
    if (ce != cudaSuccess) {
        destroy_plan(e);
        return p2cu::cuda_error(ce, "p2cu_encoder_create: set-up");
    }
    e->lazy = lazy;
    if (lazy) {   // the first run is the eager pass; it must see the position table's quantised rows
        ce = cudaStreamSynchronize(e->stream);
        if (ce != cudaSuccess) {
            destroy_plan(e);
            return p2cu::cuda_error(ce, "p2cu_encoder_create: set-up");
        }
        *out = e;
        return P2CU_OK;
    }
    // One eager pass (checks every launch and loads every kernel), then the capture.
    int rc = forward(*e, e->stream);
    if (rc == P2CU_OK) rc = p2cu_check_device(e->stream);
    if (rc != P2CU_OK) {
        destroy_plan(e);
        return rc;
    }
    const char* eager = getenv("P2CU_ENCODER_EAGER");
    if (!(eager && eager[0] == '1')) {
        ce = cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal);
        if (ce == cudaSuccess) {
            rc = forward(*e, e->stream);
            ce = cudaStreamEndCapture(e->stream, &e->graph);
            if (rc == P2CU_OK && ce == cudaSuccess) ce = cudaGraphInstantiate(&e->exec, e->graph, 0);
        }
        if (rc != P2CU_OK || ce != cudaSuccess) {
            destroy_plan(e);
            return rc != P2CU_OK ? rc : p2cu::cuda_error(ce, "p2cu_encoder_create: graph capture");
        }
    }
    *out = e;
    return P2CU_OK;
}

}  // namespace

extern "C" {

int p2cu_model_upload(const P2Model* m, int codes, P2cuModel** out) { return upload_model(m, codes, out); }

void p2cu_model_free(P2cuModel* m) {
    if (!m) return;
    if (m->arena) cudaFree(m->arena);
    delete m;
}

size_t p2cu_model_bytes(const P2cuModel* m) { return m ? m->bytes : 0; }

int p2cu_encoder_create(const P2cuModel* m, const int* n_frames, int n_windows, int mode, int chunk_frames,
                        int chunk_overlap, P2cuEncoder** out) {
    return create_plan(m, n_frames, n_windows, mode, chunk_frames, chunk_overlap, out, false);
}

// For the library's host entry points (not exported): a lazy plan (see P2cuEncoder::lazy).
int p2cu_encoder_create_lazy(const P2cuModel* m, const int* n_frames, int n_windows, int mode, int chunk_frames,
                             int chunk_overlap, P2cuEncoder** out) {
    return create_plan(m, n_frames, n_windows, mode, chunk_frames, chunk_overlap, out, true);
}

void p2cu_encoder_destroy(P2cuEncoder* e) { destroy_plan(e); }

int p2cu_encoder_frames(const P2cuEncoder* e, int window) {
    if (!e) return -1;
    if (window < 0) return e->R_sub;
    return window < e->n_mel_win ? e->Tp[window] : -1;
}

float* p2cu_encoder_mel(P2cuEncoder* e) { return e ? e->mel : nullptr; }

float* p2cu_encoder_out(P2cuEncoder* e) { return e ? e->out : nullptr; }

int p2cu_encoder_run(P2cuEncoder* e, void* stream) {
    if (!e) return fail_fmt(P2CU_EINVAL, "p2cu_encoder_run: NULL plan");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const char* eager = getenv("P2CU_ENCODER_EAGER");
    if (!e->exec && e->lazy && e->eager_runs > 0 && !e->capture_failed && !(eager && eager[0] == '1')) {
        // second run of a lazy plan: capture it now (recorded on the plan's own stream, launched on the caller's)
        cudaError_t ce = cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal);
        if (ce == cudaSuccess) {
            const int rc = forward(*e, e->stream);
            ce = cudaStreamEndCapture(e->stream, &e->graph);
            if (rc == P2CU_OK && ce == cudaSuccess) ce = cudaGraphInstantiate(&e->exec, e->graph, 0);
            if (rc != P2CU_OK || ce != cudaSuccess) {
                if (e->graph) cudaGraphDestroy(e->graph);
                e->graph = nullptr;
                e->exec = nullptr;
                e->capture_failed = true;
                cudaGetLastError();
            }
        } else {
            e->capture_failed = true;
            cudaGetLastError();
        }
    }
    if (!e->exec) {
        ++e->eager_runs;
        return forward(*e, s);
    }
    cudaError_t ce = cudaGraphLaunch(e->exec, s);
    return ce == cudaSuccess ? P2CU_OK : p2cu::cuda_error(ce, "p2cu_encoder_run");
}

}  // extern "C"
