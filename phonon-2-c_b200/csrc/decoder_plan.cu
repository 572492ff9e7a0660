// decoder_plan.cu - the device decoder's C ABI (include/p2cuda.h): a P2cuDecoder holds the state and token buffers of
// up to max_windows windows of up to max_frames encoder frames together, allocated once; p2cu_decode runs the greedy
// TDT decode of csrc/decoder.c:100-141 over a batch of windows in one cooperative launch (decoder.cu), and
// p2cu_decoder_step / p2cu_joint are the single-step calls of csrc/decoder.c:62-88 on device pointers.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <vector>
#include <cuda_runtime.h>
#include "p2cuda.h"
#include "gemm.h"
#include "model.h"
#include "decoder.h"

using p2cu::fail_fmt;

namespace {
constexpr int HD = P2_JOINT_DIM;
size_t align256(size_t n) { return (n + 255) & ~size_t(255); }
}  // namespace

struct P2cuDecoder {
    const P2cuModel* m = nullptr;
    int device = 0, max_windows = 0, max_frames = 0, grid = 0;
    char* arena = nullptr;
    size_t bytes = 0;
    // device buffers
    unsigned* bar = nullptr;   // [0] arrival count (zeroed per launch), [1] generation; h and c follow
    float* hc = nullptr;       // h [2][2][B][640] then c [2][B][640] for the launch's B
    float *dec = nullptr, *cand = nullptr, *dur = nullptr, *logits = nullptr, *enc1 = nullptr;
    int *win_off = nullptr, *tokens = nullptr, *tok_out = nullptr, *tok_off = nullptr, *count = nullptr;
    // host staging of the window offsets (pinned), reused once the copy that read it has completed
    int* h_off = nullptr;
    cudaEvent_t staged = nullptr;
    int n_windows = 0;         // of the last p2cu_decode
};

namespace {

void destroy(P2cuDecoder* d) {
    if (!d) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(d->device);
    if (d->staged) cudaEventSynchronize(d->staged), cudaEventDestroy(d->staged);
    if (d->h_off) cudaFreeHost(d->h_off);
    if (d->arena) cudaFree(d->arena);
    cudaSetDevice(prev);
    delete d;
}

p2cu::DecParams params(const P2cuDecoder* d, int B) {
    const P2cuModel* m = d->m;
    p2cu::DecParams p{};
    p.embed = m->embed;
    p.wih0 = m->wih[0]; p.whh0 = m->whh[0]; p.bih0 = m->bih[0]; p.bhh0 = m->bhh[0];
    p.wih1 = m->wih[1]; p.whh1 = m->whh[1]; p.bih1 = m->bih[1]; p.bhh1 = m->bhh[1];
    p.proj = m->dproj; p.projb = m->dproj_b; p.head = m->head; p.headb = m->head_b;
    p.win_off = d->win_off;
    p.B = B;
    p.h = d->hc;
    p.c = d->hc + static_cast<size_t>(4) * B * HD;
    p.dec = d->dec;
    p.cand = d->cand;
    p.dur = d->dur;
    p.tokens = d->tokens;
    p.tok_out = d->tok_out;
    p.tok_off = d->tok_off;
    p.count = d->count;
    p.logits = d->logits;
    p.bar_count = d->bar;
    p.err = p2cu::device_error_word();
    return p;
}

// Zero the barrier's arrival count and the LSTM state of B windows (one memset: they are adjacent).
cudaError_t zero_state(const P2cuDecoder* d, int B, cudaStream_t s) {
    return cudaMemsetAsync(d->bar, 0, 256 + static_cast<size_t>(6) * B * HD * sizeof(float), s);
}

int check_model(const P2cuModel* m, const char* who) {
    if (!m) return fail_fmt(P2CU_EINVAL, "%s: NULL model", who);
    if (!m->has_dec) return fail_fmt(P2CU_EINVAL, "%s: the model was uploaded without decoder tables", who);
    return P2CU_OK;
}

}  // namespace

extern "C" {

int p2cu_decoder_create(const P2cuModel* m, int max_windows, int max_frames, P2cuDecoder** out) {
    if (!out) return fail_fmt(P2CU_EINVAL, "p2cu_decoder_create: NULL out");
    *out = nullptr;
    if (int rc = check_model(m, "p2cu_decoder_create")) return rc;
    if (max_windows < 1 || max_windows > p2cu::decoder_max_windows())
        return fail_fmt(P2CU_EINVAL, "p2cu_decoder_create: max_windows %d outside [1, %d]", max_windows,
                        p2cu::decoder_max_windows());
    if (max_frames < 1 || max_frames > (1 << 26))
        return fail_fmt(P2CU_EINVAL, "p2cu_decoder_create: max_frames %d outside [1, 2^26]", max_frames);
    auto* d = new P2cuDecoder();
    d->m = m;
    d->device = m->device;
    d->max_windows = max_windows;
    d->max_frames = max_frames;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(d->device);
    if (e != cudaSuccess) {
        delete d;
        return p2cu::cuda_error(e, "p2cu_decoder_create: cudaSetDevice");
    }
    d->grid = p2cu::decoder_max_grid(d->device);
    if (d->grid == 0 || (HD + d->grid - 1) / d->grid > p2cu::decoder_max_units()) {
        cudaSetDevice(prev);
        delete d;
        return fail_fmt(P2CU_EUNSUPPORTED, "p2cu_decoder_create: the decoder needs one %d-byte CTA on each of at "
                        "least %d SMs", p2cu::decoder_smem_bytes(148), (HD + p2cu::decoder_max_units() - 1) /
                        p2cu::decoder_max_units());
    }
    const size_t W = max_windows, F = max_frames;
    struct Slot { void** p; size_t bytes; };
    const Slot slots[] = {
        {reinterpret_cast<void**>(&d->bar), 256 + 6 * W * HD * sizeof(float)},   // barrier + h + c
        {reinterpret_cast<void**>(&d->dec), W * HD * sizeof(float)},
        {reinterpret_cast<void**>(&d->cand), 2 * static_cast<size_t>(d->grid) * W * 8},
        {reinterpret_cast<void**>(&d->dur), 2 * W * 5 * sizeof(float)},
        {reinterpret_cast<void**>(&d->logits), P2_N_LOGITS * sizeof(float)},
        {reinterpret_cast<void**>(&d->enc1), HD * sizeof(float)},
        {reinterpret_cast<void**>(&d->win_off), (W + 1) * sizeof(int)},
        {reinterpret_cast<void**>(&d->tokens), P2CU_DEC_MAX_SYMBOLS * F * 3 * sizeof(int)},
        {reinterpret_cast<void**>(&d->tok_out), P2CU_DEC_MAX_SYMBOLS * F * 3 * sizeof(int)},
        {reinterpret_cast<void**>(&d->tok_off), (W + 1) * sizeof(int)},
        {reinterpret_cast<void**>(&d->count), W * sizeof(int)},
    };
    size_t total = 0;
    for (const Slot& s : slots) total += align256(s.bytes);
    e = cudaMalloc(&d->arena, total);
    if (e == cudaSuccess) e = cudaMallocHost(&d->h_off, (W + 1) * sizeof(int));
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&d->staged, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaMemset(d->arena, 0, total);
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        destroy(d);
        return p2cu::cuda_error(e, "p2cu_decoder_create");
    }
    d->bytes = total;
    size_t off = 0;
    for (const Slot& s : slots) {
        *s.p = d->arena + off;
        off += align256(s.bytes);
    }
    d->hc = reinterpret_cast<float*>(reinterpret_cast<char*>(d->bar) + 256);
    *out = d;
    return P2CU_OK;
}

void p2cu_decoder_destroy(P2cuDecoder* d) { destroy(d); }

int p2cu_decode(P2cuDecoder* d, const float* enc, const int* n_frames, int n_windows, void* stream) {
    if (!d || !enc || !n_frames) return fail_fmt(P2CU_EINVAL, "p2cu_decode: NULL argument");
    if (n_windows < 1 || n_windows > d->max_windows)
        return fail_fmt(P2CU_EINVAL, "p2cu_decode: %d windows, the plan holds 1 to %d", n_windows, d->max_windows);
    if (reinterpret_cast<uintptr_t>(enc) % 16)
        return fail_fmt(P2CU_EINVAL, "p2cu_decode: enc is not 16-byte aligned");
    long long total = 0;
    int tmax = 0;
    for (int w = 0; w < n_windows; ++w) {
        if (n_frames[w] < 0) return fail_fmt(P2CU_EINVAL, "p2cu_decode: window %d has %d frames", w, n_frames[w]);
        total += n_frames[w];
        tmax = std::max(tmax, n_frames[w]);
    }
    if (total > d->max_frames)
        return fail_fmt(P2CU_EINVAL, "p2cu_decode: %lld frames, the plan holds %d", total, d->max_frames);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaEventSynchronize(d->staged);   // the last copy out of h_off has completed
    if (e != cudaSuccess) return p2cu::cuda_error(e, "p2cu_decode: staging");
    d->h_off[0] = 0;
    for (int w = 0; w < n_windows; ++w) d->h_off[w + 1] = d->h_off[w] + n_frames[w];
    e = cudaMemcpyAsync(d->win_off, d->h_off, (n_windows + 1) * sizeof(int), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaEventRecord(d->staged, s);
    if (e == cudaSuccess) e = zero_state(d, n_windows, s);
    if (e != cudaSuccess) return p2cu::cuda_error(e, "p2cu_decode: staging");
    p2cu::DecParams p = params(d, n_windows);
    p.mode = p2cu::DEC_DECODE;
    p.first_token = P2_BLANK;
    p.enc = enc;
    p.max_iters = 11 * tmax + 1;   // per frame at most 10 tokens and one blank
    e = p2cu::tdt_decode_launch(p, d->grid, s);
    if (e != cudaSuccess) return p2cu::cuda_error(e, "p2cu_decode: launch");
    d->n_windows = n_windows;
    return P2CU_OK;
}

int p2cu_decoder_read(P2cuDecoder* d, int* offsets, P2Token* tokens, int cap, void* stream) {
    if (!d || !offsets || (cap > 0 && !tokens)) return fail_fmt(P2CU_EINVAL, "p2cu_decoder_read: NULL argument");
    if (d->n_windows == 0) return fail_fmt(P2CU_EINVAL, "p2cu_decoder_read: nothing decoded yet");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(offsets, d->tok_off, (d->n_windows + 1) * sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) return p2cu::cuda_error(e, "p2cu_decoder_read");
    if (int rc = p2cu_check_device(stream)) return rc;
    const int n = offsets[d->n_windows];
    const int k = std::min(n, std::max(cap, 0));
    if (k > 0) {
        static_assert(sizeof(P2Token) == 3 * sizeof(int), "P2Token is id, frame, duration");
        e = cudaMemcpyAsync(tokens, d->tok_out, static_cast<size_t>(k) * sizeof(P2Token), cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return p2cu::cuda_error(e, "p2cu_decoder_read");
    }
    return n;
}

const int* p2cu_decoder_tokens(const P2cuDecoder* d) { return d ? d->tok_out : nullptr; }

const int* p2cu_decoder_offsets(const P2cuDecoder* d) { return d ? d->tok_off : nullptr; }

int p2cu_decoder_step(P2cuDecoder* d, int token_id, float* state, float* dec_out, void* stream) {
    if (!d || !state || !dec_out) return fail_fmt(P2CU_EINVAL, "p2cu_decoder_step: NULL argument");
    if (token_id < 0 || token_id >= P2_VOCAB)
        return fail_fmt(P2CU_EINVAL, "p2cu_decoder_step: token %d outside [0, %d)", token_id, P2_VOCAB);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    p2cu::DecParams p = params(d, 1);
    p.mode = p2cu::DEC_STEP;
    p.first_token = token_id;
    const size_t hb = 2 * HD * sizeof(float);   // LSTMState: h[2][640], then c[2][640]
    cudaError_t e = cudaMemsetAsync(d->bar, 0, sizeof(unsigned), s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(p.h, state, hb, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(p.c, state + 2 * HD, hb, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = p2cu::tdt_decode_launch(p, d->grid, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(state, p.h + 2 * HD, hb, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(state + 2 * HD, p.c, hb, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dec_out, p.dec, HD * sizeof(float), cudaMemcpyDeviceToDevice, s);
    return e == cudaSuccess ? P2CU_OK : p2cu::cuda_error(e, "p2cu_decoder_step");
}

int p2cu_joint(P2cuDecoder* d, const float* enc_t, const float* dec_out, float* logits, void* stream) {
    if (!d || !enc_t || !dec_out || !logits) return fail_fmt(P2CU_EINVAL, "p2cu_joint: NULL argument");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    p2cu::DecParams p = params(d, 1);
    p.mode = p2cu::DEC_JOINT;
    p.enc = d->enc1;
    cudaError_t e = cudaMemcpyAsync(d->enc1, enc_t, HD * sizeof(float), cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d->dec, dec_out, HD * sizeof(float), cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = p2cu::tdt_decode_launch(p, d->grid, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(logits, d->logits, P2_N_LOGITS * sizeof(float), cudaMemcpyDeviceToDevice, s);
    return e == cudaSuccess ? P2CU_OK : p2cu::cuda_error(e, "p2cu_joint");
}

}  // extern "C"
