// mel.cu - the log-mel front end on the device (csrc/mel.c of phonon-2-c) for a batch of audio windows.
//
// Per window of n samples (16 kHz): pre-emphasis 0.97; n / 160 frames of a 512-point STFT (hop 160, 256 zeros of
// padding on each side, a symmetric 400-tap Hann window centred in the 512); power; a 128-bin slaney mel filterbank
// (0-8 kHz); log(x + 2^-24); then per-bin normalisation over the window's frames, (x - mean) / (std + 1e-5) with the
// unbiased variance, statistics in double. Constants (window, filterbank) are built on the host in double exactly as
// the reference builds them (csrc/mel.c:65-103, 186-190) and rounded to float.
//
// The arithmetic differs from the compiled reference only in rounding: the FFT here takes exact twiddles where the
// reference advances them by a recurrence (csrc/mel.c:45-60), and logf comes from CUDA's math library. Features agree
// to ~1e-5 after normalisation (tested against the reference's own p2_mel_spectrogram).
//
// frames kernel: one CTA of 256 threads per frame (FFT in shared memory, one butterfly per thread per stage; each mel
// bin sums only its filter's nonzero bins, in increasing frequency - the order of the reference's loop, whose other
// terms are zeros). norm kernel: one CTA per (window, 32 mel bins).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>
#include <cuda_runtime.h>
#include "p2cuda.h"
#include "gemm.h"

using p2cu::fail_fmt;

namespace {

constexpr int NFFT = 512, NFREQ = NFFT / 2 + 1, WIN = 400, HOP = 160, NMEL = P2_N_MELS, SR = 16000;
constexpr float PREEMPH = 0.97f;
constexpr float LOG_GUARD = 5.9604644775390625e-08f;   // 2^-24
constexpr float NORM_EPS = 1e-5f;
constexpr int FB_MAX = 1024;                            // nonzero filterbank weights (about 2 per frequency bin)

// Device constants, built once per device: window, twiddles, the filterbank's nonzero runs.
struct MelConsts {
    float window[NFFT];
    float tw_re[NFFT / 2], tw_im[NFFT / 2];   // exp(-2 pi i k / 512)
    int fb_lo[NMEL], fb_len[NMEL], fb_off[NMEL];
    float fb_w[FB_MAX];
};

__global__ void __launch_bounds__(256) mel_frames_kernel(const float* __restrict__ audio, const long long* sample_off,
                                                         const int* frame_off, int n_windows, int n_frames,
                                                         const MelConsts* __restrict__ k, float* __restrict__ mel) {
    __shared__ float re[NFFT], im[NFFT];
    __shared__ float power[NFREQ];
    const int f = blockIdx.x;
    if (f >= n_frames) return;
    int lo = 0, hi = n_windows;   // the window holding frame f: frame_off[w] <= f < frame_off[w + 1]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (frame_off[mid] <= f) lo = mid;
        else hi = mid;
    }
    const int w = lo;
    const int fl = f - frame_off[w];                  // frame within its window
    const long long s0 = sample_off[w];
    const int n = static_cast<int>(sample_off[w + 1] - s0);
    const float* a = audio + s0;
    // windowed frame, bit-reversed into the FFT buffers: padded[p] (p = 160 fl + i) is audio sample t = p - 256 after
    // pre-emphasis (the first sample kept as is), zero outside [0, n)
    for (int i = threadIdx.x; i < NFFT; i += blockDim.x) {
        const int t = fl * HOP + i - NFFT / 2;
        float x = 0.f;
        if (t >= 0 && t < n) x = t == 0 ? a[0] : __fsub_rn(a[t], __fmul_rn(PREEMPH, a[t - 1]));
        const int r = static_cast<int>(__brev(static_cast<unsigned>(i)) >> (32 - 9));
        re[r] = __fmul_rn(x, k->window[i]);
        im[r] = 0.f;
    }
    __syncthreads();
    // radix-2 decimation in time: stage with butterflies of span `half`
    for (int half = 1; half < NFFT; half <<= 1) {
        const int b = threadIdx.x;                     // butterfly b of 256
        const int j = b & (half - 1), u = ((b - j) << 1) + j, v = u + half;
        const int ti = j * (NFFT / (2 * half));
        const float wr = k->tw_re[ti], wi = k->tw_im[ti];
        const float vr = re[v], vi = im[v];
        const float tr = __fsub_rn(__fmul_rn(vr, wr), __fmul_rn(vi, wi));
        const float tim = __fadd_rn(__fmul_rn(vr, wi), __fmul_rn(vi, wr));
        const float ur = re[u], ui = im[u];   // (u and v belong to this thread alone within the stage)
        re[v] = __fsub_rn(ur, tr);
        im[v] = __fsub_rn(ui, tim);
        re[u] = __fadd_rn(ur, tr);
        im[u] = __fadd_rn(ui, tim);
        __syncthreads();
    }
    for (int q = threadIdx.x; q < NFREQ; q += blockDim.x)
        power[q] = __fadd_rn(__fmul_rn(re[q], re[q]), __fmul_rn(im[q], im[q]));
    __syncthreads();
    if (threadIdx.x < NMEL) {
        const int m = threadIdx.x, lo = k->fb_lo[m], len = k->fb_len[m], off = k->fb_off[m];
        float v = 0.f;
        for (int q = 0; q < len; ++q) v = __fadd_rn(v, __fmul_rn(k->fb_w[off + q], power[lo + q]));
        mel[static_cast<size_t>(f) * NMEL + m] = logf(__fadd_rn(v, LOG_GUARD));
    }
}

// Per-bin normalisation of each window's frames (csrc/mel.c:197-217): mean and unbiased variance in double.
__global__ void __launch_bounds__(256) mel_norm_kernel(const int* frame_off, float* __restrict__ mel) {
    __shared__ double red[8][32];
    __shared__ float mu_s[32], inv_s[32];
    const int w = blockIdx.y, m = blockIdx.x * 32 + (threadIdx.x & 31), row = threadIdx.x >> 5;
    const int f0 = frame_off[w], nf = frame_off[w + 1] - f0;
    float* x = mel + static_cast<size_t>(f0) * NMEL;
    double s = 0.0;
    for (int f = row; f < nf; f += 8) s += x[static_cast<size_t>(f) * NMEL + m];
    red[row][threadIdx.x & 31] = s;
    __syncthreads();
    if (row == 0) {
        double t = 0.0;
        for (int r = 0; r < 8; ++r) t += red[r][threadIdx.x];
        red[0][threadIdx.x] = t / nf;   // the mean, in double
    }
    __syncthreads();
    const double mean = red[0][threadIdx.x & 31];
    __syncthreads();
    double v = 0.0;
    for (int f = row; f < nf; f += 8) {
        const double d = x[static_cast<size_t>(f) * NMEL + m] - mean;
        v += d * d;
    }
    red[row][threadIdx.x & 31] = v;
    __syncthreads();
    if (row == 0) {
        double t = 0.0;
        for (int r = 0; r < 8; ++r) t += red[r][threadIdx.x];
        const float sd = static_cast<float>(sqrt(t / (nf - 1)));
        inv_s[threadIdx.x] = __fdiv_rn(1.0f, __fadd_rn(sd, NORM_EPS));
        mu_s[threadIdx.x] = static_cast<float>(mean);
    }
    __syncthreads();
    const float mu = mu_s[threadIdx.x & 31], inv = inv_s[threadIdx.x & 31];
    for (int f = row; f < nf; f += 8) {
        float* p = x + static_cast<size_t>(f) * NMEL + m;
        *p = __fmul_rn(__fsub_rn(*p, mu), inv);
    }
}

// The reference's constants (csrc/mel.c:65-103, 186-190), in double, rounded to float.
double hz_to_mel(double hz) { return hz < 1000.0 ? hz * 3.0 / 200.0 : 15.0 + 27.0 * std::log(hz / 1000.0) / std::log(6.4); }
double mel_to_hz(double m) { return m < 15.0 ? m * 200.0 / 3.0 : 1000.0 * std::exp((m - 15.0) * std::log(6.4) / 27.0); }

bool build_consts(MelConsts* c) {
    memset(c, 0, sizeof(*c));
    const int off = (NFFT - WIN) / 2;
    for (int i = 0; i < WIN; ++i)
        c->window[off + i] = static_cast<float>(0.5 - 0.5 * std::cos(2.0 * M_PI * i / (WIN - 1)));
    for (int q = 0; q < NFFT / 2; ++q) {
        const double ang = -2.0 * M_PI * q / NFFT;
        c->tw_re[q] = static_cast<float>(std::cos(ang));
        c->tw_im[q] = static_cast<float>(std::sin(ang));
    }
    const double mel_lo = hz_to_mel(0.0), mel_hi = hz_to_mel(SR / 2.0);
    double mels[NMEL + 2];
    for (int i = 0; i < NMEL + 2; ++i) mels[i] = mel_to_hz(mel_lo + (mel_hi - mel_lo) * i / (NMEL + 1));
    int used = 0;
    for (int m = 0; m < NMEL; ++m) {
        const double lo = mels[m], center = mels[m + 1], hi = mels[m + 2], norm = 2.0 / (hi - lo);
        int first = -1, last = -1;
        float w[NFREQ];
        for (int q = 0; q < NFREQ; ++q) {
            const double hz = static_cast<double>(SR) * q / NFFT;
            double val = 0.0;
            if (hz >= lo && hz <= center) val = (hz - lo) / (center - lo);
            else if (hz > center && hz <= hi) val = (hi - hz) / (hi - center);
            w[q] = static_cast<float>(val * norm);
            if (w[q] != 0.f) {
                if (first < 0) first = q;
                last = q;
            }
        }
        if (first < 0) first = last = 0;   // an empty filter: one zero weight
        const int len = last - first + 1;
        if (used + len > FB_MAX) return false;
        c->fb_lo[m] = first;
        c->fb_len[m] = len;
        c->fb_off[m] = used;
        for (int q = 0; q < len; ++q) c->fb_w[used + q] = w[first + q];   // zeros inside the run kept: same sum
        used += len;
    }
    return true;
}

}  // namespace

struct P2cuMel {
    int device = 0, max_windows = 0;
    long long max_samples = 0;
    MelConsts* consts = nullptr;      // device
    long long* sample_off = nullptr;  // device [max_windows + 1]
    int* frame_off = nullptr;         // device [max_windows + 1]
    std::vector<long long> h_soff;
    std::vector<int> h_foff;
};

extern "C" {

int p2cu_mel_create(int max_windows, long long max_samples, P2cuMel** out) {
    if (!out) return fail_fmt(P2CU_EINVAL, "p2cu_mel_create: NULL out");
    *out = nullptr;
    if (max_windows < 1 || max_samples < 2 * HOP)
        return fail_fmt(P2CU_EINVAL, "p2cu_mel_create: %d windows, %lld samples", max_windows, max_samples);
    MelConsts h;
    if (!build_consts(&h)) return fail_fmt(P2CU_EUNSUPPORTED, "p2cu_mel_create: filterbank larger than expected");
    auto* d = new P2cuMel();
    cudaGetDevice(&d->device);
    d->max_windows = max_windows;
    d->max_samples = max_samples;
    cudaError_t e = cudaMalloc(&d->consts, sizeof(MelConsts));
    if (e == cudaSuccess) e = cudaMalloc(&d->sample_off, (max_windows + 1) * sizeof(long long));
    if (e == cudaSuccess) e = cudaMalloc(&d->frame_off, (max_windows + 1) * sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpy(d->consts, &h, sizeof(h), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(d->consts);
        cudaFree(d->sample_off);
        cudaFree(d->frame_off);
        delete d;
        return p2cu::cuda_error(e, "p2cu_mel_create");
    }
    *out = d;
    return P2CU_OK;
}

void p2cu_mel_destroy(P2cuMel* d) {
    if (!d) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(d->device);
    cudaFree(d->consts);
    cudaFree(d->sample_off);
    cudaFree(d->frame_off);
    cudaSetDevice(prev);
    delete d;
}

int p2cu_mel_frames(long long n_samples) { return static_cast<int>(n_samples / HOP); }

int p2cu_mel_run(P2cuMel* d, const float* audio, const long long* n_samples, int n_windows, float* mel,
                 void* stream) {
    if (!d || !audio || !n_samples || !mel) return fail_fmt(P2CU_EINVAL, "p2cu_mel_run: NULL argument");
    if (n_windows < 1 || n_windows > d->max_windows)
        return fail_fmt(P2CU_EINVAL, "p2cu_mel_run: %d windows, the plan holds 1 to %d", n_windows, d->max_windows);
    d->h_soff.assign(n_windows + 1, 0);
    d->h_foff.assign(n_windows + 1, 0);
    for (int w = 0; w < n_windows; ++w) {
        const int nf = static_cast<int>(n_samples[w] / HOP);
        if (nf < 2) return fail_fmt(P2CU_EINVAL, "p2cu_mel_run: window %d: audio too short: %lld samples", w,
                                    n_samples[w]);
        d->h_soff[w + 1] = d->h_soff[w] + n_samples[w];
        d->h_foff[w + 1] = d->h_foff[w] + nf;
    }
    if (d->h_soff[n_windows] > d->max_samples)
        return fail_fmt(P2CU_EINVAL, "p2cu_mel_run: %lld samples, the plan holds %lld", d->h_soff[n_windows],
                        d->max_samples);
    const int nf = d->h_foff[n_windows];
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // pageable sources: these copies complete before the calls return, so the host tables may change afterwards
    cudaError_t e = cudaMemcpyAsync(d->sample_off, d->h_soff.data(), (n_windows + 1) * sizeof(long long),
                                    cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d->frame_off, d->h_foff.data(), (n_windows + 1) * sizeof(int), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return p2cu::cuda_error(e, "p2cu_mel_run: tables");
    mel_frames_kernel<<<nf, 256, 0, s>>>(audio, d->sample_off, d->frame_off, n_windows, nf, d->consts, mel);
    mel_norm_kernel<<<dim3(NMEL / 32, n_windows), 256, 0, s>>>(d->frame_off, mel);
    e = cudaGetLastError();
    return e == cudaSuccess ? P2CU_OK : p2cu::cuda_error(e, "p2cu_mel_run");
}

}  // extern "C"
