// segment.cu - the energy measures of phonon-2-c's segmenter (csrc/segment.c) with the block RMS on the device, and
// the decisions the reference takes from them, restated on the host: where a window of long audio ends (the longest
// pause in the last 10 s before the maximum length), where a window that went quiet is split (the longest pause in its
// middle third), and whether a decoded window went quiet over speech (csrc/engine.c:213-251).
//
// Block RMS: blocks of 50 ms (800 samples at 16 kHz) aligned to the window's start, zero-padded at its end,
// rms = sqrt(sum x^2 / block) with the sum in double (csrc/segment.c:36-48). One warp per block: each lane sums every
// 32nd sample (x*x is exact in double, so the sum differs from the reference's loop only in the order of its double
// additions, ~1e-16 relative - far below the float the value is rounded to). The kernel reads each sample once:
// HBM-bound, 4 bytes per sample.
//
// The decisions read only block RMS values and integer sample positions, so they are restated exactly: the same
// comparisons in the same float and integer arithmetic as csrc/segment.c:50-184 and csrc/engine.c:224-251.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>
#include <cuda_runtime.h>
#include "p2cuda.h"
#include "gemm.h"

using p2cu::fail_fmt;

namespace {

// csrc/segment.c:27-32
constexpr double WINDOW_MAX_S = 35.0, WINDOW_BAND_S = 10.0, WINDOW_BLOCK_S = 0.05;
constexpr float WINDOW_FLOOR_RMS = 0.004f, WINDOW_GATE_RATIO = 0.18f, SPEECH_FLOOR_RATIO = 3.0f;
// csrc/engine.c:213-223
constexpr double DROPOUT_S = 2.0;
constexpr float DROPOUT_SPEECH = 0.40f, DROPOUT_TONE = 0.90f;

int block_of(int sample_rate) { return static_cast<int>(WINDOW_BLOCK_S * sample_rate); }

double window_max_seconds() {   // csrc/segment.c:75-83: P2_WINDOW_MAX moves the band, if at least 15 s
    const char* env = getenv("P2_WINDOW_MAX");
    if (env && *env) {
        const double v = atof(env);
        if (v >= WINDOW_BAND_S + 5.0) return v;
    }
    return WINDOW_MAX_S;
}

// The gate for a stretch of blocks: 0.18 of its peak, never below the room-tone floor.
float gate_for(const float* rms, int b_from, int b_to) {
    float peak = 0.0f;
    for (int b = b_from; b < b_to; ++b) peak = rms[b] > peak ? rms[b] : peak;
    const float gate = WINDOW_GATE_RATIO * peak;
    return gate < WINDOW_FLOOR_RMS ? WINDOW_FLOOR_RMS : gate;
}

// The middle (in samples) of the longest run of blocks at or under `gate` inside [b0, b1); of equally long runs the
// one whose middle is nearest `target` (the first of equally near ones); -1 when no block is that quiet.
int quiet_cut(const float* rms, int b0, int b1, int block, float gate, int target) {
    int cut = -1, best_len = 0, best_dist = 0;
    int i = b0;
    while (i < b1) {
        if (rms[i] > gate) {
            ++i;
            continue;
        }
        int j = i;
        while (j < b1 && rms[j] <= gate) ++j;
        if (j == i) {   // a NaN block: neither loud nor quiet (the callers pass finite audio)
            ++i;
            continue;
        }
        const int mid = static_cast<int>((static_cast<long long>(i) + j) * block / 2);
        const int run = j - i, dist = std::abs(mid - target);
        if (run > best_len || (run == best_len && dist < best_dist)) {
            best_len = run;
            best_dist = dist;
            cut = mid;
        }
        i = j;
    }
    return cut;
}

// ---- device: block RMS of many windows in one launch ----------------------------------------------------------------

constexpr int SPANS_PER_LAUNCH = 1024;
constexpr int RMS_WARPS = 8;

struct RmsSpans {   // passed by value (16 KB of kernel parameters)
    long long start[SPANS_PER_LAUNCH];
    int len[SPANS_PER_LAUNCH];
    int first[SPANS_PER_LAUNCH + 1];   // output index of each span's block 0; first[n] = total blocks
    int n, block;
};

__global__ void __launch_bounds__(RMS_WARPS * 32) block_rms_kernel(const float* __restrict__ audio,
                                                                   const __grid_constant__ RmsSpans sp,
                                                                   float* __restrict__ out) {
    const int w = blockIdx.x * RMS_WARPS + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (w >= sp.first[sp.n]) return;
    int lo = 0, hi = sp.n - 1;   // the span holding block w: the last with first <= w
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (sp.first[mid] <= w) lo = mid;
        else hi = mid - 1;
    }
    const int b = w - sp.first[lo];
    const int i0 = b * sp.block, i1 = min(i0 + sp.block, sp.len[lo]);
    const float* x = audio + sp.start[lo];
    double acc = 0.0;
    for (int i = i0 + lane; i < i1; i += 32) {
        const double v = x[i];
        acc = fma(v, v, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) out[w] = static_cast<float>(sqrt(acc / sp.block));
}

}  // namespace

extern "C" {

int p2cu_seg_block(int sample_rate) { return block_of(sample_rate); }

int p2cu_seg_blocks(int n_samples, int sample_rate) {
    const int block = block_of(sample_rate);
    return n_samples > 0 && block > 0 ? (n_samples + block - 1) / block : 0;
}

int p2cu_seg_window_max_samples(int sample_rate) { return static_cast<int>(window_max_seconds() * sample_rate); }

int p2cu_block_rms(const float* audio, const long long* starts, const int* lens, int n_windows, int sample_rate,
                   float* rms, void* stream) {
    if (!audio || !starts || !lens || !rms || n_windows < 0) return fail_fmt(P2CU_EINVAL, "p2cu_block_rms: NULL argument");
    const int block = block_of(sample_rate);
    if (block < 1) return fail_fmt(P2CU_EINVAL, "p2cu_block_rms: sample rate %d", sample_rate);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    long long out_at = 0;
    for (int w0 = 0; w0 < n_windows; w0 += SPANS_PER_LAUNCH) {
        RmsSpans sp;
        sp.n = std::min(SPANS_PER_LAUNCH, n_windows - w0);
        sp.block = block;
        long long total = 0;
        for (int i = 0; i < sp.n; ++i) {
            if (lens[w0 + i] < 0 || starts[w0 + i] < 0)
                return fail_fmt(P2CU_EINVAL, "p2cu_block_rms: window %d: start %lld, %d samples", w0 + i,
                                starts[w0 + i], lens[w0 + i]);
            sp.start[i] = starts[w0 + i];
            sp.len[i] = lens[w0 + i];
            sp.first[i] = static_cast<int>(total);
            total += (lens[w0 + i] + block - 1) / block;
            if (total > (1LL << 30)) return fail_fmt(P2CU_EINVAL, "p2cu_block_rms: too many blocks in one call");
        }
        sp.first[sp.n] = static_cast<int>(total);
        if (total > 0) {
            const int grid = static_cast<int>((total + RMS_WARPS - 1) / RMS_WARPS);
            block_rms_kernel<<<grid, RMS_WARPS * 32, 0, s>>>(audio, sp, rms + out_at);
            const cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) return fail_fmt(P2CU_ECUDA, "p2cu_block_rms: %s", cudaGetErrorString(e));
        }
        out_at += total;
    }
    return P2CU_OK;
}

// csrc/segment.c:90-118. rms: the block RMS of the first min(n_samples, window max) samples.
int p2cu_seg_first_cut(const float* rms, int n_blocks, int n_samples, int sample_rate) {
    const double max_s = window_max_seconds();
    const int single = static_cast<int>(max_s * sample_rate);
    const int lo = static_cast<int>((max_s - WINDOW_BAND_S) * sample_rate);
    const int target = static_cast<int>((max_s - WINDOW_BAND_S / 2) * sample_rate);
    if (n_samples <= single) return n_samples;
    const int block = block_of(sample_rate);
    if (!rms || n_blocks < (single + block - 1) / block) return -1;
    const int b0 = (lo + block - 1) / block;   // first block fully inside the band
    const int b1 = single / block;             // one past the last block inside it
    int cut = quiet_cut(rms, b0, b1, block, gate_for(rms, 0, b1), target);
    if (cut < 0) cut = target;
    if (cut < lo) cut = lo;
    if (cut > single) cut = single;
    return cut;
}

// csrc/segment.c:142-151. rms: the window's block RMS (n_blocks = its ceil(n_samples / block)).
int p2cu_seg_split_point(const float* rms, int n_blocks, int n_samples, int sample_rate) {
    const int block = block_of(sample_rate);
    if (!rms) return n_samples / 2;
    const int b0 = (n_samples / 3 + block - 1) / block, b1 = (2 * n_samples / 3) / block;
    const int cut = quiet_cut(rms, b0, std::min(b1, n_blocks), block, gate_for(rms, 0, n_blocks), n_samples / 2);
    return cut < 0 ? n_samples / 2 : cut;
}

// csrc/segment.c:165-177: three times the 10th-percentile block RMS, never under the floor.
float p2cu_seg_speech_gate(const float* rms, int n_blocks) {
    if (n_blocks <= 0) return WINDOW_FLOOR_RMS;
    std::vector<float> v(rms, rms + n_blocks);
    std::nth_element(v.begin(), v.begin() + n_blocks / 10, v.end());
    const float gate = SPEECH_FLOOR_RATIO * v[n_blocks / 10];
    return gate < WINDOW_FLOOR_RMS ? WINDOW_FLOOR_RMS : gate;
}

// csrc/segment.c:179-184: the share of the blocks over samples [from, to) above `gate`.
float p2cu_seg_speech_share(const float* rms, int n_blocks, int sample_rate, int from, int to, float gate) {
    if (to <= from || n_blocks <= 0) return 0.0f;
    const int block = block_of(sample_rate);
    const int b0 = from / block;
    int b1 = (to + block - 1) / block, loud = 0;
    if (b1 > n_blocks) b1 = n_blocks;
    for (int b = b0; b < b1; ++b) loud += rms[b] > gate;
    return b1 > b0 ? static_cast<float>(loud) / (b1 - b0) : 0.0f;
}

// The first stretch of at least 2 s between tokens (from the window's start, between one token's end and the next
// token, or from the last token to the window's end), as csrc/engine.c:230-248 walks them: 1 and its bounds, else 0.
// Needs no RMS: a window without such a stretch cannot have gone quiet.
int p2cu_seg_long_gap(const P2Token* toks, int n_toks, int n_samples) {
    const int frame = P2_HOP_LEN * P2_SUB_FACTOR, min_gap = static_cast<int>(DROPOUT_S * P2_SAMPLE_RATE);
    int prev = 0;
    for (int i = 0; i <= n_toks; ++i) {
        int cur = i < n_toks ? toks[i].frame * frame : n_samples;
        if (cur > n_samples) cur = n_samples;
        if (cur - prev >= min_gap) return 1;
        if (i < n_toks) prev = cur + (toks[i].duration > 0 ? toks[i].duration : 1) * frame;
    }
    return 0;
}

// csrc/engine.c:224-251: whether the window went quiet over speech - a stretch of at least 2 s with no token whose
// speech share (blocks above three times the window's 10th-percentile RMS) is in [0.40, 0.90]; the first such
// stretch's bounds and share go to *gap_from, *gap_to, *speech. rms: the window's block RMS at 16 kHz.
int p2cu_seg_dropped_out(const float* rms, int n_blocks, int n_samples, const P2Token* toks, int n_toks,
                         int* gap_from, int* gap_to, float* speech) {
    const int frame = P2_HOP_LEN * P2_SUB_FACTOR, min_gap = static_cast<int>(DROPOUT_S * P2_SAMPLE_RATE);
    bool have_gate = false;
    float gate = 0.0f;
    int prev = 0;
    for (int i = 0; i <= n_toks; ++i) {
        int cur = i < n_toks ? toks[i].frame * frame : n_samples;
        if (cur > n_samples) cur = n_samples;
        if (cur - prev >= min_gap) {
            if (!have_gate) {
                if (!rms || n_blocks <= 0) return 0;   // the reference skips the check without an energy profile
                gate = p2cu_seg_speech_gate(rms, n_blocks);
                have_gate = true;
            }
            const float s = p2cu_seg_speech_share(rms, n_blocks, P2_SAMPLE_RATE, prev, cur, gate);
            if (s >= DROPOUT_SPEECH && s <= DROPOUT_TONE) {
                if (gap_from) *gap_from = prev;
                if (gap_to) *gap_to = cur;
                if (speech) *speech = s;
                return 1;
            }
        }
        if (i < n_toks) prev = cur + (toks[i].duration > 0 ? toks[i].duration : 1) * frame;
    }
    return 0;
}

}  // extern "C"
