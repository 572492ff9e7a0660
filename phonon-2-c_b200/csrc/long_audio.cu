// long_audio.cu - long audio as phonon-2-c's engine transcribes it (csrc/engine.c:253-357), scheduled in batches.
//
// The reference cuts audio longer than 35 s into pause-aligned windows (csrc/segment.c:120-140), decodes each window
// on its own, and re-decodes a window that went quiet over speech as two halves split at its longest pause, at most
// two levels deep (csrc/engine.c:253-292) - one window after another, depth first. Here every window of one split
// depth goes through log-mel, encoder and decoder as one batch spread over the GPUs (p2_b200_transcribe_audio_windows'
// machinery), the quiet ones are found on the host from block RMS computed on the device, and their halves form the
// next batch. The decisions are the reference's (segment.cu), so the same windows come out with the same tokens; they
// are returned in the order the reference's recursion appends them, which is the order of their start samples (the
// halves of a window tile it, left before right).
//
// The audio goes to the first GPU once, for the block RMS of the planning (one small launch per planned window: each
// cut depends on the one before) and of the dropout checks (one launch per split depth).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>
#include <cuda_runtime.h>
#include "p2cuda.h"

extern "C" {
int p2b_thread_device(void);   // blas_host.c
int p2b_transcribe_slices(const P2Model* m, const float* audio, const long long* starts, const long long* n_samples,
                          int n_windows, const int* devices, int n_devices, P2Token** tokens, int* n_tokens,
                          int* enc_frames);   // host_entry.cu
}

namespace {

constexpr int SPLIT_MAX_DEPTH = 2;                               // csrc/engine.c:221-222
constexpr double SPLIT_MIN_S = 6.0;
constexpr int MIN_DECODE = P2_SUB_FACTOR * P2_HOP_LEN;           // under 80 ms nothing is decoded (engine.c:259)

bool env_enabled(const char* name) {   // csrc/engine.c:201-205: on unless "0..." or "off"
    const char* env = getenv(name);
    return !(env && (env[0] == '0' || strcmp(env, "off") == 0));
}

// The audio on one GPU and the buffers of the block RMS calls.
struct DeviceAudio {
    int device = -1;
    cudaStream_t stream = nullptr;
    float* audio = nullptr;
    float* rms = nullptr;
    size_t rms_cap = 0;
    std::vector<float> host_rms;
    std::string err;

    ~DeviceAudio() {
        if (device < 0) return;
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        cudaFree(audio);
        cudaFree(rms);
        if (stream) cudaStreamDestroy(stream);
        cudaSetDevice(prev);
    }

    bool fail(const std::string& what) {
        err = what;
        return false;
    }

    bool upload(int dev, const float* x, int n) {
        device = dev;
        if (cudaSetDevice(dev) != cudaSuccess) return fail("cannot use GPU " + std::to_string(dev));
        if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess)
            return fail("cannot create a CUDA stream");
        if (cudaMalloc(&audio, static_cast<size_t>(std::max(n, 1)) * sizeof(float)) != cudaSuccess)
            return fail("out of device memory for the audio");
        if (n > 0 && cudaMemcpyAsync(audio, x, static_cast<size_t>(n) * sizeof(float), cudaMemcpyHostToDevice,
                                     stream) != cudaSuccess)
            return fail("audio copy failed");
        return true;
    }

    // Block RMS of windows [starts[i], starts[i] + lens[i]) into host_rms, window i's blocks from offs[i].
    bool block_rms(const std::vector<long long>& starts, const std::vector<int>& lens, std::vector<size_t>& offs) {
        offs.assign(lens.size() + 1, 0);
        for (size_t i = 0; i < lens.size(); ++i)
            offs[i + 1] = offs[i] + static_cast<size_t>(p2cu_seg_blocks(lens[i], P2_SAMPLE_RATE));
        const size_t total = offs.back();
        if (cudaSetDevice(device) != cudaSuccess) return fail("cannot use GPU " + std::to_string(device));
        if (total > rms_cap) {
            cudaFree(rms);
            rms = nullptr;
            rms_cap = 0;
            if (cudaMalloc(&rms, total * sizeof(float)) != cudaSuccess) return fail("out of device memory");
            rms_cap = total;
        }
        host_rms.resize(std::max<size_t>(total, 1));
        if (total == 0) return true;
        if (p2cu_block_rms(audio, starts.data(), lens.data(), static_cast<int>(lens.size()), P2_SAMPLE_RATE, rms,
                           stream) != P2CU_OK)
            return fail(p2cu_last_error());
        if (cudaMemcpyAsync(host_rms.data(), rms, total * sizeof(float), cudaMemcpyDeviceToHost, stream) !=
                cudaSuccess ||
            cudaStreamSynchronize(stream) != cudaSuccess)
            return fail(std::string("block RMS: ") + cudaGetErrorString(cudaGetLastError()));
        return true;
    }
};

// csrc/segment.c:120-140: windows up to the maximum length, each ending at the cut p2cu_seg_first_cut picks from the
// block RMS of the maximum length that follows its start. False on a device error.
bool plan_windows(DeviceAudio& da, int n, std::vector<P2Window>& out) {
    out.clear();
    const int single = p2cu_seg_window_max_samples(P2_SAMPLE_RATE);
    std::vector<size_t> offs;
    int start = 0;
    for (;;) {
        int cut = n - start;
        if (n - start > single) {
            if (!da.block_rms({start}, {single}, offs)) return false;
            cut = p2cu_seg_first_cut(da.host_rms.data(), static_cast<int>(offs[1]), n - start, P2_SAMPLE_RATE);
            if (cut < 0) return da.fail("window planning failed");
        }
        out.push_back({start, start + cut});
        if (start + cut >= n) break;
        start += cut;
    }
    return true;
}

struct Node {
    int start, end, depth;
};

}  // namespace

extern "C" {

__attribute__((visibility("default"))) int p2_b200_plan_windows(const float* audio, int n_samples, int sample_rate,
                                                                P2Window** out) {
    if (!out) return 0;
    *out = nullptr;
    if (n_samples <= 0 || sample_rate != P2_SAMPLE_RATE || !audio) {
        if (n_samples > 0 && sample_rate > 0 && sample_rate != P2_SAMPLE_RATE)
            fprintf(stderr, "p2_b200_plan_windows: %d Hz audio (16 kHz expected)\n", sample_rate);
        return 0;
    }
    DeviceAudio da;
    std::vector<P2Window> w;
    if (!da.upload(p2b_thread_device(), audio, n_samples) || !plan_windows(da, n_samples, w)) {
        fprintf(stderr, "p2_b200_plan_windows: %s\n", da.err.c_str());
        return 0;
    }
    *out = static_cast<P2Window*>(malloc(w.size() * sizeof(P2Window)));
    if (!*out) return 0;
    memcpy(*out, w.data(), w.size() * sizeof(P2Window));
    return static_cast<int>(w.size());
}

__attribute__((visibility("default"))) int p2_b200_split_point(const float* audio, int n_samples, int sample_rate) {
    if (!audio || n_samples <= 0 || sample_rate != P2_SAMPLE_RATE) return n_samples / 2;
    DeviceAudio da;
    std::vector<size_t> offs;
    if (!da.upload(p2b_thread_device(), audio, n_samples) || !da.block_rms({0}, {n_samples}, offs)) {
        fprintf(stderr, "p2_b200_split_point: %s\n", da.err.c_str());
        return n_samples / 2;
    }
    return p2cu_seg_split_point(da.host_rms.data(), static_cast<int>(offs[1]), n_samples, sample_rate);
}

__attribute__((visibility("default"))) void p2_b200_windows_free(P2B200Window* w, int n) {
    if (!w) return;
    for (int i = 0; i < n; ++i) free(w[i].tokens);
    free(w);
}

__attribute__((visibility("default"))) int p2_b200_transcribe_long(const P2Model* m, const float* audio, int n_samples,
                                                                   const int* devices, int n_devices,
                                                                   P2B200Window** out, int* n_out,
                                                                   long long* encoder_frames) {
    const char* who = "p2_b200_transcribe_long";
    if (!m || !out || !n_out || n_samples < 0 || (n_samples > 0 && !audio) || n_devices < 0 ||
        (n_devices > 0 && !devices)) {
        fprintf(stderr, "%s: bad arguments\n", who);
        return -1;
    }
    *out = nullptr;
    *n_out = 0;
    if (encoder_frames) *encoder_frames = 0;
    // non-finite samples become zeros, as the reference's engine does before anything else (csrc/engine.c:295-309)
    std::vector<float> cleaned;
    const float* x = audio;
    for (int i = 0; i < n_samples; ++i)
        if (!std::isfinite(audio[i])) {
            cleaned.assign(audio, audio + n_samples);
            for (float& v : cleaned) v = std::isfinite(v) ? v : 0.0f;
            x = cleaned.data();
            break;
        }

    int first_dev = 0;
    if (n_devices > 0) {
        first_dev = devices[0];
    } else {
        int count = 0;
        if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
            fprintf(stderr, "%s: no CUDA device\n", who);
            return -1;
        }
    }
    int prev = 0;
    cudaGetDevice(&prev);
    DeviceAudio da;
    std::vector<Node> level;
    const bool redecode = env_enabled("P2_REDECODE");
    if (env_enabled("P2_SEGMENT")) {
        std::vector<P2Window> w;
        if (n_samples > 0 && (!da.upload(first_dev, x, n_samples) || !plan_windows(da, n_samples, w))) {
            fprintf(stderr, "%s: %s\n", who, da.err.c_str());
            cudaSetDevice(prev);
            return -1;
        }
        for (const P2Window& v : w) level.push_back({v.start, v.end, 0});
    } else {   // the whole audio as one window, never re-decoded (csrc/engine.c:336-341)
        level.push_back({0, n_samples, SPLIT_MAX_DEPTH});
    }

    std::vector<P2B200Window> leaves;
    auto drop_all = [&] {
        for (P2B200Window& l : leaves) free(l.tokens);
        leaves.clear();
    };
    long long frames_total = 0;
    int rc = 0;
    while (rc == 0 && !level.empty()) {
        const int nl = static_cast<int>(level.size());
        std::vector<P2Token*> toks(nl, nullptr);
        std::vector<int> counts(nl, 0), frames(nl, 0);
        // one batch: every window of this depth long enough to frame
        std::vector<long long> st, ln;
        std::vector<int> which;
        for (int i = 0; i < nl; ++i)
            if (level[i].end - level[i].start >= MIN_DECODE) {
                which.push_back(i);
                st.push_back(level[i].start);
                ln.push_back(level[i].end - level[i].start);
            }
        if (!which.empty()) {
            const int nb = static_cast<int>(which.size());
            std::vector<P2Token*> bt(nb, nullptr);
            std::vector<int> bc(nb, 0), bf(nb, 0);
            rc = p2b_transcribe_slices(m, x, st.data(), ln.data(), nb, devices, n_devices, bt.data(), bc.data(),
                                       bf.data());
            for (int k = 0; k < nb; ++k) {
                toks[which[k]] = bt[k];
                counts[which[k]] = bc[k];
                frames[which[k]] = bf[k];
                frames_total += bf[k];
            }
        }
        // the dropout checks of the windows that may still be split
        std::vector<int> cand;
        std::vector<long long> cst;
        std::vector<int> clen;
        if (rc == 0 && redecode)
            for (int i = 0; i < nl; ++i) {
                const int len = level[i].end - level[i].start;
                if (level[i].depth < SPLIT_MAX_DEPTH && len >= 2 * SPLIT_MIN_S * P2_SAMPLE_RATE &&
                    p2cu_seg_long_gap(toks[i], counts[i], len)) {
                    cand.push_back(i);
                    cst.push_back(level[i].start);
                    clen.push_back(len);
                }
            }
        std::vector<int> split_at(nl, -1);
        if (!cand.empty()) {
            std::vector<size_t> offs;
            if (!da.audio && !da.upload(first_dev, x, n_samples)) {
                rc = -1;
            } else if (!da.block_rms(cst, clen, offs)) {
                rc = -1;
            } else {
                for (size_t c = 0; c < cand.size(); ++c) {
                    const int i = cand[c];
                    const float* r = da.host_rms.data() + offs[c];
                    const int nb = static_cast<int>(offs[c + 1] - offs[c]);
                    if (p2cu_seg_dropped_out(r, nb, clen[c], toks[i], counts[i], nullptr, nullptr, nullptr))
                        split_at[i] = level[i].start + p2cu_seg_split_point(r, nb, clen[c], P2_SAMPLE_RATE);
                }
            }
            if (rc != 0) fprintf(stderr, "%s: %s\n", who, da.err.c_str());
        }
        std::vector<Node> next;
        for (int i = 0; i < nl; ++i) {
            if (rc == 0 && split_at[i] >= 0) {
                free(toks[i]);
                next.push_back({level[i].start, split_at[i], level[i].depth + 1});
                next.push_back({split_at[i], level[i].end, level[i].depth + 1});
            } else {
                leaves.push_back({level[i].start, level[i].end, level[i].depth, frames[i], toks[i], counts[i]});
            }
        }
        level.swap(next);
    }
    cudaSetDevice(prev);
    if (rc != 0) {
        drop_all();
        return -1;
    }
    std::stable_sort(leaves.begin(), leaves.end(),
                     [](const P2B200Window& a, const P2B200Window& b) { return a.start < b.start; });
    if (!leaves.empty()) {
        *out = static_cast<P2B200Window*>(malloc(leaves.size() * sizeof(P2B200Window)));
        if (!*out) {
            drop_all();
            fprintf(stderr, "%s: out of host memory\n", who);
            return -1;
        }
        memcpy(*out, leaves.data(), leaves.size() * sizeof(P2B200Window));
    }
    *n_out = static_cast<int>(leaves.size());
    if (encoder_frames) *encoder_frames = frames_total;
    return 0;
}

}  // extern "C"
