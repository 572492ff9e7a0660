// host_entry.cu - phonon-2-c's encoder and decoder entry points on host pointers (include/phonon2.h): p2_encoder,
// p2_encoder_chunked, p2_verbose (the drop-in for csrc/encoder.c), p2_decoder_step, p2_joint, p2_greedy_decode (for
// csrc/decoder.c), and the batched p2_b200_encode_windows / p2_b200_transcribe_windows.
//
// The model's weights are uploaded to the calling thread's GPU the first time a P2Model is seen there and found again
// by its address (the reference's weights are read-only for the model's life, csrc/phonon2.h:204-205); the inputs go
// up, one graph launch runs the whole encoder (one cooperative launch the whole decode), the results come back. Each
// host thread keeps its last plans (buffers and captured graph for one length and mode) and a stream of its own, so
// concurrent callers on one model do not share buffers (the reference allows concurrent p2_transcribe calls on one
// engine, csrc/phonon2.h:277-279).
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <numeric>
#include <string>
#include <thread>
#include <vector>
#include <cuda_runtime.h>
#include "p2cuda.h"

extern "C" {
int p2b_gemm_mode(void);       // blas_host.c
int p2b_thread_device(void);   // blas_host.c
int p2cu_encoder_create_lazy(const P2cuModel* m, const int* n_frames, int n_windows, int mode, int chunk_frames,
                             int chunk_overlap, P2cuEncoder** out);   // encoder.cu
}

extern "C" {
__attribute__((visibility("default"))) int p2_verbose = 1;
}

namespace {

struct ModelEntry {
    const P2Model* key;
    int device;
    uint64_t print;
    P2cuModel* dev;
};

std::mutex g_mu;
std::vector<ModelEntry> g_models;

uint64_t mix(uint64_t h, uint64_t v) { return (h ^ v) * 0x100000001b3ull; }

// A fingerprint of the model: its weight pointers and the first bytes of two of its planes, to notice a P2Model
// address reused for other weights.
uint64_t fingerprint(const P2Model* m) {
    uint64_t h = 0xcbf29ce484222325ull;
    const Weight* ws[] = {&m->enc.subsampling.linear_w, &m->enc.blocks[0].ff1.linear1_w,
                          &m->enc.blocks[P2_N_BLOCKS - 1].ff2.linear2_w, &m->enc.projector_w};
    for (const Weight* w : ws) {
        h = mix(h, reinterpret_cast<uintptr_t>(w->signs));
        h = mix(h, reinterpret_cast<uintptr_t>(w->q8));
        h = mix(h, reinterpret_cast<uintptr_t>(w->f32));
    }
    h = mix(h, reinterpret_cast<uintptr_t>(m->dec.embed_w));
    h = mix(h, reinterpret_cast<uintptr_t>(m->dec.head_w));
    const Weight& a = m->enc.blocks[0].ff1.linear1_w;
    if (a.kind == P2_W_FV && a.signs)
        for (int i = 0; i < 64; ++i) h = mix(h, a.signs[i]);
    if (m->enc.subsampling.conv0_w)
        for (int i = 0; i < 16; ++i) {
            uint32_t bits;
            memcpy(&bits, m->enc.subsampling.conv0_w + i, 4);
            h = mix(h, bits);
        }
    return h;
}

int env_int(const char* name, int fallback) {   // csrc/encoder.c:647-655
    const char* v = getenv(name);
    if (!v || !*v) return fallback;
    char* end;
    const long n = strtol(v, &end, 10);
    return (*end == '\0' && n > 0) ? static_cast<int>(n) : fallback;
}

bool should_chunk(int Tp) {   // csrc/encoder.c:715-723
    const char* env = getenv("P2_CHUNK");
    if (env) {
        if (env[0] == '0' || strcmp(env, "off") == 0) return false;
        if (env[0] == '1' || strcmp(env, "on") == 0) return true;
    }
    return Tp > 500;
}

struct ThreadCtx {
    int device = -1;
    cudaStream_t stream = nullptr;
    P2cuEncoder* plan = nullptr;
    const P2cuModel* plan_model = nullptr;
    int plan_frames = 0, plan_mode = -1, plan_chunk = 0, plan_overlap = 0;
    // the decoder entry points: a one-window decoder plan and a device buffer for their inputs and outputs
    P2cuDecoder* dec = nullptr;
    const P2cuModel* dec_model = nullptr;
    int dec_frames = 0;
    float* io = nullptr;
    size_t io_floats = 0;
    P2cuMel* mel = nullptr;   // p2_mel_spectrogram's one-window plan
    long long mel_samples = 0;

    void drop_plan() {
        if (plan) p2cu_encoder_destroy(plan);
        plan = nullptr;
        plan_model = nullptr;
        if (dec) p2cu_decoder_destroy(dec);
        dec = nullptr;
        dec_model = nullptr;
        dec_frames = 0;
        if (mel) p2cu_mel_destroy(mel);
        mel = nullptr;
        mel_samples = 0;
    }
    void drop_all() {
        if (device >= 0) cudaSetDevice(device);
        drop_plan();
        if (io) cudaFree(io);
        io = nullptr;
        io_floats = 0;
        if (stream) cudaStreamDestroy(stream);
        stream = nullptr;
    }
    ~ThreadCtx() { drop_all(); }
};

thread_local ThreadCtx t_ctx;

const P2cuModel* model_on(const P2Model* m, int device) {
    const uint64_t print = fingerprint(m);
    std::lock_guard<std::mutex> lock(g_mu);
    for (const ModelEntry& e : g_models)
        if (e.key == m && e.device == device && e.print == print) return e.dev;
    const char* cc = getenv("P2_CACHE_CODES");
    P2cuModel* d = nullptr;
    if (p2cu_model_upload(m, cc && cc[0] && cc[0] != '0', &d) != P2CU_OK) return nullptr;
    g_models.push_back({m, device, print, d});
    return d;
}

// The calling thread's context on its GPU (p2_b200_set_device), with a stream; null after a message on stderr.
ThreadCtx* thread_ctx(const char* who) {
    ThreadCtx& c = t_ctx;
    const int device = p2b_thread_device();
    if (cudaSetDevice(device) != cudaSuccess) {
        fprintf(stderr, "%s: cannot use GPU %d\n", who, device);
        return nullptr;
    }
    if (c.device != device) {   // the thread moved to another GPU: start over there
        c.drop_all();
        c.device = device;
        cudaSetDevice(device);
    }
    if (!c.stream && cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking) != cudaSuccess) {
        fprintf(stderr, "%s: cannot create a CUDA stream\n", who);
        return nullptr;
    }
    return &c;
}

int encode(const P2Model* m, const float* mel, int n_frames, bool force_chunk, float** out, int* out_len) {
    if (!m || !mel || n_frames < 1 || !out || !out_len) {
        fprintf(stderr, "p2_encoder: bad arguments\n");
        return -1;
    }
    ThreadCtx* cp = thread_ctx("p2_encoder");
    if (!cp) return -1;
    ThreadCtx& c = *cp;
    const P2cuModel* dm = model_on(m, c.device);
    if (!dm) {
        fprintf(stderr, "p2_encoder: %s\n", p2cu_last_error());
        return -1;
    }
    const int Tp = ((((n_frames - 1) / 2 + 1) - 1) / 2 + 1 - 1) / 2 + 1;
    const bool chunked = force_chunk || should_chunk(Tp);
    const int chunk = chunked ? env_int("P2_CHUNK_SIZE", 400) : 0;
    const int overlap = chunked ? env_int("P2_CHUNK_OVERLAP", 8) : 0;
    const int mode = p2b_gemm_mode();
    if (!c.plan || c.plan_model != dm || c.plan_frames != n_frames || c.plan_mode != mode || c.plan_chunk != chunk ||
        c.plan_overlap != overlap) {
        if (c.plan) p2cu_encoder_destroy(c.plan);
        c.plan = nullptr;
        if (p2cu_encoder_create_lazy(dm, &n_frames, 1, mode, chunk, overlap, &c.plan) != P2CU_OK) {
            fprintf(stderr, "p2_encoder: %s\n", p2cu_last_error());
            c.plan = nullptr;
            return -1;
        }
        c.plan_model = dm; c.plan_frames = n_frames; c.plan_mode = mode; c.plan_chunk = chunk;
        c.plan_overlap = overlap;
    }
    const int T = p2cu_encoder_frames(c.plan, -1);
    float* res = static_cast<float*>(malloc(static_cast<size_t>(T) * P2_JOINT_DIM * sizeof(float)));
    if (!res) {
        fprintf(stderr, "p2_encoder: out of memory\n");
        return -1;
    }
    cudaError_t e = cudaMemcpyAsync(p2cu_encoder_mel(c.plan), mel, static_cast<size_t>(n_frames) * P2_N_MELS * 4,
                                    cudaMemcpyHostToDevice, c.stream);
    int rc = e == cudaSuccess ? p2cu_encoder_run(c.plan, c.stream) : P2CU_ECUDA;
    if (rc == P2CU_OK)
        e = cudaMemcpyAsync(res, p2cu_encoder_out(c.plan), static_cast<size_t>(T) * P2_JOINT_DIM * 4,
                            cudaMemcpyDeviceToHost, c.stream);
    if (rc == P2CU_OK && e == cudaSuccess) rc = p2cu_check_device(c.stream);
    if (rc != P2CU_OK || e != cudaSuccess) {
        fprintf(stderr, "p2_encoder: %s\n", e != cudaSuccess ? cudaGetErrorString(e) : p2cu_last_error());
        free(res);
        return -1;
    }
    *out = res;
    *out_len = T;
    return 0;
}

// The thread's one-window decoder plan for `m`, holding at least `frames` frames, and its io buffer of `floats`.
bool thread_decoder(ThreadCtx& c, const P2Model* m, int frames, size_t floats, const char* who) {
    const P2cuModel* dm = model_on(m, c.device);
    if (!dm) {
        fprintf(stderr, "%s: %s\n", who, p2cu_last_error());
        return false;
    }
    if (!c.dec || c.dec_model != dm || c.dec_frames < frames) {
        if (c.dec) p2cu_decoder_destroy(c.dec);
        c.dec = nullptr;
        const int f = std::max(frames, std::max(2 * c.dec_frames, 1024));
        if (p2cu_decoder_create(dm, 1, f, &c.dec) != P2CU_OK) {
            fprintf(stderr, "%s: %s\n", who, p2cu_last_error());
            c.dec_model = nullptr;
            c.dec_frames = 0;
            return false;
        }
        c.dec_model = dm;
        c.dec_frames = f;
    }
    if (c.io_floats < floats) {
        if (c.io) cudaFree(c.io);
        c.io = nullptr;
        c.io_floats = 0;
        if (cudaMalloc(&c.io, floats * sizeof(float)) != cudaSuccess) {
            fprintf(stderr, "%s: cannot allocate %zu bytes on GPU %d\n", who, floats * sizeof(float), c.device);
            return false;
        }
        c.io_floats = floats;
    }
    return true;
}

int conv3(int n) {   // encoder frames of n mel frames: three stride-2 convolutions
    for (int i = 0; i < 3; ++i) n = (n - 1) / 2 + 1;
    return n;
}

// Windows to GPUs: longest first, each to the GPU with the fewest frames so far; each GPU keeps its windows in their
// original order.
std::vector<std::vector<int>> shard_windows(const int* n_frames, int n, int n_dev) {
    std::vector<int> order(n);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return n_frames[a] > n_frames[b]; });
    std::vector<long long> load(n_dev, 0);
    std::vector<std::vector<int>> out(n_dev);
    for (int w : order) {
        const int d = static_cast<int>(std::min_element(load.begin(), load.end()) - load.begin());
        out[d].push_back(w);
        load[d] += n_frames[w];
    }
    for (auto& v : out) std::sort(v.begin(), v.end());
    return out;
}

// One GPU's share of the batched entry points: its cached encoder plans (one per distinct window set and chunking),
// its decoder plan and its stream.
struct DeviceSlot {
    std::mutex mu;
    cudaStream_t stream = nullptr;
    struct Cached {
        const P2cuModel* model;
        std::vector<int> frames;
        int mode, chunk, overlap;
        P2cuEncoder* plan;
    };
    std::vector<Cached> plans;   // the two most recent
    P2cuDecoder* dec = nullptr;
    const P2cuModel* dec_model = nullptr;
    int dec_windows = 0, dec_frames = 0;
    P2cuMel* mel = nullptr;          // the log-mel plan and the audio it reads (p2_b200_transcribe_audio_windows)
    int mel_windows = 0;
    long long mel_samples = 0;
    float* audio = nullptr;

    P2cuMel* mel_for(int windows, long long samples) {
        if (mel && mel_windows >= windows && mel_samples >= samples) return mel;
        drop_mel();
        const int w = std::max(windows, 1);
        const long long n = std::max(samples, static_cast<long long>(P2_N_MELS));
        if (p2cu_mel_create(w, n, &mel) != P2CU_OK) return nullptr;
        if (cudaMalloc(&audio, static_cast<size_t>(n) * sizeof(float)) != cudaSuccess) {
            drop_mel();
            return nullptr;
        }
        mel_windows = w;
        mel_samples = n;
        return mel;
    }
    void drop_mel() {
        if (mel) p2cu_mel_destroy(mel);
        if (audio) cudaFree(audio);
        mel = nullptr;
        audio = nullptr;
        mel_windows = 0;
        mel_samples = 0;
    }

    P2cuEncoder* plan_for(const P2cuModel* dm, const std::vector<int>& frames, int mode, int chunk, int overlap) {
        for (Cached& c : plans)
            if (c.model == dm && c.frames == frames && c.mode == mode && c.chunk == chunk && c.overlap == overlap)
                return c.plan;
        P2cuEncoder* e = nullptr;
        if (p2cu_encoder_create_lazy(dm, frames.data(), static_cast<int>(frames.size()), mode, chunk, overlap, &e) !=
            P2CU_OK)
            return nullptr;
        if (plans.size() >= 2) {
            p2cu_encoder_destroy(plans.front().plan);
            plans.erase(plans.begin());
        }
        plans.push_back({dm, frames, mode, chunk, overlap, e});
        return e;
    }
    P2cuDecoder* decoder_for(const P2cuModel* dm, int windows, int frames) {
        if (dec && dec_model == dm && dec_windows >= windows && dec_frames >= frames) return dec;
        if (dec) p2cu_decoder_destroy(dec);
        dec = nullptr;
        const int w = std::max(windows, dec_windows), f = std::max(frames, dec_frames);
        if (p2cu_decoder_create(dm, w, f, &dec) != P2CU_OK) {
            dec_model = nullptr;
            dec_windows = dec_frames = 0;
            return nullptr;
        }
        dec_model = dm;
        dec_windows = w;
        dec_frames = f;
        return dec;
    }
};

DeviceSlot g_slots[64];

// What a batched entry point does with one encoder plan's output on the device: the plan, its stream, the slot, the
// caller's window indices of the plan's windows in order.
using AfterEncode = std::function<int(P2cuEncoder*, cudaStream_t, DeviceSlot&, const P2cuModel*,
                                      const std::vector<int>&, std::string*)>;
// How a batched entry point fills an encoder plan's input (its mel frames, windows stacked) from the caller's data.
using FeedEncoder = std::function<int(P2cuEncoder*, cudaStream_t, DeviceSlot&, const std::vector<int>&,
                                      std::string*)>;

// Encode `wins` (indices into the caller's windows) on `device` with one plan, its input written by `feed`, then run
// `after` on its output.
int encode_on_device(const P2Model* m, int device, const std::vector<int>& wins, const int* n_frames, int chunk,
                     int overlap, const FeedEncoder& feed, const AfterEncode& after, std::string* err) {
    if (wins.empty()) return 0;
    if (cudaSetDevice(device) != cudaSuccess) {
        *err = "cannot use GPU " + std::to_string(device);
        return -1;
    }
    DeviceSlot& slot = g_slots[device];
    std::lock_guard<std::mutex> lock(slot.mu);
    if (!slot.stream && cudaStreamCreateWithFlags(&slot.stream, cudaStreamNonBlocking) != cudaSuccess) {
        *err = "cannot create a CUDA stream";
        return -1;
    }
    const P2cuModel* dm = model_on(m, device);
    if (!dm) {
        *err = p2cu_last_error();
        return -1;
    }
    std::vector<int> frames;
    for (int w : wins) frames.push_back(n_frames[w]);
    P2cuEncoder* e = slot.plan_for(dm, frames, p2b_gemm_mode(), chunk, overlap);
    if (!e) {
        *err = p2cu_last_error();
        return -1;
    }
    if (feed(e, slot.stream, slot, wins, err) != 0) return -1;
    if (p2cu_encoder_run(e, slot.stream) != P2CU_OK) {
        *err = p2cu_last_error();
        return -1;
    }
    return after(e, slot.stream, slot, dm, wins, err);
}

// FeedEncoder from host mel frames ([sum n_frames][128], windows one after another).
FeedEncoder feed_host_mel(const float* mel, const int* n_frames, int n_windows) {
    auto off = std::make_shared<std::vector<long long>>(n_windows + 1, 0);
    for (int w = 0; w < n_windows; ++w) (*off)[w + 1] = (*off)[w] + n_frames[w];
    return [mel, n_frames, off](P2cuEncoder* e, cudaStream_t s, DeviceSlot&, const std::vector<int>& wins,
                                std::string* err) {
        float* dmel = p2cu_encoder_mel(e);
        size_t row = 0;
        for (int w : wins) {
            const cudaError_t ce = cudaMemcpyAsync(dmel + row * P2_N_MELS, mel + (*off)[w] * P2_N_MELS,
                                                   static_cast<size_t>(n_frames[w]) * P2_N_MELS * sizeof(float),
                                                   cudaMemcpyHostToDevice, s);
            if (ce != cudaSuccess) {
                *err = cudaGetErrorString(ce);
                return -1;
            }
            row += n_frames[w];
        }
        return 0;
    };
}

// FeedEncoder from windows that are slices of host audio (16 kHz): window w is audio[starts[w], starts[w] + n[w]).
// The windows' samples go up, the log-mel front end writes the plan's input on the device.
FeedEncoder feed_host_slices(const float* audio, std::vector<long long> starts, std::vector<long long> n_samples) {
    auto st = std::make_shared<std::vector<long long>>(std::move(starts));
    auto ns_all = std::make_shared<std::vector<long long>>(std::move(n_samples));
    return [audio, st, ns_all](P2cuEncoder* e, cudaStream_t s, DeviceSlot& slot, const std::vector<int>& wins,
                               std::string* err) {
        long long total = 0;
        std::vector<long long> ns;
        for (int w : wins) {
            ns.push_back((*ns_all)[w]);
            total += (*ns_all)[w];
        }
        P2cuMel* mp = slot.mel_for(static_cast<int>(wins.size()), total);
        if (!mp) {
            *err = std::string("log-mel plan: ") + p2cu_last_error();
            return -1;
        }
        long long at = 0;
        for (int w : wins) {
            const cudaError_t ce = cudaMemcpyAsync(slot.audio + at, audio + (*st)[w],
                                                   static_cast<size_t>((*ns_all)[w]) * sizeof(float),
                                                   cudaMemcpyHostToDevice, s);
            if (ce != cudaSuccess) {
                *err = cudaGetErrorString(ce);
                return -1;
            }
            at += (*ns_all)[w];
        }
        if (p2cu_mel_run(mp, slot.audio, ns.data(), static_cast<int>(wins.size()), p2cu_encoder_mel(e), s) !=
            P2CU_OK) {
            *err = p2cu_last_error();
            return -1;
        }
        return 0;
    };
}

// FeedEncoder from host audio ([sum n_samples] at 16 kHz, the windows one after another).
FeedEncoder feed_host_audio(const float* audio, const long long* n_samples, int n_windows) {
    std::vector<long long> starts(n_windows, 0), ns(n_samples, n_samples + n_windows);
    for (int w = 1; w < n_windows; ++w) starts[w] = starts[w - 1] + n_samples[w - 1];
    return feed_host_slices(audio, std::move(starts), std::move(ns));
}

// The window checks, the sharding over GPUs and one host thread per GPU, shared by the batched entry points: `after`
// runs on every plan's output. The reference's chunking rule applies per window (csrc/encoder.c:715-723): windows it
// would chunk go in a plan of their own on the same GPU.
// A GPU whose share fails (a CUDA error, a kernel that reported a timeout, no memory) hands the share to a GPU whose
// share succeeded, which runs it after its own; every window's result depends on the window alone, so the output is
// the same. The call fails only when no GPU succeeded or the second attempt fails too. For tests, P2_B200_FAIL_SLOT=i
// makes the share at position i of the device list report a failure before it runs anything (a host-side fault; no
// GPU is disturbed).
int run_windows(const char* who, const P2Model* m, const int* n_frames, int n_windows, const int* devices,
                int n_devices, const FeedEncoder& feed, const AfterEncode& after) {
    std::vector<int> devs;
    if (n_devices == 0) {
        // No list from the caller: P2_DEVICES (GPU indices separated by commas; an index may repeat, its shares then
        // run one after the other), else every GPU.
        const char* env = getenv("P2_DEVICES");
        for (const char* c = env; c && *c;) {
            char* end = nullptr;
            const long v = strtol(c, &end, 10);
            if (end == c || v < 0 || v >= 64) {
                fprintf(stderr, "%s: P2_DEVICES=\"%s\" is not a list of GPU indices\n", who, env);
                return -1;
            }
            devs.push_back(static_cast<int>(v));
            c = *end == ',' ? end + 1 : end;
            if (*end && *end != ',') {
                fprintf(stderr, "%s: P2_DEVICES=\"%s\" is not a list of GPU indices\n", who, env);
                return -1;
            }
        }
        if (devs.empty()) {
            int n = 0;
            if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
                fprintf(stderr, "%s: no CUDA device\n", who);
                return -1;
            }
            for (int i = 0; i < n; ++i) devs.push_back(i);
        }
    } else {
        devs.assign(devices, devices + n_devices);
    }
    for (int d : devs)
        if (d < 0 || d >= 64) {
            fprintf(stderr, "%s: device %d out of range\n", who, d);
            return -1;
        }
    for (int w = 0; w < n_windows; ++w)
        if (n_frames[w] < 1) {
            fprintf(stderr, "%s: window %d has %d frames\n", who, w, n_frames[w]);
            return -1;
        }
    const int chunk = env_int("P2_CHUNK_SIZE", 400), overlap = env_int("P2_CHUNK_OVERLAP", 8);
    int prev = 0;
    cudaGetDevice(&prev);
    const auto shards = shard_windows(n_frames, n_windows, static_cast<int>(devs.size()));
    if (p2_verbose && devs.size() > 1) {
        size_t busy = 0;
        for (const auto& sh : shards) busy += sh.empty() ? 0 : 1;
        fprintf(stderr, "  %s: %d window(s) over %zu GPU slot(s) of %zu listed\n", who, n_windows, busy, devs.size());
    }
    int fail_slot = -1;
    if (const char* fs = getenv("P2_B200_FAIL_SLOT")) {
        char* end;
        const long v = strtol(fs, &end, 10);
        if (*fs && *end == '\0' && v >= 0 && v < 64) fail_slot = static_cast<int>(v);
    }
    auto run_share = [&](const std::vector<int>& share, int device, std::string* err) {
        std::vector<int> plain, chunked;
        for (int w : share) (should_chunk(conv3(n_frames[w])) ? chunked : plain).push_back(w);
        int rc = encode_on_device(m, device, plain, n_frames, 0, 0, feed, after, err);
        if (rc == 0) rc = encode_on_device(m, device, chunked, n_frames, chunk, overlap, feed, after, err);
        return rc;
    };
    // The same GPU may appear twice in `devices`: its shares then run one after the other (the slot's mutex).
    std::vector<std::string> errs(devs.size());
    std::vector<int> rcs(devs.size(), 0);
    std::vector<std::thread> threads;
    for (size_t i = 0; i < devs.size(); ++i) {
        threads.emplace_back([&, i] {
            if (static_cast<int>(i) == fail_slot && !shards[i].empty()) {
                errs[i] = "failure injected by P2_B200_FAIL_SLOT";
                rcs[i] = -1;
                return;
            }
            rcs[i] = run_share(shards[i], devs[i], &errs[i]);
        });
    }
    for (auto& t : threads) t.join();
    std::vector<size_t> healthy;
    for (size_t i = 0; i < devs.size(); ++i)
        if (rcs[i] == 0) healthy.push_back(i);
    int rc = 0;
    for (size_t i = 0, k = 0; i < devs.size() && rc == 0; ++i) {
        if (rcs[i] == 0) continue;
        fprintf(stderr, "%s: GPU %d: %s\n", who, devs[i], errs[i].c_str());
        if (healthy.empty()) {
            rc = -1;
            break;
        }
        const size_t j = healthy[k++ % healthy.size()];
        fprintf(stderr, "%s: GPU %d's %zu window(s) re-run on GPU %d\n", who, devs[i], shards[i].size(), devs[j]);
        std::string err;
        if (run_share(shards[i], devs[j], &err) != 0) {
            fprintf(stderr, "%s: GPU %d: %s\n", who, devs[j], err.c_str());
            rc = -1;
        }
    }
    cudaSetDevice(prev);
    return rc;
}

}  // namespace

extern "C" {

// No counterpart in the reference, whose engine encodes the windows of long audio one after another on its thread
// pool (csrc/engine.c:311-357): here they are spread over GPUs, one batch per GPU, with no collective.
__attribute__((visibility("default"))) int p2_b200_encode_windows(const P2Model* m, const float* mel,
                                                                  const int* n_frames, int n_windows,
                                                                  const int* devices, int n_devices, float* out) {
    if (!m || !mel || !n_frames || n_windows <= 0 || !out || n_devices < 0 || (n_devices > 0 && !devices)) {
        fprintf(stderr, "p2_b200_encode_windows: bad arguments\n");
        return -1;
    }
    std::vector<long long> out_off(n_windows + 1, 0);
    for (int w = 0; w < n_windows; ++w) out_off[w + 1] = out_off[w] + conv3(std::max(n_frames[w], 1));
    auto copy_out = [&](P2cuEncoder* e, cudaStream_t s, DeviceSlot&, const P2cuModel*, const std::vector<int>& wins,
                        std::string* err) {
        const float* dout = p2cu_encoder_out(e);
        cudaError_t ce = cudaSuccess;
        size_t row = 0;
        for (size_t i = 0; ce == cudaSuccess && i < wins.size(); ++i) {
            const int w = wins[i];
            const int t = p2cu_encoder_frames(e, static_cast<int>(i));
            ce = cudaMemcpyAsync(out + out_off[w] * P2_JOINT_DIM, dout + row * P2_JOINT_DIM,
                                 static_cast<size_t>(t) * P2_JOINT_DIM * sizeof(float), cudaMemcpyDeviceToHost, s);
            row += t;
        }
        const int rc = ce == cudaSuccess ? p2cu_check_device(s) : P2CU_ECUDA;
        if (rc != P2CU_OK) {
            *err = ce != cudaSuccess ? cudaGetErrorString(ce) : p2cu_last_error();
            return -1;
        }
        return 0;
    };
    return run_windows("p2_b200_encode_windows", m, n_frames, n_windows, devices, n_devices,
                       feed_host_mel(mel, n_frames, n_windows), copy_out);
}

}  // extern "C"

namespace {

// AfterEncode that decodes each plan's output on the device and hands every window's tokens to the caller (malloc'd
// arrays in tokens[w], counts in n_tokens[w], and the window's encoder frames in enc_frames[w] when it is given).
AfterEncode decode_after(P2Token** tokens, int* n_tokens, int* enc_frames) {
    return [tokens, n_tokens, enc_frames](P2cuEncoder* e, cudaStream_t s, DeviceSlot& slot, const P2cuModel* dm,
                                          const std::vector<int>& wins, std::string* err) {
        const int nw = static_cast<int>(wins.size());
        std::vector<int> T(nw);
        for (int i = 0; i < nw; ++i) T[i] = p2cu_encoder_frames(e, i);
        if (enc_frames)
            for (int i = 0; i < nw; ++i) enc_frames[wins[i]] = T[i];
        // one decoder launch per group of at most kDecodeWindows windows
        constexpr int kDecodeWindows = 512;
        const float* enc = p2cu_encoder_out(e);
        for (int g0 = 0; g0 < nw; g0 += kDecodeWindows) {
            const int gn = std::min(kDecodeWindows, nw - g0);
            long long frames = 0;
            for (int i = 0; i < gn; ++i) frames += T[g0 + i];
            P2cuDecoder* d = slot.decoder_for(dm, gn, static_cast<int>(std::max(frames, 1LL)));
            std::vector<int> offs(gn + 1);
            int total = -1;
            if (d && p2cu_decode(d, enc, T.data() + g0, gn, s) == P2CU_OK)
                total = p2cu_decoder_read(d, offs.data(), nullptr, 0, s);
            std::vector<P2Token> all(std::max(total, 1));
            if (total > 0 && p2cu_decoder_read(d, offs.data(), all.data(), total, s) != total) total = -1;
            if (total < 0) {
                *err = p2cu_last_error();
                return -1;
            }
            for (int i = 0; i < gn; ++i) {
                const int n = offs[i + 1] - offs[i], w = wins[g0 + i];
                free(tokens[w]);   // a share re-run after a failed attempt replaces what that attempt wrote
                tokens[w] = nullptr;
                n_tokens[w] = n;
                if (n == 0) continue;
                tokens[w] = static_cast<P2Token*>(malloc(static_cast<size_t>(n) * sizeof(P2Token)));
                if (!tokens[w]) {
                    *err = "out of host memory";
                    return -1;
                }
                memcpy(tokens[w], all.data() + offs[i], static_cast<size_t>(n) * sizeof(P2Token));
            }
            enc += frames * P2_JOINT_DIM;
        }
        return 0;
    };
}

// The shared part of the transcribe entry points: checks, token arrays reset, run, arrays freed on failure.
int transcribe(const char* who, const P2Model* m, const int* n_frames, int n_windows, const int* devices,
               int n_devices, const FeedEncoder& feed, P2Token** tokens, int* n_tokens, int* enc_frames = nullptr) {
    if (!m->dec.embed_w) {
        fprintf(stderr, "%s: the model has no decoder tables\n", who);
        return -1;
    }
    for (int w = 0; w < n_windows; ++w) {
        tokens[w] = nullptr;
        n_tokens[w] = 0;
    }
    const int rc = run_windows(who, m, n_frames, n_windows, devices, n_devices, feed,
                               decode_after(tokens, n_tokens, enc_frames));
    if (rc != 0)
        for (int w = 0; w < n_windows; ++w) {
            free(tokens[w]);
            tokens[w] = nullptr;
            n_tokens[w] = 0;
        }
    return rc;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) int p2_b200_transcribe_windows(const P2Model* m, const float* mel,
                                                                      const int* n_frames, int n_windows,
                                                                      const int* devices, int n_devices,
                                                                      P2Token** tokens, int* n_tokens) {
    if (!m || !mel || !n_frames || n_windows <= 0 || !tokens || !n_tokens || n_devices < 0 ||
        (n_devices > 0 && !devices)) {
        fprintf(stderr, "p2_b200_transcribe_windows: bad arguments\n");
        return -1;
    }
    return transcribe("p2_b200_transcribe_windows", m, n_frames, n_windows, devices, n_devices,
                      feed_host_mel(mel, n_frames, n_windows), tokens, n_tokens);
}

__attribute__((visibility("default"))) int p2_b200_transcribe_audio_windows(const P2Model* m, const float* audio,
                                                                            const long long* n_samples,
                                                                            int n_windows, const int* devices,
                                                                            int n_devices, P2Token** tokens,
                                                                            int* n_tokens) {
    if (!m || !audio || !n_samples || n_windows <= 0 || !tokens || !n_tokens || n_devices < 0 ||
        (n_devices > 0 && !devices)) {
        fprintf(stderr, "p2_b200_transcribe_audio_windows: bad arguments\n");
        return -1;
    }
    std::vector<int> frames(n_windows);
    for (int w = 0; w < n_windows; ++w) {
        frames[w] = p2cu_mel_frames(n_samples[w]);
        if (frames[w] < 2) {
            fprintf(stderr, "p2_b200_transcribe_audio_windows: window %d: audio too short: %lld samples\n", w,
                    n_samples[w]);
            return -1;
        }
    }
    return transcribe("p2_b200_transcribe_audio_windows", m, frames.data(), n_windows, devices, n_devices,
                      feed_host_audio(audio, n_samples, n_windows), tokens, n_tokens);
}

// For long_audio.cu (not exported): windows that are slices of one host audio buffer, window w being
// audio[starts[w], starts[w] + n_samples[w]) with at least 1280 samples; tokens and counts as
// p2_b200_transcribe_audio_windows, each window's encoder frames in enc_frames[w].
int p2b_transcribe_slices(const P2Model* m, const float* audio, const long long* starts, const long long* n_samples,
                          int n_windows, const int* devices, int n_devices, P2Token** tokens, int* n_tokens,
                          int* enc_frames) {
    std::vector<int> frames(n_windows);
    for (int w = 0; w < n_windows; ++w) frames[w] = p2cu_mel_frames(n_samples[w]);
    return transcribe("p2_b200_transcribe_long", m, frames.data(), n_windows, devices, n_devices,
                      feed_host_slices(audio, std::vector<long long>(starts, starts + n_windows),
                                       std::vector<long long>(n_samples, n_samples + n_windows)),
                      tokens, n_tokens, enc_frames);
}

__attribute__((visibility("default"))) int p2_mel_spectrogram(const float* audio, int n_samples, float** out_mel,
                                                              int* out_frames) {
    if (!audio || !out_mel || !out_frames || n_samples < 0) {
        fprintf(stderr, "p2_mel_spectrogram: bad arguments\n");
        return -1;
    }
    const int nf = p2cu_mel_frames(n_samples);
    if (nf < 2) {
        fprintf(stderr, "audio too short: %d samples\n", n_samples);   // the reference's message
        return -1;
    }
    ThreadCtx* cp = thread_ctx("p2_mel_spectrogram");
    if (!cp) return -1;
    ThreadCtx& c = *cp;
    const size_t need = static_cast<size_t>(n_samples) + static_cast<size_t>(nf) * P2_N_MELS;
    if (!c.mel || c.mel_samples < n_samples) {
        if (c.mel) p2cu_mel_destroy(c.mel);
        c.mel = nullptr;
        const long long cap = std::max<long long>(n_samples, 2 * c.mel_samples);
        if (p2cu_mel_create(1, cap, &c.mel) != P2CU_OK) {
            fprintf(stderr, "p2_mel_spectrogram: %s\n", p2cu_last_error());
            c.mel_samples = 0;
            return -1;
        }
        c.mel_samples = cap;
    }
    if (c.io_floats < need) {
        if (c.io) cudaFree(c.io);
        c.io = nullptr;
        c.io_floats = 0;
        if (cudaMalloc(&c.io, need * sizeof(float)) != cudaSuccess) {
            fprintf(stderr, "p2_mel_spectrogram: cannot allocate device memory\n");
            return -1;
        }
        c.io_floats = need;
    }
    float* res = static_cast<float*>(malloc(static_cast<size_t>(nf) * P2_N_MELS * sizeof(float)));
    if (!res) {
        fprintf(stderr, "p2_mel_spectrogram: out of memory\n");
        return -1;
    }
    const long long ns = n_samples;
    float* dmel = c.io + n_samples;
    cudaError_t ce = cudaMemcpyAsync(c.io, audio, static_cast<size_t>(n_samples) * sizeof(float),
                                     cudaMemcpyHostToDevice, c.stream);
    int rc = ce == cudaSuccess ? p2cu_mel_run(c.mel, c.io, &ns, 1, dmel, c.stream) : P2CU_ECUDA;
    if (rc == P2CU_OK)
        ce = cudaMemcpyAsync(res, dmel, static_cast<size_t>(nf) * P2_N_MELS * sizeof(float), cudaMemcpyDeviceToHost,
                             c.stream);
    if (rc == P2CU_OK && ce == cudaSuccess) rc = p2cu_check_device(c.stream);
    if (rc != P2CU_OK || ce != cudaSuccess) {
        fprintf(stderr, "p2_mel_spectrogram: %s\n", ce != cudaSuccess ? cudaGetErrorString(ce) : p2cu_last_error());
        free(res);
        return -1;
    }
    *out_mel = res;
    *out_frames = nf;
    return 0;
}

__attribute__((visibility("default"))) int p2_greedy_decode(const P2Model* m, const float* enc_out, int T,
                                                            P2Token** out_tokens) {
    if (!m || (!enc_out && T > 0) || T < 0 || !out_tokens) {
        fprintf(stderr, "p2_greedy_decode: bad arguments\n");
        return -1;
    }
    if (!m->dec.embed_w) {
        fprintf(stderr, "p2_greedy_decode: the model has no decoder tables\n");
        return -1;
    }
    ThreadCtx* cp = thread_ctx("p2_greedy_decode");
    if (!cp || !thread_decoder(*cp, m, std::max(T, 1), static_cast<size_t>(std::max(T, 1)) * P2_JOINT_DIM,
                               "p2_greedy_decode"))
        return -1;
    ThreadCtx& c = *cp;
    int offs[2] = {0, 0};
    int n = 0;
    cudaError_t ce = cudaSuccess;
    if (T > 0) {
        ce = cudaMemcpyAsync(c.io, enc_out, static_cast<size_t>(T) * P2_JOINT_DIM * sizeof(float),
                             cudaMemcpyHostToDevice, c.stream);
        n = ce != cudaSuccess ? -1 : p2cu_decode(c.dec, c.io, &T, 1, c.stream) != P2CU_OK
                                         ? -1 : p2cu_decoder_read(c.dec, offs, nullptr, 0, c.stream);
    }
    // at least one element, as the reference's buffer of T + 16 (csrc/decoder.c:105-106) is never NULL
    P2Token* toks = static_cast<P2Token*>(malloc(static_cast<size_t>(std::max(n, 1)) * sizeof(P2Token)));
    if (n > 0 && toks && p2cu_decoder_read(c.dec, offs, toks, n, c.stream) != n) n = -1;
    if (n < 0 || !toks) {
        fprintf(stderr, "p2_greedy_decode: %s\n",
                !toks ? "out of host memory" : ce != cudaSuccess ? cudaGetErrorString(ce) : p2cu_last_error());
        free(toks);
        return -1;
    }
    *out_tokens = toks;
    return n;
}

// The reference's p2_decoder_step and p2_joint return nothing: a failure here prints its message and leaves the
// outputs as they were.
__attribute__((visibility("default"))) void p2_decoder_step(const P2Model* m, int token_id, LSTMState* state,
                                                            float* dec_out) {
    if (!m || !state || !dec_out || !m->dec.embed_w || token_id < 0 || token_id >= P2_VOCAB) {
        fprintf(stderr, "p2_decoder_step: bad arguments\n");
        return;
    }
    ThreadCtx* cp = thread_ctx("p2_decoder_step");
    const size_t nst = sizeof(LSTMState) / sizeof(float);
    if (!cp || !thread_decoder(*cp, m, 1, nst + P2_JOINT_DIM, "p2_decoder_step")) return;
    ThreadCtx& c = *cp;
    float* dst = c.io;
    float* ddec = c.io + nst;
    cudaError_t ce = cudaMemcpyAsync(dst, state, sizeof(LSTMState), cudaMemcpyHostToDevice, c.stream);
    int rc = ce == cudaSuccess ? p2cu_decoder_step(c.dec, token_id, dst, ddec, c.stream) : P2CU_ECUDA;
    if (rc == P2CU_OK) rc = p2cu_check_device(c.stream);   // the state is not touched unless the step completed
    if (rc == P2CU_OK) {
        ce = cudaMemcpyAsync(state, dst, sizeof(LSTMState), cudaMemcpyDeviceToHost, c.stream);
        if (ce == cudaSuccess)
            ce = cudaMemcpyAsync(dec_out, ddec, P2_JOINT_DIM * sizeof(float), cudaMemcpyDeviceToHost, c.stream);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(c.stream);
    }
    if (rc != P2CU_OK || ce != cudaSuccess)
        fprintf(stderr, "p2_decoder_step: %s\n", ce != cudaSuccess ? cudaGetErrorString(ce) : p2cu_last_error());
}

__attribute__((visibility("default"))) void p2_joint(const P2Model* m, const float* enc_t, const float* dec_out,
                                                     float* logits) {
    if (!m || !enc_t || !dec_out || !logits || !m->dec.embed_w) {
        fprintf(stderr, "p2_joint: bad arguments\n");
        return;
    }
    ThreadCtx* cp = thread_ctx("p2_joint");
    if (!cp || !thread_decoder(*cp, m, 1, 2 * P2_JOINT_DIM + P2_N_LOGITS, "p2_joint")) return;
    ThreadCtx& c = *cp;
    float* denc = c.io;
    float* ddec = c.io + P2_JOINT_DIM;
    float* dlog = c.io + 2 * P2_JOINT_DIM;
    cudaError_t ce = cudaMemcpyAsync(denc, enc_t, P2_JOINT_DIM * sizeof(float), cudaMemcpyHostToDevice, c.stream);
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(ddec, dec_out, P2_JOINT_DIM * sizeof(float), cudaMemcpyHostToDevice, c.stream);
    int rc = ce == cudaSuccess ? p2cu_joint(c.dec, denc, ddec, dlog, c.stream) : P2CU_ECUDA;
    if (rc == P2CU_OK) rc = p2cu_check_device(c.stream);
    if (rc == P2CU_OK) {
        ce = cudaMemcpyAsync(logits, dlog, P2_N_LOGITS * sizeof(float), cudaMemcpyDeviceToHost, c.stream);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(c.stream);
    }
    if (rc != P2CU_OK || ce != cudaSuccess)
        fprintf(stderr, "p2_joint: %s\n", ce != cudaSuccess ? cudaGetErrorString(ce) : p2cu_last_error());
}

__attribute__((visibility("default"))) int p2_encoder(const P2Model* m, const float* mel, int n_frames, float** out,
                                                      int* out_len) {
    return encode(m, mel, n_frames, false, out, out_len);
}

__attribute__((visibility("default"))) int p2_encoder_chunked(const P2Model* m, const float* mel, int n_frames,
                                                              float** out, int* out_len) {
    return encode(m, mel, n_frames, true, out, out_len);
}

// Called by p2_b200_release_weights: drop the calling thread's plans and every uploaded model with the plans made
// on it.
void p2b_release_encoder_models(void) {
    t_ctx.drop_all();
    for (int d = 0; d < 64; ++d) {
        DeviceSlot& slot = g_slots[d];
        std::lock_guard<std::mutex> lock(slot.mu);
        if (slot.plans.empty() && !slot.dec && !slot.mel) continue;
        cudaSetDevice(d);
        for (auto& c : slot.plans) p2cu_encoder_destroy(c.plan);
        slot.plans.clear();
        if (slot.dec) p2cu_decoder_destroy(slot.dec);
        slot.dec = nullptr;
        slot.dec_model = nullptr;
        slot.dec_windows = slot.dec_frames = 0;
        slot.drop_mel();
    }
    std::lock_guard<std::mutex> lock(g_mu);
    int prev = 0;
    cudaGetDevice(&prev);
    for (ModelEntry& e : g_models) {
        cudaSetDevice(e.device);
        cudaDeviceSynchronize();
        p2cu_model_free(e.dev);
    }
    g_models.clear();
    cudaSetDevice(prev);
}

}  // extern "C"
