// encoder_host.cu - phonon-2-c's encoder entry points on host pointers (include/phonon2.h): p2_encoder,
// p2_encoder_chunked and p2_verbose, the drop-in for csrc/encoder.c.
//
// The model's weights are uploaded to the calling thread's GPU the first time a P2Model is seen there and found again
// by its address (the reference's weights are read-only for the model's life, csrc/phonon2.h:204-205); the mel
// frames go up, one graph launch runs the whole encoder, the frames come back. Each host thread keeps its last plan
// (buffers and captured graph for one length and mode) and a stream of its own, so concurrent callers on one model
// do not share buffers (the reference allows concurrent p2_transcribe calls on one engine, csrc/phonon2.h:277-279).
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
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

    void drop_plan() {
        if (plan) p2cu_encoder_destroy(plan);
        plan = nullptr;
        plan_model = nullptr;
    }
    ~ThreadCtx() {
        if (device >= 0) cudaSetDevice(device);
        drop_plan();
        if (stream) cudaStreamDestroy(stream);
    }
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

int encode(const P2Model* m, const float* mel, int n_frames, bool force_chunk, float** out, int* out_len) {
    if (!m || !mel || n_frames < 1 || !out || !out_len) {
        fprintf(stderr, "p2_encoder: bad arguments\n");
        return -1;
    }
    ThreadCtx& c = t_ctx;
    const int device = p2b_thread_device();
    if (cudaSetDevice(device) != cudaSuccess) {
        fprintf(stderr, "p2_encoder: cannot use GPU %d\n", device);
        return -1;
    }
    if (c.device != device) {   // the thread moved to another GPU: start over there
        c.drop_plan();
        if (c.stream) cudaStreamDestroy(c.stream);
        c.stream = nullptr;
        c.device = device;
    }
    if (!c.stream && cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking) != cudaSuccess) {
        fprintf(stderr, "p2_encoder: cannot create a CUDA stream\n");
        return -1;
    }
    const P2cuModel* dm = model_on(m, device);
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
        c.drop_plan();
        if (p2cu_encoder_create(dm, &n_frames, 1, mode, chunk, overlap, &c.plan) != P2CU_OK) {
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

// One GPU's share of p2_b200_encode_windows: its cached plans (one per distinct window set and chunking) and stream.
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

    P2cuEncoder* plan_for(const P2cuModel* dm, const std::vector<int>& frames, int mode, int chunk, int overlap) {
        for (Cached& c : plans)
            if (c.model == dm && c.frames == frames && c.mode == mode && c.chunk == chunk && c.overlap == overlap)
                return c.plan;
        P2cuEncoder* e = nullptr;
        if (p2cu_encoder_create(dm, frames.data(), static_cast<int>(frames.size()), mode, chunk, overlap, &e) !=
            P2CU_OK)
            return nullptr;
        if (plans.size() >= 2) {
            p2cu_encoder_destroy(plans.front().plan);
            plans.erase(plans.begin());
        }
        plans.push_back({dm, frames, mode, chunk, overlap, e});
        return e;
    }
};

DeviceSlot g_slots[64];

// Encode `wins` (indices into the caller's windows) on `device` with one plan; mel / out are the caller's host
// arrays with per-window row offsets.
int encode_on_device(const P2Model* m, int device, const std::vector<int>& wins, const float* mel,
                     const std::vector<long long>& mel_off, const int* n_frames, const std::vector<long long>& out_off,
                     float* out, int chunk, int overlap, std::string* err) {
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
    float* dmel = p2cu_encoder_mel(e);
    float* dout = p2cu_encoder_out(e);
    cudaError_t ce = cudaSuccess;
    size_t row = 0;
    for (int w : wins) {
        ce = cudaMemcpyAsync(dmel + row * P2_N_MELS, mel + mel_off[w] * P2_N_MELS,
                             static_cast<size_t>(n_frames[w]) * P2_N_MELS * sizeof(float), cudaMemcpyHostToDevice,
                             slot.stream);
        if (ce != cudaSuccess) break;
        row += n_frames[w];
    }
    int rc = ce == cudaSuccess ? p2cu_encoder_run(e, slot.stream) : P2CU_ECUDA;
    row = 0;
    for (size_t i = 0; rc == P2CU_OK && ce == cudaSuccess && i < wins.size(); ++i) {
        const int w = wins[i];
        const int t = p2cu_encoder_frames(e, static_cast<int>(i));
        ce = cudaMemcpyAsync(out + out_off[w] * P2_JOINT_DIM, dout + row * P2_JOINT_DIM,
                             static_cast<size_t>(t) * P2_JOINT_DIM * sizeof(float), cudaMemcpyDeviceToHost,
                             slot.stream);
        row += t;
    }
    if (rc == P2CU_OK && ce == cudaSuccess) rc = p2cu_check_device(slot.stream);
    if (rc != P2CU_OK || ce != cudaSuccess) {
        *err = ce != cudaSuccess ? cudaGetErrorString(ce) : p2cu_last_error();
        return -1;
    }
    return 0;
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
    std::vector<int> devs;
    if (n_devices == 0) {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
            fprintf(stderr, "p2_b200_encode_windows: no CUDA device\n");
            return -1;
        }
        for (int i = 0; i < n; ++i) devs.push_back(i);
    } else {
        devs.assign(devices, devices + n_devices);
    }
    for (int d : devs)
        if (d < 0 || d >= 64) {
            fprintf(stderr, "p2_b200_encode_windows: device %d out of range\n", d);
            return -1;
        }
    std::vector<long long> mel_off(n_windows + 1, 0), out_off(n_windows + 1, 0);
    for (int w = 0; w < n_windows; ++w) {
        if (n_frames[w] < 1) {
            fprintf(stderr, "p2_b200_encode_windows: window %d has %d frames\n", w, n_frames[w]);
            return -1;
        }
        mel_off[w + 1] = mel_off[w] + n_frames[w];
        out_off[w + 1] = out_off[w] + conv3(n_frames[w]);
    }
    // The reference's chunking rule per window (csrc/encoder.c:715-723): windows it would chunk go in a plan of
    // their own on the same GPU.
    const int chunk = env_int("P2_CHUNK_SIZE", 400), overlap = env_int("P2_CHUNK_OVERLAP", 8);
    int prev = 0;
    cudaGetDevice(&prev);
    const auto shards = shard_windows(n_frames, n_windows, static_cast<int>(devs.size()));
    // The same GPU may appear twice in `devices`: its shares then run one after the other (the slot's mutex).
    std::vector<std::string> errs(devs.size());
    std::vector<int> rcs(devs.size(), 0);
    std::vector<std::thread> threads;
    for (size_t i = 0; i < devs.size(); ++i) {
        threads.emplace_back([&, i] {
            std::vector<int> plain, chunked;
            for (int w : shards[i]) (should_chunk(conv3(n_frames[w])) ? chunked : plain).push_back(w);
            rcs[i] = encode_on_device(m, devs[i], plain, mel, mel_off, n_frames, out_off, out, 0, 0, &errs[i]);
            if (rcs[i] == 0)
                rcs[i] = encode_on_device(m, devs[i], chunked, mel, mel_off, n_frames, out_off, out, chunk, overlap,
                                          &errs[i]);
        });
    }
    for (auto& t : threads) t.join();
    cudaSetDevice(prev);
    for (size_t i = 0; i < devs.size(); ++i)
        if (rcs[i]) {
            fprintf(stderr, "p2_b200_encode_windows: GPU %d: %s\n", devs[i], errs[i].c_str());
            return -1;
        }
    return 0;
}

__attribute__((visibility("default"))) int p2_encoder(const P2Model* m, const float* mel, int n_frames, float** out,
                                                      int* out_len) {
    return encode(m, mel, n_frames, false, out, out_len);
}

__attribute__((visibility("default"))) int p2_encoder_chunked(const P2Model* m, const float* mel, int n_frames,
                                                              float** out, int* out_len) {
    return encode(m, mel, n_frames, true, out, out_len);
}

// Called by p2_b200_release_weights: drop the calling thread's plan and every uploaded encoder model.
void p2b_release_encoder_models(void) {
    t_ctx.drop_plan();
    for (int d = 0; d < 64; ++d) {
        DeviceSlot& slot = g_slots[d];
        std::lock_guard<std::mutex> lock(slot.mu);
        if (slot.plans.empty()) continue;
        cudaSetDevice(d);
        for (auto& c : slot.plans) p2cu_encoder_destroy(c.plan);
        slot.plans.clear();
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
