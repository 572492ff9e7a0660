// encoder_host.cu - phonon-2-c's encoder entry points on host pointers (include/phonon2.h): p2_encoder,
// p2_encoder_chunked and p2_verbose, the drop-in for csrc/encoder.c.
//
// The model's weights are uploaded to the calling thread's GPU the first time a P2Model is seen there and found again
// by its address (the reference's weights are read-only for the model's life, csrc/phonon2.h:204-205); the mel
// frames go up, one graph launch runs the whole encoder, the frames come back. Each host thread keeps its last plan
// (buffers and captured graph for one length and mode) and a stream of its own, so concurrent callers on one model
// do not share buffers (the reference allows concurrent p2_transcribe calls on one engine, csrc/phonon2.h:277-279).
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
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

}  // namespace

extern "C" {

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
