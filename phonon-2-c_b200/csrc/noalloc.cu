// noalloc.cu - p2cu_sgemm_fvb_noalloc: the fp32-activation five-value GEMM with its scratch memory in a fixed
// device array that the library owns, for callers that cannot allocate device memory.
//
// Who needs it: a caller that must not call cudaMalloc, e.g. a real-time audio callback (cudaMalloc can block and
// implicitly synchronise the device) or a plugin host that only hands out a fixed memory budget. p2cu_sgemm_fvb needs a workspace for the quantised
// activations and, when K > 1024, for the per-1024-row-block partial results; here that workspace is the array below.
//
// The array is a file-scope __device__ variable: every GPU that loads this library holds its P2CU_NOALLOC_SCRATCH_BYTES
// until the process exits. In host code the name g_noalloc_scratch is only a stand-in for the symbol, not a device
// address, so it is never passed to a kernel; its device address is looked up once per device with
// cudaGetSymbolAddress, with that device current, on the first call made on that device; make that first call before
// any stream capture. The address is kept for the process's life: after cudaDeviceReset the module (and the array) of
// the old context are gone, so the entry point must not be called on that device again.
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <cuda_runtime.h>
#include "p2cuda.h"

namespace p2cu {
void set_error_message(int code, const char* msg);   // api.cu: the text p2cu_last_error() returns
}

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[P2CU_NOALLOC_SCRATCH_BYTES];

struct DeviceScratch {
    void* ptr = nullptr;
    bool ready = false;
};

// The array's device address, looked up on the first call on the current device (mutex-protected).
int scratch_on_current_device(void** out) {
    static DeviceScratch table[64];
    static std::mutex mu;
    char msg[256];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        snprintf(msg, sizeof(msg), "p2cu_sgemm_fvb_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
        p2cu::set_error_message(P2CU_ECUDA, msg);
        return P2CU_ECUDA;
    }
    if (dev < 0 || dev >= 64) {
        snprintf(msg, sizeof(msg), "p2cu_sgemm_fvb_noalloc: device %d out of range", dev);
        p2cu::set_error_message(P2CU_EINVAL, msg);
        return P2CU_EINVAL;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!table[dev].ready) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            snprintf(msg, sizeof(msg),
                     "p2cu_sgemm_fvb_noalloc: cudaGetSymbolAddress of the scratch array failed on device %d: %s", dev,
                     cudaGetErrorString(e));
            p2cu::set_error_message(P2CU_ECUDA, msg);
            return P2CU_ECUDA;
        }
        table[dev].ptr = p;
        table[dev].ready = true;
    }
    *out = table[dev].ptr;
    return P2CU_OK;
}

}  // namespace

extern "C" {

int p2cu_sgemm_fvb_noalloc(int M, int N, int K, float alpha, const float* A, int lda, const P2cuFiveValue* B, int mode,
                           float beta, float* C, int ldc, void* stream) {
    const size_t need = p2cu_gemm_workspace_bytes(M, N, K, mode);
    if (need > P2CU_NOALLOC_SCRATCH_BYTES) {
        char msg[256];
        snprintf(msg, sizeof(msg),
                 "p2cu_sgemm_fvb_noalloc: M=%d N=%d K=%d needs %zu bytes of scratch, the fixed array holds %zu "
                 "(use p2cu_sgemm_fvb with a workspace of your own)",
                 M, N, K, need, static_cast<size_t>(P2CU_NOALLOC_SCRATCH_BYTES));
        p2cu::set_error_message(P2CU_EINVAL, msg);
        return P2CU_EINVAL;
    }
    void* scratch = nullptr;
    int rc = scratch_on_current_device(&scratch);
    if (rc != P2CU_OK) return rc;
    // Nothing in the scratch has to start at zero: the quantised rows and the per-block partials are written in
    // full by this call's kernels before they are read, so the previous call's contents do no harm.
    return p2cu_sgemm_fvb(M, N, K, alpha, A, lda, B, mode, beta, C, ldc, scratch, P2CU_NOALLOC_SCRATCH_BYTES, stream);
}

}  // extern "C"
