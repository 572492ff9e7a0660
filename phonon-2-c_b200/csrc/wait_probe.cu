// wait_probe.cu - the kernels' bounded-wait path exercised without a fault (p2cu_probe_wait_timeout): one warp waits,
// through the kernels' own mbar_wait, on an mbarrier phase that nothing completes, gives up after a given number of
// polls, records its code in the device error word and returns; the host reads the error through p2cu_check_device
// with the context still usable. No counterpart in the reference (its CPU loops have no waits to bound).
#include <cstdint>
#include <cuda_runtime.h>
#include "p2cuda.h"
#include "gemm.h"
#include "ptx.cuh"

using p2cu::fail_fmt;

namespace p2cu {
namespace {

// One warp; its barrier expects one arrival and gets none, so phase 0 never completes and lane 0's wait runs out
// after `limit` polls (DEV_TIMEOUT_FULL into the error word, the abort flag set).
__global__ void __launch_bounds__(32) wait_timeout_kernel(uint32_t limit, uint32_t* err) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncwarp();
    int ok = 1;
    if (threadIdx.x == 0) ok = mbar_wait(&bar, 0, DEV_TIMEOUT_FULL, err, &abort_flag, limit) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok && err) atomicCAS(err, DEV_OK, DEV_BAD_ARGS);   // a phase nobody completed cannot have completed
}

}  // namespace
}  // namespace p2cu

extern "C" {

// The device timeout path: a wait on a barrier nothing completes gives up after `limit` polls (1 .. 2^20) and
// reports it. Returns what p2cu_check_device returns afterwards: P2CU_EDEVICE with code 1 when the path works.
int p2cu_probe_wait_timeout(unsigned limit, double* seconds) {
    using namespace p2cu;
    if (!seconds || limit < 1 || limit > (1u << 20)) return fail_fmt(P2CU_EINVAL, "p2cu_probe_wait_timeout: arguments");
    if (int rc = p2cu_check_device(nullptr)) return rc;   // start from a clear error word
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaError_t e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    if (e == cudaSuccess) e = cudaEventRecord(e0);
    if (e == cudaSuccess) {
        wait_timeout_kernel<<<1, 32>>>(limit, device_error_word());
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaEventRecord(e1);
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (e != cudaSuccess) return cuda_error(e, "p2cu_probe_wait_timeout");
    *seconds = ms * 1e-3;
    return p2cu_check_device(nullptr);
}

}  // extern "C"
