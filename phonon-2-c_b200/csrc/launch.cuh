// launch.cuh - kernel launches with programmatic dependent launch (PDL).
//
// A launch with cudaLaunchAttributeProgrammaticStreamSerialization may begin while the previous kernel in the stream
// is still running (once that kernel's CTAs have all issued griddepcontrol.launch_dependents or exited), so its launch
// and set-up overlap the predecessor's tail instead of following its completion. Every kernel launched this way must
// execute griddepcontrol.wait (ptx.cuh: griddep_wait) before it reads anything an earlier kernel wrote or writes
// anything an earlier kernel reads; the kernels here do so first thing, so only the launch is overlapped. The wait
// returns once every preceding kernel has completed and its writes are visible, so the order of a chain of such
// kernels is the stream's order.
#pragma once
#include <utility>
#include <cuda_runtime.h>

namespace p2cu {

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace p2cu
