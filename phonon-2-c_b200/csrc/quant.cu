// quant.cu - per-row symmetric int8 quantisation of fp32 activations (csrc/blas.c:1114-1144, quant_pack_row):
//   amax = max |x|, scale = amax > 0 ? amax / 127 : 1, q = saturate_int8(round_half_even(x * (1 / scale))).
// Division is IEEE (the C source as written; the reference's -ffast-math build may use a reciprocal, see the oracle).
// Output is row-major int8 [M, K] plus one fp32 scale per row; the GEMM's TMA loads tile it.
#include <cstdint>
#include <cuda_runtime.h>
#include "kernels.h"
#include "ptx.cuh"

namespace p2cu {

__device__ __forceinline__ int8_t quant_one(float x, float inv) {
    int v = __float2int_rn(__fmul_rn(x, inv));
    v = v > 127 ? 127 : (v < -128 ? -128 : v);
    return static_cast<int8_t>(v);
}

// One warp per row; K % 4 == 0 and 16-byte aligned rows (lda % 4 == 0) take the vector path.
__global__ void __launch_bounds__(128) quant_rows_kernel(const float* __restrict__ A, int M, int K, int lda,
                                                         int8_t* __restrict__ q, float* __restrict__ scales) {
    griddep_launch_dependents();
    griddep_wait();   // A may come from the previous kernel in the stream
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M) return;
    const float* row = A + static_cast<size_t>(warp) * lda;
    int8_t* qrow = q + static_cast<size_t>(warp) * K;
    float amax = 0.f;
    const bool vec = (K % 4 == 0) && (lda % 4 == 0) && ((reinterpret_cast<uintptr_t>(A) & 15) == 0);
    if (vec) {
        for (int k = 4 * lane; k < K; k += 128) {
            const float4 v = *reinterpret_cast<const float4*>(row + k);
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    } else {
        for (int k = lane; k < K; k += 32) amax = fmaxf(amax, fabsf(row[k]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = amax > 0.f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, scale);
    if (vec) {
        for (int k = 4 * lane; k < K; k += 128) {
            const float4 v = *reinterpret_cast<const float4*>(row + k);
            char4 o;
            o.x = quant_one(v.x, inv); o.y = quant_one(v.y, inv); o.z = quant_one(v.z, inv); o.w = quant_one(v.w, inv);
            *reinterpret_cast<char4*>(qrow + k) = o;
        }
    } else {
        for (int k = lane; k < K; k += 32) qrow[k] = quant_one(row[k], inv);
    }
    if (lane == 0) scales[warp] = scale;
}

cudaError_t quant_rows_launch(const float* A, int M, int K, int lda, int8_t* q, float* scales, cudaStream_t stream) {
    const int rows_per_block = 4;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((M + rows_per_block - 1) / rows_per_block);
    cfg.blockDim = dim3(32 * rows_per_block);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // set-up overlaps the previous kernel
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, quant_rows_kernel, A, M, K, lda, q, scales);
}

// The int8w codes of a whole five-value weight as a row-major [K, N] int8 plane:
// code = sign * (flag ? 127 : clo[n]), clo[n] = clamp(rint(127 * lo / hi), 0, 127) (csrc/blas.c:1222-1240, 1316-1324).
// One thread per 4 consecutive columns of one row (one sign byte, half a flag byte).
__global__ void __launch_bounds__(256) fv_codes_kernel(const uint8_t* __restrict__ signs,
                                                       const uint8_t* __restrict__ flags,
                                                       const float* __restrict__ lo, const float* __restrict__ hi,
                                                       int K, int N, int8_t* __restrict__ codes) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;   // index of a 4-column group
    const size_t groups = static_cast<size_t>(K) * (N / 4);
    if (i >= groups) return;
    const int k = static_cast<int>(i / (N / 4)), g = static_cast<int>(i % (N / 4));
    const uint32_t sb = signs[static_cast<size_t>(k) * (N / 4) + g];
    const uint32_t fb = flags[static_cast<size_t>(k) * (N / 8) + (g >> 1)] >> (4 * (g & 1));
    char4 out;
    int8_t* o = reinterpret_cast<int8_t*>(&out);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int n = 4 * g + j;
        const int s = static_cast<int>((sb >> (2 * j)) & 3u) - 1;
        int mag = 127;
        if (!((fb >> j) & 1u)) {
            const float l = lo[n], h = hi[n];
            const int c = h > 0.f ? __float2int_rn(__fdiv_rn(__fmul_rn(127.0f, l), h)) : 0;
            mag = c < 0 ? 0 : c > 127 ? 127 : c;
        }
        o[j] = static_cast<int8_t>(s * mag);
    }
    *reinterpret_cast<char4*>(codes + static_cast<size_t>(k) * N + 4 * g) = out;
}

cudaError_t fv_codes_launch(const uint8_t* signs, const uint8_t* flags, const float* lo, const float* hi, int K, int N,
                            int8_t* codes, cudaStream_t stream) {
    const size_t groups = static_cast<size_t>(K) * (N / 4);
    fv_codes_kernel<<<static_cast<unsigned>((groups + 255) / 256), 256, 0, stream>>>(signs, flags, lo, hi, K, N, codes);
    return cudaGetLastError();
}

}  // namespace p2cu
