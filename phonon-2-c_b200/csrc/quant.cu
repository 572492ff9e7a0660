// quant.cu - per-row symmetric int8 quantisation of fp32 activations (csrc/blas.c:1114-1144, quant_pack_row):
//   amax = max |x|, scale = amax > 0 ? amax / 127 : 1, q = saturate_int8(round_half_even(x * (1 / scale))), and for
//   the last K % 16 values of a row the reference's scalar tail, clamp(round_half_even(x / scale), -127, 127).
// Division is IEEE (the C source as written); with the opt-in rule (p2cu_set_quant_fast_math, P2CU_QUANT_FAST_MATH)
// the scale and reciprocal are those of the reference's -ffast-math build (numerics.cuh, quant_rule).
// Output is row-major int8 [M, K] plus one fp32 scale per row; the GEMM's TMA loads tile it.
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cuda_runtime.h>
#include "kernels.h"
#include "numerics.cuh"
#include "ptx.cuh"

namespace p2cu {

// One CTA of 128 threads per row. Rows up to 4096 wide with K % 4 == 0 and 16-byte aligned rows stay in registers
// (one read of A); other shapes take a strided two-pass path.
constexpr int QT = 128;            // threads per row
constexpr int QV = 4096 / (4 * QT);   // float4 per thread when the row is held in registers

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    v = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    return v;
}

__global__ void __launch_bounds__(QT) quant_rows_kernel(const float* __restrict__ A, int M, int K, int lda,
                                                        int8_t* __restrict__ q, float* __restrict__ scales, int fm) {
    griddep_launch_dependents();
    {   // the row into L2 while the previous kernel finishes (cold rows then cost no DRAM latency after the wait)
        const char* rb = reinterpret_cast<const char*>(A + static_cast<size_t>(blockIdx.x) * lda);
        for (int off = threadIdx.x * 128; off < K * 4; off += QT * 128) prefetch_l2(rb + off);
    }
    griddep_wait();   // A may come from the previous kernel in the stream
    __shared__ float red[QT / 32];
    const int m = blockIdx.x;
    const float* row = A + static_cast<size_t>(m) * lda;
    int8_t* qrow = q + static_cast<size_t>(m) * K;
    const bool vec = (K % 4 == 0) && (K <= 4 * QT * QV) && (lda % 4 == 0) &&
                     ((reinterpret_cast<uintptr_t>(A) & 15) == 0);
    if (vec) {
        float4 v[QV];
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < QV; ++i) {
            const int k = 4 * (threadIdx.x + i * QT);
            v[i] = k < K ? *reinterpret_cast<const float4*>(row + k) : make_float4(0.f, 0.f, 0.f, 0.f);
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
        }
        amax = block_max(amax, red);
        const QuantRule qr = quant_rule(amax, fm);
        const float scale = qr.scale, inv = qr.inv;
#pragma unroll
        for (int i = 0; i < QV; ++i) {
            const int k = 4 * (threadIdx.x + i * QT);
            if (k < K) {   // k is a multiple of 4 and so is K & ~15: the four values are all in the tail or none
                char4 o;
                if (k < (K & ~15)) {
                    o.x = quant_one(v[i].x, inv); o.y = quant_one(v[i].y, inv);
                    o.z = quant_one(v[i].z, inv); o.w = quant_one(v[i].w, inv);
                } else {
                    o.x = quant_tail(v[i].x, scale, inv, fm); o.y = quant_tail(v[i].y, scale, inv, fm);
                    o.z = quant_tail(v[i].z, scale, inv, fm); o.w = quant_tail(v[i].w, scale, inv, fm);
                }
                *reinterpret_cast<char4*>(qrow + k) = o;
            }
        }
        if (threadIdx.x == 0) scales[m] = scale;
        return;
    }
    float amax = 0.f;
    for (int k = threadIdx.x; k < K; k += QT) amax = fmaxf(amax, fabsf(row[k]));
    amax = block_max(amax, red);
    const QuantRule qr = quant_rule(amax, fm);
    for (int k = threadIdx.x; k < K; k += QT) qrow[k] = quant_at(row[k], qr, k, K, fm);
    if (threadIdx.x == 0) scales[m] = qr.scale;
}

namespace {
std::atomic<int> g_quant_fm{-1};   // -1: not read from the environment yet
}

int quant_fast_math() {
    int v = g_quant_fm.load(std::memory_order_relaxed);
    if (v < 0) {
        const char* e = getenv("P2CU_QUANT_FAST_MATH");
        int expected = -1;
        g_quant_fm.compare_exchange_strong(expected, (e && *e && *e != '0') ? 1 : 0);
        v = g_quant_fm.load(std::memory_order_relaxed);
    }
    return v;
}

void set_quant_fast_math(int on) { g_quant_fm.store(on ? 1 : 0, std::memory_order_relaxed); }

cudaError_t quant_rows_launch(const float* A, int M, int K, int lda, int8_t* q, float* scales, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(M);
    cfg.blockDim = dim3(QT);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // set-up overlaps the previous kernel
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, quant_rows_kernel, A, M, K, lda, q, scales, quant_fast_math());
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
