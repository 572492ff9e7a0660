// probes.cu - measurements of the B200 features the GEMM kernels are built around, for the roofline and the design:
//   * p2cu_probe_int8_mma: the tcgen05 kind::i8 MMA rate with shared-memory operands (M = 128, N = 256, K = 32 per
//     instruction, one CTA per SM; or M = 256 on CTA pairs), i.e. the measured int8 dense peak;
//   * p2cu_probe_tma_load: tiled TMA load throughput per SM from an L2-resident int8 matrix, with the loads issued
//     by 1-4 warps of a CTA - one warp's loads complete one after another, which is why the GEMM kernels spread their
//     K steps over several producer warps;
//   * p2cu_probe_int8_ring: the CTA-pair MMA stream fed through the stage ring of the pair GEMM kernel without any
//     copies - six stages of 32 KB per CTA, each released by the MMAs' commit to both CTAs' "empty" barriers and
//     handed back by a producer thread's arrive, the odd CTA's stages relayed to the even one (mode 1) or arrived
//     remotely on the even CTA's barrier (mode 2), against the same MMAs issued without waiting (mode 0). The gap is
//     what the handshake alone costs: the MMAs of a step can start only after the MMAs six steps back have
//     completed and their release has travelled round the ring.
//   * p2cu_probe_packed_math: the encoder's packed fp32x2 SiLU and exp (numerics.cuh) against their scalar forms,
//     and the packed reciprocal against __frcp_rn, bit for bit over every input in their ranges.
// Each allocates its own buffers, runs a few launches, and reports through out-parameters. Every wait is bounded.
// Built as its own library (libphonon2_probes.so, declared in probes.h): the product library does not carry them.
#include <cstdint>
#include <cstdio>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdarg>
#include "probes.h"
#include "ptx.cuh"
#include "numerics.cuh"

namespace p2cu {
namespace {

// This library's own error text, device error word and tensor maps (it is built apart from libphonon2_b200.so).
char g_probe_msg[256] = "";
__device__ uint32_t g_probe_err;

int fail_fmt(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_probe_msg, sizeof(g_probe_msg), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_error(cudaError_t e, const char* what) { return fail_fmt(-2, "%s: %s", what, cudaGetErrorString(e)); }

uint32_t* device_error_word() {
    void* p = nullptr;
    return cudaGetSymbolAddress(&p, g_probe_err) == cudaSuccess ? static_cast<uint32_t*>(p) : nullptr;
}

// Synchronise and read (then clear) the error word: -3 when a probe's bounded wait ran out.
int check_device() {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_error(e, "probe");
    uint32_t v = 0, zero = 0;
    if ((e = cudaMemcpyFromSymbol(&v, g_probe_err, sizeof(v))) != cudaSuccess) return cuda_error(e, "error word");
    if (v) {
        cudaMemcpyToSymbol(g_probe_err, &zero, sizeof(zero));
        return fail_fmt(-3, "a probe's wait ran out (device error code %u)", v);
    }
    return 0;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// An int8 [outer][inner] tensor map, rows `stride` bytes apart, boxes box_in x box_out, 128-byte swizzle.
int make_tile_map(CUtensorMap* map, const void* base, int, uint64_t inner, uint64_t outer, uint64_t stride,
                  uint32_t box_in, uint32_t box_out, int, const char* what) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
        return fail_fmt(-2, "cuTensorMapEncodeTiled is not available");
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {stride};
    const cuuint32_t box[2] = {box_in, box_out};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = reinterpret_cast<EncodeTiledFn>(p)(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base),
                                                    dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : fail_fmt(-2, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
}

constexpr int PROBE_THREADS = 128;
constexpr uint32_t PROBE_TIMEOUT = 30;

// One CTA per SM: `iters` K = 128 steps of four MMAs on zero operands (128 x 128 A, 256-column B, MN-major).
__global__ void __launch_bounds__(PROBE_THREADS, 1) mma_probe_kernel(int iters, uint32_t* err) {
    extern __shared__ uint8_t raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a = smem;                 // 16 KB
    uint8_t* b = smem + 16384;         // 32 KB
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 16384 + 32768);
    uint32_t* holder = reinterpret_cast<uint32_t*>(bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(holder + 1);
    for (int i = threadIdx.x; i < (16384 + 32768) / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    fence_proxy_async_smem();
    if (threadIdx.x < 32) {
        tmem_alloc(holder, 256);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *holder;
    if (threadIdx.x == 0) {
        constexpr uint32_t IDESC = idesc_i8(128, 256, false, true);
        const uint32_t ab = smem_u32(a), bb = smem_u32(b);
        for (int it = 0; it < iters; ++it)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
                mma_i8(tmem, smem_desc(ab + ks * 32, 16, 1024, SWZ_128B),
                       smem_desc(bb + ks * 4 * 1024, 16384, 1024, SWZ_128B), IDESC, (it > 0 || ks > 0) ? 1u : 0u);
        mma_commit(bar);
        mbar_wait(bar, 0, PROBE_TIMEOUT, err, abort_flag);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x < 32) tmem_dealloc(tmem, 256);
}

// Clusters of two: the even CTA issues M = 256 MMAs over both CTAs' operands (each: 128 x 128 A, 128 B columns).
__global__ void __launch_bounds__(PROBE_THREADS, 1) mma_pair_probe_kernel(int iters, uint32_t* err) {
    extern __shared__ uint8_t raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a = smem;
    uint8_t* b = smem + 16384;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 16384 + 32768);
    uint32_t* holder = reinterpret_cast<uint32_t*>(bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(holder + 1);
    for (int i = threadIdx.x; i < (16384 + 32768) / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    fence_proxy_async_smem();
    if (threadIdx.x < 32) {
        tmem_alloc_pair(holder, 256);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = *holder;
    if (threadIdx.x == 0 && cluster_ctarank() == 0) {
        constexpr uint32_t IDESC = idesc_i8(256, 256, false, true);
        const uint32_t ab = smem_u32(a), bb = smem_u32(b);
        for (int it = 0; it < iters; ++it)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
                mma_i8_pair(tmem, smem_desc(ab + ks * 32, 16, 1024, SWZ_128B),
                            smem_desc(bb + ks * 4 * 1024, 1024, 1024, SWZ_128B), IDESC, (it > 0 || ks > 0) ? 1u : 0u);
        mma_commit_pair(bar, 0x1);
        mbar_wait(bar, 0, PROBE_TIMEOUT, err, abort_flag);
    }
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    if (threadIdx.x < 32) tmem_dealloc_pair(tmem, 256);
}

constexpr int RING_STAGES = 6;
constexpr int RING_STAGE_BYTES = 32768;   // 16 KB of A, 16 KB of B per CTA, as a pair GEMM stage

// Clusters of two over a six-stage ring of zero operands: mode 0 issues every step at once (the first round waits
// like the others), mode 1 hands stages back through the even CTA's producer and the odd CTA's relay, mode 2 has the
// odd CTA's producer arrive on the even CTA's barrier directly.
__global__ void __launch_bounds__(PROBE_THREADS, 1) mma_ring_probe_kernel(int iters, int mode, uint32_t* err) {
    extern __shared__ uint8_t raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + RING_STAGES * RING_STAGE_BYTES);
    uint64_t* peer = full + RING_STAGES;
    uint64_t* empty = peer + RING_STAGES;
    uint64_t* done = empty + RING_STAGES;
    uint32_t* holder = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(holder + 1);
    const uint32_t rank = cluster_ctarank();
    for (int i = threadIdx.x; i < RING_STAGES * RING_STAGE_BYTES / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x == 0) {
        for (int s = 0; s < RING_STAGES; ++s) {
            mbar_init(&full[s], mode == 2 && rank == 0 ? 2 : 1);
            mbar_init(&peer[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    fence_proxy_async_smem();
    if (threadIdx.x < 32) {
        tmem_alloc_pair(holder, 256);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = *holder;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int handed = mode == 0 ? RING_STAGES : iters;   // stages passed through the ring
    if (warp == 1 && lane == 0) {
        // producer of this CTA: a stage is refilled (here: handed back) once the pair's MMAs are done with it
        const uint32_t full0 = cluster_map(&full[0], 0);
        for (int g = 0; g < handed; ++g) {
            const int s = g % RING_STAGES, r = g / RING_STAGES;
            if (g >= RING_STAGES && !mbar_wait(&empty[s], (r & 1) ^ 1, PROBE_TIMEOUT, err, abort_flag)) break;
            if (mode == 2 && rank == 1) mbar_arrive_remote_relaxed(full0 + static_cast<uint32_t>(s) * 8u);
            else mbar_arrive(&full[s]);
        }
    } else if (warp == 0 && lane == 0 && rank == 1 && mode != 2) {
        // relay of the odd CTA's stages to the even CTA
        const uint32_t peer0 = cluster_map(&peer[0], 0);
        for (int g = 0; g < handed; ++g) {
            const int s = g % RING_STAGES, r = g / RING_STAGES;
            if (!mbar_wait(&full[s], r & 1, PROBE_TIMEOUT, err, abort_flag)) break;
            mbar_arrive_remote_relaxed(peer0 + static_cast<uint32_t>(s) * 8u);
        }
    } else if (warp == 0 && lane == 0 && rank == 0) {
        constexpr uint32_t IDESC = idesc_i8(256, 256, false, true);
        const uint32_t base = smem_u32(smem);
        for (int g = 0; g < iters; ++g) {
            const int s = g % RING_STAGES, r = g / RING_STAGES;
            if (g < handed) {
                if (!mbar_wait(&full[s], r & 1, PROBE_TIMEOUT, err, abort_flag)) break;
                if (mode != 2 && !mbar_wait(&peer[s], r & 1, PROBE_TIMEOUT, err, abort_flag)) break;
            }
            tc_fence_after();
            const uint32_t ab = base + s * RING_STAGE_BYTES, bb = ab + 16384;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
                mma_i8_pair(tmem, smem_desc(ab + ks * 32, 16, 1024, SWZ_128B),
                            smem_desc(bb + ks * 4 * 1024, 1024, 1024, SWZ_128B), IDESC, (g > 0 || ks > 0) ? 1u : 0u);
            mma_commit_pair(&empty[s], 0x3);
        }
        mma_commit_pair(done, 0x1);
        mbar_wait(done, 0, PROBE_TIMEOUT, err, abort_flag);
    }
    __syncwarp();
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    if (threadIdx.x < 32) tmem_dealloc_pair(tmem, 256);
}

// One CTA per SM: `warps` warps each stream boxes of `box_bytes` (128-byte rows) through a ring of two slots.
__global__ void __launch_bounds__(PROBE_THREADS, 1)
tma_probe_kernel(const __grid_constant__ CUtensorMap tm, int boxes, int warps, int box_bytes, int row_blocks,
                 uint32_t* err) {
    extern __shared__ uint8_t raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 2 * warps * box_bytes);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bar + 8);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < 8; ++s) mbar_init(&bar[s], 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tm);
    }
    __syncthreads();
    if (warp < warps && lane == 0) {
        const int box_rows = box_bytes / 128, mine = boxes / warps;
        for (int i = 0; i < mine + 2; ++i) {
            const int slot = 2 * warp + (i & 1);
            if (i >= 2 && !mbar_wait(&bar[slot], ((i - 2) >> 1) & 1, PROBE_TIMEOUT, err, abort_flag)) break;
            if (i < mine) {
                const int blk = static_cast<int>((blockIdx.x * 7919u + (i * warps + warp) * 104729u) % row_blocks);
                mbar_arrive_expect_tx(&bar[slot], box_bytes);
                tma_load_2d(smem + slot * box_bytes, &tm, &bar[slot], 0, blk * box_rows);
            }
        }
    }
    __syncthreads();
}

// exp_poly as first written: k by rintf and an integer conversion (the reference's formula, step for step)
__device__ __forceinline__ float exp_rint(float x) {
    x = fminf(fmaxf(x, -87.0f), 87.0f);
    const float kf = rintf(__fmul_rn(x, 1.44269504088896341f));
    const int ki = static_cast<int>(kf);
    const float r = __fmaf_rn(-kf, 0.69314718055994529f, x);
    float y = 1.0f / 120.0f;
    y = __fmaf_rn(y, r, 1.0f / 24.0f);
    y = __fmaf_rn(y, r, 1.0f / 6.0f);
    y = __fmaf_rn(y, r, 0.5f);
    y = __fmaf_rn(y, r, 1.0f);
    y = __fmaf_rn(y, r, 1.0f);
    return __fmul_rn(y, __int_as_float((ki + 127) << 23));
}

__device__ __forceinline__ bool same_bits(float a, float b) {
    return __float_as_uint(a) == __float_as_uint(b) || (a != a && b != b);
}

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16; x *= 0x7feb352du; x ^= x >> 15; x *= 0x846ca68bu; x ^= x >> 16;
    return x;
}

// Over every 32-bit pattern u (x = the float with those bits, x' = -x): bad[0] exp_poly(x) != exp_rint(x); bad[1]
// exp_poly2 on (x, x') != exp_poly on each; bad[2] swish2 on (x', x) != swish1 on each; bad[3] f2_fma != __fmaf_rn
// on hashed operand triples (normal, subnormal and special values); bad[4] rcp2_ge1 != __frcp_rn over [1, 2^126).
__global__ void packed_math_kernel(unsigned long long* bad) {
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    unsigned long long b0 = 0, b1 = 0, b2 = 0, b3 = 0, b4 = 0;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < (1ull << 32); i += stride) {
        const uint32_t u = static_cast<uint32_t>(i);
        const float x = __uint_as_float(u), xn = __uint_as_float(u ^ 0x80000000u);
        const float ex = exp_poly(x);
        b0 += !same_bits(ex, exp_rint(x));
        const float2 e2 = exp_poly2(make_float2(x, xn));
        b1 += !same_bits(e2.x, ex) || !same_bits(e2.y, exp_poly(xn));
        const float2 s2 = swish2(make_float2(xn, x));
        b2 += !same_bits(s2.y, swish1(x)) || !same_bits(s2.x, swish1(xn));
        const uint32_t h1 = mix32(u), h2 = mix32(u ^ 0x9e3779b9u), h3 = mix32(u + 0x632be5abu);
        const float a = __uint_as_float(h1), bb = __uint_as_float(h2), c = __uint_as_float(h3);
        const float as = __uint_as_float(h1 & 0x807fffffu), cs = __uint_as_float(h3 >> 9);
        const float2 f = f2_fma(make_float2(a, as), make_float2(bb, bb), make_float2(c, cs));
        b3 += !same_bits(f.x, __fmaf_rn(a, bb, c)) || !same_bits(f.y, __fmaf_rn(as, bb, cs));
        if (u >= 0x3F800000u && u < 0x7E800000u && !(u & 1u)) {
            const float2 d = make_float2(x, __uint_as_float(u + 1));
            const float2 r = rcp2_ge1(d, make_float2(-d.x, -d.y));
            b4 += (__float_as_uint(r.x) != __float_as_uint(__frcp_rn(d.x))) +
                  (__float_as_uint(r.y) != __float_as_uint(__frcp_rn(d.y)));
        }
    }
    if (b0) atomicAdd(&bad[0], b0);
    if (b1) atomicAdd(&bad[1], b1);
    if (b2) atomicAdd(&bad[2], b2);
    if (b3) atomicAdd(&bad[3], b3);
    if (b4) atomicAdd(&bad[4], b4);
}

int sms_of_device() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

}  // namespace
}  // namespace p2cu

extern "C" {

const char* p2cu_probes_last_error(void) { return p2cu::g_probe_msg; }

// The int8 MMA rate (MACs per second, all SMs) over `iters` K = 128 steps per SM; pair != 0 on CTA pairs.
int p2cu_probe_int8_mma(int pair, int iters, double* macs_per_s) {
    using namespace p2cu;
    if (!macs_per_s || iters < 1 || iters > (1 << 20)) return fail_fmt(-1, "p2cu_probe_int8_mma: arguments");
    const int sms = sms_of_device();
    const int smem = 1024 + 16384 + 32768 + 64;
    cudaError_t e = cudaFuncSetAttribute(pair ? mma_pair_probe_kernel : mma_probe_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (e == cudaSuccess) e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    float best = 0.f;
    for (int rep = 0; e == cudaSuccess && rep < 3; ++rep) {
        cudaEventRecord(e0);
        if (pair) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(sms / 2 * 2);
            cfg.blockDim = dim3(PROBE_THREADS);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = 2;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            e = cudaLaunchKernelEx(&cfg, mma_pair_probe_kernel, iters, device_error_word());
        } else {
            mma_probe_kernel<<<sms, PROBE_THREADS, smem>>>(iters, device_error_word());
            e = cudaGetLastError();
        }
        cudaEventRecord(e1);
        if (e == cudaSuccess) e = cudaEventSynchronize(e1);
        float ms = 0.f;
        if (e == cudaSuccess) cudaEventElapsedTime(&ms, e0, e1);
        if (rep > 0 && (best == 0.f || ms < best)) best = ms;
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (e != cudaSuccess) return cuda_error(e, "p2cu_probe_int8_mma");
    if (int rc = check_device()) return rc;
    const double macs = (pair ? 256.0 : 128.0) * 256.0 * 128.0 * iters * (pair ? sms / 2 : sms);
    *macs_per_s = macs / (best * 1e-3);
    return 0;
}

int p2cu_probe_int8_ring(int mode, int iters, double* macs_per_s) {
    using namespace p2cu;
    if (!macs_per_s || mode < 0 || mode > 2 || iters < 1 || iters > (1 << 20))
        return fail_fmt(-1, "p2cu_probe_int8_ring: arguments");
    const int sms = sms_of_device();
    const int smem = 1024 + RING_STAGES * RING_STAGE_BYTES + 256;
    cudaError_t e = cudaFuncSetAttribute(mma_ring_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (e == cudaSuccess) e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    float best = 0.f;
    for (int rep = 0; e == cudaSuccess && rep < 3; ++rep) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(sms / 2 * 2);
        cfg.blockDim = dim3(PROBE_THREADS);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaEventRecord(e0);
        e = cudaLaunchKernelEx(&cfg, mma_ring_probe_kernel, iters, mode, device_error_word());
        cudaEventRecord(e1);
        if (e == cudaSuccess) e = cudaEventSynchronize(e1);
        float ms = 0.f;
        if (e == cudaSuccess) cudaEventElapsedTime(&ms, e0, e1);
        if (rep > 0 && (best == 0.f || ms < best)) best = ms;
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (e != cudaSuccess) return cuda_error(e, "p2cu_probe_int8_ring");
    if (int rc = check_device()) return rc;
    *macs_per_s = 256.0 * 256.0 * 128.0 * iters * (sms / 2) / (best * 1e-3);
    return 0;
}

// Tiled TMA load throughput (bytes per second per SM) with `warps` issuing warps per CTA and boxes of `box_rows`
// 128-byte rows (1-256), from an 8 MB matrix (L2-resident) with 128-byte swizzle.
int p2cu_probe_tma_load(int warps, int box_rows, double* bytes_per_s_per_sm) {
    using namespace p2cu;
    if (!bytes_per_s_per_sm || warps < 1 || warps > 4 || box_rows < 8 || box_rows > 256 || (box_rows & 7) ||
        2 * warps * 128 * box_rows > 196608)
        return fail_fmt(-1, "p2cu_probe_tma_load: warps 1-4, box rows 8-256 (multiple of 8), "
                        "2 x warps x box <= 192 KB");
    const int rows = 8192, width = 128;   // an [8192][1024] matrix read as 128-byte columns of its first 128 bytes
    const int stride = 1024;
    uint8_t* buf = nullptr;
    cudaError_t e = cudaMalloc(&buf, static_cast<size_t>(rows) * stride);
    if (e != cudaSuccess) return cuda_error(e, "p2cu_probe_tma_load: cudaMalloc");
    cudaMemset(buf, 1, static_cast<size_t>(rows) * stride);
    CUtensorMap tm;
    int rc = make_tile_map(&tm, buf, 1, width, rows, stride, 128, static_cast<uint32_t>(box_rows), 128,
                           "p2cu_probe_tma_load");
    const int sms = sms_of_device();
    const int smem = 1024 + 196608 + 128;
    const int boxes = 400;
    float best = 0.f;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (rc == 0) {
        e = cudaFuncSetAttribute(tma_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e == cudaSuccess) e = cudaEventCreate(&e0);
        if (e == cudaSuccess) e = cudaEventCreate(&e1);
        for (int rep = 0; e == cudaSuccess && rep < 3; ++rep) {
            cudaEventRecord(e0);
            tma_probe_kernel<<<sms, PROBE_THREADS, smem>>>(tm, boxes, warps, 128 * box_rows, rows / box_rows,
                                                          device_error_word());
            e = cudaGetLastError();
            cudaEventRecord(e1);
            if (e == cudaSuccess) e = cudaEventSynchronize(e1);
            float ms = 0.f;
            if (e == cudaSuccess) cudaEventElapsedTime(&ms, e0, e1);
            if (rep > 0 && (best == 0.f || ms < best)) best = ms;
        }
        if (e != cudaSuccess) rc = cuda_error(e, "p2cu_probe_tma_load");
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaFree(buf);
    if (rc == 0) rc = check_device();
    if (rc == 0) *bytes_per_s_per_sm = static_cast<double>(boxes / warps * warps) * 128 * box_rows /
                                              (best * 1e-3);
    return rc;
}

// The packed fp32x2 forms against the scalar ones (packed_math_kernel): mismatches[0..4] as listed there.
int p2cu_probe_packed_math(unsigned long long* mismatches) {
    using namespace p2cu;
    if (!mismatches) return fail_fmt(-1, "p2cu_probe_packed_math: arguments");
    unsigned long long* bad = nullptr;
    cudaError_t e = cudaMalloc(&bad, 5 * sizeof(unsigned long long));
    if (e != cudaSuccess) return cuda_error(e, "p2cu_probe_packed_math: buffer");
    int rc = 0;
    e = cudaMemset(bad, 0, 5 * sizeof(unsigned long long));
    if (e == cudaSuccess) {
        packed_math_kernel<<<sms_of_device() * 8, 256>>>(bad);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(mismatches, bad, 5 * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) rc = cuda_error(e, "p2cu_probe_packed_math");
    cudaFree(bad);
    return rc;
}

}  // extern "C"
