// fv_gemm_t.cu - the int8w five-value GEMM for few rows (one encoder window: M up to about a thousand), with the
// weights expanded straight into tensor memory.
//
// At M = 375 the block GEMMs are bound by shared-memory traffic and plane expansion, not by the tensor cores: with the
// weights as the MMA's B operand in shared memory, every weight code is written to shared memory by the expanding
// threads and read back by the MMA, and each 128-row tile of A expands the same planes again. This kernel turns the
// product around, C^T = B^T A^T: the weights are the MMA's A operand (M = 128 output columns per CTA, one TMEM lane
// each) and are written by the expanding threads straight into tensor memory (tcgen05.st); the quantised activations
// are the B operand (N = MT output rows) and are the only operand in shared memory. The int32 sums land in TMEM with
// one output column per lane and one output row per TMEM column, so the epilogue's global stores are whole 128-byte
// rows of C per warp.
//
// The weights come in the device-side value-index plane `vindex` (p2cu_fv_pack_vindex): one 4-bit index per weight
// into the weight's possible int8w codes, eight consecutive K rows of one column per 32-bit word (row 8r + t at bits
// 4t .. 4t + 3 of word [r][n]). A thread that owns column n keeps that column's codes as an 8-byte palette in two
// registers - {0, clo, -clo, 127, -127, 2 clo, -2} for the reference's 2-bit codes 1, 2 and 0 with flag 0 / 1 and
// the unused code 3, whose sign +2 the reference multiplies in with wrap-around (csrc/blas.c:1197-1238) - and a
// single byte permute (prmt) with 16 bits of the word as selectors turns four indices into the TMEM word of four
// K rows (four K values per 32-bit column, byte j = row 4c + j). Two permutes and one shift per 8 weights, against
// about twenty integer operations to decode the reference's 3-bit planes; 4 bits per weight on the device (302 MB for
// the whole model, between the planes' 229 MB and the code cache's 604 MB).
//
// Arithmetic: the int8w codes sign * (flag ? 127 : clo), clo = round(127 lo / hi) (csrc/blas.c:1222-1240), int32 sums
// over each 1024-row block of K, f = (float)acc * (hi * (1/127)), C = (beta == 0) ? f * as : fma(f, as, C_old),
// as = a_scale[m] * alpha (csrc/blas.c:1316-1366) - bit for bit the other kernels' results. K > 1024: one CTA per
// block writes f to the workspace slice of its block and fv_combine_kernel folds the slices in block order.
//
// One CTA: a 128-column x MT-row output tile and one 1024-row K block in eight 128-row stages, all resident at once
// (no ring: each barrier completes once). Warps 0-15 expand (warp w: TMEM lanes 32 (w % 4).., K rows 32 (w / 4) .. of every
// stage) and then run the epilogue; warp 16 issues the TMA loads (the weight planes before griddepcontrol.wait, A
// after it); warp 17 owns TMEM and issues the MMAs. Every wait is bounded.
#include <cstdint>
#include <utility>
#include <cuda.h>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "fv_gemm.h"
#include "fv_common.cuh"

namespace p2cu {

namespace {

constexpr int TN = 128;                    // output columns per CTA (the MMA's M)
constexpr int TBK = 128;                   // K rows per stage
constexpr int TNK = 8;                     // stages per CTA: one 1024-row K block
constexpr int EXP_WARPS = 16;
constexpr int PROD_WARP = 16, MMA_WARP = 17;
constexpr int NTHREADS = 18 * 32;
constexpr uint32_t VI_BYTES = (TBK / 8) * TN * 4;        // one stage of the index plane: 16 words x 128 columns
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t W_COL = 256;            // weight stage kb at TMEM columns W_COL + 32 kb (8 per MMA K step)
constexpr uint32_t MIN_SMEM = 120 * 1024;  // one CTA per SM: each CTA allocates the whole tensor memory

template <int MT>
struct TCfg {
    static_assert(MT % 16 == 0 && MT >= 16 && MT <= 128, "rows per CTA");
    static constexpr uint32_t A_BYTES = MT * 128;                        // one stage of A, K-major, 128-byte swizzle
    static constexpr uint32_t BAR_OFF = TNK * (A_BYTES + VI_BYTES);
    static constexpr uint32_t USED = 1024 + BAR_OFF + 256 + MT * 4;
    static constexpr uint32_t SMEM_BYTES = USED > MIN_SMEM ? USED : MIN_SMEM;
    static constexpr uint32_t IDESC = idesc_i8(TN, MT, false, false);
};

// Diagnostic builds (-DP2CU_TRACE) record %globaltimer at pipeline events of every CTA of 16 consecutive launches
// (ring by p.trace_slot) into g_t_trace; p2cu_debug_ttrace reads them. Events: 0 entry, 1 set-up done, 2 first
// weight stage landed, 3 expansion done, 4 dependency wait returned (producer), 5 last MMA issued, 6 accumulator
// ready, 7 stores issued; slot 8 holds the SM id; 9 + i / 17 + i: the i-th weight / A stage of the CTA's walk landed
// (observed by idle lanes of the producer warp).
#ifdef P2CU_TRACE
constexpr int TR_CTAS = 256, TR_EV = 25, TR_LAUNCHES = 16;
__device__ unsigned long long g_t_trace[TR_LAUNCHES * TR_CTAS * TR_EV];
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
#define TTRACE(ev) do { const int cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);          \
                        if (cta_ < TR_CTAS) g_t_trace[((p.trace_slot % TR_LAUNCHES) * TR_CTAS + cta_) * TR_EV + (ev)] \
                            = gtimer(); } while (0)
#else
#define TTRACE(ev) do { } while (0)
#endif

// Four int8w codes from four 4-bit indices (the low 16 bits of sel) and the column's palette (bytes 0-3 in lo,
// 4-7 in hi).
__device__ __forceinline__ uint32_t decode4(uint32_t lo, uint32_t hi, uint32_t sel) { return __byte_perm(lo, hi, sel); }

template <int MT>
__global__ void __launch_bounds__(NTHREADS, 1)
fv_gemm_t_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmVI,
                 const FvGemmTParams p) {
    using G = TCfg<MT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a_tiles = smem;
    uint32_t* vi_tiles = reinterpret_cast<uint32_t*>(smem + TNK * G::A_BYTES);
    uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + G::BAR_OFF);
    uint64_t* full_vi = full_a + TNK;
    uint64_t* wfull = full_vi + TNK;   // weight stage kb is in tensor memory (one arrival per expanding warp)
    uint64_t* accfull = wfull + TNK;
    uint64_t* drain = accfull + 1;
    uint64_t* sready = drain + 1;   // the row scales are in shared memory
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sready + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    float* row_scale = reinterpret_cast<float*>(smem + G::BAR_OFF + 256);   // [MT]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * TN, m0 = blockIdx.y * MT, z = blockIdx.z;
    const int k_begin = z * 1024;
    const int k_len = p.K - k_begin < 1024 ? p.K - k_begin : 1024;
    const int nk = (k_len + TBK - 1) / TBK;
    const bool partial = p.ksplit > 1;
    // Each CTA walks its K stages from a rotated start (int32 sums do not depend on the order): the CTAs that share
    // an A tile (one per column tile) or a weight tile (one per row tile) then ask L2 for different lines at any one
    // time instead of all for the same ones. Position i of the walk is stage stage_at(i).
    const int rot = (blockIdx.x + blockIdx.y) % nk;
    auto stage_at = [&](int i) { return i + rot < nk ? i + rot : i + rot - nk; };

    if (threadIdx.x == 0) {
        TTRACE(0);
#ifdef P2CU_TRACE
        {
            unsigned smid;
            asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
            const int cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
            if (cta_ < TR_CTAS) g_t_trace[((p.trace_slot % TR_LAUNCHES) * TR_CTAS + cta_) * TR_EV + 8] = smid;
        }
#endif
        for (int s = 0; s < TNK; ++s) {
            mbar_init(&full_a[s], 1);
            mbar_init(&full_vi[s], 1);
            mbar_init(&wfull[s], EXP_WARPS);
        }
        mbar_init(accfull, 1);
        mbar_init(drain, 1);
        mbar_init(sready, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == PROD_WARP && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmVI);
    }
    if (warp == MMA_WARP) {
        tmem_alloc(tmem_holder, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    if (threadIdx.x == 0) TTRACE(1);
    griddep_launch_dependents();

    if (warp == PROD_WARP) {
        // ---------------- TMA: the weight planes now, A once the previous kernel's writes are visible ----------------
        if (lane == 0) {
            const int vi_row0 = k_begin / 8;
            for (int i = 0; i < nk; ++i) {
                const int kb = stage_at(i);
                mbar_arrive_expect_tx(&full_vi[kb], VI_BYTES);
                tma_load_2d(vi_tiles + kb * (VI_BYTES / 4), &tmVI, &full_vi[kb], n0, vi_row0 + kb * (TBK / 8));
            }
            griddep_wait();
            TTRACE(4);
            for (int i = 0; i < nk; ++i) {
                const int kb = stage_at(i);
                mbar_arrive_expect_tx(&full_a[kb], G::A_BYTES);
                tma_load_2d(a_tiles + kb * G::A_BYTES, &tmA, &full_a[kb], k_begin + kb * TBK, m0);
            }
        }
#ifdef P2CU_TRACE
        if (lane == 1)   // when each TMA stage lands, as seen by otherwise idle lanes
            for (int i = 0; i < nk; ++i)
                if (mbar_wait(&full_vi[stage_at(i)], 0, DEV_TIMEOUT_FULL, p.err, abort_flag)) TTRACE(9 + i);
        if (lane == 2)
            for (int i = 0; i < nk; ++i)
                if (mbar_wait(&full_a[stage_at(i)], 0, DEV_TIMEOUT_FULL, p.err, abort_flag)) TTRACE(17 + i);
#endif
        // The tile's row scales a_scale[m] * alpha into shared memory for the epilogue (a_scales belong to the
        // previous kernels until the dependency wait).
        griddep_wait();
        for (int i = lane; i < MT; i += 32) {
            const int m = m0 + i;
            row_scale[i] = m < p.M ? __fmul_rn(p.a_scales[m], p.alpha) : 0.f;
        }
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(sready);
            // No copy may still be landing when the CTA exits (the abort path).
            for (int kb = 0; kb < nk; ++kb) {
                for (uint32_t i = 0; i < WAIT_LIMIT && !mbar_try_wait(smem_u32(&full_vi[kb]), 0); ++i) {}
                for (uint32_t i = 0; i < WAIT_LIMIT && !mbar_try_wait(smem_u32(&full_a[kb]), 0); ++i) {}
            }
        }
    } else if (warp == MMA_WARP) {
        // ---------------- MMA issue: D[128 cols x MT rows] += W^T[tmem] * A^T[smem] ----------------
        if (lane == 0) {
            for (int i = 0; i < nk; ++i) {
                const int kb = stage_at(i);
                if (!mbar_wait(&wfull[kb], 0, DEV_TIMEOUT_READY, p.err, abort_flag)) break;
                if (!mbar_wait(&full_a[kb], 0, DEV_TIMEOUT_FULL, p.err, abort_flag)) break;
                tc_fence_after();
                const uint32_t a_base = smem_u32(a_tiles + kb * G::A_BYTES);
#pragma unroll
                for (int ks = 0; ks < TBK / 32; ++ks) {
                    // A rows of 128 bytes (K-major), 8-row groups 1024 bytes apart; a K step of 32 moves 32 bytes
                    // inside the swizzle atom. The weights of K step ks: TMEM columns W_COL + 32 kb + 8 ks.
                    const uint64_t bdesc = smem_desc(a_base + ks * 32, 16, 1024, SWZ_128B);
                    mma_i8_ts(tmem, tmem + W_COL + 32 * kb + 8 * ks, bdesc, G::IDESC, (i > 0 || ks > 0) ? 1u : 0u);
                }
            }
            TTRACE(5);
            mma_commit(accfull);
            mma_commit(drain);   // every MMA issued has completed once this flips (also on the abort path)
            mbar_wait(drain, 0, DEV_TIMEOUT_DRAIN, p.err, abort_flag);
        }
        __syncwarp();
    } else {
        // ---------------- expansion (warps 0-15), then the epilogue ----------------
        const int g = warp >> 2, q = warp & 3;
        const int nl = 32 * q + lane, n = n0 + nl;
        const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
        const uint32_t clo = static_cast<uint32_t>(clo_of(p.lo[n], p.hi[n]));
        const uint32_t pal_lo = (clo << 8) | (((0x100u - clo) & 0xFFu) << 16) | (0x7Fu << 24);
        const uint32_t pal_hi = 0x81u | (((2u * clo) & 0xFFu) << 8) | (0xFEu << 16);
        const float c1 = __fmul_rn(p.hi[n], 1.0f / 127.0f);
        // Stages go to tensor memory two at a time: one wait for the stores of both (a store's completion is only
        // observable through tcgen05.wait::st, a round trip of several hundred cycles), then both are released.
        bool live = true;
        for (int i = 0; i < nk && live; i += 2) {
            const int kn = i + 1 < nk ? 2 : 1;
            for (int u = 0; u < kn; ++u) {
                const int kb = stage_at(i + u);
                if (!warp_wait(&full_vi[kb], 0, DEV_TIMEOUT_FULL, p.err, abort_flag)) {
                    live = false;
                    break;
                }
                if (i + u == 0 && warp == 0 && lane == 0) TTRACE(2);
                const uint32_t* vi = vi_tiles + kb * (VI_BYTES / 4) + (4 * g) * TN + nl;
                uint32_t w[8];
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const uint32_t x = vi[v * TN];   // K rows 32 g + 8 v .. + 7 of the stage
                    w[2 * v] = decode4(pal_lo, pal_hi, x);
                    w[2 * v + 1] = decode4(pal_lo, pal_hi, x >> 16);
                }
                tmem_st_32x32b_x8(tmem + lane_base + W_COL + 32 * kb + 8 * g, w);
            }
            if (!live) break;
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                for (int u = 0; u < kn; ++u) mbar_arrive(&wfull[stage_at(i + u)]);
        }
        if (warp == 0 && lane == 0) TTRACE(3);
        // The epilogue: each warp owns 8-row chunks ch = g, g + 4, ... of its 32 columns. C_old (when accumulating)
        // comes into registers while the MMAs run.
        constexpr int CPW = (MT / 8 + 3) / 4;
        float* out = partial ? p.ws + (static_cast<size_t>(z) * p.m_pad) * p.N + n : p.C + n;
        const size_t ld = partial ? static_cast<size_t>(p.N) : static_cast<size_t>(p.ldc);
        const bool load_old = !partial && !p.beta_zero;
        griddep_wait();   // C belongs to the previous kernels until here
        float old[CPW][8];
#pragma unroll
        for (int j = 0; j < CPW; ++j) {
            const int mb = m0 + 8 * (g + 4 * j);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                old[j][i] = load_old && g + 4 * j < MT / 8 && mb + i < p.M ? out[static_cast<size_t>(mb + i) * ld]
                                                                           : 0.f;
        }
        const bool ok = warp_wait(accfull, 0, DEV_TIMEOUT_ACC, p.err, abort_flag) &&
                        warp_wait(sready, 0, DEV_TIMEOUT_ACC, p.err, abort_flag);
        tc_fence_after();
        if (warp == 0 && lane == 0) TTRACE(6);
        if (ok) {
            uint32_t r[CPW][8];
#pragma unroll
            for (int j = 0; j < CPW; ++j)
                if (g + 4 * j < MT / 8) tmem_ld_32x32b_x8(tmem + lane_base + 8 * (g + 4 * j), r[j]);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < CPW; ++j) {
                const int ch = g + 4 * j;
                if (ch >= MT / 8 || m0 + 8 * ch >= p.M) break;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int m = m0 + 8 * ch + i;
                    if (m >= p.M) break;
                    const float f = __fmul_rn(__int2float_rn(static_cast<int>(r[j][i])), c1);
                    const float as = row_scale[8 * ch + i];
                    out[static_cast<size_t>(m) * ld] =
                        partial ? f : (load_old ? __fmaf_rn(f, as, old[j][i]) : __fmul_rn(f, as));
                }
            }
        }
        if (warp == 0 && lane == 0) TTRACE(7);
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == MMA_WARP) tmem_dealloc(tmem, TMEM_COLS);
}

// The value-index plane: thread (r, n) encodes K rows 8 r .. 8 r + 7 of column n from the reference's planes (signs
// [K][N/4], 2-bit code at bits 2 (n & 3); flags [K][N/8], bit n & 7). Index: code 1 -> 0 (zero), code 2 -> 1 / 3
// (+clo / +127 by the flag), code 0 -> 2 / 4 (-clo / -127), code 3 -> 5 / 6 (the reference's sign 2). Rows past K
// get index 0.
__global__ void __launch_bounds__(256) fv_vindex_kernel(const uint8_t* __restrict__ signs,
                                                        const uint8_t* __restrict__ flags, int K, int N,
                                                        uint32_t* __restrict__ out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int rows = (K + 7) / 8;
    if (i >= static_cast<size_t>(rows) * N) return;
    const int n = static_cast<int>(i % N), r = static_cast<int>(i / N);
    uint32_t word = 0;
    for (int t = 0; t < 8; ++t) {
        const int k = 8 * r + t;
        if (k >= K) break;
        const uint32_t code = (signs[static_cast<size_t>(k) * (N / 4) + n / 4] >> (2 * (n & 3))) & 3u;
        const uint32_t fl = (flags[static_cast<size_t>(k) * (N / 8) + n / 8] >> (n & 7)) & 1u;
        const uint32_t idx = code == 1 ? 0u : code == 2 ? 1u + 2u * fl : code == 0 ? 2u + 2u * fl : 5u + fl;
        word |= idx << (4 * t);
    }
    out[i] = word;
}

template <int MT>
cudaError_t launch_t(const CUtensorMap& a, const CUtensorMap& vi, const FvGemmTParams& p, cudaStream_t stream) {
    using G = TCfg<MT>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(fv_gemm_t_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(G::SMEM_BYTES));
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.N / TN, (p.M + MT - 1) / MT, p.ksplit);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = G::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fv_gemm_t_kernel<MT>, a, vi, p);
}

}  // namespace

#ifdef P2CU_TRACE
extern "C" __attribute__((visibility("default"))) int p2cu_debug_ttrace(unsigned long long* out, int n) {
    const int total = TR_LAUNCHES * TR_CTAS * TR_EV;
    return cudaMemcpyFromSymbol(out, g_t_trace, sizeof(unsigned long long) * (n < total ? n : total)) == cudaSuccess
               ? 0 : -1;
}
#endif

int fv_gemm_t_rows(int M, int N, int ksplit, int sms) {
    // As many row tiles as keep the launch within one CTA per SM: more CTAs spread the A loads and the stores of C,
    // and the expansion of the weights, repeated per row tile, costs two permutes per eight weights.
    const long col_tiles = static_cast<long>(N / 128) * ksplit;
    long tiles = col_tiles > 0 ? sms / col_tiles : 1;
    const long max_tiles = (M + 15) / 16;
    if (tiles < 1) tiles = 1;
    if (tiles > max_tiles) tiles = max_tiles;
    for (;;) {
        const int per = static_cast<int>((M + tiles - 1) / tiles);
        const int mt = (per + 15) / 16 * 16;
        if (mt <= 128 || tiles >= max_tiles) return mt <= 128 ? mt : 128;
        ++tiles;
    }
}

cudaError_t fv_gemm_t_launch(int mt, const CUtensorMap& a, const CUtensorMap& vi, const FvGemmTParams& p,
                             cudaStream_t stream) {
    switch (mt) {
    case 16: return launch_t<16>(a, vi, p, stream);
    case 32: return launch_t<32>(a, vi, p, stream);
    case 48: return launch_t<48>(a, vi, p, stream);
    case 64: return launch_t<64>(a, vi, p, stream);
    case 80: return launch_t<80>(a, vi, p, stream);
    case 96: return launch_t<96>(a, vi, p, stream);
    case 112: return launch_t<112>(a, vi, p, stream);
    case 128: return launch_t<128>(a, vi, p, stream);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t fv_vindex_launch(const uint8_t* signs, const uint8_t* flags, int K, int N, uint32_t* out,
                             cudaStream_t stream) {
    const size_t threads = static_cast<size_t>((K + 7) / 8) * N;
    fv_vindex_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(signs, flags, K, N, out);
    return cudaGetLastError();
}

}  // namespace p2cu
