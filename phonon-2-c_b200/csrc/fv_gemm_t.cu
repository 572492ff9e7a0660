// fv_gemm_t.cu - the int8w five-value GEMM for few rows (one encoder window: M up to about a thousand), with the
// weights expanded straight into tensor memory.
//
// At M = 375 a block GEMM is short (a few microseconds) and what bounds it is how fast each SM can take in its operands
// and how much each CTA must take in, not the tensor cores. With the weights as the MMA's B operand in shared memory
// (fv_gemm.cu), every weight code is written to shared memory by the expanding threads and read back by the MMA, and
// each 128-row tile of A expands the same planes again. This kernel turns the product around, C^T = B^T A^T: the
// weights are the MMA's A operand (M = 128 output columns per CTA, one TMEM lane each) and are written by the
// expanding threads straight into tensor memory (tcgen05.st); the quantised activations are the B operand (N = MT
// output rows) and are the only operand in shared memory. The int32 sums land in TMEM with one output column per lane
// and one output row per TMEM column, so the epilogue's global stores are whole 128-byte rows of C per warp.
//
// The weights come as the device-side value-index plane `vindex` (p2cu_fv_pack_vindex): one 4-bit index per weight
// into the weight's possible int8w codes, grouped so that the 32 K rows of one column in one 32-row chunk are 16
// contiguous bytes (four words; word v holds rows 8 v .. 8 v + 7 at bits 4 t). A thread that owns column n loads those
// 16 bytes with one vector load per stage (the LSU path, beside the TMA that brings A) and keeps the column's codes as
// an 8-byte palette in two registers - {0, clo, -clo, 127, -127, 2 clo, -2} for the reference's 2-bit codes 1, 2 and 0
// with flag 0 / 1 and the unused code 3, whose sign +2 the reference multiplies in with wrap-around
// (csrc/blas.c:1197-1238) - so that one byte permute (prmt) with 16 bits of a word as selectors gives the TMEM word of
// four K rows (four K values per 32-bit column, byte j = row 4c + j). 4 bits per weight on the device (302 MB for the
// whole model, between the reference planes' 229 MB and the code cache's 604 MB); two permutes and a shift per eight
// weights against about twenty integer operations to decode the 3-bit planes.
//
// Arithmetic: the int8w codes sign * (flag ? 127 : clo), clo = round(127 lo / hi) (csrc/blas.c:1222-1240), int32 sums
// over each 1024-row block of K, f = (float)acc * (hi * (1/127)), C = (beta == 0) ? f * as : fma(f, as, C_old),
// as = a_scale[m] * alpha (csrc/blas.c:1316-1366) - bit for bit the other kernels' results. K > 1024: one CTA per
// block writes f to the workspace slice of its block and fv_combine_kernel folds the slices in block order.
//
// One CTA: a 128-column x MT-row output tile and one 1024-row K block in eight 128-row stages, all resident at once
// (no ring: each barrier completes once). Warps 0-15 expand (warp w: TMEM lanes 32 (w % 4).., K rows 32 (w / 4) .. of
// every stage; four stages per tcgen05.wait::st) and then run the epilogue; warps 16-23 issue the TMA loads of A (after griddepcontrol.wait), stage i from
// warp 16 + i: one SM's TMA takes in about 57 GB/s from boxes one thread issues and about twice that from four or more
// issuing warps; warp 24 owns TMEM and issues the MMAs (converged, one elected lane issuing).
// Every wait is bounded.
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
constexpr int PROD_WARP = 16, NPROD = 8, MMA_WARP = PROD_WARP + NPROD;
constexpr int NTHREADS = (MMA_WARP + 1) * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t W_COL = 256;            // weight stage kb at TMEM columns W_COL + 32 kb (8 per MMA K step)
constexpr uint32_t MIN_SMEM = 120 * 1024;  // one CTA per SM: each CTA allocates the whole tensor memory

template <int MT>
struct TCfg {
    static_assert(MT % 16 == 0 && MT >= 16 && MT <= 128, "rows per CTA");
    static constexpr uint32_t A_BYTES = MT * 128;                        // one stage of A, K-major, 128-byte swizzle
    static constexpr uint32_t VI_OFF = TNK * A_BYTES;                    // weight indices: [stage][thread][16 B]
    static constexpr uint32_t BAR_OFF = VI_OFF + TNK * EXP_WARPS * 32 * 16;
    static constexpr uint32_t USED = 1024 + BAR_OFF + 256 + MT * 4;
    static constexpr uint32_t SMEM_BYTES = USED > MIN_SMEM ? USED : MIN_SMEM;
    static constexpr uint32_t IDESC = idesc_i8(TN, MT, false, false);
};

// Diagnostic builds (-DP2CU_TRACE) record clock64 at pipeline events of every CTA of 16 consecutive launches
// (ring by p.trace_slot) into g_t_trace; p2cu_debug_ttrace reads them. Events: 0 entry, 1 set-up done, 2 first
// weight stage in registers, 3 expansion done, 4 dependency wait returned (producer), 5 last MMA issued,
// 6 accumulator ready, 7 stores issued; slot 8 holds the SM id; 9 + kb: A stage kb landed (its producer warp);
// 17 + kb: the MMAs of stage kb issued; 25 + kb: weight stage kb seen complete by the MMA issuer; 33 + w: expanding
// warp w done; 41: the epilogue's accumulator loads returned (warp 0); 42: the epilogue's dependency wait returned
// (warp 0); 49: %globaltimer at entry (reading it takes a fraction of a microsecond, so it is read once).
#ifdef P2CU_TRACE
constexpr int TR_CTAS = 256, TR_EV = 50, TR_LAUNCHES = 16;
__device__ unsigned long long g_t_trace[TR_LAUNCHES * TR_CTAS * TR_EV];
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
#define TTRACE(ev) do { const int cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);          \
                        if (cta_ < TR_CTAS) g_t_trace[((p.trace_slot % TR_LAUNCHES) * TR_CTAS + cta_) * TR_EV + (ev)] \
                            = clock64(); } while (0)
#else
#define TTRACE(ev) do { } while (0)
#endif

// Four int8w codes from four 4-bit indices (the low 16 bits of sel) and the column's palette (bytes 0-3 in lo,
// 4-7 in hi).
__device__ __forceinline__ uint32_t decode4(uint32_t lo, uint32_t hi, uint32_t sel) { return __byte_perm(lo, hi, sel); }

// 16 bytes global -> shared through the LSU path (cp.async, L2 only), zero-filled when `valid` is false; completion
// per commit group of the issuing thread.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

// ACC: the epilogue accumulates into C (beta != 0 and a single K block), C_old read while the MMAs run.
template <int MT, bool ACC>
__global__ void __launch_bounds__(NTHREADS, 1)
fv_gemm_t_kernel(const __grid_constant__ CUtensorMap tmA, const FvGemmTParams p) {
    using G = TCfg<MT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a_tiles = smem;
    uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + G::BAR_OFF);
    uint64_t* wfull = full_a + TNK;   // weight stage kb is in tensor memory (one arrival per expanding warp)
    uint64_t* accfull = wfull + TNK;
    uint64_t* drain = accfull + 1;
    uint64_t* sready = drain + 1;     // the row scales are in shared memory
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sready + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    float* row_scale = reinterpret_cast<float*>(smem + G::BAR_OFF + 256);   // [MT]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * TN, m0 = blockIdx.y * MT, z = blockIdx.z;
    const int k_begin = z * 1024;
    const int k_len = p.K - k_begin < 1024 ? p.K - k_begin : 1024;
    const int nk = (k_len + TBK - 1) / TBK;
    const bool partial = p.ksplit > 1;

    // The expanding threads' copies of their weight indices go out first of all (they need no barrier and no tensor
    // memory, and their first bytes take about a microsecond to arrive): thread t of warps 0-15 copies, for stage kb,
    // the 16 bytes of chunk k_begin / 32 + 4 kb + (t / 128) of column n0 + t % 128, one commit group per stage; rows
    // past K read as zeros.
    if (warp < EXP_WARPS) {
        const int n = n0 + 32 * (warp & 3) + lane;
        const uint4* vsrc = reinterpret_cast<const uint4*>(p.vindex) + n;
        const int kc0 = k_begin / 32 + (warp >> 2);
        uint4* vdst = reinterpret_cast<uint4*>(smem + G::VI_OFF) + threadIdx.x;
#pragma unroll
        for (int kb = 0; kb < TNK; ++kb) {
            const int kc = kc0 + 4 * kb;
            const bool valid = kb < nk && kc < p.kchunks;
            cp_async16(vdst + kb * (EXP_WARPS * 32), valid ? vsrc + static_cast<size_t>(kc) * p.N : vsrc, valid);
            cp_async_commit();
        }
    }

    if (threadIdx.x == 0) {
        TTRACE(0);
#ifdef P2CU_TRACE
        {
            unsigned smid;
            asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
            const int cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
            if (cta_ < TR_CTAS) {
                g_t_trace[((p.trace_slot % TR_LAUNCHES) * TR_CTAS + cta_) * TR_EV + 8] = smid;
                g_t_trace[((p.trace_slot % TR_LAUNCHES) * TR_CTAS + cta_) * TR_EV + 49] = gtimer();
            }
        }
#endif
        for (int s = 0; s < TNK; ++s) {
            mbar_init(&full_a[s], 1);
            mbar_init(&wfull[s], EXP_WARPS);
        }
        mbar_init(accfull, 1);
        mbar_init(drain, 1);
        mbar_init(sready, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == PROD_WARP && lane == 0) tma_prefetch_desc(&tmA);
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

    if (warp >= PROD_WARP && warp < PROD_WARP + NPROD) {
        // ---------------- TMA: A once the previous kernel's writes are visible ----------------
        griddep_wait();
        if (lane == 0) {
            if (warp == PROD_WARP) TTRACE(4);
            for (int kb = warp - PROD_WARP; kb < nk; kb += NPROD) {
                mbar_arrive_expect_tx(&full_a[kb], G::A_BYTES);
                tma_load_2d(a_tiles + kb * G::A_BYTES, &tmA, &full_a[kb], k_begin + kb * TBK, m0);
            }
        }
        if (warp == PROD_WARP) {
            // The tile's row scales a_scale[m] * alpha into shared memory for the epilogue.
            for (int i = lane; i < MT; i += 32) {
                const int m = m0 + i;
                row_scale[i] = m < p.M ? __fmul_rn(p.a_scales[m], p.alpha) : 0.f;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(sready);
        }
        if (lane == 0) {
            // No copy this warp issued may still be landing when the CTA exits (the abort path).
            for (int kb = warp - PROD_WARP; kb < nk; kb += NPROD) {
                for (uint32_t i = 0; i < (WAIT_LIMIT >> 5) && !mbar_test_wait(smem_u32(&full_a[kb]), 0); ++i)
                    __nanosleep(64);
                TTRACE(9 + kb);
            }
        }
    } else if (warp == MMA_WARP) {
        // ---------------- MMA issue: D[128 cols x MT rows] += W^T[tmem] * A^T[smem] ----------------
        // The whole warp runs this loop converged and waits with all lanes at once; one elected lane issues each MMA
        // through a predicate. (Issued from code that lane 0 ran alone, with the waits' branches inside it, the same
        // MMAs went out at ~65 ns each; converged, ~37 ns, against ~27 ns of tensor-core work at N = 96.)
        const uint32_t lead = elect_one();
        // A rows of 128 bytes (K-major), 8-row groups 1024 bytes apart; a K step of 32 moves 32 bytes inside the
        // swizzle atom. The descriptor's start-address field holds the address >> 4 (14 bits; shared memory addresses
        // stay below 256 KB), so the descriptor of stage s, K step ks is the first one plus (s * A_BYTES + 32 ks) >> 4.
        // The weights of K step ks of stage s: TMEM columns W_COL + 32 s + 8 ks.
        const uint64_t bdesc0 = smem_desc(smem_u32(a_tiles), 16, 1024, SWZ_128B);
        const uint32_t wcol0 = tmem + W_COL;
        // A pair of stages per wait and fence (the expanding warps release four at a time).
        for (int kb = 0; kb < nk; kb += 2) {
            const int kn = kb + 1 < nk ? 2 : 1;
            if (!warp_wait_all(&wfull[kb + kn - 1], 0, DEV_TIMEOUT_READY, p.err, abort_flag)) break;
            TTRACE(25 + kb);
            if (!warp_wait_all(&full_a[kb], 0, DEV_TIMEOUT_FULL, p.err, abort_flag)) break;
            if (kn == 2 && !warp_wait_all(&full_a[kb + 1], 0, DEV_TIMEOUT_FULL, p.err, abort_flag)) break;
            tc_fence_after();
            for (int u = 0; u < kn; ++u) {
                const int s = kb + u;
                const uint64_t bd = bdesc0 + static_cast<uint64_t>(s * (G::A_BYTES >> 4));
                const uint32_t wa = wcol0 + 32 * s;
                mma_i8_ts_lead(lead, tmem, wa, bd, G::IDESC, s > 0 ? 1u : 0u);
#pragma unroll
                for (int ks = 1; ks < TBK / 32; ++ks) mma_i8_ts_lead(lead, tmem, wa + 8 * ks, bd + 2 * ks, G::IDESC, 1u);
            }
            TTRACE(17 + kb);
        }
        TTRACE(5);
        mma_commit_lead(lead, accfull);
        mma_commit_lead(lead, drain);   // every MMA issued has completed once this flips (also on the abort path)
        volatile int keep_waiting = 0;  // on the abort path too: tensor memory is freed only after the MMAs are done
        warp_wait_all(drain, 0, DEV_TIMEOUT_DRAIN, p.err, &keep_waiting);
        __syncwarp();
    } else {
        // ---------------- expansion (warps 0-15), then the epilogue ----------------
        const int g = warp >> 2, q = warp & 3;
        const int nl = 32 * q + lane, n = n0 + nl;
        const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
        const uint4* vdst = reinterpret_cast<const uint4*>(smem + G::VI_OFF) + threadIdx.x;   // this thread's copies
        const uint32_t clo = static_cast<uint32_t>(clo_of(p.lo[n], p.hi[n]));
        const uint32_t pal_lo = (clo << 8) | (((0x100u - clo) & 0xFFu) << 16) | (0x7Fu << 24);
        const uint32_t pal_hi = 0x81u | (((2u * clo) & 0xFFu) << 8) | (0xFEu << 16);
        const float c1 = __fmul_rn(p.hi[n], 1.0f / 127.0f);
        // Stages go to tensor memory EG at a time: one wait for the stores of the group (a store's completion is only
        // observable through tcgen05.wait::st, a round trip of several hundred cycles, so the groups' waits are the
        // expansion's serial chain), then the group's stages are released.
        constexpr int EG = 4;
        static_assert(TNK == 2 * EG, "two groups of stages");
#pragma unroll
        for (int kb = 0; kb < TNK; kb += EG) {
            if (kb >= nk) break;
            if (kb == 0) cp_async_wait<TNK - EG>();   // the first group's commit groups have landed (own copies)
            else cp_async_wait<0>();
#pragma unroll
            for (int u = 0; u < EG; ++u) {
                if (kb + u < nk) {
                    const uint4 vv = vdst[(kb + u) * (EXP_WARPS * 32)];
                    const uint32_t x[4] = {vv.x, vv.y, vv.z, vv.w};
                    uint32_t w[8];
#pragma unroll
                    for (int v = 0; v < 4; ++v) {   // word v: K rows 32 g + 8 v .. + 7 of the stage
                        w[2 * v] = decode4(pal_lo, pal_hi, x[v]);
                        w[2 * v + 1] = decode4(pal_lo, pal_hi, x[v] >> 16);
                    }
                    tmem_st_32x32b_x8(tmem + lane_base + W_COL + 32 * (kb + u) + 8 * g, w);
                    if (kb + u == 0 && warp == 0 && lane == 0) TTRACE(2);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
#pragma unroll
                for (int u = 0; u < EG; ++u)
                    if (kb + u < nk) mbar_arrive(&wfull[kb + u]);
            }
        }
        cp_async_wait<0>();   // none of this thread's copies is still landing (the loop may have stopped early)
        if (warp == 0 && lane == 0) TTRACE(3);
        if (lane == 0) TTRACE(33 + warp);
        // The epilogue: each warp owns 8-row chunks ch = g, g + 4, ... of its 32 columns. C_old (when accumulating)
        // comes into registers while the MMAs run.
        constexpr int CPW = (MT / 8 + 3) / 4;
        float* out = partial ? p.ws + (static_cast<size_t>(z) * p.m_pad) * p.N + n : p.C + n;
        const size_t ld = partial ? static_cast<size_t>(p.N) : static_cast<size_t>(p.ldc);
        griddep_wait();   // C belongs to the previous kernels until here
        if (warp == 0 && lane == 0) TTRACE(42);
        float old[ACC ? CPW : 1][8];
        if (ACC) {
#pragma unroll
            for (int j = 0; j < CPW; ++j) {
                const int mb = m0 + 8 * (g + 4 * j);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    old[ACC ? j : 0][i] = g + 4 * j < MT / 8 && mb + i < p.M ? out[static_cast<size_t>(mb + i) * ld]
                                                                             : 0.f;
            }
        }
        const bool ok = warp_wait_all(accfull, 0, DEV_TIMEOUT_ACC, p.err, abort_flag) &&
                        warp_wait_all(sready, 0, DEV_TIMEOUT_ACC, p.err, abort_flag);
        tc_fence_after();
        if (warp == 0 && lane == 0) TTRACE(6);
        if (ok) {
            uint32_t r[CPW][8];
#pragma unroll
            for (int j = 0; j < CPW; ++j)
                if (g + 4 * j < MT / 8) tmem_ld_32x32b_x8(tmem + lane_base + 8 * (g + 4 * j), r[j]);
            tmem_wait_ld();
            if (warp == 0 && lane == 0) TTRACE(41);
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
                        ACC ? __fmaf_rn(f, as, old[ACC ? j : 0][i]) : (partial ? f : __fmul_rn(f, as));
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

// The value-index plane: thread (kc, n) encodes K rows 32 kc .. 32 kc + 31 of column n from the reference's planes
// (signs [K][N/4], 2-bit code at bits 2 (n & 3); flags [K][N/8], bit n & 7) as four words at out[(kc N + n) 4 + v],
// word v holding rows 32 kc + 8 v + t at bits 4 t. Index: code 1 -> 0 (zero), code 2 -> 1 / 3 (+clo / +127 by the
// flag), code 0 -> 2 / 4 (-clo / -127), code 3 -> 5 / 6 (the reference's sign 2). Rows past K get index 0.
__global__ void __launch_bounds__(256) fv_vindex_kernel(const uint8_t* __restrict__ signs,
                                                        const uint8_t* __restrict__ flags, int K, int N,
                                                        uint32_t* __restrict__ out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int chunks = (K + 31) / 32;
    if (i >= static_cast<size_t>(chunks) * N) return;
    const int n = static_cast<int>(i % N), kc = static_cast<int>(i / N);
    uint32_t words[4] = {0u, 0u, 0u, 0u};
    for (int t = 0; t < 32; ++t) {
        const int k = 32 * kc + t;
        if (k >= K) break;
        const uint32_t code = (signs[static_cast<size_t>(k) * (N / 4) + n / 4] >> (2 * (n & 3))) & 3u;
        const uint32_t fl = (flags[static_cast<size_t>(k) * (N / 8) + n / 8] >> (n & 7)) & 1u;
        const uint32_t idx = code == 1 ? 0u : code == 2 ? 1u + 2u * fl : code == 0 ? 2u + 2u * fl : 5u + fl;
        words[t >> 3] |= idx << (4 * (t & 7));
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(words[0], words[1], words[2], words[3]);
}

template <int MT, bool ACC>
cudaError_t launch_t(const CUtensorMap& a, const FvGemmTParams& p, cudaStream_t stream) {
    using G = TCfg<MT>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(fv_gemm_t_kernel<MT, ACC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
    return cudaLaunchKernelEx(&cfg, fv_gemm_t_kernel<MT, ACC>, a, p);
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

template <int MT>
cudaError_t launch_rows(const CUtensorMap& a, const FvGemmTParams& p, cudaStream_t stream) {
    return p.ksplit == 1 && !p.beta_zero ? launch_t<MT, true>(a, p, stream) : launch_t<MT, false>(a, p, stream);
}

cudaError_t fv_gemm_t_launch(int mt, const CUtensorMap& a, const FvGemmTParams& p, cudaStream_t stream) {
    switch (mt) {
    case 16: return launch_rows<16>(a, p, stream);
    case 32: return launch_rows<32>(a, p, stream);
    case 48: return launch_rows<48>(a, p, stream);
    case 64: return launch_rows<64>(a, p, stream);
    case 80: return launch_rows<80>(a, p, stream);
    case 96: return launch_rows<96>(a, p, stream);
    case 112: return launch_rows<112>(a, p, stream);
    case 128: return launch_rows<128>(a, p, stream);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t fv_vindex_launch(const uint8_t* signs, const uint8_t* flags, int K, int N, uint32_t* out,
                             cudaStream_t stream) {
    const size_t threads = static_cast<size_t>((K + 31) / 32) * N;
    fv_vindex_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(signs, flags, K, N, out);
    return cudaGetLastError();
}

}  // namespace p2cu
