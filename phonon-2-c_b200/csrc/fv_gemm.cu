// fv_gemm.cu - the five-value int8 GEMM on sm_100a tensor cores (tcgen05, TMEM accumulators, TMA operand loads).
//
// C[M, N] = alpha * A * B + beta * C with A int8 [M, K] (one fp32 scale per row, produced by a quantising kernel)
// and B one of
//   * a five-value weight as stored by phonon-2-c: 2-bit sign plane [K, N/4] + 1-bit magnitude plane [K, N/8] and
//     per-column lo / hi (csrc/blas.h:38-45). The planes are streamed by TMA into shared memory and expanded there
//     into two int8 planes, S = sign and T = sign * flag, which feed two MMAs into two TMEM accumulators.
//       int8  mode (csrc/blas.c:1329-1333, 1362): f = fma((float)accT, hi - lo, (float)accS * lo)
//       int8w mode (csrc/blas.c:1319-1328, 1222-1240): the reference multiplies by the one code plane
//         code = sign * (flag ? 127 : clo), clo = round(127 lo / hi); its int32 sum equals, exactly,
//         clo * accS + (127 - clo) * accT, which is what the epilogue forms before f = (float)acc * (hi / 127).
//   * a plain int8 table [K, N] with one fp32 scale per column (the int8-table weights, csrc/blas.c:1243-1254, and
//     the pre-expanded int8w codes of the code cache): loaded by TMA straight into the MMA layout, one MMA.
// The int32 sums restart every 1024 rows of K, and the fp32 epilogue runs per 1024-row block in the reference order
// (csrc/blas.c:1339-1366): C = (beta == 0 && first block) ? f * as : fma(f, as, C), as = a_scale[m] * alpha.
//
// Tile: 128 rows (one TMEM lane per row) x 128 columns per CTA, K staged 128 at a time. Roles:
//   warps 0-3  epilogue (TMEM -> registers -> rescale -> C), one row per thread
//   warps 4-7  expand the sign / flag planes into the S and T operand tiles (planes mode only)
//   warp  8    TMA producer
//   warp  9    TMEM allocation and MMA issue (one elected lane)
// Accumulators are double-buffered in TMEM so that the epilogue of one 1024-row block overlaps the next block's MMAs.
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "fv_gemm.h"

namespace p2cu {

constexpr int BM = 128, BN = 128, BK = 128, KBLK = 1024;
constexpr int NTHREADS = 320;
constexpr uint32_t A_BYTES = BM * BK;            // int8 A tile, K-major, 128-byte swizzle
constexpr uint32_t B_BYTES = BK * BN;            // int8 B tile, MN-major, 128-byte swizzle
constexpr uint32_t SG_BYTES = BK * (BN / 4);     // sign-plane tile
constexpr uint32_t FL_BYTES = BK * (BN / 8);     // flag-plane tile

template <bool PLANES> struct Cfg {
    static constexpr int STAGES = PLANES ? 3 : 4;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES * (PLANES ? 2 : 1) + (PLANES ? SG_BYTES + FL_BYTES : 0);
    static constexpr uint32_t TX_BYTES = A_BYTES + (PLANES ? SG_BYTES + FL_BYTES : B_BYTES);
    static constexpr uint32_t ACC_COLS = PLANES ? 2 * BN : BN;   // S | T, or the single plane
    static constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;          // two accumulator buffers
    static constexpr uint32_t BAR_BYTES = 1024;                  // barriers, flags, per-column constants
    static constexpr uint32_t CONST_BYTES = 3 * BN * 4;
    static constexpr uint32_t SMEM_BYTES = 1024 /*alignment slack*/ + STAGES * STAGE_BYTES + BAR_BYTES + CONST_BYTES;
};

// Expand 32 columns of one K row: x0, x1 = the 8 sign bytes of the columns, fw = their 32 flag bits.
// Output word j holds, at byte p, the operand for column 8p + j of the group (a 4 x 8 transpose of the natural order
// that keeps the expansion to shifts and masks); the epilogue undoes it with compile-time register indexing.
__device__ __forceinline__ void expand32(uint32_t x0, uint32_t x1, uint32_t fw, uint32_t (&S)[8], uint32_t (&T)[8]) {
    const uint32_t u = __byte_perm(x0, x1, 0x6420);   // sign bytes of columns 0-3, 8-11, 16-19, 24-27
    const uint32_t v = __byte_perm(x0, x1, 0x7531);   // sign bytes of columns 4-7, 12-15, 20-23, 28-31
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t src = j < 4 ? u : v;
        const uint32_t code = (src >> (2 * (j & 3))) & 0x03030303u;     // 2-bit codes 0, 1, 2 per byte
        const uint32_t s = (code + 0x7F7F7F7Fu) ^ 0x80808080u;            // code - 1 per byte: -1, 0, +1
        const uint32_t f = (fw >> j) & 0x01010101u;                        // magnitude flag per byte
        S[j] = s;
        T[j] = s & (f * 0xFFu);
    }
}

// Byte offset of (row k, 16-byte chunk c) inside an MN-major, 128-byte-swizzled 128 x 128 int8 tile.
__device__ __forceinline__ uint32_t mn_sw128_offset(int k, int c) {
    return static_cast<uint32_t>((k >> 3) * 1024 + (k & 7) * 128 + ((c ^ (k & 7)) << 4));
}

template <bool PLANES>
__global__ void __launch_bounds__(NTHREADS, 1)
fv_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
               const __grid_constant__ CUtensorMap tmB1, const FvGemmParams p) {
    using G = Cfg<PLANES>;
    constexpr int STAGES = G::STAGES;
    constexpr uint32_t IDESC = idesc_i8(BM, BN, /*A K-major*/ false, /*B MN-major*/ true);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* bar_region = smem + STAGES * G::STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(bar_region);
    uint64_t* bready = full + STAGES;
    uint64_t* empty = bready + STAGES;
    uint64_t* accfull = empty + STAGES;
    uint64_t* accempty = accfull + 2;
    uint64_t* drain = accempty + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    float* cc1 = reinterpret_cast<float*>(bar_region + G::BAR_BYTES);
    float* cc2 = cc1 + BN;
    int* cclo = reinterpret_cast<int*>(cc2 + BN);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int nk = (p.K + BK - 1) / BK;
    const int nblk = (p.K + KBLK - 1) / KBLK;

    auto stage_ptr = [&](int s) { return smem + s * G::STAGE_BYTES; };
    auto a_tile = [&](int s) { return stage_ptr(s); };
    auto b0_tile = [&](int s) { return stage_ptr(s) + A_BYTES; };
    auto b1_tile = [&](int s) { return stage_ptr(s) + A_BYTES + B_BYTES; };
    auto sg_tile = [&](int s) { return stage_ptr(s) + A_BYTES + 2 * B_BYTES; };
    auto fl_tile = [&](int s) { return stage_ptr(s) + A_BYTES + 2 * B_BYTES + SG_BYTES; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&bready[s], 128);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accfull[b], 1);
            mbar_init(&accempty[b], 128);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 8 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB0);
        if (PLANES) tma_prefetch_desc(&tmB1);
    }
    if (warp == 9) {
        tmem_alloc(tmem_holder, G::TMEM_COLS);
        tmem_relinquish();
    }
    if (threadIdx.x < BN) {   // per-column epilogue constants
        const int n = n0 + threadIdx.x;
        float c1 = 0.f, c2 = 0.f;
        int clo = 0;
        if (n < p.N) {
            if (p.cmode == CM_Q8B) {
                c1 = p.scales[n];
            } else if (p.cmode == CM_INT8) {
                c1 = p.lo[n];
                c2 = __fsub_rn(p.hi[n], p.lo[n]);
            } else {   // int8w: c1 = hi * (1 / 127); clo = clamp(rint(127 * lo / hi), 0, 127)
                const float lo = p.lo[n], hi = p.hi[n];
                c1 = __fmul_rn(hi, 1.0f / 127.0f);
                const int c = hi > 0.f ? __float2int_rn(__fdiv_rn(__fmul_rn(127.0f, lo), hi)) : 0;
                clo = c < 0 ? 0 : c > 127 ? 127 : c;
            }
        }
        cc1[threadIdx.x] = c1;
        cc2[threadIdx.x] = c2;
        cclo[threadIdx.x] = clo;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 8) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int issued = 0;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % STAGES, r = kb / STAGES;
                if (!mbar_wait(&empty[s], (r & 1) ^ 1, DEV_TIMEOUT_EMPTY, p.err, abort_flag)) break;
                issued = kb + 1;
                mbar_arrive_expect_tx(&full[s], G::TX_BYTES);
                tma_load_2d(a_tile(s), &tmA, &full[s], kb * BK, m0);
                if (PLANES) {
                    tma_load_2d(sg_tile(s), &tmB0, &full[s], n0 / 4, kb * BK);
                    tma_load_2d(fl_tile(s), &tmB1, &full[s], n0 / 8, kb * BK);
                } else {
                    tma_load_2d(b0_tile(s), &tmB0, &full[s], n0, kb * BK);
                }
            }
            // No copy may still be landing in shared memory when the CTA exits (matters on the abort path only):
            // wait, bounded, for the last round issued on every stage.
            for (int kb = issued - STAGES < 0 ? 0 : issued - STAGES; kb < issued; ++kb) {
                const int s = kb % STAGES, r = kb / STAGES;
                for (uint32_t i = 0; i < WAIT_LIMIT && !mbar_try_wait(smem_u32(&full[s]), r & 1); ++i) {}
            }
        }
    } else if (warp == 9) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % STAGES, r = kb / STAGES;
                const int b = (kb * BK) / KBLK, ab = b & 1;
                const bool first = (kb * BK) % KBLK == 0;
                const bool last = ((kb + 1) * BK) % KBLK == 0 || kb == nk - 1;
                if (first && !mbar_wait(&accempty[ab], ((b >> 1) & 1) ^ 1, DEV_TIMEOUT_ACC, p.err, abort_flag)) break;
                if (!mbar_wait(PLANES ? &bready[s] : &full[s], r & 1, DEV_TIMEOUT_READY, p.err, abort_flag)) break;
                tc_fence_after();
                const uint32_t a_base = smem_u32(a_tile(s));
                const uint32_t b0_base = smem_u32(b0_tile(s)), b1_base = smem_u32(b1_tile(s));
                const uint32_t d = tmem + ab * G::ACC_COLS;
#pragma unroll
                for (int ks = 0; ks < BK / 32; ++ks) {
                    // A: K-major rows of 128 bytes, 8-row groups 1024 bytes apart; a K step of 32 advances 32 bytes
                    // inside the swizzle atom. B: MN-major, 8-row K groups 1024 bytes apart, one 128-column atom
                    // (its leading offset is never used; it is set to the group stride so that no reading of the
                    // descriptor reaches past the tile).
                    const uint64_t adesc = smem_desc(a_base + ks * 32, 16, 1024, SWZ_128B);
                    const uint32_t acc = (!first || ks > 0) ? 1u : 0u;
                    mma_i8(d, adesc, smem_desc(b0_base + ks * 4096, 1024, 1024, SWZ_128B), IDESC, acc);
                    if (PLANES)
                        mma_i8(d + BN, adesc, smem_desc(b1_base + ks * 4096, 1024, 1024, SWZ_128B), IDESC, acc);
                }
                mma_commit(&empty[s]);
                if (last) mma_commit(&accfull[ab]);
            }
            // Every MMA this thread issued has completed once `drain` flips (bounded: also on the abort path).
            mma_commit(drain);
            mbar_wait(drain, 0, DEV_TIMEOUT_DRAIN, p.err, abort_flag);
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ---------------- plane expansion (planes mode) ----------------
        if (PLANES) {
            const int et = threadIdx.x - 128, h = et & 3;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % STAGES, r = kb / STAGES;
                if (!mbar_wait(&full[s], r & 1, DEV_TIMEOUT_FULL, p.err, abort_flag)) break;
                const uint8_t* sg = sg_tile(s);
                const uint8_t* fl = fl_tile(s);
                uint8_t* bS = b0_tile(s);
                uint8_t* bT = b1_tile(s);
#pragma unroll
                for (int it = 0; it < BK / 32; ++it) {
                    const int k = it * 32 + (et >> 2);
                    const uint2 x = *reinterpret_cast<const uint2*>(sg + k * (BN / 4) + 8 * h);
                    const uint32_t fw = *reinterpret_cast<const uint32_t*>(fl + k * (BN / 8) + 4 * h);
                    uint32_t S[8], T[8];
                    expand32(x.x, x.y, fw, S, T);
                    const uint32_t o0 = mn_sw128_offset(k, 2 * h), o1 = mn_sw128_offset(k, 2 * h + 1);
                    *reinterpret_cast<uint4*>(bS + o0) = make_uint4(S[0], S[1], S[2], S[3]);
                    *reinterpret_cast<uint4*>(bS + o1) = make_uint4(S[4], S[5], S[6], S[7]);
                    *reinterpret_cast<uint4*>(bT + o0) = make_uint4(T[0], T[1], T[2], T[3]);
                    *reinterpret_cast<uint4*>(bT + o1) = make_uint4(T[4], T[5], T[6], T[7]);
                }
                fence_proxy_async_smem();
                mbar_arrive(&bready[s]);
            }
        }
    } else {
        // ---------------- epilogue: warps 0-3, TMEM lanes 32w .. 32w + 31 ----------------
        const int row = m0 + warp * 32 + lane;
        const bool live = row < p.M;
        const float as = live ? __fmul_rn(p.a_scales[row], p.alpha) : 0.f;
        float* crow = p.C + static_cast<size_t>(live ? row : 0) * p.ldc + n0;
        const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
        for (int b = 0; b < nblk; ++b) {
            const int ab = b & 1;
            if (!mbar_wait(&accfull[ab], (b >> 1) & 1, DEV_TIMEOUT_ACC, p.err, abort_flag)) break;
            tc_fence_after();
            const bool store = p.beta_zero && b == 0;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t rS[32], rT[32];
                tmem_ld_32x32b_x32(tmem + lane_base + ab * G::ACC_COLS + 32 * c, rS);
                if (PLANES) tmem_ld_32x32b_x32(tmem + lane_base + ab * G::ACC_COLS + BN + 32 * c, rT);
                tmem_wait_ld();
                if (live && n0 + 32 * c < p.N) {
#pragma unroll
                    for (int t4 = 0; t4 < 8; ++t4) {
                        float4 old = make_float4(0.f, 0.f, 0.f, 0.f);
                        if (!store) old = *reinterpret_cast<const float4*>(crow + 32 * c + 4 * t4);
                        float o[4] = {old.x, old.y, old.z, old.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int t = 4 * t4 + e;                              // column within the group
                            const int ph = PLANES ? 4 * (t & 7) + (t >> 3) : t;    // its TMEM column
                            const int nl = 32 * c + t;
                            float f;
                            if (PLANES && p.cmode == CM_INT8W) {
                                const int clo = cclo[nl];
                                const int acc = clo * static_cast<int>(rS[ph]) + (127 - clo) * static_cast<int>(rT[ph]);
                                f = __fmul_rn(__int2float_rn(acc), cc1[nl]);
                            } else if (PLANES) {
                                f = __fmaf_rn(__int2float_rn(static_cast<int>(rT[ph])), cc2[nl],
                                              __fmul_rn(__int2float_rn(static_cast<int>(rS[ph])), cc1[nl]));
                            } else {
                                f = __fmul_rn(__int2float_rn(static_cast<int>(rS[ph])), cc1[nl]);
                            }
                            o[e] = store ? __fmul_rn(f, as) : __fmaf_rn(f, as, o[e]);
                        }
                        *reinterpret_cast<float4*>(crow + 32 * c + 4 * t4) = make_float4(o[0], o[1], o[2], o[3]);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&accempty[ab]);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 9) tmem_dealloc(tmem, G::TMEM_COLS);
}

template <bool PLANES>
static cudaError_t launch(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                          const FvGemmParams& p, cudaStream_t stream) {
    using G = Cfg<PLANES>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(fv_gemm_kernel<PLANES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(G::SMEM_BYTES));
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM);
    fv_gemm_kernel<PLANES><<<grid, NTHREADS, G::SMEM_BYTES, stream>>>(a, b0, b1, p);
    return cudaGetLastError();
}

cudaError_t fv_gemm_launch_planes(const CUtensorMap& a, const CUtensorMap& signs, const CUtensorMap& flags,
                                  const FvGemmParams& p, cudaStream_t stream) {
    return launch<true>(a, signs, flags, p, stream);
}

cudaError_t fv_gemm_launch_table(const CUtensorMap& a, const CUtensorMap& table, const FvGemmParams& p,
                                 cudaStream_t stream) {
    return launch<false>(a, table, table, p, stream);
}

}  // namespace p2cu
