// attn_tc.cu - the attention products on the tensor cores with fp32 accuracy: grouped GEMMs C = A op(B) through
// tcgen05.mma kind::tf32, each operand split into two tf32 parts on its way into shared memory.
//
// The reference computes attention in fp32 (csrc/encoder.c:282-316, 505-519): AC = (Q + bias_u) K^T, BD = (Q +
// bias_v) P^T, then the context S V. A tf32 product keeps 10 explicit mantissa bits, too few for that. Here every
// operand value x becomes hi = x rounded to the tf32 grid and lo = x - hi (exact in fp32), and every K step runs
// three MMAs into the same fp32 accumulator: hi*hi + hi*lo + lo*hi. The dropped lo*lo term and the tf32 truncation
// of lo leave a relative error of about 2^-21 per product, the accuracy of an fp32 dot product; the summation order
// inside the tensor core differs from the reference's FMA chain, so results agree to an ulp or two, not bit for bit.
//
// One CTA computes one 128 x 128 output tile of one group (a (window, head, product) problem). Four loader warps
// read fp32 tiles of 128 rows x 16 K from global memory into registers one K step ahead (a [k][n] B is transposed
// on the way), split them and store the four operand tiles (A hi / lo, B hi / lo) K-major with the 64-byte swizzle
// the MMA reads; one thread issues the
// MMAs (TMEM accumulator, 128 columns); the loader warps then read the accumulator out (one TMEM lane per row).
// Every wait is bounded (ptx.cuh).
#include <cstdint>
#include <cuda_runtime.h>
#include "attn_tc.h"
#include "ptx.cuh"
#include "tf32_split.cuh"

namespace p2cu {

namespace {

// K steps of 16 fp32 (64-byte rows, 64-byte swizzle) and two stages keep a CTA at 66 KB of shared memory, so three
// CTAs share an SM and hide each other's global-load latency.
constexpr int TM = 128, TN = 128, TK = 16, TSTAGES = 2;
constexpr uint32_t PART = TM * TK * 4;      // one operand part of one stage: 128 rows x 16 fp32 = 8 KB
constexpr uint32_t STAGE = 4 * PART;        // A hi, A lo, B hi, B lo
constexpr uint32_t SMEM_BYTES = 1024 + TSTAGES * STAGE + 256;
constexpr int NTHREADS = 160;               // warps 0-3 load / split / read out, warp 4 issues the MMAs
constexpr int PER = TM * TK / 4 / 128;      // float4 per loader thread per operand and stage

__device__ __forceinline__ float4 load4(const float* row, int k, int K, bool vec) {   // row[k .. k+3], zero past K
    if (vec && k + 3 < K) return __ldg(reinterpret_cast<const float4*>(row + k));
    float4 v;
    v.x = k < K ? __ldg(row + k) : 0.f;
    v.y = k + 1 < K ? __ldg(row + k + 1) : 0.f;
    v.z = k + 2 < K ? __ldg(row + k + 2) : 0.f;
    v.w = k + 3 < K ? __ldg(row + k + 3) : 0.f;
    return v;
}

template <bool B_KN>
__global__ void __launch_bounds__(NTHREADS, 3) attn_tc_kernel(const TcGroup* __restrict__ groups, int n_groups,
                                                              TcArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + TSTAGES * STAGE);
    uint64_t* empty = full + TSTAGES;
    uint64_t* accfull = empty + TSTAGES;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accfull + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int tile = blockIdx.x;
    int lo = 0, hi = n_groups - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (groups[mid].tile0 <= tile) lo = mid; else hi = mid - 1;
    }
    const TcGroup g = groups ? groups[lo] : args.single;
    const int tn = (g.N + TN - 1) / TN;
    const int m0 = ((tile - g.tile0) / tn) * TM, n0 = ((tile - g.tile0) % tn) * TN;
    const float* A = args.src[g.a_src] + g.a_off;
    const float* B = args.src[g.b_src] + g.b_off;
    float* C = args.dst[g.c_dst] + g.c_off;
    const float* bias = g.bias_sel >= 0 ? args.bias[g.bias_sel] + g.bias_off : nullptr;
    const int nk = (g.K + TK - 1) / TK;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TSTAGES; ++s) {
            mbar_init(&full[s], 128);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accfull, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 4) {
        tmem_alloc(tmem_holder, TN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp < 4) {
        // ---------------- loaders: one K step ahead in registers ----------------
        const int t = threadIdx.x;   // 0 .. 127
        const bool avec = (g.lda & 3) == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0;
        const bool bvec = !B_KN && (g.ldb & 3) == 0 && (reinterpret_cast<uintptr_t>(B) & 15) == 0;
        const bool biasvec = (reinterpret_cast<uintptr_t>(bias) & 15) == 0;
        float4 ra[PER], rb[PER];
        auto fetch = [&](int kb) {
            const int k0 = kb * TK;
#pragma unroll
            for (int i = 0; i < PER; ++i) {
                const int e = t + 128 * i;
                {   // A: row e / 4, chunk e % 4 (a warp reads eight 64-byte row segments)
                    const int r = e >> 2, c = e & 3, m = m0 + r, k = k0 + 4 * c;
                    ra[i] = m < g.M ? load4(A + static_cast<size_t>(m) * g.lda, k, g.K, avec) : make_float4(0, 0, 0, 0);
                    if (bias && m < g.M) {
                        const float4 b4 = load4(bias, k, g.K, biasvec);
                        ra[i].x = k < g.K ? __fadd_rn(ra[i].x, b4.x) : 0.f;
                        ra[i].y = k + 1 < g.K ? __fadd_rn(ra[i].y, b4.y) : 0.f;
                        ra[i].z = k + 2 < g.K ? __fadd_rn(ra[i].z, b4.z) : 0.f;
                        ra[i].w = k + 3 < g.K ? __fadd_rn(ra[i].w, b4.w) : 0.f;
                    }
                }
                if (!B_KN) {   // B [n][k]: like A
                    const int r = e >> 2, c = e & 3, n = n0 + r, k = k0 + 4 * c;
                    rb[i] = n < g.N ? load4(B + static_cast<size_t>(n) * g.ldb, k, g.K, bvec) : make_float4(0, 0, 0, 0);
                } else {       // B [k][n], transposed on the way: column n = e % 128 (consecutive across a warp),
                               // the four K rows 4 (e / 128) .. + 3 of it
                    const int r = e & 127, c = e >> 7, n = n0 + r, k = k0 + 4 * c;
                    const float* col = B + n;
                    float4 v = make_float4(0, 0, 0, 0);
                    if (n < g.N) {
                        v.x = k < g.K ? __ldg(col + static_cast<size_t>(k) * g.ldb) : 0.f;
                        v.y = k + 1 < g.K ? __ldg(col + static_cast<size_t>(k + 1) * g.ldb) : 0.f;
                        v.z = k + 2 < g.K ? __ldg(col + static_cast<size_t>(k + 2) * g.ldb) : 0.f;
                        v.w = k + 3 < g.K ? __ldg(col + static_cast<size_t>(k + 3) * g.ldb) : 0.f;
                    }
                    rb[i] = v;
                }
            }
        };
        // The common case - 16-byte aligned rows of A, B [n][k] and the bias - loads every whole K step without any
        // branch: rows past the problem read row 0 instead and are zeroed when stored, and the bias is added then
        // too, so nothing waits for a load before the stage it feeds is free. A last, partial K step takes the
        // bounds-checked loads above (zeros past K, bias included).
        const bool fast = !B_KN && avec && bvec && (!bias || biasvec);
        if (fast) {
            float4 ba[PER];
            uint32_t live = 0;   // bit i: A row of chunk i inside the problem; bit PER + i: B row
#pragma unroll
            for (int i = 0; i < PER; ++i) {
                const int e = t + 128 * i, r = e >> 2;
                live |= (m0 + r < g.M ? 1u : 0u) << i;
                live |= (n0 + r < g.N ? 1u : 0u) << (PER + i);
            }
            auto fetch_fast = [&](int kb) {
                const int k0 = kb * TK;
#pragma unroll
                for (int i = 0; i < PER; ++i) {
                    const int e = t + 128 * i, r = e >> 2, c = e & 3, k = k0 + 4 * c;
                    const int m = (live >> i) & 1 ? m0 + r : 0, n = (live >> (PER + i)) & 1 ? n0 + r : 0;
                    ra[i] = __ldg(reinterpret_cast<const float4*>(A + static_cast<size_t>(m) * g.lda + k));
                    rb[i] = __ldg(reinterpret_cast<const float4*>(B + static_cast<size_t>(n) * g.ldb + k));
                    if (bias) ba[i] = __ldg(reinterpret_cast<const float4*>(bias + k));
                }
            };
            auto fetch_step = [&](int kb) {
                if ((kb + 1) * TK <= g.K) fetch_fast(kb);
                else fetch(kb);
            };
            if (nk > 0) fetch_step(0);
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % TSTAGES, r = kb / TSTAGES;
                if (!warp_wait(&empty[s], (r & 1) ^ 1, DEV_TIMEOUT_EMPTY, args.err, abort_flag)) break;
                uint8_t* st = smem + s * STAGE;
                const bool whole = (kb + 1) * TK <= g.K;   // loaded by fetch_fast: bias and row masks still to apply
#pragma unroll
                for (int i = 0; i < PER; ++i) {
                    const int e = t + 128 * i;
                    float4 a = ra[i], b = rb[i];
                    if (whole) {
                        if (bias)
                            a = make_float4(__fadd_rn(a.x, ba[i].x), __fadd_rn(a.y, ba[i].y), __fadd_rn(a.z, ba[i].z),
                                            __fadd_rn(a.w, ba[i].w));
                        if (!((live >> i) & 1)) a = make_float4(0.f, 0.f, 0.f, 0.f);
                        if (!((live >> (PER + i)) & 1)) b = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                    store_split(st, st + PART, kmaj_off(e >> 2, e & 3), a);
                    store_split(st + 2 * PART, st + 3 * PART, kmaj_off(e >> 2, e & 3), b);
                }
                fence_proxy_async_smem();
                mbar_arrive(&full[s]);
                if (kb + 1 < nk) fetch_step(kb + 1);
            }
        } else {
            if (nk > 0) fetch(0);
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % TSTAGES, r = kb / TSTAGES;
                if (!warp_wait(&empty[s], (r & 1) ^ 1, DEV_TIMEOUT_EMPTY, args.err, abort_flag)) break;
                uint8_t* st = smem + s * STAGE;
#pragma unroll
                for (int i = 0; i < PER; ++i) {
                    const int e = t + 128 * i;
                    store_split(st, st + PART, kmaj_off(e >> 2, e & 3), ra[i]);
                    store_split(st + 2 * PART, st + 3 * PART,
                                B_KN ? kmaj_off(e & 127, e >> 7) : kmaj_off(e >> 2, e & 3), rb[i]);
                }
                fence_proxy_async_smem();
                mbar_arrive(&full[s]);
                if (kb + 1 < nk) fetch(kb + 1);
            }
        }
    } else if (lane == 0) {
        // ---------------- MMA issue ----------------
        constexpr uint32_t IDESC = idesc_tf32(TM, TN, false);
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % TSTAGES, r = kb / TSTAGES;
            if (!mbar_wait(&full[s], r & 1, DEV_TIMEOUT_FULL, args.err, abort_flag)) break;
            tc_fence_after();
            const uint32_t base = smem_u32(smem + s * STAGE);
#pragma unroll
            for (int ks = 0; ks < TK / 8; ++ks) {   // K = 8 tf32 (32 bytes) per MMA
                const uint64_t ah = smem_desc(base + ks * 32, 16, 512, SWZ_64B);
                const uint64_t al = smem_desc(base + PART + ks * 32, 16, 512, SWZ_64B);
                const uint64_t bh = smem_desc(base + 2 * PART + ks * 32, 16, 512, SWZ_64B);
                const uint64_t bl = smem_desc(base + 3 * PART + ks * 32, 16, 512, SWZ_64B);
                mma_tf32(tmem, ah, bh, IDESC, (kb > 0 || ks > 0) ? 1u : 0u);
                mma_tf32(tmem, ah, bl, IDESC, 1u);
                mma_tf32(tmem, al, bh, IDESC, 1u);
            }
            mma_commit(&empty[s]);
        }
        mma_commit(accfull);
    }

    if (warp < 4) {
        // ---------------- read-out: TMEM lane = tile row ----------------
        // Each warp drains its 32 rows 32 columns at a time through a 4 KB block of the (now idle) stage buffers:
        // thread = row on the way in, then four whole 128-byte rows per store instruction on the way out.
        const bool ok = nk > 0 && warp_wait(accfull, 0, DEV_TIMEOUT_ACC, args.err, abort_flag);
        tc_fence_after();
        const bool cvec = (g.ldc & 3) == 0 && (reinterpret_cast<uintptr_t>(C) & 15) == 0;
        uint8_t* blk = smem + warp * 4096;   // the MMAs are done with every stage once the accumulator is full
        if (ok) {
#pragma unroll 1
            for (int c = 0; c < TN / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + 32 * c, v);
                const int n = n0 + 32 * c;
                float ob[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) ob[j] = args.out_bias && n + j < g.N ? __ldg(args.out_bias + n + j) : 0.f;
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 8; ++q) {   // row `lane`, columns 4q .. 4q + 3, at 16-byte slot q ^ (lane % 8)
                    float x[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        x[e] = __uint_as_float(v[4 * q + e]);
                        if (args.out_bias) x[e] = __fadd_rn(x[e], ob[4 * q + e]);
                        if (args.out_relu) x[e] = x[e] > 0.f ? x[e] : 0.f;
                    }
                    *reinterpret_cast<float4*>(blk + lane * 128 + ((q ^ (lane & 7)) << 4)) =
                        make_float4(x[0], x[1], x[2], x[3]);
                }
                __syncwarp();
                const int q = lane & 7;
#pragma unroll
                for (int it = 0; it < 8; ++it) {   // rows 4 it .. 4 it + 3, eight lanes per row
                    const int r = 4 * it + (lane >> 3);
                    const int row = m0 + warp * 32 + r, col = n + 4 * q;
                    const float4 y = *reinterpret_cast<const float4*>(blk + r * 128 + ((q ^ (r & 7)) << 4));
                    if (row < g.M) {
                        float* dst = C + static_cast<size_t>(row) * g.ldc + col;
                        if (cvec && col + 4 <= g.N) {
                            *reinterpret_cast<float4*>(dst) = y;
                        } else {
                            if (col < g.N) dst[0] = y.x;
                            if (col + 1 < g.N) dst[1] = y.y;
                            if (col + 2 < g.N) dst[2] = y.z;
                            if (col + 3 < g.N) dst[3] = y.w;
                        }
                    }
                }
                __syncwarp();   // the block is read before the next chunk overwrites it
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tmem, TN);
    }
}

}  // namespace

int tc_gemm_tiles(int M, int N) { return ((M + TM - 1) / TM) * ((N + TN - 1) / TN); }

cudaError_t attn_tc_launch(const TcGroup* groups, int n_groups, int total_tiles, const TcArgs& args, bool b_kn,
                           cudaStream_t s) {
    if (total_tiles <= 0 || (groups && n_groups <= 0)) return cudaSuccess;
    auto* k = b_kn ? attn_tc_kernel<true> : attn_tc_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    k<<<total_tiles, NTHREADS, SMEM_BYTES, s>>>(groups, n_groups, args);
    return cudaGetLastError();
}

}  // namespace p2cu
