// fv_gemm_p.cu - the persistent form of the five-value / int8-table GEMM, for launches with more output tiles than
// the GPU has SMs (large M: a batch of windows stacked along the rows).
//
// The arithmetic is fv_gemm.cu's, bit for bit (the same operand kinds, the same per-1024-row-block epilogue; see the
// comment there). What changes is the schedule: one CTA per SM walks a list of 128 x BN output tiles (tile t, t +
// gridDim.x, ...; M fastest, so consecutive tiles of an SM share their weight columns in L2) and
//   * the TMA producer and the plane expanders run ahead across tile boundaries through one ring of stages;
//   * the accumulator is double-buffered in TMEM (2 x MMA_N columns): the MMAs of tile i + 1 run while the epilogue
//     drains tile i, so the fp32 stores - at K = 1024 they cost as much HBM time as the MMAs cost tensor time -
//     overlap the tensor work instead of following it;
//   * the epilogue stages 128 x 32 output chunks in two shared-memory buffers and stores them by TMA, loading C_old
//     by TMA into the same buffer first when it accumulates.
// Warps: 8 plane expanders (planes kinds only), 4 epilogue warps (TMEM lane quarters 0-3), the TMA producer, the MMA
// issuer. Every wait is bounded (ptx.cuh); a timeout aborts every role and is reported through the error word.
#include <cstdint>
#include <utility>
#include <cuda.h>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "fv_gemm.h"
#include "fv_common.cuh"

namespace p2cu {

namespace {

constexpr int PBM = 128, PBK = 128, PKBLK = 1024;

template <int BN_, int KIND_> struct PCfg {
    static constexpr int BN = BN_;
    static constexpr int KIND = KIND_;
    static constexpr bool PLANES = KIND != KIND_TABLE;
    static constexpr bool ST = KIND == KIND_ST;
    static constexpr int MMA_N = ST ? 2 * BN : BN;
    static constexpr int ATOM_W = ST ? BN : (BN < 128 ? BN : 128);
    static constexpr int N_ATOMS = MMA_N / ATOM_W;
    static constexpr uint32_t REGION = PBK * ATOM_W;
    static constexpr uint32_t B_SWZ = ATOM_W == 128 ? SWZ_128B : SWZ_64B;
    static constexpr uint32_t SBO = 8 * ATOM_W;
    static constexpr int NEXP = PLANES ? 8 : 0;                 // expander warps 0 .. NEXP - 1
    static constexpr int EPI0 = NEXP;                           // epilogue warps EPI0 .. EPI0 + 3

    static constexpr uint32_t A_BYTES = PBM * PBK;
    static constexpr uint32_t B_BYTES = PBK * MMA_N;
    static constexpr uint32_t SG_BYTES = PBK * (BN / 4);
    static constexpr uint32_t FL_ROW = BN / 8 < 16 ? 16 : BN / 8;
    static constexpr uint32_t FL_BYTES = PBK * FL_ROW;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES + (PLANES ? SG_BYTES + FL_BYTES : 0);
    static constexpr uint32_t B_TX_BYTES = PLANES ? SG_BYTES + FL_BYTES : B_BYTES;
    static constexpr uint32_t STG_BYTES = PBM * 32 * 4;         // one 128 x 32 fp32 output chunk
    static constexpr uint32_t BAR_BYTES = 512;
    static constexpr uint32_t FIXED = 1024 + 2 * STG_BYTES + BAR_BYTES;
    static constexpr int STAGES = (220 * 1024 - FIXED) / STAGE_BYTES > 4 ? 4 : (220 * 1024 - FIXED) / STAGE_BYTES;
    // TMA producer warps: one warp's tile loads complete one after another (about 0.4 us each on B200, whatever the
    // box size), so warp PROD + w issues the loads of the K steps g with g % NPROD == w. NPROD <= STAGES keeps each
    // warp's parity wait on a stage unambiguous (its own previous wait proves the round before last complete).
    static constexpr int NPROD = STAGES < 4 ? STAGES : 4;
    static constexpr int PROD = EPI0 + 4, MMAW = PROD + NPROD;
    static constexpr int NTHREADS = (MMAW + 1) * 32;
    static constexpr uint32_t SMEM_BYTES = FIXED + STAGES * STAGE_BYTES;
    static constexpr uint32_t TMEM_COLS = 2 * MMA_N <= 128 ? 128 : 2 * MMA_N <= 256 ? 256 : 512;
    static constexpr int CHUNKS = BN / 32;
    static_assert(STAGES >= 2, "pipeline depth");
    static_assert(NPROD <= STAGES, "producer warps and stage phases");
    static_assert(2 * MMA_N <= 512, "two accumulators must fit in TMEM");
};

struct TileDesc {
    int m0, n0, z, k_begin, nk;
};

__device__ __forceinline__ TileDesc tile_of(int t, int m_tiles, int n_tiles, int BN, int K) {
    TileDesc d;
    const int mt = t % m_tiles, rest = t / m_tiles;
    d.m0 = mt * PBM;
    d.n0 = (rest % n_tiles) * BN;
    d.z = rest / n_tiles;
    d.k_begin = d.z * PKBLK;
    const int k_len = K - d.k_begin < PKBLK ? K - d.k_begin : PKBLK;
    d.nk = (k_len + PBK - 1) / PBK;
    return d;
}

template <int BN, int KIND>
__global__ void __launch_bounds__(PCfg<BN, KIND>::NTHREADS, 1)
fv_gemm_p_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                 const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmOut,
                 const FvGemmParams p) {
    using G = PCfg<BN, KIND>;
    constexpr int STAGES = G::STAGES;
    constexpr bool PLANES = G::PLANES;
    constexpr uint32_t IDESC = idesc_i8(PBM, G::MMA_N, false, true);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stg = smem + STAGES * G::STAGE_BYTES;                  // two staging chunks
    uint8_t* bar_region = stg + 2 * G::STG_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(bar_region);       // weights of a stage landed
    uint64_t* afull = full + STAGES;                                // A of a stage landed
    uint64_t* bready = afull + STAGES;                              // planes expanded
    uint64_t* empty = bready + STAGES;                              // the MMAs are done with a stage
    uint64_t* tfull = empty + STAGES;                               // [2] accumulator complete
    uint64_t* tempty = tfull + 2;                                   // [2] accumulator drained
    uint64_t* cfull = tempty + 2;                                   // [2] C_old chunk in a staging buffer
    uint64_t* drain = cfull + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    // Abort decisions of the warps that meet at named barriers, taken by one thread between two barriers so that
    // every warp of the group leaves its loop at the same tile (a barrier some warps never reach would never open).
    volatile int* decide_epi = abort_flag + 1;
    volatile int* decide_exp = abort_flag + 2;
    uint8_t* clo_s = reinterpret_cast<uint8_t*>(tmem_holder + 4);   // BN bytes: the tile's clo values

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tiles = (p.M + PBM - 1) / PBM, n_tiles = p.N / BN;
    const int total = m_tiles * n_tiles * p.ksplit;
    const bool partial = p.ksplit > 1;

    auto stage_ptr = [&](int s) { return smem + s * G::STAGE_BYTES; };
    auto a_tile = [&](int s) { return stage_ptr(s); };
    auto b_tile = [&](int s) { return stage_ptr(s) + G::A_BYTES; };
    auto sg_tile = [&](int s) { return stage_ptr(s) + G::A_BYTES + G::B_BYTES; };
    auto fl_tile = [&](int s) { return stage_ptr(s) + G::A_BYTES + G::B_BYTES + G::SG_BYTES; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&afull[s], 1);
            mbar_init(&bready[s], G::NEXP > 0 ? G::NEXP * 32 : 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
            mbar_init(&cfull[b], 1);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == G::PROD && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB0);
        if (PLANES) tma_prefetch_desc(&tmB1);
        tma_prefetch_desc(&tmOut);
    }
    if (warp == G::MMAW) {
        tmem_alloc(tmem_holder, G::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    griddep_launch_dependents();

    if (warp >= G::PROD && warp < G::PROD + G::NPROD) {
        // ---------------- TMA producers: one ring of stages across all of this CTA's tiles ----------------
        const int pw = warp - G::PROD;
        if (lane == 0) {
            auto load_b = [&](int s, int n0, int kx) {
                mbar_arrive_expect_tx(&full[s], G::B_TX_BYTES);
                if (PLANES) {
                    tma_load_2d(sg_tile(s), &tmB0, &full[s], n0 / 4, kx);
                    tma_load_2d(fl_tile(s), &tmB1, &full[s], (n0 / 8) & ~15, kx);   // 16-byte aligned box
                } else {
#pragma unroll
                    for (int a = 0; a < G::N_ATOMS; ++a)
                        tma_load_2d(b_tile(s) + a * G::REGION, &tmB0, &full[s], n0 + a * G::ATOM_W, kx);
                }
            };
            // The first stages' weights before the dependency wait (they are constant), then everything else.
            int pre = 0;
            if (static_cast<int>(blockIdx.x) < total) {
                const TileDesc d = tile_of(blockIdx.x, m_tiles, n_tiles, BN, p.K);
                pre = d.nk < STAGES ? d.nk : STAGES;
                for (int kb = pw; kb < pre; kb += G::NPROD) load_b(kb, d.n0, d.k_begin + kb * PBK);
            }
            griddep_wait();
            int g = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
                const TileDesc d = tile_of(t, m_tiles, n_tiles, BN, p.K);
                for (int kb = 0; kb < d.nk; ++kb, ++g) {
                    if (g % G::NPROD != pw) continue;
                    const int s = g % STAGES, r = g / STAGES;
                    if (g >= pre) {
                        if (!mbar_wait(&empty[s], (r & 1) ^ 1, DEV_TIMEOUT_EMPTY, p.err, abort_flag)) { ok = false; break; }
                        load_b(s, d.n0, d.k_begin + kb * PBK);
                    }
                    mbar_arrive_expect_tx(&afull[s], G::A_BYTES);
                    tma_load_2d(a_tile(s), &tmA, &afull[s], d.k_begin + kb * PBK, d.m0);
                }
            }
            // No copy this warp issued may still be landing in shared memory when the CTA exits.
            for (int k = g - STAGES < 0 ? 0 : g - STAGES; k < g; ++k) {
                if (k % G::NPROD != pw) continue;
                const int s = k % STAGES, r = k / STAGES;
                for (uint32_t i = 0; i < WAIT_LIMIT && !mbar_try_wait(smem_u32(&full[s]), r & 1); ++i) {}
                for (uint32_t i = 0; i < WAIT_LIMIT && !mbar_try_wait(smem_u32(&afull[s]), r & 1); ++i) {}
            }
        }
    } else if (warp == G::MMAW) {
        // ---------------- MMA issue: tile i into accumulator i % 2 ----------------
        // The whole warp runs the loop converged and waits with all lanes; one elected lane issues (issue from code
        // one lane runs alone, branches inside it, was measured at about half the rate).
        const uint32_t el = elect_one();
        int g = 0, it = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < total; t += gridDim.x, ++it) {
            const TileDesc d = tile_of(t, m_tiles, n_tiles, BN, p.K);
            const int b = it & 1;
            if (!warp_wait_all(&tempty[b], ((it >> 1) & 1) ^ 1, DEV_TIMEOUT_ACC, p.err, abort_flag)) break;
            tc_fence_after();
            const uint32_t acc = tmem + static_cast<uint32_t>(b * G::MMA_N);
            for (int kb = 0; kb < d.nk; ++kb, ++g) {
                const int s = g % STAGES, r = g / STAGES;
                if (!warp_wait_all(PLANES ? &bready[s] : &full[s], r & 1, DEV_TIMEOUT_READY, p.err, abort_flag) ||
                    !warp_wait_all(&afull[s], r & 1, DEV_TIMEOUT_READY, p.err, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_base = smem_u32(a_tile(s));
                const uint32_t b_base = smem_u32(b_tile(s));
#pragma unroll
                for (int ks = 0; ks < PBK / 32; ++ks) {
                    const uint64_t adesc = smem_desc(a_base + ks * 32, 16, 1024, SWZ_128B);
                    const uint64_t bdesc = smem_desc(b_base + ks * 4 * G::SBO, G::N_ATOMS > 1 ? G::REGION : G::SBO,
                                                     G::SBO, G::B_SWZ);
                    mma_i8_lead(el, acc, adesc, bdesc, IDESC, (kb > 0 || ks > 0) ? 1u : 0u);
                }
                mma_commit_lead(el, &empty[s]);
            }
            if (ok) mma_commit_lead(el, &tfull[b]);
        }
        mma_commit_lead(el, drain);
        volatile int keep_waiting = 0;   // tensor memory is freed only after the MMAs are done, on every path
        warp_wait_all(drain, 0, DEV_TIMEOUT_DRAIN, p.err, &keep_waiting);
        __syncwarp();
    } else if (PLANES && warp < G::NEXP) {
        // ---------------- plane expansion, one ring with the producer ----------------
        const int et = threadIdx.x;                  // 0 .. 255
        constexpr int GROUPS = BN / 32;
        constexpr int ITEMS = PBK * GROUPS / 256;
        const int h = et % GROUPS;
        const uint32_t atom = static_cast<uint32_t>((32 * h) / G::ATOM_W) * G::REGION;
        const int cc = ((32 * h) % G::ATOM_W) / 16;
        int g = 0;
        bool ok = true;   // (KIND_ST: each expander warp stops on its own; no barrier joins them)
        for (int t = blockIdx.x; (KIND == KIND_CODES || ok) && t < total; t += gridDim.x) {
            const TileDesc d = tile_of(t, m_tiles, n_tiles, BN, p.K);
            const int fl_off = (d.n0 / 8) & 15;
            uint32_t clo[8], nclo[8];
            if (KIND == KIND_CODES) {   // this tile's clo bytes, through shared memory
                named_barrier_sync(5, 256);   // everyone is done with the previous tile and its table
                if (et == 0) *decide_exp = *abort_flag;
                for (int nl = et; nl < BN; nl += 256) clo_s[nl] = static_cast<uint8_t>(clo_of(p.lo[d.n0 + nl],
                                                                                               p.hi[d.n0 + nl]));
                named_barrier_sync(5, 256);
                if (*decide_exp) break;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    uint32_t c = 0, nc = 0;
#pragma unroll
                    for (int pb = 0; pb < 4; ++pb) {
                        const uint32_t v = clo_s[32 * h + 8 * pb + j];
                        c |= v << (8 * pb);
                        nc |= ((0x100u - v) & 0xFFu) << (8 * pb);
                    }
                    clo[j] = c;
                    nclo[j] = nc;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) clo[j] = nclo[j] = 0;
            }
            for (int kb = 0; kb < d.nk; ++kb, ++g) {
                const int s = g % STAGES, r = g / STAGES;
                if (!warp_wait(&full[s], r & 1, DEV_TIMEOUT_FULL, p.err, abort_flag)) {
                    ok = false;
                    g += d.nk - kb;   // keep the ring position in step with the other roles
                    break;
                }
                const uint8_t* sg = sg_tile(s);
                const uint8_t* fl = fl_tile(s);
                uint8_t* bt = b_tile(s);
#pragma unroll
                for (int itm = 0; itm < ITEMS; ++itm) {
                    const int k = (itm * 256 + et) / GROUPS;
                    const uint2 x = *reinterpret_cast<const uint2*>(sg + k * (BN / 4) + 8 * h);
                    const uint32_t fw = *reinterpret_cast<const uint32_t*>(fl + k * G::FL_ROW + fl_off + 4 * h);
                    Planes32 pl;
                    pl.load(x.x, x.y, fw);
                    const uint32_t q0 = atom + b_offset<G::ATOM_W>(k, cc), q1 = atom + b_offset<G::ATOM_W>(k, cc + 1);
                    if (KIND == KIND_ST) {
                        uint32_t S[8], T[8];
                        expand_st(pl, S, T);
                        *reinterpret_cast<uint4*>(bt + q0) = make_uint4(S[0], S[1], S[2], S[3]);
                        *reinterpret_cast<uint4*>(bt + q1) = make_uint4(S[4], S[5], S[6], S[7]);
                        *reinterpret_cast<uint4*>(bt + G::REGION + q0) = make_uint4(T[0], T[1], T[2], T[3]);
                        *reinterpret_cast<uint4*>(bt + G::REGION + q1) = make_uint4(T[4], T[5], T[6], T[7]);
                    } else {
                        uint32_t W[8];
                        expand_codes(pl, clo, nclo, W);
                        *reinterpret_cast<uint4*>(bt + q0) = make_uint4(W[0], W[1], W[2], W[3]);
                        *reinterpret_cast<uint4*>(bt + q1) = make_uint4(W[4], W[5], W[6], W[7]);
                    }
                }
                fence_proxy_async_smem();
                mbar_arrive(&bready[s]);
            }
        }
    } else if (warp >= G::EPI0 && warp < G::EPI0 + 4) {
        // ---------------- epilogue: warp EPI0 + q reads TMEM lanes 32 q .. 32 q + 31 ----------------
        const int quarter = warp & 3;
        const int rloc = quarter * 32 + lane;
        const bool leader = warp == G::EPI0 && lane == 0;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const bool load_old = !partial && !p.beta_zero;
        griddep_wait();   // a_scales, C_old and C belong to the previous kernels until here
        int cc = 0, it = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
            const TileDesc d = tile_of(t, m_tiles, n_tiles, BN, p.K);
            const int b = it & 1;
            const int row = d.m0 + rloc;
            const float as = row < p.M ? __fmul_rn(p.a_scales[row], p.alpha) : 0.f;
            const int out_row = partial ? d.z * p.m_pad + d.m0 : d.m0;
            warp_wait(&tfull[b], (it >> 1) & 1, DEV_TIMEOUT_ACC, p.err, abort_flag);   // a timeout sets the flag
            named_barrier_sync(6, 128);
            if (leader) *decide_epi = *abort_flag;
            named_barrier_sync(6, 128);
            if (*decide_epi) break;
            tc_fence_after();
            const uint32_t acc = tmem + lane_base + static_cast<uint32_t>(b * G::MMA_N);
#pragma unroll 1
            for (int c = 0; c < G::CHUNKS; ++c, ++cc) {
                const int sb = cc & 1;
                uint8_t* tile = stg + sb * G::STG_BYTES;
                if (leader) {
                    tma_store_wait_read_1();   // the store that last read this buffer has finished reading it
                    if (load_old) {
                        mbar_arrive_expect_tx(&cfull[sb], G::STG_BYTES);
                        tma_load_2d(tile, &tmOut, &cfull[sb], d.n0 + 32 * c, d.m0);
                    }
                }
                named_barrier_sync(6, 128);
                // (a timed-out C_old load sets the abort flag; every warp still meets the barriers below, the chunk
                // is stored with whatever the buffer holds and the error is reported through the error word)
                if (load_old) warp_wait(&cfull[sb], (cc >> 1) & 1, DEV_TIMEOUT_ACC, p.err, abort_flag);
                const int n = d.n0 + 32 * c;
                if (!G::ST) {
                    uint32_t r32[32];
                    tmem_ld_32x32b_x32(acc + 32 * c, r32);
                    float c1a[32];
#pragma unroll
                    for (int t4 = 0; t4 < 8; ++t4) {
                        float4 a;
                        if (p.cmode == CM_Q8B) {
                            a = __ldg(reinterpret_cast<const float4*>(p.scales + n) + t4);
                        } else {   // int8w: hi * (1 / 127)
                            const float4 hv = __ldg(reinterpret_cast<const float4*>(p.hi + n) + t4);
                            a = make_float4(__fmul_rn(hv.x, 1.0f / 127.0f), __fmul_rn(hv.y, 1.0f / 127.0f),
                                            __fmul_rn(hv.z, 1.0f / 127.0f), __fmul_rn(hv.w, 1.0f / 127.0f));
                        }
                        c1a[4 * t4] = a.x; c1a[4 * t4 + 1] = a.y; c1a[4 * t4 + 2] = a.z; c1a[4 * t4 + 3] = a.w;
                    }
                    tmem_wait_ld();
#pragma unroll
                    for (int t4 = 0; t4 < 8; ++t4) {
                        float4 old = make_float4(0.f, 0.f, 0.f, 0.f);
                        if (load_old) old = *reinterpret_cast<const float4*>(tile + out_offset(rloc, t4));
                        const float ov[4] = {old.x, old.y, old.z, old.w};
                        float o[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int tt = 4 * t4 + e;
                            const int ph = PLANES ? 4 * (tt & 7) + (tt >> 3) : tt;   // column-transposed with planes
                            const float f = __fmul_rn(__int2float_rn(static_cast<int>(r32[ph])), c1a[tt]);
                            o[e] = partial ? f : (load_old ? __fmaf_rn(f, as, ov[e]) : __fmul_rn(f, as));
                        }
                        *reinterpret_cast<float4*>(tile + out_offset(rloc, t4)) = make_float4(o[0], o[1], o[2], o[3]);
                    }
                } else {
#pragma unroll 1
                    for (int half = 0; half < 2; ++half) {
                        uint32_t rS[16], rT[16];
                        tmem_ld_32x32b_x16(acc + 32 * c + 16 * half, rS);
                        tmem_ld_32x32b_x16(acc + BN + 32 * c + 16 * half, rT);
                        float c1a[16], c2a[16];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int t4 = 2 * i + half;
                            const float4 lo4 = __ldg(reinterpret_cast<const float4*>(p.lo + n) + t4);
                            const float4 hi4 = __ldg(reinterpret_cast<const float4*>(p.hi + n) + t4);
                            c1a[4 * i] = lo4.x; c1a[4 * i + 1] = lo4.y; c1a[4 * i + 2] = lo4.z; c1a[4 * i + 3] = lo4.w;
                            c2a[4 * i] = __fsub_rn(hi4.x, lo4.x); c2a[4 * i + 1] = __fsub_rn(hi4.y, lo4.y);
                            c2a[4 * i + 2] = __fsub_rn(hi4.z, lo4.z); c2a[4 * i + 3] = __fsub_rn(hi4.w, lo4.w);
                        }
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int t4 = 2 * i + half;
                            float4 old = make_float4(0.f, 0.f, 0.f, 0.f);
                            if (load_old) old = *reinterpret_cast<const float4*>(tile + out_offset(rloc, t4));
                            const float ov[4] = {old.x, old.y, old.z, old.w};
                            float o[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int ph = 4 * e + i;
                                const float f = __fmaf_rn(__int2float_rn(static_cast<int>(rT[ph])), c2a[4 * i + e],
                                                          __fmul_rn(__int2float_rn(static_cast<int>(rS[ph])),
                                                                    c1a[4 * i + e]));
                                o[e] = partial ? f : (load_old ? __fmaf_rn(f, as, ov[e]) : __fmul_rn(f, as));
                            }
                            *reinterpret_cast<float4*>(tile + out_offset(rloc, t4)) =
                                make_float4(o[0], o[1], o[2], o[3]);
                        }
                    }
                }
                fence_proxy_async_smem();
                named_barrier_sync(6, 128);
                if (leader) {
                    tma_store_2d(&tmOut, tile, n, out_row);
                    tma_store_commit();
                }
            }
            // every TMEM read of accumulator b is complete: hand it back to the MMA issuer
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
        }
        if (leader) tma_store_wait_all();   // the staging buffers must outlive the stores reading them
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == G::MMAW) tmem_dealloc(tmem, G::TMEM_COLS);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_p(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
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

int sm_count() {
    static int n[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
    return n[dev] > 0 ? n[dev] : 148;
}

template <int BN, int KIND>
cudaError_t launch_p(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1, const CUtensorMap& out,
                     const FvGemmParams& p, cudaStream_t stream) {
    using G = PCfg<BN, KIND>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(fv_gemm_p_kernel<BN, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(G::SMEM_BYTES));
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const int total = ((p.M + PBM - 1) / PBM) * (p.N / BN) * p.ksplit;
    const int grid = total < sm_count() ? total : sm_count();
    return launch_pdl_p(fv_gemm_p_kernel<BN, KIND>, dim3(grid), dim3(G::NTHREADS), G::SMEM_BYTES, stream, a, b0, b1,
                        out, p);
}

}  // namespace

int fv_gemm_p_tiles(int M, int N, int bn, int ksplit) { return ((M + PBM - 1) / PBM) * (N / bn) * ksplit; }

int fv_gemm_p_min_tiles() { return sm_count(); }

cudaError_t fv_gemm_p_launch(int bn, int kind, const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                             const CUtensorMap& out, const FvGemmParams& p, cudaStream_t stream) {
    switch (kind) {
    case KIND_ST:
        if (bn == 64) return launch_p<64, KIND_ST>(a, b0, b1, out, p, stream);
        if (bn == 128) return launch_p<128, KIND_ST>(a, b0, b1, out, p, stream);
        break;
    case KIND_CODES:
        if (bn == 64) return launch_p<64, KIND_CODES>(a, b0, b1, out, p, stream);
        if (bn == 128) return launch_p<128, KIND_CODES>(a, b0, b1, out, p, stream);
        if (bn == 256) return launch_p<256, KIND_CODES>(a, b0, b1, out, p, stream);
        break;
    default:
        if (bn == 64) return launch_p<64, KIND_TABLE>(a, b0, b1, out, p, stream);
        if (bn == 128) return launch_p<128, KIND_TABLE>(a, b0, b1, out, p, stream);
        if (bn == 256) return launch_p<256, KIND_TABLE>(a, b0, b1, out, p, stream);
        break;
    }
    return cudaErrorInvalidValue;
}

}  // namespace p2cu
