// fv_gemm_2sm.cu - the five-value / int8-table GEMM on CTA pairs (tcgen05 cta_group::2), for launches with many
// output tiles (large M: windows stacked along the rows).
//
// The arithmetic is fv_gemm.cu's, bit for bit (int8 products summed exactly in int32 per 1024-row K block, the same
// epilogue). What changes is the tile: a cluster of two CTAs on two SMs computes a 256 x 256 output tile with one
// M = 256 MMA stream. CTA r of the pair holds rows [128 r, 128 r + 128) of the A tile and columns
// [128 r, 128 r + 128) of the B tile in its own shared memory and rows [128 r, 128 r + 128) of the accumulator in its
// own TMEM, so each SM streams 32 KB of operands per 128-deep K step for 4.2 M MACs - two thirds of what a one-SM
// 128 x 256 tile needs - which is what the tensor cores' rate asks of L2 at large M.
//
// Roles in each CTA: the TMA producer (its A and B halves, into its own shared memory, on its own barriers); 8 plane
// expanders when the weights are five-value planes (its B half); 8 epilogue warps (its TMEM rows -> fp32 C); and one
// warp that in the even CTA issues the pair's MMAs and in the odd CTA relays "this stage of mine has landed" to it.
// The epilogue warps work independently: warp (h, q) drains TMEM lanes 32 q .. 32 q + 31 and accumulator columns
// 128 h .. 128 h + 127, 32 at a time, through two 4 KB staging blocks of its own (one being written while the other's
// store reads it), each 32 x 32 block leaving by its own TMA store (one thread's bulk copies complete in order, so
// spreading them over eight warps keeps the stores apace);
// the column constants of a tile are read into shared memory once, C_old straight from global memory.
// The even CTA's MMA completions are committed to the barriers of both CTAs at once (tcgen05.commit multicast); the
// odd CTA's epilogue hands each drained accumulator back with a remote mbarrier arrive. With an int8 table (the code
// cache) the odd CTA's TMA loads complete on the even CTA's stage barrier (the cta_group::2 form of the load, no
// multicast), which expects both CTAs' bytes, so the MMA issuer waits on one barrier per stage and no relay hop lies
// in the stage's round trip; with planes the odd CTA's expanders finish the stage, and its relay thread announces it.
// Barriers that the other CTA completes (by a multicast commit or a remote arrive with release semantics at cluster
// scope) are waited on like local ones, with the CTA-scope try_wait: a cluster-scope acquire there cost about 0.6 us
// per K step on the critical path, and the operands the MMAs read are ordered by the tensor-core proxy's own commits
// and by the TMA completions the relaying thread observed. Every wait is bounded (ptx.cuh); a timeout is reported
// through the error word.
#include <cstdint>
#include <utility>
#include <cuda.h>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "fv_gemm.h"
#include "fv_common.cuh"

namespace p2cu {

namespace {

constexpr int QBM = 128;            // rows per CTA (a pair tile has 256)
constexpr int QBN = 256;            // columns per pair tile (the MMA's N)
constexpr int QHN = 128;            // columns of B per CTA
constexpr int QBK = 128, QKBLK = 1024;

template <int KIND_> struct QCfg {
    static constexpr int KIND = KIND_;
    static constexpr bool PLANES = KIND == KIND_CODES;
    static constexpr int NEXP = PLANES ? 8 : 0;                 // expander warps 0 .. NEXP - 1
    static constexpr int EPI0 = NEXP;                           // epilogue warps EPI0 .. EPI0 + 7
    static constexpr int NEPI = 8;
    // TMA producer warps. One warp's tile loads complete one after another (about 0.4 us each on B200, whatever the
    // box size), so the stages are spread over several producer warps: warp PROD + w issues every load of the
    // K steps g with g % NPROD == w. NPROD <= STAGES (asserted below) keeps each warp's parity wait on a stage
    // unambiguous: its own previous wait proves the round before last complete.
    static constexpr int NPROD = 4;
    static constexpr int PROD = EPI0 + NEPI, MMAW = PROD + NPROD;
    static constexpr int NTHREADS = (MMAW + 1) * 32;
    static constexpr uint32_t A_BYTES = QBM * QBK;              // 16 KB, K-major, 128-byte swizzle
    static constexpr uint32_t B_BYTES = QBK * QHN;              // 16 KB, MN-major, one 128-byte swizzle atom wide
    static constexpr uint32_t SG_BYTES = QBK * (QHN / 4);       // sign plane rows of the half
    static constexpr uint32_t FL_ROW = QHN / 8;
    static constexpr uint32_t FL_BYTES = QBK * FL_ROW;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES + (PLANES ? SG_BYTES + FL_BYTES : 0);
    static constexpr uint32_t SBO = 8 * QHN;
    static constexpr uint32_t WBUF = 32 * 32 * 4;               // one 32 x 32 fp32 output block
    static constexpr uint32_t STG_BYTES = NEPI * 2 * WBUF;      // two per epilogue warp: one written, one storing
    static constexpr uint32_t C1_BYTES = QBN * 4;               // the tile's column constants
    static constexpr uint32_t BAR_BYTES = 512;
    static constexpr uint32_t FIXED = 1024 + STG_BYTES + C1_BYTES + BAR_BYTES;
    static constexpr int STAGES_FIT = static_cast<int>((227 * 1024 - FIXED) / STAGE_BYTES);
    static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
    static constexpr uint32_t SMEM_BYTES = FIXED + STAGES * STAGE_BYTES;
    static constexpr uint32_t TMEM_COLS = 2 * QBN;              // two accumulators
    static_assert(STAGES >= 3, "pipeline depth");
    static_assert(NPROD <= STAGES, "producer warps and stage phases");
    static_assert(5 * STAGES * 8 + 5 * 8 + 32 + QHN <= BAR_BYTES, "barrier region");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};

struct PairTile {
    int m0, n0, z, k_begin, nk;
};

__device__ __forceinline__ PairTile pair_tile(int t, int m_tiles, int n_tiles, int K) {
    PairTile d;
    const int mt = t % m_tiles, rest = t / m_tiles;
    d.m0 = mt * 2 * QBM;
    d.n0 = (rest % n_tiles) * QBN;
    d.z = rest / n_tiles;
    d.k_begin = d.z * QKBLK;
    const int k_len = K - d.k_begin < QKBLK ? K - d.k_begin : QKBLK;
    d.nk = (k_len + QBK - 1) / QBK;
    return d;
}

// Diagnostic builds (-DP2CU_TRACE) record globaltimer nanoseconds at pipeline events of the first CTA pair into
// p.trace[256 * rank + slot]: 0+g MMA warp has the stage's own data, 40+g it has the peer's, 80+g producer issues the
// stage's A load, 120+g (odd CTA) relay fired, 160+i epilogue warp 0 sees accumulator i, 168+i it finished tile i,
// 176+i tile i committed, 250 start.
#ifdef P2CU_TRACE
__device__ __forceinline__ long long trace_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return static_cast<long long>(t);
}
#define QTRACE(slot, cond) do { if (p.trace && blockIdx.x < 2 && (cond)) \
                                    p.trace[256 * rank + (slot)] = trace_ns(); } while (0)
#else
#define QTRACE(slot, cond) do { } while (0)
#endif

template <int KIND>
__global__ void __launch_bounds__(QCfg<KIND>::NTHREADS, 1)
fv_gemm_2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                   const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmOut,
                   const FvGemmParams p) {
    using G = QCfg<KIND>;
    constexpr int STAGES = G::STAGES;
    constexpr bool PLANES = G::PLANES;
    constexpr uint32_t IDESC = idesc_i8(2 * QBM, QBN, false, true);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stg = smem + STAGES * G::STAGE_BYTES;                  // the epilogue warps' staging blocks
    float* c1_s = reinterpret_cast<float*>(stg + G::STG_BYTES);     // [QBN] column constants of the current tile
    uint8_t* bar_region = stg + G::STG_BYTES + G::C1_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(bar_region);       // this CTA's A (and table B) of a stage landed
    uint64_t* pfull = full + STAGES;                                // this CTA's planes of a stage landed
    uint64_t* bready = pfull + STAGES;                              // this CTA's planes expanded
    uint64_t* peer = bready + STAGES;                               // (even CTA) the odd CTA's stage is ready
    uint64_t* empty = peer + STAGES;                                // the pair's MMAs are done with a stage
    uint64_t* tfull = empty + STAGES;                               // [2] accumulator complete
    uint64_t* tempty = tfull + 2;                                   // [2] (even CTA) accumulator drained by both
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    volatile int* decide_epi = abort_flag + 1;
    volatile int* decide_exp = abort_flag + 2;
    uint8_t* clo_s = reinterpret_cast<uint8_t*>(tmem_holder + 8);   // QHN bytes: the half's clo values

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool lead = rank == 0;
    const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
    const int mrow = static_cast<int>(rank) * QBM, ncol = static_cast<int>(rank) * QHN;
    const int m_tiles = (p.M + 2 * QBM - 1) / (2 * QBM), n_tiles = p.N / QBN;
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
            mbar_init(&pfull[s], 1);
            mbar_init(&bready[s], G::NEXP > 0 ? G::NEXP * 32 : 1);
            mbar_init(&peer[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * G::NEPI);   // the epilogue warps of both CTAs
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
        tmem_alloc_pair(tmem_holder, G::TMEM_COLS);
        tmem_relinquish_pair();
    }
    // Both CTAs' barriers are initialised and their TMEM allocated before either CTA signals the other.
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    griddep_launch_dependents();
    QTRACE(250, threadIdx.x == 0);

    if (warp >= G::PROD && warp < G::PROD + G::NPROD) {
        // ---------------- TMA producers: this CTA's halves, one ring of stages across its tiles ----------------
        const int pw = warp - G::PROD;
        if (lane == 0) {
            constexpr uint32_t FULL_TX = PLANES ? G::A_BYTES : G::A_BYTES + G::B_BYTES;
            // table: both CTAs' copies of a stage complete on the even CTA's barrier, which expects them all
            const uint32_t full_lead = cluster_map(&full[0], 0);
            auto load_b = [&](int s, int n0, int kx) {
                if (PLANES) {
                    mbar_arrive_expect_tx(&pfull[s], G::SG_BYTES + G::FL_BYTES);
                    tma_load_2d(sg_tile(s), &tmB0, &pfull[s], (n0 + ncol) / 4, kx);
                    tma_load_2d(fl_tile(s), &tmB1, &pfull[s], (n0 + ncol) / 8, kx);
                } else {
                    if (lead) mbar_arrive_expect_tx(&full[s], 2 * FULL_TX);   // the A loads of the stage follow
                    tma_load_2d_pair(b_tile(s), &tmB0, full_lead + static_cast<uint32_t>(s) * 8u, n0 + ncol, kx);
                }
            };
            // The first stages' weights before the dependency wait (they are constant), then everything else.
            int pre = 0;
            if (pair < total) {
                const PairTile d = pair_tile(pair, m_tiles, n_tiles, p.K);
                pre = d.nk < STAGES ? d.nk : STAGES;
                for (int kb = pw; kb < pre; kb += G::NPROD) load_b(kb, d.n0, d.k_begin + kb * QBK);
            }
            griddep_wait();
            int g = 0;
            bool ok = true;
            for (int t = pair; ok && t < total; t += npairs) {
                const PairTile d = pair_tile(t, m_tiles, n_tiles, p.K);
                for (int kb = 0; kb < d.nk; ++kb, ++g) {
                    if (g % G::NPROD != pw) continue;
                    const int s = g % STAGES, r = g / STAGES;
                    if (g >= pre) {
                        if (!mbar_wait(&empty[s], (r & 1) ^ 1, DEV_TIMEOUT_EMPTY, p.err, abort_flag)) {
                            ok = false;
                            break;
                        }
                        load_b(s, d.n0, d.k_begin + kb * QBK);
                    }
                    QTRACE(80 + g, g < 40);
                    if (PLANES) {
                        mbar_arrive_expect_tx(&full[s], FULL_TX);
                        tma_load_2d(a_tile(s), &tmA, &full[s], d.k_begin + kb * QBK, d.m0 + mrow);
                    } else {
                        tma_load_2d_pair(a_tile(s), &tmA, full_lead + static_cast<uint32_t>(s) * 8u,
                                         d.k_begin + kb * QBK, d.m0 + mrow);
                    }
                }
            }
            // No copy this warp issued may still be landing in this CTA's shared memory when it exits. With a table
            // the even CTA's barrier counts both CTAs' copies: the even CTA waits for them, and the odd one, which
            // cannot observe that barrier, leaves only after the even one (the cluster barrier at the end) and,
            // after a timeout, after a bounded pause for copies still in flight.
            if (!PLANES && !lead) {
                if (*abort_flag) {
                    const long long t0 = clock64();
                    while (clock64() - t0 < 20000) {}
                }
                g = 0;
            }
            for (int k = g - STAGES < 0 ? 0 : g - STAGES; k < g; ++k) {
                if (k % G::NPROD != pw) continue;
                const int s = k % STAGES, r = k / STAGES;
                for (uint32_t i = 0; i < WAIT_LIMIT && !mbar_try_wait(smem_u32(&full[s]), r & 1); ++i) {}
                if (PLANES)
                    for (uint32_t i = 0; i < WAIT_LIMIT && !mbar_try_wait(smem_u32(&pfull[s]), r & 1); ++i) {}
            }
        }
    } else if (warp == G::MMAW) {
        if (lead) {
            // ---------------- MMA issue for the pair: tile i into accumulator i % 2 ----------------
            // The whole warp runs the loop converged and waits with all lanes; one elected lane issues (issue from
            // code one lane runs alone, branches inside it, was measured at about half the rate).
            const uint32_t el = elect_one();
            int g = 0, it = 0;
            bool ok = true;
            for (int t = pair; ok && t < total; t += npairs, ++it) {
                const PairTile d = pair_tile(t, m_tiles, n_tiles, p.K);
                const int b = it & 1;
                if (!warp_wait_all(&tempty[b], ((it >> 1) & 1) ^ 1, DEV_TIMEOUT_ACC, p.err, abort_flag)) break;
                tc_fence_after();
                const uint32_t acc = tmem + static_cast<uint32_t>(b * QBN);
                for (int kb = 0; kb < d.nk; ++kb, ++g) {
                    const int s = g % STAGES, r = g / STAGES;
                    if (!warp_wait_all(&full[s], r & 1, DEV_TIMEOUT_READY, p.err, abort_flag) ||
                        (PLANES && !warp_wait_all(&bready[s], r & 1, DEV_TIMEOUT_READY, p.err, abort_flag))) {
                        ok = false;
                        break;
                    }
                    QTRACE(g, g < 40 && el);
                    if (PLANES && !warp_wait_all(&peer[s], r & 1, DEV_TIMEOUT_READY, p.err, abort_flag)) {
                        ok = false;
                        break;
                    }
                    QTRACE(40 + g, g < 40 && el);
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(a_tile(s));
                    const uint32_t b_base = smem_u32(b_tile(s));
#pragma unroll
                    for (int ks = 0; ks < QBK / 32; ++ks) {
                        const uint64_t adesc = smem_desc(a_base + ks * 32, 16, 1024, SWZ_128B);
                        const uint64_t bdesc = smem_desc(b_base + ks * 4 * G::SBO, G::SBO, G::SBO, SWZ_128B);
                        mma_i8_pair_lead(el, acc, adesc, bdesc, IDESC, (kb > 0 || ks > 0) ? 1u : 0u);
                    }
                    mma_commit_pair_lead(el, &empty[s], 0x3);
                }
                if (ok) mma_commit_pair_lead(el, &tfull[b], 0x3);
                QTRACE(176 + it, it < 8 && el);
            }
            mma_commit_pair_lead(el, drain, 0x1);
            volatile int keep_waiting = 0;   // tensor memory is freed only after the MMAs are done, on every path
            warp_wait_all(drain, 0, DEV_TIMEOUT_DRAIN, p.err, &keep_waiting);
        } else {
            // ---------------- relay (planes): each of this CTA's stages, once expanded, to the even CTA --------
            if (PLANES && lane == 0) {
                const uint32_t peer0 = cluster_map(&peer[0], 0);
                int g = 0;
                bool ok = true;
                for (int t = pair; ok && t < total; t += npairs) {
                    const PairTile d = pair_tile(t, m_tiles, n_tiles, p.K);
                    for (int kb = 0; kb < d.nk; ++kb, ++g) {
                        const int s = g % STAGES, r = g / STAGES;
                        if (!mbar_wait(&full[s], r & 1, DEV_TIMEOUT_READY, p.err, abort_flag) ||
                            (PLANES && !mbar_wait(&bready[s], r & 1, DEV_TIMEOUT_READY, p.err, abort_flag))) {
                            ok = false;
                            break;
                        }
                        QTRACE(120 + g, g < 40);
                        mbar_arrive_remote_relaxed(peer0 + static_cast<uint32_t>(s) * 8u);
                    }
                }
            }
        }
        __syncwarp();
    } else if (PLANES && warp < G::NEXP) {
        // ---------------- plane expansion of this CTA's B half ----------------
        const int et = threadIdx.x;                  // 0 .. 255
        constexpr int GROUPS = QHN / 32;
        constexpr int ITEMS = QBK * GROUPS / 256;
        const int h = et % GROUPS;
        const int cc = (32 * h) / 16;
        int g = 0;
        for (int t = pair; t < total; t += npairs) {
            const PairTile d = pair_tile(t, m_tiles, n_tiles, p.K);
            uint32_t clo[8], nclo[8];
            named_barrier_sync(5, 256);   // everyone is done with the previous tile and its table
            if (et == 0) *decide_exp = *abort_flag;
            for (int nl = et; nl < QHN; nl += 256)
                clo_s[nl] = static_cast<uint8_t>(clo_of(p.lo[d.n0 + ncol + nl], p.hi[d.n0 + ncol + nl]));
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
            for (int kb = 0; kb < d.nk; ++kb, ++g) {
                const int s = g % STAGES, r = g / STAGES;
                if (!warp_wait(&pfull[s], r & 1, DEV_TIMEOUT_FULL, p.err, abort_flag)) {
                    g += d.nk - kb;   // keep the ring position in step with the other roles
                    break;
                }
                const uint8_t* sg = sg_tile(s);
                const uint8_t* fl = fl_tile(s);
                uint8_t* bt = b_tile(s);
#pragma unroll
                for (int itm = 0; itm < ITEMS; ++itm) {
                    const int k = (itm * 256 + et) / GROUPS;
                    const uint2 x = *reinterpret_cast<const uint2*>(sg + k * (QHN / 4) + 8 * h);
                    const uint32_t fw = *reinterpret_cast<const uint32_t*>(fl + k * G::FL_ROW + 4 * h);
                    Planes32 pl;
                    pl.load(x.x, x.y, fw);
                    const uint32_t q0 = b_offset<QHN>(k, cc), q1 = b_offset<QHN>(k, cc + 1);
                    uint32_t W[8];
                    expand_codes(pl, clo, nclo, W);
                    *reinterpret_cast<uint4*>(bt + q0) = make_uint4(W[0], W[1], W[2], W[3]);
                    *reinterpret_cast<uint4*>(bt + q1) = make_uint4(W[4], W[5], W[6], W[7]);
                }
                fence_proxy_async_smem();
                mbar_arrive(&bready[s]);
            }
        }
    } else if (warp >= G::EPI0 && warp < G::EPI0 + G::NEPI) {
        // ---------------- epilogue: warp (h, q) drains TMEM lanes 32 q .. + 31, columns 128 h .. + 127 ----------------
        const int ew = warp - G::EPI0;
        const int quarter = warp & 3;               // a warp reads the TMEM lane quarter of its warp id modulo 4
        const int half = ew >> 2;
        const int rloc = quarter * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const bool load_old = !partial && !p.beta_zero;
        const uint32_t tempty_lead = cluster_map(&tempty[0], 0);
        uint8_t* bufs = stg + ew * 2 * G::WBUF;
        int nblk_done = 0;   // blocks this warp has handed to TMA stores (which of its two staging blocks is next)
        griddep_wait();   // a_scales, C_old and C belong to the previous kernels until here
        int it = 0;
        for (int t = pair; t < total; t += npairs, ++it) {
            const PairTile d = pair_tile(t, m_tiles, n_tiles, p.K);
            const int b = it & 1;
            const int row0 = d.m0 + mrow;
            const int row = row0 + rloc;
            const bool row_ok = row < p.M;
            const float as = row_ok ? __fmul_rn(p.a_scales[row], p.alpha) : 0.f;
            const int out_row = (partial ? d.z * p.m_pad + row0 : row0) + 32 * quarter;
            const bool live = row0 < p.M;   // an odd CTA wholly below the last row stores nothing
            warp_wait(&tfull[b], (it >> 1) & 1, DEV_TIMEOUT_ACC, p.err, abort_flag);
            QTRACE(160 + it, ew == 0 && lane == 0 && it < 8);
            named_barrier_sync(6, 32 * G::NEPI);   // every warp is done with the previous tile's constants
            if (ew == 0 && lane == 0) *decide_epi = *abort_flag;
            for (int i = ew * 32 + lane; i < QBN; i += 32 * G::NEPI) {
                const int n = d.n0 + i;
                c1_s[i] = p.cmode == CM_Q8B ? p.scales[n] : __fmul_rn(p.hi[n], 1.0f / 127.0f);   // int8w: hi / 127
            }
            named_barrier_sync(6, 32 * G::NEPI);
            if (*decide_epi) break;
            tc_fence_after();
            const uint32_t acc = tmem + lane_base + static_cast<uint32_t>(b * QBN);
#pragma unroll 1
            for (int c = 0; live && c < 4; ++c) {
                const int col = 128 * half + 32 * c;
                const int n = d.n0 + col;
                uint32_t r32[32];
                tmem_ld_32x32b_x32(acc + col, r32);
                float4 old[8];
                if (load_old) {   // this thread's row of C_old, 32 columns
                    const float4* src = reinterpret_cast<const float4*>(p.C + static_cast<size_t>(row) * p.ldc + n);
#pragma unroll
                    for (int t4 = 0; t4 < 8; ++t4) old[t4] = row_ok ? src[t4] : make_float4(0.f, 0.f, 0.f, 0.f);
                }
                uint8_t* buf = bufs + (nblk_done & 1) * G::WBUF;
                if (lane == 0) tma_store_wait_read_1();   // the store before last (this block's) has finished reading it
                __syncwarp();
                tmem_wait_ld();
#pragma unroll
                for (int t4 = 0; t4 < 8; ++t4) {
                    const float ov[4] = {old[t4].x, old[t4].y, old[t4].z, old[t4].w};
                    float o[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int tt = 4 * t4 + e;
                        const int ph = PLANES ? 4 * (tt & 7) + (tt >> 3) : tt;   // column-transposed with planes
                        const float f = __fmul_rn(__int2float_rn(static_cast<int>(r32[ph])), c1_s[col + tt]);
                        o[e] = partial ? f : (load_old ? __fmaf_rn(f, as, ov[e]) : __fmul_rn(f, as));
                    }
                    *reinterpret_cast<float4*>(buf + out_offset(lane, t4)) = make_float4(o[0], o[1], o[2], o[3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tmOut, buf, n, out_row);
                    tma_store_commit();
                }
                ++nblk_done;
            }
            QTRACE(168 + it, ew == 0 && lane == 0 && it < 8);
            // every TMEM read of accumulator b by this warp is complete: hand it back to the pair's MMA issuer
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (lead) mbar_arrive(&tempty[b]);
                else mbar_arrive_remote(tempty_lead + static_cast<uint32_t>(b) * 8u);
            }
        }
        if (lane == 0) tma_store_wait_all();   // the staging block must outlive the stores reading it
    }

    // Neither CTA leaves (and frees its TMEM or shared memory) while the other may still signal or read it.
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    if (warp == G::MMAW) tmem_dealloc_pair(tmem, G::TMEM_COLS);
}

int sm_count_2sm() {
    static int n[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
    return n[dev] > 0 ? n[dev] : 148;
}

template <int KIND>
cudaError_t launch_2sm(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1, const CUtensorMap& out,
                       const FvGemmParams& p, cudaStream_t stream) {
    using G = QCfg<KIND>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(fv_gemm_2sm_kernel<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(G::SMEM_BYTES));
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const int total = ((p.M + 2 * QBM - 1) / (2 * QBM)) * (p.N / QBN) * p.ksplit;
    const int pairs = sm_count_2sm() / 2;
    const int grid = 2 * (total < pairs ? total : pairs);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(G::NTHREADS);
    cfg.dynamicSmemBytes = G::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, fv_gemm_2sm_kernel<KIND>, a, b0, b1, out, p);
}

}  // namespace

int fv_gemm_2sm_tiles(int M, int N, int ksplit) { return ((M + 2 * QBM - 1) / (2 * QBM)) * (N / QBN) * ksplit; }

cudaError_t fv_gemm_2sm_launch(int kind, const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                               const CUtensorMap& out, const FvGemmParams& p, cudaStream_t stream) {
    if (p.N % QBN) return cudaErrorInvalidValue;
    switch (kind) {
    case KIND_CODES: return launch_2sm<KIND_CODES>(a, b0, b1, out, p, stream);
    case KIND_TABLE: return launch_2sm<KIND_TABLE>(a, b0, b1, out, p, stream);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace p2cu
