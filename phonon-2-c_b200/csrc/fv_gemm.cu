// fv_gemm.cu - the five-value int8 GEMM on sm_100a tensor cores (tcgen05, TMEM accumulators, TMA operand loads and
// result stores).
//
// C[M, N] = alpha * A * B + beta * C with A int8 [M, K] (one fp32 scale per row, from a quantising kernel) and B one
// of three operand kinds:
//   KIND_CODES  five-value planes as phonon-2-c stores them (2-bit sign plane [K, N/4], 1-bit magnitude plane
//               [K, N/8], per-column lo / hi; csrc/blas.h:38-45), streamed by TMA and expanded in shared memory into
//               the int8w code plane sign * (flag ? 127 : clo), clo = round(127 lo / hi) (csrc/blas.c:1222-1240,
//               1316-1328); f = (float)acc * (hi * (1 / 127)).
//   KIND_ST     the same planes expanded into the two int8 planes of the int8 mode, S = sign and T = sign * flag,
//               multiplied by one MMA over [S | T] into adjacent TMEM columns (csrc/blas.c:1190-1220, 1329-1362):
//               f = fma((float)accT, hi - lo, (float)accS * lo).
//   KIND_TABLE  an int8 table [K, N] with one fp32 scale per column (the int8-table weights, csrc/blas.c:1243-1254,
//               and the cached int8w codes), loaded by TMA straight into the operand layout.
// The reference restarts its int32 sums every 1024 rows of K and rescales per block into C in block order
// (csrc/blas.c:1339-1366): C = (beta == 0 && first block) ? f * as : fma(f, as, C), as = a_scale[m] * alpha.
// Here one CTA owns exactly one 1024-row block of one 128 x BN output tile:
//   * K <= 1024: the CTA finishes the tile: C = f * as or fma(f, as, C_old);
//   * K > 1024: CTA z writes its block's f to a workspace slice, and fv_combine_kernel folds the slices into C in
//     block order afterwards, which is the reference's arithmetic bit for bit.
// Output chunks (128 rows x 32 columns) are staged in shared memory (128-byte swizzle) and written by TMA stores as
// soon as each is ready; C_old comes in by TMA.
//
// Roles (warps): epilogue groups of four warps (one TMEM lane quarter each); with planes, groups 1 and 2 expand the
// planes during the main loop; then the TMA producer and the MMA issuer (one elected lane, also the TMEM owner).
// Launched with programmatic dependent launch: the set-up, the weight loads and the plane expansion overlap the
// previous kernel's tail; A, its scales and C (everything a previous kernel may write) are touched only after
// griddepcontrol.wait. The weights must therefore not be written by a kernel that triggers dependent launches early.
#include <cstdint>
#include <utility>
#include <cuda.h>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "launch.cuh"
#include "fv_gemm.h"
#include "fv_common.cuh"

namespace p2cu {

// Diagnostic builds (-DP2CU_TRACE) record clock64() at pipeline events of CTA (0, 0, 0) into p.trace[slot].
#ifdef P2CU_TRACE
#define TRACE(slot) do { if (p.trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) \
                             p.trace[(slot)] = clock64(); } while (0)
#else
#define TRACE(slot) do { } while (0)
#endif
// Trace slots: 0 start, 1 after set-up, 8+kb producer issue, 80+kb MMA ready, 160+kb expansion done (first
// expander thread), 240 accumulator ready, 241 first chunk staged, 242 all chunks staged, 250 stores read, 260 end.

constexpr int BM = 128, BK = 128, KBLK = 1024;

template <int BN_, int KIND_> struct Cfg {
    static constexpr int BN = BN_;                                 // output columns per CTA
    static constexpr int KIND = KIND_;
    static constexpr bool PLANES = KIND != KIND_TABLE;             // B arrives as sign / magnitude planes
    static constexpr bool ST = KIND == KIND_ST;
    // B operand of the single MMA per K step: [S | T] (2 BN columns) or one plane of BN columns, MN-major, in atom
    // columns ATOM_W bytes wide (an atom = 8 K rows of ATOM_W bytes, swizzled).
    static constexpr int MMA_N = ST ? 2 * BN : BN;
    static constexpr int ATOM_W = ST ? BN : (BN < 128 ? BN : 128);
    static constexpr int N_ATOMS = MMA_N / ATOM_W;
    static constexpr uint32_t REGION = BK * ATOM_W;               // bytes of one atom column = the leading offset
    static constexpr uint32_t B_SWZ = ATOM_W == 128 ? SWZ_128B : SWZ_64B;
    static constexpr uint32_t SBO = 8 * ATOM_W;                    // 8-row K groups
    static constexpr int EPI_GROUPS = PLANES ? 3 : 2;
    static constexpr int NEXP = PLANES ? 8 : 0;                    // expander warps (= epilogue groups 1 and 2)
    static constexpr uint32_t A_BYTES = BM * BK;                   // int8 A tile, K-major, 128-byte swizzle
    static constexpr uint32_t B_BYTES = BK * MMA_N;                // the MMA's B operand
    static constexpr uint32_t SG_BYTES = BK * (BN / 4);            // sign-plane tile
    static constexpr uint32_t FL_ROW = BN / 8 < 16 ? 16 : BN / 8;  // a TMA box row is at least 16 bytes
    static constexpr uint32_t FL_BYTES = BK * FL_ROW;              // flag-plane tile
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES + (PLANES ? SG_BYTES + FL_BYTES : 0);
    static constexpr uint32_t B_TX_BYTES = PLANES ? SG_BYTES + FL_BYTES : B_BYTES;   // bytes TMA brings per stage
                                                                                      // besides the A tile
    static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 6 ? 6 : (200 * 1024) / STAGE_BYTES;
    // TMA producer warps: one warp's tile loads complete one after another (about 0.4 us each on B200, whatever the
    // box size), so warp PROD + w issues the loads of the K steps kb with kb % NPROD == w. NPROD <= STAGES: a warp's
    // wait for round r of a stage (by phase parity) is unambiguous only if round r - 2 is known to be complete, which
    // its own previous wait (for step kb - NPROD) guarantees exactly when NPROD <= STAGES.
    static constexpr int NPROD = STAGES < 4 ? STAGES : 4;
    static constexpr int PROD = 4 * EPI_GROUPS, MMAW = PROD + NPROD;
    static constexpr int NTHREADS = (MMAW + 1) * 32;
    static constexpr uint32_t TMEM_COLS = MMA_N <= 32 ? 32 : MMA_N <= 64 ? 64 : MMA_N <= 128 ? 128 : 256;
    static constexpr int CHUNKS = BN / 32;                         // 32-column output chunks
    static constexpr uint32_t OUT_BYTES = BM * BN * 4;             // fp32 output tile, aliases the stage buffers
    static constexpr uint32_t BAR_BYTES = 512;
    static constexpr uint32_t CONST_BYTES = 2 * BN * 4;
    static constexpr uint32_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + BAR_BYTES + CONST_BYTES;
    static_assert(MMA_N <= 256 && MMA_N % 16 == 0, "MMA N");
    static_assert(ATOM_W == 64 || ATOM_W == 128, "atom width");
    static_assert(STAGES >= 2, "pipeline depth");
    static_assert(NPROD <= STAGES, "producer warps and stage phases");
    static_assert(OUT_BYTES <= STAGES * STAGE_BYTES, "the output tile must fit in the stage buffers");
};

template <int BN, int KIND>
__global__ void __launch_bounds__(Cfg<BN, KIND>::NTHREADS, 1)
fv_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
               const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmOut,
               const FvGemmParams p) {
    using G = Cfg<BN, KIND>;
    constexpr int STAGES = G::STAGES;
    constexpr bool PLANES = G::PLANES;
    constexpr uint32_t IDESC = idesc_i8(BM, G::MMA_N, /*A MN-major*/ false, /*B MN-major*/ true);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* bar_region = smem + STAGES * G::STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(bar_region);
    uint64_t* bready = full + STAGES;
    uint64_t* empty = bready + STAGES;
    uint64_t* accfull = empty + STAGES;
    uint64_t* cfull = accfull + 1;
    uint64_t* drain = cfull + 1;
    uint64_t* afull = drain + 1;   // the A tile of a stage has landed (full[] covers the weights)
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(afull + STAGES);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    float* cc1 = reinterpret_cast<float*>(bar_region + G::BAR_BYTES);
    float* cc2 = cc1 + BN;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM, z = blockIdx.z;
    const int k_begin = z * KBLK;
    const int k_len = p.K - k_begin < KBLK ? p.K - k_begin : KBLK;
    const int nk = (k_len + BK - 1) / BK;
    const bool partial = p.ksplit > 1;   // this CTA writes f for its block to the workspace slice z

    auto stage_ptr = [&](int s) { return smem + s * G::STAGE_BYTES; };
    auto a_tile = [&](int s) { return stage_ptr(s); };
    auto b_tile = [&](int s) { return stage_ptr(s) + G::A_BYTES; };
    auto sg_tile = [&](int s) { return stage_ptr(s) + G::A_BYTES + G::B_BYTES; };
    auto fl_tile = [&](int s) { return stage_ptr(s) + G::A_BYTES + G::B_BYTES + G::SG_BYTES; };

    if (threadIdx.x == 0) {
        TRACE(0);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&afull[s], 1);
            mbar_init(&bready[s], G::NEXP > 0 ? G::NEXP * 32 : 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accfull, 1);
        mbar_init(cfull, 1);
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
    if (threadIdx.x == 0) TRACE(1);
    griddep_launch_dependents();   // the next kernel in the stream may start its set-up
    // Only what the previous kernels write (A, its scales, C_old, and C itself) waits for them (griddepcontrol.wait,
    // below, in the producer before the first A load and in the epilogue before the first read): the weights are
    // constant, so their loads and expansion overlap the previous kernel's tail.

    if (warp >= G::PROD && warp < G::PROD + G::NPROD) {
        // ---------------- TMA producers ----------------
        const int pw = warp - G::PROD;
        if (lane == 0) {
            auto load_b = [&](int kb) {
                const int s = kb % STAGES;
                const int kx = k_begin + kb * BK;
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
            // The stages are empty at the start (kb < pre). This warp's first stage's weights load before the
            // dependency wait; those of its later first-round stages follow its first A tile, because a warp's TMA
            // loads complete one after another and the first MMA must not queue behind weights it does not need.
            const int pre = nk < STAGES ? nk : STAGES;
            if (pw < pre) load_b(pw);
            griddep_wait();
            int issued = 0;
            for (int kb = pw; kb < nk; kb += G::NPROD) {
                const int s = kb % STAGES, r = kb / STAGES;
                if (kb >= pre) {
                    if (!mbar_wait(&empty[s], (r & 1) ^ 1, DEV_TIMEOUT_EMPTY, p.err, abort_flag)) break;
                    load_b(kb);
                } else if (kb != pw) {
                    load_b(kb);
                }
                issued = kb + 1;
                TRACE(8 + kb);
                mbar_arrive_expect_tx(&afull[s], G::A_BYTES);
                tma_load_2d(a_tile(s), &tmA, &afull[s], k_begin + kb * BK, m0);
            }
            // No copy this warp issued may still be landing in shared memory when the CTA exits (matters on the abort
            // path only).
            for (int kb = issued - STAGES < 0 ? 0 : issued - STAGES; kb < issued; ++kb) {
                if (kb % G::NPROD != pw) continue;
                const int s = kb % STAGES, r = kb / STAGES;
                for (uint32_t i = 0; i < WAIT_LIMIT && !mbar_try_wait(smem_u32(&full[s]), r & 1); ++i) {}
                for (uint32_t i = 0; i < WAIT_LIMIT && !mbar_try_wait(smem_u32(&afull[s]), r & 1); ++i) {}
            }
        }
    } else if (warp == G::MMAW) {
        // ---------------- MMA issue ----------------
        // The whole warp runs the loop converged and waits with all lanes; one elected lane issues (issue from code
        // one lane runs alone, branches inside it, was measured at about half the rate).
        const uint32_t el = elect_one();
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % STAGES, r = kb / STAGES;
            if (!warp_wait_all(PLANES ? &bready[s] : &full[s], r & 1, DEV_TIMEOUT_READY, p.err, abort_flag)) break;
            if (!warp_wait_all(&afull[s], r & 1, DEV_TIMEOUT_READY, p.err, abort_flag)) break;
            tc_fence_after();
            TRACE(80 + kb);
            const uint32_t a_base = smem_u32(a_tile(s));
            const uint32_t b_base = smem_u32(b_tile(s));
#pragma unroll
            for (int ks = 0; ks < BK / 32; ++ks) {
                // A: K-major 128-byte rows, 8-row groups 1024 bytes apart; a K step of 32 moves 32 bytes inside
                // the swizzle atom. B: MN-major atom columns ATOM_W bytes wide, REGION bytes apart (the leading
                // offset; with a single atom column it is never used and is set to SBO so that no reading of it
                // leaves the tile), 8-row K groups SBO bytes apart; a K step of 32 rows moves 4 groups.
                const uint64_t adesc = smem_desc(a_base + ks * 32, 16, 1024, SWZ_128B);
                const uint64_t bdesc = smem_desc(b_base + ks * 4 * G::SBO, G::N_ATOMS > 1 ? G::REGION : G::SBO,
                                                 G::SBO, G::B_SWZ);
                mma_i8_lead(el, tmem, adesc, bdesc, IDESC, (kb > 0 || ks > 0) ? 1u : 0u);
            }
            mma_commit_lead(el, &empty[s]);
        }
        mma_commit_lead(el, accfull);
        // Every MMA issued has completed once `drain` flips (bounded, and waited for on the abort path too).
        mma_commit_lead(el, drain);
        volatile int keep_waiting = 0;
        warp_wait_all(drain, 0, DEV_TIMEOUT_DRAIN, p.err, &keep_waiting);
        __syncwarp();
    } else {
        if (PLANES && warp >= 4) {
            // ---------------- plane expansion: warps 4-11 during the main loop ----------------
            const int et = threadIdx.x - 128;            // 0 .. 255
            constexpr int GROUPS = BN / 32;              // 32-column groups per K row
            constexpr int ITEMS = BK * GROUPS / 256;     // (row, group) items per expander thread per stage
            const int h = et % GROUPS;                   // this thread's 32-column group, the same in every item
            const int fl_off = (n0 / 8) & 15;            // this tile's flags inside the 16-byte box rows
            uint32_t clo[8], nclo[8];                    // codes: clo and -clo of the group's columns, word layout
            if (KIND == KIND_CODES) {
                // one column per expander thread into shared memory, then each thread packs its group's bytes
                uint8_t* clo_s = reinterpret_cast<uint8_t*>(cc2);   // cc2 is free in the int8w mode
                for (int nl = et; nl < BN; nl += 256) {
                    const int n = n0 + nl;
                    clo_s[nl] = n < p.N ? static_cast<uint8_t>(clo_of(p.lo[n], p.hi[n])) : 0;
                }
                named_barrier_sync(5, 256);
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
            // where this thread's 32 columns sit in the operand: atom column and 16-byte chunk within its rows
            const uint32_t atom = static_cast<uint32_t>((32 * h) / G::ATOM_W) * G::REGION;
            const int cc = ((32 * h) % G::ATOM_W) / 16;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % STAGES, r = kb / STAGES;
                if (!warp_wait(&full[s], r & 1, DEV_TIMEOUT_FULL, p.err, abort_flag)) break;
                const uint8_t* sg = sg_tile(s);
                const uint8_t* fl = fl_tile(s);
                uint8_t* bt = b_tile(s);
#pragma unroll
                for (int it = 0; it < ITEMS; ++it) {
                    const int k = (it * 256 + et) / GROUPS;
                    const uint2 x = *reinterpret_cast<const uint2*>(sg + k * (BN / 4) + 8 * h);
                    const uint32_t fw = *reinterpret_cast<const uint32_t*>(fl + k * G::FL_ROW + fl_off + 4 * h);
                    Planes32 pl;
                    pl.load(x.x, x.y, fw);
                    const uint32_t q0 = atom + b_offset<G::ATOM_W>(k, cc), q1 = atom + b_offset<G::ATOM_W>(k, cc + 1);
                    if (KIND == KIND_ST) {   // S in the first atom column, T in the second
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
                if (et == 0) TRACE(160 + kb);
                mbar_arrive(&bready[s]);
            }
        }
        // ---------------- epilogue: all groups; warp w reads TMEM lanes 32 (w % 4) .. + 31 ----------------
        constexpr int NEPI = 128 * G::EPI_GROUPS;
        const int grp = warp >> 2, quarter = warp & 3;
        const int rloc = quarter * 32 + lane, row = m0 + rloc;
        const bool live = row < p.M;
        if (grp == 0) {   // per-column constants, while the main loop runs
            for (int nl = rloc; nl < BN; nl += 128) {
                const int n = n0 + nl;
                float c1 = 0.f, c2 = 0.f;
                if (n < p.N) {
                    if (p.cmode == CM_Q8B) {
                        c1 = p.scales[n];
                    } else if (p.cmode == CM_INT8) {
                        c1 = p.lo[n];
                        c2 = __fsub_rn(p.hi[n], p.lo[n]);
                    } else {   // int8w: c1 = hi * (1 / 127)
                        c1 = __fmul_rn(p.hi[n], 1.0f / 127.0f);
                    }
                }
                cc1[nl] = c1;
                if (G::ST) cc2[nl] = c2;   // in the int8w mode the expanders keep their clo table there
            }
        }
        if (grp == 0 && !partial && !p.beta_zero) {   // C_old into L2 meanwhile: its TMA load after the wait hits L2
            for (int i = rloc; i < BM * G::CHUNKS; i += 128) {
                const int r = m0 + i / G::CHUNKS, c = n0 + 32 * (i % G::CHUNKS);
                if (r < p.M && c < p.N) prefetch_l2(p.C + static_cast<size_t>(r) * p.ldc + c);
            }
        }
        griddep_wait();   // a_scales, C_old and C belong to the previous kernels until here
        const float as = live ? __fmul_rn(p.a_scales[row], p.alpha) : 0.f;
        named_barrier_sync(1, NEPI);   // constants visible; the expanders are done with the stage buffers
        const bool ok = warp_wait(accfull, 0, DEV_TIMEOUT_ACC, p.err, abort_flag);
        tc_fence_after();
        if (threadIdx.x == 0) TRACE(240);
        const bool load_old = !partial && !p.beta_zero;
        bool have_old = ok && load_old;
        if (have_old && threadIdx.x == 0) {   // C_old into the staging tiles (the stage buffers are free now)
            mbar_arrive_expect_tx(cfull, G::OUT_BYTES);
            for (int c = 0; c < G::CHUNKS; ++c) tma_load_2d(smem + c * (BM * 128), &tmOut, cfull, n0 + 32 * c, m0);
        }
        if (have_old) have_old = warp_wait(cfull, 0, DEV_TIMEOUT_ACC, p.err, abort_flag);
        const bool go = ok && (!load_old || have_old);
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const int out_row = partial ? z * p.m_pad + m0 : m0;   // the workspace slice of block z, or C
        if (go) {
#pragma unroll 1
            for (int c = grp; c < G::CHUNKS; c += G::EPI_GROUPS) {
                uint8_t* tile = smem + c * (BM * 128);
                if (!G::ST) {
                    // one plane: the chunk's 32 TMEM columns in one load, its constants loaded meanwhile
                    uint32_t r32[32];
                    tmem_ld_32x32b_x32(tmem + lane_base + 32 * c, r32);
                    float c1a[32];
#pragma unroll
                    for (int t4 = 0; t4 < 8; ++t4) {
                        const float4 a = *reinterpret_cast<const float4*>(cc1 + 32 * c + 4 * t4);
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
                            const int t = 4 * t4 + e;
                            const int ph = PLANES ? 4 * (t & 7) + (t >> 3) : t;   // column-transposed with planes
                            const float f = __fmul_rn(__int2float_rn(static_cast<int>(r32[ph])), c1a[t]);
                            o[e] = partial ? f : (load_old ? __fmaf_rn(f, as, ov[e]) : __fmul_rn(f, as));
                        }
                        *reinterpret_cast<float4*>(tile + out_offset(rloc, t4)) = make_float4(o[0], o[1], o[2], o[3]);
                    }
                } else {
                // S and T: two halves of 16 TMEM columns each. The columns are column-transposed (TMEM column
                // 16 h + 4 e + i holds output column 8 i + 4 h + e), so half h covers the float4 groups 2 i + h.
#pragma unroll 1
                for (int half = 0; half < 2; ++half) {
                    uint32_t rS[16], rT[16];
                    tmem_ld_32x32b_x16(tmem + lane_base + 32 * c + 16 * half, rS);
                    tmem_ld_32x32b_x16(tmem + lane_base + BN + 32 * c + 16 * half, rT);
                    // the constants of these 16 output columns, while the TMEM loads are in flight
                    float c1a[16], c2a[16];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int t4 = 2 * i + half;   // float4 group of output columns
                        const float4 a = *reinterpret_cast<const float4*>(cc1 + 32 * c + 4 * t4);
                        c1a[4 * i] = a.x; c1a[4 * i + 1] = a.y; c1a[4 * i + 2] = a.z; c1a[4 * i + 3] = a.w;
                        const float4 b = *reinterpret_cast<const float4*>(cc2 + 32 * c + 4 * t4);
                        c2a[4 * i] = b.x; c2a[4 * i + 1] = b.y; c2a[4 * i + 2] = b.z; c2a[4 * i + 3] = b.w;
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
                            const int ph = 4 * e + i;   // its register among the 16
                            const float f = __fmaf_rn(__int2float_rn(static_cast<int>(rT[ph])), c2a[4 * i + e],
                                                      __fmul_rn(__int2float_rn(static_cast<int>(rS[ph])), c1a[4 * i + e]));
                            o[e] = partial ? f : (load_old ? __fmaf_rn(f, as, ov[e]) : __fmul_rn(f, as));
                        }
                        *reinterpret_cast<float4*>(tile + out_offset(rloc, t4)) = make_float4(o[0], o[1], o[2], o[3]);
                    }
                }
                }
                // the chunk is staged: the group's first thread stores it while the group moves on
                fence_proxy_async_smem();
                named_barrier_sync(2 + grp, 128);
                if (quarter == 0 && lane == 0) {
                    tma_store_2d(&tmOut, tile, n0 + 32 * c, out_row);
                    tma_store_commit();
                    if (c == 0) TRACE(241);
                }
            }
        }
        if (threadIdx.x == 0) TRACE(242);
        if (go && quarter == 0 && lane == 0) {
            tma_store_wait_read();   // the staging tiles must stay valid until the stores have read them
            if (threadIdx.x == 0) TRACE(250);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == G::MMAW) tmem_dealloc(tmem, G::TMEM_COLS);
    if (threadIdx.x == 0) TRACE(260);
}

// K > 1024: fold the per-block values f_b of the workspace slices into C in block order, as the reference's
// epilogue does block after block (csrc/blas.c:1354-1366). One thread per four consecutive columns.
__global__ void __launch_bounds__(256) fv_combine_kernel(const float* __restrict__ f, int m_pad, int nblk,
                                                         const float* __restrict__ a_scales, float alpha,
                                                         int beta_zero, float* __restrict__ C, int M, int N,
                                                         int ldc) {
    griddep_launch_dependents();
    griddep_wait();
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int groups = N / 4;
    if (i >= static_cast<size_t>(M) * groups) return;
    const int m = static_cast<int>(i / groups), n = static_cast<int>(i % groups) * 4;
    const float as = __fmul_rn(a_scales[m], alpha);
    float4 c = beta_zero ? make_float4(0.f, 0.f, 0.f, 0.f)
                         : *reinterpret_cast<const float4*>(C + static_cast<size_t>(m) * ldc + n);
    for (int b = 0; b < nblk; ++b) {
        const float4 v = *reinterpret_cast<const float4*>(f + (static_cast<size_t>(b) * m_pad + m) * N + n);
        if (b == 0 && beta_zero) {
            c = make_float4(__fmul_rn(v.x, as), __fmul_rn(v.y, as), __fmul_rn(v.z, as), __fmul_rn(v.w, as));
        } else {
            c = make_float4(__fmaf_rn(v.x, as, c.x), __fmaf_rn(v.y, as, c.y), __fmaf_rn(v.z, as, c.z),
                            __fmaf_rn(v.w, as, c.w));
        }
    }
    *reinterpret_cast<float4*>(C + static_cast<size_t>(m) * ldc + n) = c;
}


template <int BN, int KIND>
static cudaError_t launch(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                          const CUtensorMap& out, const FvGemmParams& p, cudaStream_t stream) {
    using G = Cfg<BN, KIND>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(fv_gemm_kernel<BN, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(G::SMEM_BYTES));
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM, p.ksplit);
    return launch_pdl(fv_gemm_kernel<BN, KIND>, grid, dim3(G::NTHREADS), G::SMEM_BYTES, stream, a, b0, b1, out, p);
}

cudaError_t fv_gemm_launch(int bn, int kind, const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                           const CUtensorMap& out, const FvGemmParams& p, cudaStream_t stream) {
    switch (kind) {
    case KIND_ST:
        if (bn == 64) return launch<64, KIND_ST>(a, b0, b1, out, p, stream);
        if (bn == 128) return launch<128, KIND_ST>(a, b0, b1, out, p, stream);
        break;
    case KIND_CODES:
        if (bn == 64) return launch<64, KIND_CODES>(a, b0, b1, out, p, stream);
        if (bn == 128) return launch<128, KIND_CODES>(a, b0, b1, out, p, stream);
        if (bn == 256) return launch<256, KIND_CODES>(a, b0, b1, out, p, stream);
        break;
    default:
        if (bn == 64) return launch<64, KIND_TABLE>(a, b0, b1, out, p, stream);
        if (bn == 128) return launch<128, KIND_TABLE>(a, b0, b1, out, p, stream);
        if (bn == 256) return launch<256, KIND_TABLE>(a, b0, b1, out, p, stream);
        break;
    }
    return cudaErrorInvalidValue;
}

cudaError_t fv_combine_launch(const float* f, int m_pad, int nblk, const float* a_scales, float alpha, int beta_zero,
                              float* C, int M, int N, int ldc, cudaStream_t stream) {
    const size_t threads = static_cast<size_t>(M) * (N / 4);
    return launch_pdl(fv_combine_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0, stream, f,
                      m_pad, nblk, a_scales, alpha, beta_zero, C, M, N, ldc);
}

}  // namespace p2cu
