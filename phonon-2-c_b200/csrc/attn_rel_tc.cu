// attn_rel_tc.cu - the encoder's relative-position self-attention in one kernel on the tensor cores, for windows of
// up to ATT_MAXT frames: scores, softmax and context per (window, head, 128 queries), the scores never in HBM.
//
// The reference (csrc/encoder.c:471-528, combine_softmax at :425-447) computes per window and head
//     AC = (Q + bias_u) K^T [T x T],  BD = (Q + bias_v) P^T [T x (2T - 1)],
//     S[i][j] = softmax_j((AC[i][j] + BD[i][T - 1 - i + j]) * scale),  out = S V,
// every product in fp32. Here the products run on tcgen05.mma kind::tf32 with every operand in two tf32 parts
// (hi * hi + hi * lo + lo * hi, about the accuracy of an fp32 dot product, tf32_split.cuh), and the softmax runs in
// the same kernel, one query row per thread:
//
//   * The biases enter as rank-one terms: (Q + bias_u) K^T = Q K^T + 1 (K bias_u)^T, and the same for bias_v and
//     the positions, so one copy of Q is the A operand of both products. The loader threads accumulate
//     K_j . bias_u and P_p . bias_v while they prepare the tiles; the softmax threads add them to the scores.
//   * TMA brings the raw fp32 tiles of Q, K and the positions into shared memory in the 64-byte-swizzled K-major
//     layout the MMA reads, and the MMA reads each raw tile as the operand's hi part (the tensor core takes the
//     top 19 bits of an fp32 operand, a truncation to tf32); the loader threads write only lo = x - trunc(x) beside
//     it, at the same offsets. V comes in as [16 keys][128] rows and is transposed to K-major (hi and lo) on the way.
//   * The keys come in chunks of 64. Query i and key j need position T - 1 - i + j, so a chunk of 128 queries and 64
//     keys needs a band of 191 positions; the positional product is computed in pieces of 64 positions (the MMA's
//     N), each piece once, three pieces live per chunk. TMEM (512 columns): two 64-column slots for the chunk's
//     content scores, a ring of four 64-column slots for the position pieces, 128 columns for the context.
//   * The softmax threads read their row's band from TMEM and write the 64 values the row needs into a padded row of
//     shared memory at their shifted place (the relative shift), then add the content scores and both bias terms
//     and scale.
//   * The chunk's probabilities go back into TMEM as two tf32 parts, over the content scores and over the position
//     piece the chunk no longer needs, and the context product reads them from there (A from TMEM).
//   * Online softmax with a lazily moved reference: p = exp(s - m) with m the row's largest score so far, moved (and
//     the context and the running sum rescaled by exp(m_old - m_new)) only when a chunk's largest score exceeds m by
//     more than 16, so that exp(s - m) stays below e^16. Softmax is invariant under the shift, so the result is the
//     reference's up to rounding; the sum and the division by it close the row.
//
// A launch with few query tiles (a window or two) splits each tile's key chunks over up to four CTAs: each keeps its
// own reference, sum and unnormalised context and writes them out; the last CTA of the tile to finish (an atomic count,
// no waiting) merges them in split order, out = sum_s e^(m_s - M) O_s / sum_s e^(m_s - M) l_s with M = max_s m_s.
//
// Warps 0-3: softmax and read-out (TMEM lane = query row); warps 4-7: loader threads (lo parts, V transposed, bias
// terms); warp 8: TMEM owner and MMA issue (converged, one elected lane issuing); warp 9: TMA issue (one lane). The
// MMA order, one chunk of look-ahead:
//     pieces 0, 1 | AC_0, piece 2, [scores 0] | AC_1, piece 3, [scores 1], context 0 | AC_2, piece 4, ... | context n-1
// so the tensor pipe computes chunk c + 1's scores while the softmax threads work on chunk c. Every wait is bounded.
#include <cstdint>
#include <vector>
#include <cuda.h>
#include <cuda_runtime.h>
#include "encoder_ops.h"
#include "gemm.h"
#include "numerics.cuh"
#include "ptx.cuh"
#include "tf32_split.cuh"

namespace p2cu {

namespace {

constexpr int DM = 1024, NHEAD = 8, HD = 128, LDQ = 3 * DM;
constexpr int QT = ATT_TC_QT;   // queries per CTA: the MMA's M, one TMEM lane each
constexpr int KC = 64;          // keys per chunk and positions per piece: the score products' N
constexpr int NST = 4;          // stages
// A score stage (16 of the head's 128 dimensions): raw Q [128 rows] | Q lo | raw B1 [64 rows] | B1 lo | raw B2 | B2 lo,
// every tile K-major with 64-byte rows and the 64-byte swizzle. B1 / B2: keys and the next position piece, or
// position pieces 0 and 1. A context stage (16 keys): raw V [16][128] | V^T hi [128 rows] | V^T lo.
constexpr uint32_t RAW_Q = 0, LO_Q = 8192, RAW_B1 = 16384, LO_B1 = 20480, RAW_B2 = 24576, LO_B2 = 28672;
constexpr uint32_t RAW_V = 0, VT_HI = 8192, VT_LO = 16384;
constexpr uint32_t STAGE = 32768;
constexpr uint32_t SCORE_TX = 8192 + 4096 + 4096, CTX_TX = 8192;   // TMA bytes per stage
constexpr int SROW = KC + 1;                                         // shifted-band row stride in floats (odd)
constexpr uint32_t OFF_SH = NST * STAGE;
constexpr uint32_t OFF_BIAS = OFF_SH + QT * SROW * 4;   // bias_u, bias_v of the head: 2 x 128 floats
constexpr uint32_t OFF_CB = OFF_BIAS + 2 * HD * 4;      // K_j . bias_u of a chunk's keys: 2 slots x 64 floats
constexpr uint32_t OFF_DB = OFF_CB + 2 * KC * 4;        // P_p . bias_v of a piece: 4 slots x 64 floats
constexpr uint32_t OFF_BAR = OFF_DB + 4 * KC * 4;
constexpr uint32_t SMEM_BYTES = 1024 + OFF_BAR + 256;
constexpr int NTHREADS = 320;
constexpr uint32_t COL_A = 0, COL_B = 128, COL_O = 384, TMEM_COLS = 512;
constexpr float SHIFT_SLACK = 16.f;
constexpr uint32_t IDESC_S = idesc_tf32(QT, KC, false);   // scores: 128 queries x 64 keys / positions
constexpr uint32_t IDESC_O = idesc_tf32(QT, HD, false);   // context: 128 queries x 128 head dimensions

static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
static_assert(OFF_SH % 16 == 0 && (32 * SROW * 4) % 16 == 0, "read-out blocks are 16-byte aligned");
static_assert(OFF_BAR % 8 == 0, "mbarriers are 8-byte aligned");

enum { ST_POS = 0, ST_SCORE = 1, ST_CTX = 2 };

// The four tensor maps of a launch: Q (boxes of 16 x 128 rows), K (16 x 64), V (128 x 16, no swizzle) over the qkv
// rows, and the positions P (16 x 64).
struct AttnMaps {
    CUtensorMap q, k, v, p;
};

// Stage st of a CTA with nch key chunks: 8 K steps of pieces 0 and 1; 8 of chunk 0's scores (with piece 2); then per
// chunk c >= 1 its 8 score steps (with piece c + 2) and the 4 context steps of chunk c - 1; last, the 4 context steps
// of chunk nch - 1. 8 + 12 nch stages.
__device__ __forceinline__ void stage_of(int st, int nch, int& kind, int& c, int& kk) {
    if (st < 8) { kind = ST_POS; c = 0; kk = st; return; }
    int u = st - 8;
    if (u < 8) { kind = ST_SCORE; c = 0; kk = u; return; }
    u -= 8;
    const int b = u / 12, o = u % 12;
    if (b + 1 < nch) {
        if (o < 8) { kind = ST_SCORE; c = b + 1; kk = o; }
        else { kind = ST_CTX; c = b; kk = o - 8; }
    } else {
        kind = ST_CTX; c = nch - 1; kk = o;
    }
}

// x minus its truncation to tf32 (exact in fp32): what the tensor core drops when it reads x as a tf32 operand.
__device__ __forceinline__ float4 lo4(float4 x) {
    auto lo = [](float v) { return __fsub_rn(v, __uint_as_float(__float_as_uint(v) & 0xFFFFE000u)); };
    return make_float4(lo(x.x), lo(x.y), lo(x.z), lo(x.w));
}

__device__ __forceinline__ float dot4(float4 x, const float* b) {
    float p = __fmul_rn(x.x, b[0]);
    p = __fmaf_rn(x.y, b[1], p);
    p = __fmaf_rn(x.z, b[2], p);
    return __fmaf_rn(x.w, b[3], p);
}

__global__ void __launch_bounds__(NTHREADS, 1)
attn_rel_tc_kernel(const __grid_constant__ AttnMaps maps, const float* __restrict__ bias_u,
                   const float* __restrict__ bias_v, const int* __restrict__ row_off,
                   const AttnTile* __restrict__ tiles, int Tmax, float scale, float* __restrict__ attn,
                   float* __restrict__ part_o, float2* __restrict__ part_ml, int* __restrict__ counters,
                   uint32_t* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* tfull = reinterpret_cast<uint64_t*>(smem + OFF_BAR);   // the stage's TMA bytes have landed
    uint64_t* full = tfull + NST;                                     // the stage's lo parts are written (128)
    uint64_t* empty = full + NST;                                     // the MMAs are done with the stage
    // Per-chunk barriers in pairs, chunk c on [c & 1] in phase c >> 1: no waiter can then fall two phases behind.
    uint64_t* sready = empty + NST;   // chunk c's scores are in TMEM
    uint64_t* pready = sready + 2;    // chunk c's probabilities are in TMEM (128 arrivals)
    uint64_t* pvdone = pready + 2;    // chunk c's context product has completed
    uint64_t* bready = pvdone + 2;    // chunk c's key bias terms and its pieces' position bias terms are written (128)
    uint64_t* ofull = bready + 2;     // the last context product has completed
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(ofull + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    float* bias_s = reinterpret_cast<float*>(smem + OFF_BIAS);
    float* cbuf = reinterpret_cast<float*>(smem + OFF_CB);
    float* dbuf = reinterpret_cast<float*>(smem + OFF_DB);

    const AttnTile tile = tiles[blockIdx.x];
    const int w = tile.w, q0 = tile.q0, h = blockIdx.y;
    const int r0 = row_off[w], T = row_off[w + 1] - r0;
    // this CTA's key chunks c0 + u, u < nch (every chunk index below is relative to c0 but for the keys' places)
    const int c0 = tile.c0, nch = tile.c1 - tile.c0;
    const int nstages = 8 + 12 * nch;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&tfull[s], 1);
            mbar_init(&full[s], 128);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sready[b], 1);
            mbar_init(&pready[b], 128);
            mbar_init(&pvdone[b], 1);
            mbar_init(&bready[b], 128);
        }
        mbar_init(ofull, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 8) {
        tmem_alloc(tmem_holder, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 9) {
        // ---------------- TMA issue ----------------
        if (lane == 0) {
            // the row of P holding position 0 of this CTA's piece 0 (may be < 0: zeros), and its first key's row
            const int prow0 = Tmax - QT - q0 + KC * c0, krow0 = r0 + KC * c0;
            for (int st = 0; st < nstages; ++st) {
                const int s = st % NST;
                if (!mbar_wait(&empty[s], ((st / NST) & 1) ^ 1, DEV_TIMEOUT_EMPTY, err, abort_flag)) break;
                int kind, c, kk;
                stage_of(st, nch, kind, c, kk);
                uint8_t* B = smem + s * STAGE;
                if (kind == ST_CTX) {
                    mbar_arrive_expect_tx(&tfull[s], CTX_TX);
                    tma_load_2d(B + RAW_V, &maps.v, &tfull[s], 2 * DM + h * HD, krow0 + KC * c + 16 * kk);
                } else {
                    const int x = h * HD + 16 * kk;
                    mbar_arrive_expect_tx(&tfull[s], SCORE_TX);
                    tma_load_2d(B + RAW_Q, &maps.q, &tfull[s], x, r0 + q0);
                    if (kind == ST_POS) {
                        tma_load_2d(B + RAW_B1, &maps.p, &tfull[s], x, prow0);
                        tma_load_2d(B + RAW_B2, &maps.p, &tfull[s], x, prow0 + KC);
                    } else {
                        tma_load_2d(B + RAW_B1, &maps.k, &tfull[s], DM + x, krow0 + KC * c);
                        tma_load_2d(B + RAW_B2, &maps.p, &tfull[s], x, prow0 + KC * (c + 2));
                    }
                }
            }
        }
    } else if (warp >= 4 && warp < 8) {
        // ---------------- loader threads: lo parts, V^T, bias terms ----------------
        const int t = threadIdx.x - 128;
        bias_s[t] = bias_u[h * HD + t];
        bias_s[HD + t] = bias_v[h * HD + t];
        named_barrier_sync(1, 128);
        float acc1[2] = {0.f, 0.f}, acc2[2] = {0.f, 0.f};   // this thread's share of two rows' bias dot products
        for (int st = 0; st < nstages; ++st) {
            const int s = st % NST;
            if (!warp_wait(&tfull[s], (st / NST) & 1, DEV_TIMEOUT_FULL, err, abort_flag)) break;
            int kind, c, kk;
            stage_of(st, nch, kind, c, kk);
            uint8_t* B = smem + s * STAGE;
            if (kind == ST_CTX) {   // V^T: row n of the head dimension, keys 4 c4 .. + 3 of the 16
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int e = t + 128 * i, n = e & 127, c4 = e >> 7;
                    const float* rv = reinterpret_cast<const float*>(B + RAW_V) + 4 * c4 * HD + n;
                    store_split(B + VT_HI, B + VT_LO, kmaj_off(n, c4),
                                make_float4(rv[0], rv[HD], rv[2 * HD], rv[3 * HD]));
                }
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) {   // Q: the lo part beside each raw 16-byte chunk
                    const uint32_t X = (t + 128 * i) * 16;
                    *reinterpret_cast<float4*>(B + LO_Q + X) = lo4(*reinterpret_cast<const float4*>(B + RAW_Q + X));
                }
                const float* b1 = bias_s + (kind == ST_POS ? HD : 0);   // keys take bias_u, positions bias_v
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const int e = t + 128 * i, row = e >> 2;
                    const uint32_t X = e * 16;
                    // the 16-byte chunk's dimensions: its place in the row before the 64-byte swizzle
                    const int dim = 16 * kk + 4 * ((e & 3) ^ ((row >> 1) & 3));
                    const float4 x1 = *reinterpret_cast<const float4*>(B + RAW_B1 + X);
                    const float4 x2 = *reinterpret_cast<const float4*>(B + RAW_B2 + X);
                    *reinterpret_cast<float4*>(B + LO_B1 + X) = lo4(x1);
                    *reinterpret_cast<float4*>(B + LO_B2 + X) = lo4(x2);
                    float p1 = dot4(x1, b1 + dim), p2 = dot4(x2, bias_s + HD + dim);
                    p1 = __fadd_rn(p1, __shfl_xor_sync(0xffffffffu, p1, 1));   // the row's four 16-byte chunks
                    p2 = __fadd_rn(p2, __shfl_xor_sync(0xffffffffu, p2, 1));
                    p1 = __fadd_rn(p1, __shfl_xor_sync(0xffffffffu, p1, 2));
                    p2 = __fadd_rn(p2, __shfl_xor_sync(0xffffffffu, p2, 2));
                    acc1[i] = __fadd_rn(acc1[i], p1);
                    acc2[i] = __fadd_rn(acc2[i], p2);
                }
                if (kk == 7) {
                    if ((t & 3) == 0) {
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            const int row = (t + 128 * i) >> 2;
                            if (kind == ST_POS) {
                                dbuf[row] = acc1[i];
                                dbuf[KC + row] = acc2[i];
                            } else {
                                cbuf[KC * (c & 1) + row] = acc1[i];
                                dbuf[KC * ((c + 2) & 3) + row] = acc2[i];
                            }
                        }
                    }
                    acc1[0] = acc1[1] = acc2[0] = acc2[1] = 0.f;
                }
            }
            fence_proxy_async_smem();
            mbar_arrive(&full[s]);
            if (kind == ST_SCORE && kk == 7) mbar_arrive(&bready[c & 1]);
        }
    } else if (warp == 8) {
        // ---------------- MMA issue ----------------
        const uint32_t lead = elect_one();
        for (int st = 0; st < nstages; ++st) {
            int kind, c, kk;
            stage_of(st, nch, kind, c, kk);
            if (kind == ST_CTX && kk == 0) {
                if (!warp_wait_all(&pready[c & 1], (c >> 1) & 1, DEV_TIMEOUT_READY, err, abort_flag)) break;
                tc_fence_after();
            }
            const int s = st % NST;
            if (!warp_wait_all(&full[s], (st / NST) & 1, DEV_TIMEOUT_FULL, err, abort_flag)) break;
            tc_fence_after();
            const uint32_t base = smem_u32(smem + s * STAGE);
            if (kind == ST_CTX) {
                const uint32_t a_hi = tmem + COL_A + KC * (c & 1), a_lo = tmem + COL_B + KC * (c & 3);
#pragma unroll
                for (int ks = 0; ks < 2; ++ks) {
                    const int k8 = 2 * kk + ks;
                    const uint64_t bh = smem_desc(base + VT_HI + ks * 32, 16, 512, SWZ_64B);
                    const uint64_t bl = smem_desc(base + VT_LO + ks * 32, 16, 512, SWZ_64B);
                    mma_tf32_ts_lead(lead, tmem + COL_O, a_hi + 8 * k8, bh, IDESC_O, (c > 0 || k8 > 0) ? 1u : 0u);
                    mma_tf32_ts_lead(lead, tmem + COL_O, a_hi + 8 * k8, bl, IDESC_O, 1u);
                    mma_tf32_ts_lead(lead, tmem + COL_O, a_lo + 8 * k8, bh, IDESC_O, 1u);
                }
            } else {
                // Q against B1 into d1 and against B2 into d2
                const uint32_t d1 = kind == ST_POS ? COL_B : COL_A + KC * (c & 1);
                const uint32_t d2 = kind == ST_POS ? COL_B + KC : COL_B + KC * ((c + 2) & 3);
#pragma unroll
                for (int ks = 0; ks < 2; ++ks) {
                    const uint32_t acc = (kk > 0 || ks > 0) ? 1u : 0u;
                    const uint64_t ah = smem_desc(base + RAW_Q + ks * 32, 16, 512, SWZ_64B);
                    const uint64_t al = smem_desc(base + LO_Q + ks * 32, 16, 512, SWZ_64B);
                    const uint64_t b1h = smem_desc(base + RAW_B1 + ks * 32, 16, 512, SWZ_64B);
                    const uint64_t b1l = smem_desc(base + LO_B1 + ks * 32, 16, 512, SWZ_64B);
                    const uint64_t b2h = smem_desc(base + RAW_B2 + ks * 32, 16, 512, SWZ_64B);
                    const uint64_t b2l = smem_desc(base + LO_B2 + ks * 32, 16, 512, SWZ_64B);
                    mma_tf32_lead(lead, tmem + d1, ah, b1h, IDESC_S, acc);
                    mma_tf32_lead(lead, tmem + d1, ah, b1l, IDESC_S, 1u);
                    mma_tf32_lead(lead, tmem + d1, al, b1h, IDESC_S, 1u);
                    mma_tf32_lead(lead, tmem + d2, ah, b2h, IDESC_S, acc);
                    mma_tf32_lead(lead, tmem + d2, ah, b2l, IDESC_S, 1u);
                    mma_tf32_lead(lead, tmem + d2, al, b2h, IDESC_S, 1u);
                }
            }
            mma_commit_lead(lead, &empty[s]);
            if (kind == ST_SCORE && kk == 7) mma_commit_lead(lead, &sready[c & 1]);
            if (kind == ST_CTX && kk == 3) {
                mma_commit_lead(lead, &pvdone[c & 1]);
                if (c == nch - 1) mma_commit_lead(lead, ofull);
            }
        }
    } else if (warp < 4) {
        // ---------------- softmax: TMEM lane = query row r ----------------
        const int r = threadIdx.x;
        const uint32_t lanes = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        float* shr = reinterpret_cast<float*>(smem + OFF_SH) + r * SROW;
        float m = 0.f, l = 0.f;
        bool ok = true;
        for (int c = 0; c < nch && ok; ++c) {
            if (!warp_wait(&sready[c & 1], (c >> 1) & 1, DEV_TIMEOUT_ACC, err, abort_flag)) { ok = false; break; }
            tc_fence_after();
            {   // the band: offsets o = 127 - r + jj (jj < 64) of the pieces c, c + 1, c + 2, in the 32-column
                // groups 3 - warp .. 5 - warp of the three pieces
                uint32_t v[3][32];
#pragma unroll
                for (int gi = 0; gi < 3; ++gi) {
                    const int g = 3 - warp + gi;
                    tmem_ld_32x32b_x32(lanes + COL_B + KC * ((c + (g >> 1)) & 3) + 32 * (g & 1), v[gi]);
                }
                tmem_wait_ld();
#pragma unroll
                for (int gi = 0; gi < 3; ++gi) {
#pragma unroll
                    for (int x = 0; x < 32; ++x) {
                        const int jj = 32 * (3 - warp + gi) + x - 127 + r;
                        if (static_cast<unsigned>(jj) < static_cast<unsigned>(KC)) shr[jj] = __uint_as_float(v[gi][x]);
                    }
                }
            }
            uint32_t a[2][32];
            tmem_ld_32x32b_x32(lanes + COL_A + KC * (c & 1), a[0]);
            tmem_ld_32x32b_x32(lanes + COL_A + KC * (c & 1) + 32, a[1]);
            if (!warp_wait(&bready[c & 1], (c >> 1) & 1, DEV_TIMEOUT_ACC, err, abort_flag)) { ok = false; break; }
            tmem_wait_ld();
            const float* cb = cbuf + KC * (c & 1);
            float s[KC];
            float mx = -INFINITY;
#pragma unroll
            for (int jj = 0; jj < KC; ++jj) {
                const int o = 127 - r + jj;   // the band offset: piece c + o / 64, column o % 64
                const float bd = __fadd_rn(shr[jj], dbuf[KC * ((c + (o >> 6)) & 3) + (o & 63)]);
                const float ac = __fadd_rn(__uint_as_float(a[jj >> 5][jj & 31]), cb[jj]);
                const float v = KC * (c0 + c) + jj < T ? __fmul_rn(__fadd_rn(ac, bd), scale) : -INFINITY;
                s[jj] = v;
                mx = fmaxf(mx, v);
            }
            bool move = false;
            if (c == 0) m = mx;   // key 0 is in every window
            else move = mx > m + SHIFT_SLACK;
            if (__any_sync(0xffffffffu, move)) {
                // the context so far (chunks < c) is rescaled once chunk c - 1's product has completed
                if (!warp_wait(&pvdone[(c - 1) & 1], ((c - 1) >> 1) & 1, DEV_TIMEOUT_ACC, err, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const float alpha = move ? exp_poly(__fsub_rn(m, mx)) : 1.f;
                if (move) {
                    l = __fmul_rn(l, alpha);
                    m = mx;
                }
#pragma unroll
                for (int q = 0; q < HD / 32; ++q) {
                    uint32_t o[32];
                    tmem_ld_32x32b_x32(lanes + COL_O + 32 * q, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int g8 = 0; g8 < 4; ++g8) {
                        uint32_t y[8];
#pragma unroll
                        for (int x = 0; x < 8; ++x)
                            y[x] = __float_as_uint(__fmul_rn(__uint_as_float(o[8 * g8 + x]), alpha));
                        tmem_st_32x32b_x8(lanes + COL_O + 32 * q + 8 * g8, y);
                    }
                }
            }
#pragma unroll
            for (int g8 = 0; g8 < KC / 8; ++g8) {
                uint32_t ph[8], pl[8];
#pragma unroll
                for (int x = 0; x < 8; ++x) {
                    const float sv = s[8 * g8 + x];
                    const float p = sv == -INFINITY ? 0.f : exp_poly(__fsub_rn(sv, m));
                    l = __fadd_rn(l, p);
                    float hi, lo;
                    tf32_split(p, hi, lo);
                    ph[x] = __float_as_uint(hi);
                    pl[x] = __float_as_uint(lo);
                }
                tmem_st_32x32b_x8(lanes + COL_A + KC * (c & 1) + 8 * g8, ph);   // over the content scores
                tmem_st_32x32b_x8(lanes + COL_B + KC * (c & 3) + 8 * g8, pl);   // over piece c
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&pready[c & 1]);
        }
        // ---------------- read-out: out = context / sum, or this split's part and the merge ----------------
        if (ok && warp_wait(ofull, 0, DEV_TIMEOUT_ACC, err, abort_flag, true)) {
            tc_fence_after();
            if (tile.nsplit == 1) {
                const float inv = __fdiv_rn(1.0f, l);
                uint8_t* blk = smem + OFF_SH + warp * 32 * SROW * 4;   // this warp's band rows, free now
                float* out0 = attn + static_cast<size_t>(r0 + q0) * DM + h * HD;
#pragma unroll 1
                for (int q = 0; q < HD / 32; ++q) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(lanes + COL_O + 32 * q, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int c4 = 0; c4 < 8; ++c4)   // row `lane`, columns 4 c4 .. + 3, at 16-byte slot c4 ^ (lane % 8)
                        *reinterpret_cast<float4*>(blk + lane * 128 + ((c4 ^ (lane & 7)) << 4)) =
                            make_float4(__fmul_rn(__uint_as_float(v[4 * c4]), inv),
                                        __fmul_rn(__uint_as_float(v[4 * c4 + 1]), inv),
                                        __fmul_rn(__uint_as_float(v[4 * c4 + 2]), inv),
                                        __fmul_rn(__uint_as_float(v[4 * c4 + 3]), inv));
                    __syncwarp();
                    const int c4 = lane & 7;
#pragma unroll
                    for (int it = 0; it < 8; ++it) {   // rows 4 it .. 4 it + 3, eight lanes (128 bytes) per row
                        const int rr = 4 * it + (lane >> 3), row = warp * 32 + rr;
                        const float4 y = *reinterpret_cast<const float4*>(blk + rr * 128 + ((c4 ^ (rr & 7)) << 4));
                        if (q0 + row < T)
                            *reinterpret_cast<float4*>(out0 + static_cast<size_t>(row) * DM + 32 * q + 4 * c4) = y;
                    }
                    __syncwarp();
                }
            } else {
                // this split's row: reference, sum and unnormalised context
                const size_t part = (static_cast<size_t>(blockIdx.x) * NHEAD + h) * QT + r;
                float4* po = reinterpret_cast<float4*>(part_o + part * HD);
#pragma unroll 1
                for (int q = 0; q < HD / 32; ++q) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(lanes + COL_O + 32 * q, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int c4 = 0; c4 < 8; ++c4)
                        po[8 * q + c4] = make_float4(__uint_as_float(v[4 * c4]), __uint_as_float(v[4 * c4 + 1]),
                                                     __uint_as_float(v[4 * c4 + 2]), __uint_as_float(v[4 * c4 + 3]));
                }
                part_ml[part] = make_float2(m, l);
                __threadfence();
                named_barrier_sync(2, 128);   // the four softmax warps' parts are out
                int* last_s = reinterpret_cast<int*>(tmem_holder + 2);
                if (r == 0) {
                    int* cnt = counters + static_cast<size_t>(tile.group) * NHEAD + h;
                    const int prev = atomicAdd(cnt, 1);
                    *last_s = prev == tile.nsplit - 1;
                    if (*last_s) *cnt = 0;   // ready for the next launch (the launches of a stream run in order)
                }
                named_barrier_sync(2, 128);
                if (*last_s) {
                    __threadfence();
                    // every split's row r, in split order (the same result whichever CTA merges)
                    const size_t stride = static_cast<size_t>(NHEAD) * QT;   // one tile's rows in the parts
                    const size_t base = (static_cast<size_t>(tile.first) * NHEAD + h) * QT + r;
                    float mm = -INFINITY;
                    for (int sp = 0; sp < tile.nsplit; ++sp) mm = fmaxf(mm, __ldcg(&part_ml[base + sp * stride]).x);
                    float ll = 0.f;
                    for (int sp = 0; sp < tile.nsplit; ++sp) {
                        const float2 ml = __ldcg(&part_ml[base + sp * stride]);
                        ll = __fmaf_rn(exp_poly(__fsub_rn(ml.x, mm)), ml.y, ll);
                    }
                    const float inv = __fdiv_rn(1.0f, ll);
                    float* orow = attn + static_cast<size_t>(r0 + q0 + r) * DM + h * HD;
#pragma unroll 1
                    for (int c4 = 0; c4 < HD / 4; ++c4) {
                        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                        for (int sp = 0; sp < tile.nsplit; ++sp) {
                            const float a = exp_poly(__fsub_rn(__ldcg(&part_ml[base + sp * stride]).x, mm));
                            const float4 o = __ldcg(reinterpret_cast<const float4*>(part_o + (base + sp * stride) *
                                                                                    HD) + c4);
                            acc = make_float4(__fmaf_rn(a, o.x, acc.x), __fmaf_rn(a, o.y, acc.y),
                                              __fmaf_rn(a, o.z, acc.z), __fmaf_rn(a, o.w, acc.w));
                        }
                        if (q0 + r < T)
                            *reinterpret_cast<float4*>(orow + 4 * c4) =
                                make_float4(__fmul_rn(acc.x, inv), __fmul_rn(acc.y, inv), __fmul_rn(acc.z, inv),
                                            __fmul_rn(acc.w, inv));
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace

int attn_rel_tc_plan(const int* T, int n_win, int sms, std::vector<AttnTile>& tiles, int* n_groups) {
    int base = 0;
    for (int w = 0; w < n_win; ++w) base += (T[w] + QT - 1) / QT;
    // split the key chunks when the tiles alone give fewer than half the SMs a CTA
    int want = base * NHEAD * 2 <= sms ? sms / (base * NHEAD) : 1;
    if (want > 4) want = 4;
    tiles.clear();
    int g = 0;
    for (int w = 0; w < n_win; ++w)
        for (int q0 = 0; q0 < T[w]; q0 += QT, ++g) {
            const int nch = (T[w] + KC - 1) / KC;
            const int ns = want < nch ? want : nch;
            const int first = static_cast<int>(tiles.size());
            for (int sp = 0; sp < ns; ++sp) {
                AttnTile t;
                t.w = w; t.q0 = q0;
                t.c0 = sp * nch / ns; t.c1 = (sp + 1) * nch / ns;
                t.split = sp; t.nsplit = ns; t.group = g; t.first = first;
                tiles.push_back(t);
            }
        }
    *n_groups = g;
    return static_cast<int>(tiles.size());
}

size_t attn_rel_tc_part_bytes(int n_tiles) { return static_cast<size_t>(n_tiles) * NHEAD * QT * (HD * 4 + 8); }

int attn_rel_tc_launch(const float* qkv, int rows, const float* P, const float* bias_u, const float* bias_v,
                       const int* row_off, const AttnTile* tiles, int n_tiles, int Tmax, float scale, float* attn,
                       void* parts, int* counters, uint32_t* err, cudaStream_t s) {
    if (n_tiles <= 0) return P2CU_OK;
    if (Tmax > ATT_MAXT || Tmax <= 0 || rows <= 0)
        return fail_fmt(P2CU_EINVAL, "attention: Tmax = %d, rows = %d", Tmax, rows);
    if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(P) | reinterpret_cast<uintptr_t>(attn)) & 15)
        return fail_fmt(P2CU_EINVAL, "attention: qkv, P and attn must be 16-byte aligned");
    AttnMaps maps;
    const uint64_t qstride = static_cast<uint64_t>(LDQ) * 4, pstride = static_cast<uint64_t>(DM) * 4;
    if (int rc = make_tile_map(&maps.q, qkv, 4, LDQ, rows, qstride, 16, QT, 64, "attention Q")) return rc;
    if (int rc = make_tile_map(&maps.k, qkv, 4, LDQ, rows, qstride, 16, KC, 64, "attention K")) return rc;
    if (int rc = make_tile_map(&maps.v, qkv, 4, LDQ, rows, qstride, HD, 16, 0, "attention V")) return rc;
    if (int rc = make_tile_map(&maps.p, P, 4, DM, 2 * Tmax - 1, pstride, 16, KC, 64, "attention P")) return rc;
    cudaError_t e = cudaFuncSetAttribute(attn_rel_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return cuda_error(e, "attention");
    float* part_o = static_cast<float*>(parts);
    float2* part_ml = parts ? reinterpret_cast<float2*>(part_o + static_cast<size_t>(n_tiles) * NHEAD * QT * HD)
                            : nullptr;
    attn_rel_tc_kernel<<<dim3(n_tiles, NHEAD), NTHREADS, SMEM_BYTES, s>>>(maps, bias_u, bias_v, row_off, tiles, Tmax,
                                                                         scale, attn, part_o, part_ml, counters, err);
    e = cudaGetLastError();
    return e == cudaSuccess ? P2CU_OK : cuda_error(e, "attention");
}

}  // namespace p2cu
