// decoder.cu - greedy TDT decoding on the device for a batch of windows (csrc/decoder.c of phonon-2-c).
//
// One cooperative launch runs the whole decode of every window: the loop of csrc/decoder.c:100-141 (joint network on
// the current frame, argmax over the 8193 token logits and over the 5 duration logits, the blank / max-symbols rules,
// one prediction-network step after each emitted token) for all windows in lockstep, one loop iteration per step of
// the slowest window. Each CTA owns a slice of the joint head's 8198 rows, kept in shared memory for the whole decode
// (one CTA per SM, the 21 MB head spread over them), a slice of the LSTM's hidden units (the four gate rows of each)
// and the same slice of the projector's rows. An iteration:
//   J   logits of every live window for the CTA's head rows; the CTA's best token row per window -> cand
//   --- grid barrier
//   A   every CTA reduces the candidates and takes the same decisions, so the frame pointers, symbol counts and token
//       counts live in each CTA's shared memory; CTA 0 records the tokens
//   if a live window emitted:  L0 --- L1 --- P --- (LSTM layers and projector of those windows, grid barriers between)
// The candidates and duration logits are double-buffered by iteration, so an iteration in which no window emitted
// needs only the one barrier.
//
// Dot products follow the reference's order exactly (csrc/tensor_ops.c:66-96, AVX2: 16 lanes in two 8-wide
// accumulators, added, then the horizontal-sum tree), so the logits and gate sums are those of the reference; the LSTM
// cell's expf / tanhf are CUDA's, which agree with the host's vector math library to an ulp or two. Greedy token ids
// are compared for equality.
//
// Grid barriers wait with a time bound: a barrier that does not complete records an error code and every CTA returns.
#include <cstdint>
#include <cuda_runtime.h>
#include "decoder.h"
#include "ptx.cuh"

namespace p2cu {

namespace {

constexpr int HD = 640;               // hidden, embedding and joint width
constexpr int HDP = 656;              // padded shared-memory row: the two 16-lane halves of a warp hit other banks
constexpr int NLOG = 8198;            // 8193 tokens + 5 durations
constexpr int NVOCAB = 8193, BLANK = 8192, NDUR = 5;
constexpr int THREADS = 512, WARPS = THREADS / 32, GROUPS = THREADS / 16;
constexpr int WG = 16;                // windows whose joint input (or projector input) is staged at a time
constexpr int WL = 8;                 // windows whose LSTM input (x and h rows) is staged at a time
constexpr int XTS = 20;               // staged inputs are transposed, [640][XTS]: 16 windows and 4 floats of padding,
                                      // so 8 lanes' 16-byte loads of 8 consecutive rows hit disjoint banks
constexpr int MAXW = 512;             // windows per launch
constexpr int MAXU = GROUPS / 4;      // hidden units a CTA can own: four gate rows each, one group per row
constexpr int NO_ROW = 0x7fffffff;
constexpr int STAGE_BATCH = 2;        // float4 loads per thread in flight while staging
constexpr int CAND_PER_LANE = 5;      // candidate loads a lane has in flight (148 CTAs: one round)
constexpr uint32_t DEC_TIMEOUT_BARRIER = 20, DEC_TOKEN_OVERFLOW = 21, DEC_ITER_LIMIT = 22;
constexpr unsigned long long BARRIER_NS = 2000000000ull;   // two seconds

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// The reduction of csrc/tensor_ops.c:182-190 (acc0 + acc1, then the horizontal-sum tree) for N dot products at once
// over the 16 lanes of a group (one half of a warp), lane j holding the FMA chain over i = j, j + 16, ... of each.
// The tree adds lanes (j, j + 8), then (j, j + 4), (j, j + 2), (j, j + 1); here each step pairs the same lanes, and
// while a lane holds two or more values it keeps one half of them and sends the other to its partner, so N sums take
// N/2 + N/4 + ... shuffles instead of 4 N. The sums are those of the tree, addition being commutative. On return
// lane j holds max(N / 16, 1) results in v[0..): those of dot products tree16_base<N>(j) + a. The shuffles name only
// the group's lanes: the two halves of a warp may be on different rows (or one of them on none).
template <int M, int N, int O>
__device__ __forceinline__ void tree16(float (&v)[M], unsigned mask, int j) {
    if constexpr (N >= 2) {
        const bool up = (j & O) != 0;
#pragma unroll
        for (int a = 0; a < N / 2; ++a) {
            const float send = up ? v[a] : v[a + N / 2];
            const float keep = up ? v[a + N / 2] : v[a];
            v[a] = __fadd_rn(keep, __shfl_xor_sync(mask, send, O, 16));
        }
        if constexpr (O > 1) tree16<M, N / 2, O / 2>(v, mask, j);
    } else {
        v[0] = __fadd_rn(v[0], __shfl_xor_sync(mask, v[0], O, 16));
        if constexpr (O > 1) tree16<M, 1, O / 2>(v, mask, j);
    }
}

template <int N>
__device__ __forceinline__ int tree16_base(int j) {
    int b = 0, n = N;
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1)
        if (n >= 2) {
            if (j & o) b += n / 2;
            n /= 2;
        }
    return b;
}

__device__ __forceinline__ unsigned group_mask() { return (threadIdx.x & 16) ? 0xFFFF0000u : 0x0000FFFFu; }

// Joint logits for the CTA's head rows (shared memory, rows HDP apart) and up to 4 NQ windows staged transposed in
// xt: group g takes rows g and g + GROUPS (then g + 2 GROUPS, ...), each lane the chains over i = j + 16 k of both
// rows for every window, one 16-byte load per 4 windows. out[row * ostride + s] = dot + bias[row].
template <int NQ>
__device__ __forceinline__ void joint_rows(const float* head_s, const float* xt, int nrows, int nw, int grp, int j,
                                           const float* bias, float* out, int ostride) {
    constexpr int NW = 4 * NQ, NA = 2 * NW;
    const unsigned mask = group_mask();
    for (int r = grp; r < nrows; r += 2 * GROUPS) {
        const int r2 = r + GROUPS;
        const float* ha = head_s + r * HDP;
        const float* hb = head_s + (r2 < nrows ? r2 : r) * HDP;
        float acc[NA];
#pragma unroll
        for (int a = 0; a < NA; ++a) acc[a] = 0.f;
#pragma unroll 4
        for (int i = j; i < HD; i += 16) {
            const float a0 = ha[i], a1 = hb[i];
            const float4* x = reinterpret_cast<const float4*>(xt + i * XTS);
#pragma unroll
            for (int q = 0; q < NQ; ++q) {
                const float4 xv = x[q];
                acc[4 * q + 0] = __fmaf_rn(a0, xv.x, acc[4 * q + 0]);
                acc[4 * q + 1] = __fmaf_rn(a0, xv.y, acc[4 * q + 1]);
                acc[4 * q + 2] = __fmaf_rn(a0, xv.z, acc[4 * q + 2]);
                acc[4 * q + 3] = __fmaf_rn(a0, xv.w, acc[4 * q + 3]);
                acc[NW + 4 * q + 0] = __fmaf_rn(a1, xv.x, acc[NW + 4 * q + 0]);
                acc[NW + 4 * q + 1] = __fmaf_rn(a1, xv.y, acc[NW + 4 * q + 1]);
                acc[NW + 4 * q + 2] = __fmaf_rn(a1, xv.z, acc[NW + 4 * q + 2]);
                acc[NW + 4 * q + 3] = __fmaf_rn(a1, xv.w, acc[NW + 4 * q + 3]);
            }
        }
        tree16<NA, NA, 8>(acc, mask, j);
        constexpr int R = NA >= 16 ? NA / 16 : 1;
        if (NA >= 16 || (j & (16 / NA - 1)) == 0) {
            const int base = tree16_base<NA>(j);
#pragma unroll
            for (int a = 0; a < R; ++a) {
                const int idx = base + a, row = idx < NW ? r : r2, s = idx % NW;
                if (row < nrows && s < nw) out[row * ostride + s] = __fadd_rn(acc[a], bias[row]);
            }
        }
    }
}

// The dot products of one 640-float global row w with 16 vectors staged transposed in xt (columns 0-15), by one group:
// lane j returns the dot product with column j. The row is read 20 floats per lane at a time, all loads in flight.
__device__ __forceinline__ float row_dot16(const float* __restrict__ w, const float* xt, int j) {
    float acc[16];
#pragma unroll
    for (int a = 0; a < 16; ++a) acc[a] = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        float wv[20];
#pragma unroll
        for (int k = 0; k < 20; ++k) wv[k] = w[j + 16 * (20 * h + k)];
#pragma unroll
        for (int k = 0; k < 20; ++k) {
            const float4* x = reinterpret_cast<const float4*>(xt + (j + 16 * (20 * h + k)) * XTS);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 xv = x[q];
                acc[4 * q + 0] = __fmaf_rn(wv[k], xv.x, acc[4 * q + 0]);
                acc[4 * q + 1] = __fmaf_rn(wv[k], xv.y, acc[4 * q + 1]);
                acc[4 * q + 2] = __fmaf_rn(wv[k], xv.z, acc[4 * q + 2]);
                acc[4 * q + 3] = __fmaf_rn(wv[k], xv.w, acc[4 * q + 3]);
            }
        }
    }
    tree16<16, 16, 8>(acc, group_mask(), j);
    return acc[0];
}

// The same for two rows at once against 8 vectors each: lane j < 8 returns wa . column j, lane j >= 8 returns
// wb . column j (columns 8-15 hold the vectors of wb).
__device__ __forceinline__ float row_pair_dot8(const float* __restrict__ wa, const float* __restrict__ wb,
                                               const float* xt, int j) {
    float acc[16];
#pragma unroll
    for (int a = 0; a < 16; ++a) acc[a] = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        float va[20], vb[20];
#pragma unroll
        for (int k = 0; k < 20; ++k) {
            va[k] = wa[j + 16 * (20 * h + k)];
            vb[k] = wb[j + 16 * (20 * h + k)];
        }
#pragma unroll
        for (int k = 0; k < 20; ++k) {
            const float4* x = reinterpret_cast<const float4*>(xt + (j + 16 * (20 * h + k)) * XTS);
            const float4 x0 = x[0], x1 = x[1], y0 = x[2], y1 = x[3];
            acc[0] = __fmaf_rn(va[k], x0.x, acc[0]);
            acc[1] = __fmaf_rn(va[k], x0.y, acc[1]);
            acc[2] = __fmaf_rn(va[k], x0.z, acc[2]);
            acc[3] = __fmaf_rn(va[k], x0.w, acc[3]);
            acc[4] = __fmaf_rn(va[k], x1.x, acc[4]);
            acc[5] = __fmaf_rn(va[k], x1.y, acc[5]);
            acc[6] = __fmaf_rn(va[k], x1.z, acc[6]);
            acc[7] = __fmaf_rn(va[k], x1.w, acc[7]);
            acc[8] = __fmaf_rn(vb[k], y0.x, acc[8]);
            acc[9] = __fmaf_rn(vb[k], y0.y, acc[9]);
            acc[10] = __fmaf_rn(vb[k], y0.z, acc[10]);
            acc[11] = __fmaf_rn(vb[k], y0.w, acc[11]);
            acc[12] = __fmaf_rn(vb[k], y1.x, acc[12]);
            acc[13] = __fmaf_rn(vb[k], y1.y, acc[13]);
            acc[14] = __fmaf_rn(vb[k], y1.z, acc[14]);
            acc[15] = __fmaf_rn(vb[k], y1.w, acc[15]);
        }
    }
    tree16<16, 16, 8>(acc, group_mask(), j);
    return acc[0];
}

__device__ __forceinline__ float relu_ref(float v) { return v > 0.f ? v : 0.f; }   // csrc/decoder.c:81-84

__device__ __forceinline__ float sigmoid_ref(float x) {   // csrc/phonon2.h:38-46
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(x < -87.0f ? 87.0f : -x)));
}

// Grid barrier on an arrival count that only grows during a launch (the host zeroes it before): thread 0 of each CTA
// adds one (acquire-release, so the CTA's writes before the barrier are published and, for the last arrival, everyone
// else's acquired) and polls with acquire loads until the count reaches the next multiple of the grid size. One trip
// through L2 per barrier, where a count reset by the last arrival and a generation word it then advances cost two.
// The wait is bounded: a barrier that does not complete records an error and returns false.
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ bool grid_sync(unsigned* count, unsigned nblocks, uint32_t* err, int* s_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned old = atom_add_acq_rel(count, 1u);
        const unsigned target = (old / nblocks + 1) * nblocks;
        if (old + 1 != target) {
            const unsigned long long t0 = global_ns();
            uint32_t i = 0;
            while (static_cast<int>(ld_acquire(count) - target) < 0) {
                if ((++i & 255u) == 0 && global_ns() - t0 > BARRIER_NS) {
                    ok = 0;
                    if (err) atomicCAS(err, DEV_OK, DEC_TIMEOUT_BARRIER);
                    break;
                }
            }
        }
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

struct Cand {
    float v;
    int i;
};

// Diagnostic builds (-DP2CU_TRACE) add up the globaltimer time thread 0 of CTA 0 spends in each phase (slots below)
// and count the iterations; p2cu_decoder_trace reads and clears the sums.
#ifdef P2CU_TRACE
enum { TR_SETUP, TR_J, TR_JBAR, TR_A, TR_L0, TR_L0BAR, TR_L1, TR_L1BAR, TR_P, TR_PBAR, TR_ITERS, TR_TOKITERS,
       TR_TAIL, TR_N = 16 };
__device__ unsigned long long g_dec_trace[TR_N];
#define DTRACE_START() unsigned long long tr_t = (blockIdx.x == 0 && threadIdx.x == 0) ? global_ns() : 0
#define DTRACE(slot) do { if (blockIdx.x == 0 && threadIdx.x == 0) { const unsigned long long n_ = global_ns(); \
                              g_dec_trace[slot] += n_ - tr_t; tr_t = n_; } } while (0)
#define DCOUNT(slot) do { if (blockIdx.x == 0 && threadIdx.x == 0) g_dec_trace[slot] += 1; } while (0)
#else
#define DTRACE_START() do { } while (0)
#define DTRACE(slot) do { } while (0)
#define DCOUNT(slot) do { } while (0)
#endif

// true when candidate (v, i) beats (bv, bi): the larger logit, and among equal logits the lower row - the first
// maximum in row order, as the reference's argmax (csrc/decoder.c:90-96) finds it.
__device__ __forceinline__ bool beats(float v, int i, float bv, int bi) {
    if (i == NO_ROW) return false;
    if (bi == NO_ROW) return true;
    return v > bv || (v == bv && i < bi);
}

// Appends the lanes' flagged items to list (warp-wide, in lane order); returns the new length.
__device__ __forceinline__ int warp_append(bool flag, int item, int* list, int n) {
    const unsigned bal = __ballot_sync(0xffffffffu, flag);
    const int lane = threadIdx.x & 31;
    if (flag) list[n + __popc(bal & ((1u << lane) - 1u))] = item;
    return n + __popc(bal);
}

__global__ void __launch_bounds__(THREADS, 1) tdt_decode_kernel(DecParams p) {
    extern __shared__ __align__(16) float smem[];
    const int G = gridDim.x, cta = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = tid >> 4, j = tid & 15;
    // this CTA's slices
    const int rows_max = (NLOG + G - 1) / G;
    const int r0 = static_cast<int>(static_cast<long long>(cta) * NLOG / G);
    const int nrows = static_cast<int>(static_cast<long long>(cta + 1) * NLOG / G) - r0;
    const int u0 = cta * HD / G, nu = (cta + 1) * HD / G - u0;

    float* head_s = smem;                                          // [rows_max][HDP]
    float* xt = head_s + static_cast<size_t>(rows_max) * HDP;      // [640][XTS] staged inputs, transposed
    float* logit_s = xt + HD * XTS;                                // [rows_max][WG]
    float* gate_s = logit_s + rows_max * WG;                       // [WL][GROUPS]
    float* headb_s = gate_s + WL * GROUPS;                         // [rows_max] the head bias of the CTA's rows
    int* Ts = reinterpret_cast<int*>(headb_s + rows_max);          // [MAXW] frames of each window
    int* off_s = Ts + MAXW;                                        // [MAXW] first frame of each window
    int* step_tok = off_s + MAXW;                                  // [MAXW] token of the window's next LSTM step
    int* hp = step_tok + MAXW;                                     // [MAXW] current ping-pong side of h
    int* t_s = hp + MAXW;                                          // [MAXW] frame pointer
    int* sym_s = t_s + MAXW;                                       // [MAXW] tokens emitted at the current frame
    int* cnt_s = sym_s + MAXW;                                     // [MAXW] tokens emitted
    int* act = cnt_s + MAXW;                                       // [MAXW] windows that step the LSTM
    int* live = act + MAXW;                                        // [MAXW] windows with frames left
    int* misc = live + MAXW;                                       // s_ok, n_act, n_live
    int* s_ok = misc;

    DTRACE_START();
    const int B = p.B;
    auto T_of = [&](int b) { return Ts[b]; };
    auto hrow = [&](int side, int layer, int b) { return p.h + ((static_cast<size_t>(side) * 2 + layer) * B + b) * HD; };

    if (p.mode != DEC_STEP) {
        const float4* src = reinterpret_cast<const float4*>(p.head + static_cast<size_t>(r0) * HD);
        for (int i = tid; i < nrows * (HD / 4); i += THREADS) {
            const int r = i / (HD / 4), k = i % (HD / 4);
            *reinterpret_cast<float4*>(head_s + r * HDP + 4 * k) = src[i];
        }
    }
    for (int r = tid; r < nrows; r += THREADS) headb_s[r] = p.headb[r0 + r];
    for (int b = tid; b < B; b += THREADS) {
        const int o = p.win_off[b];
        off_s[b] = o;
        Ts[b] = p.win_off[b + 1] - o;
        hp[b] = 0;
        step_tok[b] = p.first_token;   // a decode starts with one step on the blank token (zero embedding row)
        t_s[b] = 0;
        sym_s[b] = 0;
        cnt_s[b] = 0;
        act[b] = b;
    }
    if (tid == 0) misc[1] = B;
    __syncthreads();

    // one LSTM layer (csrc/decoder.c:41-59) for the windows in act: x = the token's embedding row (layer 0) or the
    // new h of layer 0 (layer 1); the state on side hp[b] is read, the new h written to the other side, c in place
    auto lstm_layer = [&](int layer) {
        const float* Wih = layer ? p.wih1 : p.wih0;
        const float* Whh = layer ? p.whh1 : p.whh0;
        const float* bih = layer ? p.bih1 : p.bih0;
        const float* bhh = layer ? p.bhh1 : p.bhh0;
        const int n_act = misc[1];
        for (int w0 = 0; w0 < n_act; w0 += WL) {
            const int nw = n_act - w0 < WL ? n_act - w0 : WL;
            __syncthreads();
            // column s: x, column 8 + s: h; each thread's loads of a batch are in flight together
            for (int i0 = 0; i0 < nw * 2 * (HD / 4); i0 += STAGE_BATCH * THREADS) {
                float4 v[STAGE_BATCH];
#pragma unroll
                for (int u = 0; u < STAGE_BATCH; ++u) {
                    const int i = i0 + tid + u * THREADS;
                    if (i < nw * 2 * (HD / 4)) {
                        const int k = i % (HD / 4), which = (i / (HD / 4)) & 1, s = i / (2 * (HD / 4));
                        const int b = act[w0 + s], cur = hp[b];
                        const float* src = which ? hrow(cur, layer, b)
                                                 : (layer ? hrow(1 - cur, 0, b)
                                                          : p.embed + static_cast<size_t>(step_tok[b]) * HD);
                        v[u] = reinterpret_cast<const float4*>(src)[k];
                    }
                }
#pragma unroll
                for (int u = 0; u < STAGE_BATCH; ++u) {
                    const int i = i0 + tid + u * THREADS;
                    if (i < nw * 2 * (HD / 4)) {
                        const int k = i % (HD / 4), which = (i / (HD / 4)) & 1, s = i / (2 * (HD / 4));
                        float* d = xt + 4 * k * XTS + 8 * which + s;
                        d[0] = v[u].x;
                        d[XTS] = v[u].y;
                        d[2 * XTS] = v[u].z;
                        d[3 * XTS] = v[u].w;
                    }
                }
            }
            // the cells' c, read while the gate rows are computed
            float c_old = 0.f;
            if (tid < nw * nu) {
                const int b = act[w0 + tid / nu];
                c_old = p.c[(static_cast<size_t>(layer) * B + b) * HD + u0 + tid % nu];
            }
            __syncthreads();
            if (grp < 4 * nu) {   // group -> gate row (gate order i, f, g, o) of one of the CTA's units
                const int r = (grp / nu) * HD + u0 + grp % nu;
                const float d = row_pair_dot8(Wih + static_cast<size_t>(r) * HD, Whh + static_cast<size_t>(r) * HD, xt, j);
                const float dh = __shfl_down_sync(group_mask(), d, 8, 16);   // lane s: W_ih x_s, lane 8 + s: W_hh h_s
                if (j < nw) gate_s[j * GROUPS + grp] = __fadd_rn(__fadd_rn(__fadd_rn(d, dh), bih[r]), bhh[r]);
            }
            __syncthreads();
            if (tid < nw * nu) {   // nw * nu <= WL * MAXU <= THREADS: one cell per thread
                const int s = tid / nu, k = tid % nu, u = u0 + k, b = act[w0 + s], cur = hp[b];
                const float* g = gate_s + s * GROUPS;
                const float gi = sigmoid_ref(g[k]), gf = sigmoid_ref(g[nu + k]);
                const float gg = tanhf(g[2 * nu + k]), go = sigmoid_ref(g[3 * nu + k]);
                const float cn = __fadd_rn(__fmul_rn(gf, c_old), __fmul_rn(gi, gg));
                p.c[(static_cast<size_t>(layer) * B + b) * HD + u] = cn;
                hrow(1 - cur, layer, b)[u] = __fmul_rn(go, tanhf(cn));
            }
        }
    };

    // dec = proj_w h1 + proj_b (csrc/decoder.c:72-73) for the CTA's rows and the windows in act
    auto projector = [&]() {
        const int n_act = misc[1];
        for (int w0 = 0; w0 < n_act; w0 += WG) {
            const int nw = n_act - w0 < WG ? n_act - w0 : WG;
            __syncthreads();
            for (int i0 = 0; i0 < nw * (HD / 4); i0 += STAGE_BATCH * THREADS) {
                float4 v[STAGE_BATCH];
#pragma unroll
                for (int u = 0; u < STAGE_BATCH; ++u) {
                    const int i = i0 + tid + u * THREADS;
                    if (i < nw * (HD / 4)) {
                        const int b = act[w0 + i / (HD / 4)];
                        v[u] = reinterpret_cast<const float4*>(hrow(1 - hp[b], 1, b))[i % (HD / 4)];
                    }
                }
#pragma unroll
                for (int u = 0; u < STAGE_BATCH; ++u) {
                    const int i = i0 + tid + u * THREADS;
                    if (i < nw * (HD / 4)) {
                        float* d = xt + 4 * (i % (HD / 4)) * XTS + i / (HD / 4);
                        d[0] = v[u].x;
                        d[XTS] = v[u].y;
                        d[2 * XTS] = v[u].z;
                        d[3 * XTS] = v[u].w;
                    }
                }
            }
            __syncthreads();
            if (grp < nu) {
                const int r = u0 + grp;
                const float d = row_dot16(p.proj + static_cast<size_t>(r) * HD, xt, j);
                if (j < nw) p.dec[static_cast<size_t>(act[w0 + j]) * HD + r] = __fadd_rn(d, p.projb[r]);
            }
        }
        __syncthreads();
        const int n = misc[1];
        for (int k = tid; k < n; k += THREADS) hp[act[k]] ^= 1;
    };

    if (p.mode == DEC_JOINT) {   // p2_joint (csrc/decoder.c:78-88): logits of enc[0] with dec[0], every row out
        for (int i = tid; i < HD * XTS; i += THREADS) {
            const int k = i / XTS, c = i % XTS;
            xt[i] = c == 0 ? relu_ref(__fadd_rn(p.enc[k], p.dec[k])) : 0.f;
        }
        __syncthreads();
        joint_rows<1>(head_s, xt, nrows, 1, grp, j, p.headb + r0, p.logits + r0, 1);
        return;
    }

    // the first prediction-network step (from zero state for a decode, csrc/decoder.c:112)
    lstm_layer(0);
    if (!grid_sync(p.bar_count, G, p.err, s_ok)) return;
    lstm_layer(1);
    if (!grid_sync(p.bar_count, G, p.err, s_ok)) return;
    projector();
    if (p.mode == DEC_STEP) return;   // p2_decoder_step: the new h is on side 1, c in place, dec written
    if (warp == 0) {
        int n = 0;
        for (int b0 = 0; b0 < B; b0 += 32) n = warp_append(b0 + lane < B && T_of(b0 + lane) > 0, b0 + lane, live, n);
        if (lane == 0) misc[2] = n;
    }
    if (!grid_sync(p.bar_count, G, p.err, s_ok)) return;
    DTRACE(TR_SETUP);

    int iter = 0;
    for (; iter < p.max_iters && misc[2] > 0; ++iter) {
        const int par = iter & 1, n_live = misc[2];
        Cand* cand = reinterpret_cast<Cand*>(p.cand) + static_cast<size_t>(par) * G * B;
        float* dur = p.dur + static_cast<size_t>(par) * B * NDUR;

        // ---- J: joint logits relu(enc[t] + dec) . head (csrc/decoder.c:78-88) for the CTA's rows ----
        for (int w0 = 0; w0 < n_live; w0 += WG) {
            const int nw = n_live - w0 < WG ? n_live - w0 : WG;
            __syncthreads();
            // relu(enc[t] + dec): v > 0 ? v : 0, as the reference writes it (a -0 sum becomes +0)
            for (int i0 = 0; i0 < nw * (HD / 4); i0 += STAGE_BATCH * THREADS) {
                float4 e[STAGE_BATCH], d[STAGE_BATCH];
#pragma unroll
                for (int u = 0; u < STAGE_BATCH; ++u) {
                    const int i = i0 + tid + u * THREADS;
                    if (i < nw * (HD / 4)) {
                        const int b = live[w0 + i / (HD / 4)], k = i % (HD / 4);
                        e[u] = reinterpret_cast<const float4*>(p.enc + (static_cast<size_t>(off_s[b]) + t_s[b]) * HD)[k];
                        d[u] = reinterpret_cast<const float4*>(p.dec + static_cast<size_t>(b) * HD)[k];
                    }
                }
#pragma unroll
                for (int u = 0; u < STAGE_BATCH; ++u) {
                    const int i = i0 + tid + u * THREADS;
                    if (i < nw * (HD / 4)) {
                        float* o = xt + 4 * (i % (HD / 4)) * XTS + i / (HD / 4);
                        o[0] = relu_ref(__fadd_rn(e[u].x, d[u].x));
                        o[XTS] = relu_ref(__fadd_rn(e[u].y, d[u].y));
                        o[2 * XTS] = relu_ref(__fadd_rn(e[u].z, d[u].z));
                        o[3 * XTS] = relu_ref(__fadd_rn(e[u].w, d[u].w));
                    }
                }
            }
            __syncthreads();
            if (nw <= 4)
                joint_rows<1>(head_s, xt, nrows, nw, grp, j, headb_s, logit_s, WG);
            else if (nw <= 8)
                joint_rows<2>(head_s, xt, nrows, nw, grp, j, headb_s, logit_s, WG);
            else
                joint_rows<4>(head_s, xt, nrows, nw, grp, j, headb_s, logit_s, WG);
            __syncthreads();
            for (int s = warp; s < nw; s += WARPS) {   // a warp per window: the CTA's first maximum
                const int b = live[w0 + s];
                float bv = -INFINITY;
                int bi = NO_ROW;
                for (int r = lane; r < nrows; r += 32) {
                    const int row = r0 + r;
                    const float v = logit_s[r * WG + s];
                    if (row < NVOCAB) {
                        if (beats(v, row, bv, bi)) { bv = v; bi = row; }
                    } else {
                        dur[static_cast<size_t>(b) * NDUR + (row - NVOCAB)] = v;   // the duration rows it owns
                    }
                }
#pragma unroll
                for (int off = 16; off; off >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                    if (beats(ov, oi, bv, bi)) { bv = ov; bi = oi; }
                }
                if (lane == 0) cand[static_cast<size_t>(cta) * B + b] = Cand{bv, bi};
            }
        }
        DTRACE(TR_J);
        if (!grid_sync(p.bar_count, G, p.err, s_ok)) return;
        DTRACE(TR_JBAR);
        DCOUNT(TR_ITERS);

        // ---- A: the decisions of csrc/decoder.c:115-140, the same in every CTA; a warp per window ----
        for (int k = warp; k < n_live; k += WARPS) {
            const int b = live[k];
            float bv = -INFINITY;
            int bi = NO_ROW;
            const float dv = lane < NDUR ? dur[static_cast<size_t>(b) * NDUR + lane] : 0.f;
            for (int c0 = 0; c0 < G; c0 += CAND_PER_LANE * 32) {   // every load of the lane in flight at once
                Cand x[CAND_PER_LANE];
#pragma unroll
                for (int u = 0; u < CAND_PER_LANE; ++u) {
                    const int c = c0 + lane + 32 * u;
                    x[u] = c < G ? cand[static_cast<size_t>(c) * B + b] : Cand{-INFINITY, NO_ROW};
                }
#pragma unroll
                for (int u = 0; u < CAND_PER_LANE; ++u)
                    if (beats(x[u].v, x[u].i, bv, bi)) { bv = x[u].v; bi = x[u].i; }
            }
#pragma unroll
            for (int off = 16; off; off >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                if (beats(ov, oi, bv, bi)) { bv = ov; bi = oi; }
            }
            float dl[NDUR];
#pragma unroll
            for (int q = 0; q < NDUR; ++q) dl[q] = __shfl_sync(0xffffffffu, dv, q);
            if (lane == 0) {
                int duration = 0;   // the durations are {0, 1, 2, 3, 4}: the argmax index itself
#pragma unroll
                for (int q = 1; q < NDUR; ++q)
                    if (dl[q] > dl[duration]) duration = q;
                const int t = t_s[b];
                if (bi == BLANK) {
                    if (duration == 0) duration = 1;
                    step_tok[b] = -1;
                } else {
                    const int n = cnt_s[b];
                    if (cta == 0) {
                        if (n < P2CU_DEC_MAX_SYMBOLS * T_of(b)) {
                            int* o = p.tokens + (static_cast<size_t>(P2CU_DEC_MAX_SYMBOLS) * off_s[b] + n) * 3;
                            o[0] = bi;
                            o[1] = t;
                            o[2] = duration;
                        } else {
                            atomicCAS(p.err, DEV_OK, DEC_TOKEN_OVERFLOW);
                        }
                    }
                    cnt_s[b] = n + 1;
                    const int sym = sym_s[b] + 1;
                    sym_s[b] = sym;
                    if (duration == 0 && sym >= P2CU_DEC_MAX_SYMBOLS) duration = 1;
                    step_tok[b] = bi;
                }
                if (duration) sym_s[b] = 0;
                t_s[b] = t + duration;
            }
        }
        __syncthreads();
        if (warp == 0) {   // windows that emitted and still have frames (the others' state is never read again)
            int n = 0;
            for (int k0 = 0; k0 < n_live; k0 += 32) {
                const int k = k0 + lane, b = k < n_live ? live[k] : 0;
                n = warp_append(k < n_live && step_tok[b] >= 0 && t_s[b] < T_of(b), b, act, n);
            }
            __syncwarp();
            int m = 0;
            for (int k0 = 0; k0 < n_live; k0 += 32) {
                const int k = k0 + lane, b = k < n_live ? live[k] : 0;
                const bool keep = k < n_live && t_s[b] < T_of(b);
                __syncwarp();
                m = warp_append(keep, b, live, m);   // in place: item k moves to m + rank <= k
            }
            if (lane == 0) {
                misc[1] = n;
                misc[2] = m;
            }
        }
        __syncthreads();
        DTRACE(TR_A);
        if (misc[1] > 0) {
            DCOUNT(TR_TOKITERS);
            lstm_layer(0);
            DTRACE(TR_L0);
            if (!grid_sync(p.bar_count, G, p.err, s_ok)) return;
            DTRACE(TR_L0BAR);
            lstm_layer(1);
            DTRACE(TR_L1);
            if (!grid_sync(p.bar_count, G, p.err, s_ok)) return;
            DTRACE(TR_L1BAR);
            projector();
            DTRACE(TR_P);
            if (!grid_sync(p.bar_count, G, p.err, s_ok)) return;
            DTRACE(TR_PBAR);
        }
    }
    if (cta != 0) return;
    __syncthreads();
    if (tid == 0 && misc[2] > 0) atomicCAS(p.err, DEV_OK, DEC_ITER_LIMIT);
    // counts, prefix offsets and the tokens packed window after window
    if (warp == 0) {
        int base = 0;
        for (int b0 = 0; b0 < B; b0 += 32) {
            const int b = b0 + lane;
            int n = 0;
            if (b < B) {
                const int cap = P2CU_DEC_MAX_SYMBOLS * T_of(b);
                n = cnt_s[b] < cap ? cnt_s[b] : cap;
                p.count[b] = cnt_s[b];
            }
            int incl = n;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += v;
            }
            if (b < B) p.tok_off[b] = base + incl - n;
            base += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) p.tok_off[B] = base;
    }
    __syncthreads();
    for (int b = warp; b < B; b += WARPS) {
        const int o = p.tok_off[b], n = p.tok_off[b + 1] - o;
        const int* src = p.tokens + static_cast<size_t>(P2CU_DEC_MAX_SYMBOLS) * off_s[b] * 3;
        for (int i = lane; i < 3 * n; i += 32) p.tok_out[static_cast<size_t>(o) * 3 + i] = src[i];
    }
    DTRACE(TR_TAIL);
}

}  // namespace

int decoder_smem_bytes(int grid) {
    const int rows_max = (NLOG + grid - 1) / grid;
    return (rows_max * HDP + HD * XTS + rows_max * WG + WL * GROUPS + rows_max) * 4 + (9 * MAXW + 4) * 4;
}

int decoder_max_windows() { return MAXW; }

int decoder_max_units() { return MAXU; }

cudaError_t tdt_decode_launch(const DecParams& p, int grid, cudaStream_t s) {
    const int bytes = decoder_smem_bytes(grid);
    cudaError_t e = cudaFuncSetAttribute(tdt_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    DecParams q = p;
    void* args[] = {&q};
    return cudaLaunchCooperativeKernel(reinterpret_cast<void*>(tdt_decode_kernel), dim3(grid), dim3(THREADS), args,
                                       static_cast<size_t>(bytes), s);
}

int decoder_max_grid(int device) {
    int sms = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    const int bytes = decoder_smem_bytes(sms);
    if (cudaFuncSetAttribute(tdt_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
        return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tdt_decode_kernel, THREADS, bytes) != cudaSuccess)
        return 0;
    return per_sm >= 1 ? sms : 0;
}

}  // namespace p2cu

#ifdef P2CU_TRACE
extern "C" __attribute__((visibility("default"))) int p2cu_decoder_trace(unsigned long long* out) {
    const unsigned long long zero[p2cu::TR_N] = {};
    if (cudaMemcpyFromSymbol(out, p2cu::g_dec_trace, sizeof(zero)) != cudaSuccess) return -1;
    return cudaMemcpyToSymbol(p2cu::g_dec_trace, zero, sizeof(zero)) == cudaSuccess ? 0 : -1;
}
#endif
