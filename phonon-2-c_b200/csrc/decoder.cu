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
constexpr int WG = 16;                // windows whose joint input is staged at a time
constexpr int WL = 8;                 // windows whose LSTM input (x and h rows) is staged at a time
constexpr int MAXW = 1024;            // windows per launch
constexpr int MAXU = GROUPS / 4;      // hidden units a CTA can own: four gate rows each, one group per row
constexpr int NO_ROW = 0x7fffffff;
constexpr uint32_t DEC_TIMEOUT_BARRIER = 20, DEC_TOKEN_OVERFLOW = 21, DEC_ITER_LIMIT = 22;
constexpr unsigned long long BARRIER_NS = 2000000000ull;   // two seconds

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Dot products of one 640-row w with nw (<= NW) vectors xs[s * xstride], by one group of 16 lanes (one half of a
// warp) in the reference's order: lane j runs the FMA chain over i = j, j + 16, ...; lanes j and j + 8 are added;
// then the horizontal-sum tree of csrc/tensor_ops.c:182-190. Every lane of the group gets the results. The shuffles
// name only the group's lanes: the two halves of a warp may be on different rows (or one of them on none).
template <int NW>
__device__ __forceinline__ void dot_rows(const float* __restrict__ w, const float* __restrict__ xs, int xstride,
                                         int nw, int j, float (&out)[NW]) {
    const unsigned mask = (threadIdx.x & 16) ? 0xFFFF0000u : 0x0000FFFFu;
    float acc[NW];
#pragma unroll
    for (int s = 0; s < NW; ++s) acc[s] = 0.f;
#pragma unroll 4
    for (int i = j; i < HD; i += 16) {
        const float wv = w[i];
#pragma unroll
        for (int s = 0; s < NW; ++s)
            if (s < nw) acc[s] = __fmaf_rn(wv, xs[s * xstride + i], acc[s]);
    }
#pragma unroll
    for (int s = 0; s < NW; ++s) {
        float a = acc[s];
        a = __fadd_rn(a, __shfl_down_sync(mask, a, 8, 16));   // acc0 + acc1
        a = __fadd_rn(a, __shfl_down_sync(mask, a, 4, 16));
        a = __fadd_rn(a, __shfl_down_sync(mask, a, 2, 16));
        a = __fadd_rn(a, __shfl_down_sync(mask, a, 1, 16));
        out[s] = __shfl_sync(mask, a, 0, 16);
    }
}

__device__ __forceinline__ float relu_ref(float v) { return v > 0.f ? v : 0.f; }   // csrc/decoder.c:81-84

__device__ __forceinline__ float sigmoid_ref(float x) {   // csrc/phonon2.h:38-46
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(x < -87.0f ? 87.0f : -x)));
}

// Grid barrier (generation counter) with a bounded wait. Returns false when it gave up.
__device__ bool grid_sync(unsigned* count, volatile unsigned* gen, unsigned nblocks, uint32_t* err, int* s_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned g = *gen;
        __threadfence();
        if (atomicAdd(count, 1u) == nblocks - 1) {
            *count = 0;
            __threadfence();
            atomicAdd(const_cast<unsigned*>(gen), 1u);
        } else {
            const unsigned long long t0 = global_ns();
            uint32_t i = 0;
            while (*gen == g) {
                if ((++i & 255u) == 0 && global_ns() - t0 > BARRIER_NS) {
                    ok = 0;
                    if (err) atomicCAS(err, DEV_OK, DEC_TIMEOUT_BARRIER);
                    break;
                }
            }
        }
        __threadfence();
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

struct Cand {
    float v;
    int i;
};

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
    float* xs_s = head_s + static_cast<size_t>(rows_max) * HDP;    // [WG][HDP] joint inputs / LSTM x, h rows
    float* logit_s = xs_s + WG * HDP;                              // [rows_max][WG]
    float* gate_s = logit_s + rows_max * WG;                       // [WL][GROUPS]
    int* step_tok = reinterpret_cast<int*>(gate_s + WL * GROUPS);  // [MAXW] token of the window's next LSTM step
    int* hp = step_tok + MAXW;                                     // [MAXW] current ping-pong side of h
    int* t_s = hp + MAXW;                                          // [MAXW] frame pointer
    int* sym_s = t_s + MAXW;                                       // [MAXW] tokens emitted at the current frame
    int* cnt_s = sym_s + MAXW;                                     // [MAXW] tokens emitted
    int* act = cnt_s + MAXW;                                       // [MAXW] windows that step the LSTM
    int* live = act + MAXW;                                        // [MAXW] windows with frames left
    int* misc = live + MAXW;                                       // s_ok, n_act, n_live
    int* s_ok = misc;

    const int B = p.B;
    auto T_of = [&](int b) { return p.win_off[b + 1] - p.win_off[b]; };
    auto hrow = [&](int side, int layer, int b) { return p.h + ((static_cast<size_t>(side) * 2 + layer) * B + b) * HD; };

    if (p.mode != DEC_STEP) {
        const float4* src = reinterpret_cast<const float4*>(p.head + static_cast<size_t>(r0) * HD);
        for (int i = tid; i < nrows * (HD / 4); i += THREADS) {
            const int r = i / (HD / 4), k = i % (HD / 4);
            *reinterpret_cast<float4*>(head_s + r * HDP + 4 * k) = src[i];
        }
    }
    for (int b = tid; b < B; b += THREADS) {
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
            for (int i = tid; i < nw * 2 * (HD / 4); i += THREADS) {   // row 2s: x, row 2s + 1: h
                const int s = i / (2 * (HD / 4)), rem = i % (2 * (HD / 4)), which = rem / (HD / 4), k = rem % (HD / 4);
                const int b = act[w0 + s], cur = hp[b];
                const float* src = which ? hrow(cur, layer, b)
                                         : (layer ? hrow(1 - cur, 0, b) : p.embed + static_cast<size_t>(step_tok[b]) * HD);
                *reinterpret_cast<float4*>(xs_s + (2 * s + which) * HDP + 4 * k) =
                    reinterpret_cast<const float4*>(src)[k];
            }
            __syncthreads();
            if (grp < 4 * nu) {   // group -> gate row (gate order i, f, g, o) of one of the CTA's units
                const int r = (grp / nu) * HD + u0 + grp % nu;
                float d1[WL], d2[WL];
                dot_rows<WL>(Wih + static_cast<size_t>(r) * HD, xs_s, 2 * HDP, nw, j, d1);
                dot_rows<WL>(Whh + static_cast<size_t>(r) * HD, xs_s + HDP, 2 * HDP, nw, j, d2);
                if (j == 0) {
                    const float bi = bih[r], bh = bhh[r];
#pragma unroll
                    for (int s = 0; s < WL; ++s)
                        if (s < nw) gate_s[s * GROUPS + grp] = __fadd_rn(__fadd_rn(__fadd_rn(d1[s], d2[s]), bi), bh);
                }
            }
            __syncthreads();
            for (int i = tid; i < nw * nu; i += THREADS) {
                const int s = i / nu, k = i % nu, u = u0 + k, b = act[w0 + s], cur = hp[b];
                const float* g = gate_s + s * GROUPS;
                const float gi = sigmoid_ref(g[k]), gf = sigmoid_ref(g[nu + k]);
                const float gg = tanhf(g[2 * nu + k]), go = sigmoid_ref(g[3 * nu + k]);
                float* c = p.c + (static_cast<size_t>(layer) * B + b) * HD + u;
                const float cn = __fadd_rn(__fmul_rn(gf, *c), __fmul_rn(gi, gg));
                *c = cn;
                hrow(1 - cur, layer, b)[u] = __fmul_rn(go, tanhf(cn));
            }
        }
    };

    // dec = proj_w h1 + proj_b (csrc/decoder.c:72-73) for the CTA's rows and the windows in act
    auto projector = [&]() {
        const int n_act = misc[1];
        for (int w0 = 0; w0 < n_act; w0 += WL) {
            const int nw = n_act - w0 < WL ? n_act - w0 : WL;
            __syncthreads();
            for (int i = tid; i < nw * (HD / 4); i += THREADS) {
                const int s = i / (HD / 4), k = i % (HD / 4), b = act[w0 + s];
                *reinterpret_cast<float4*>(xs_s + s * HDP + 4 * k) =
                    reinterpret_cast<const float4*>(hrow(1 - hp[b], 1, b))[k];
            }
            __syncthreads();
            if (grp < nu) {
                const int r = u0 + grp;
                float d[WL];
                dot_rows<WL>(p.proj + static_cast<size_t>(r) * HD, xs_s, HDP, nw, j, d);
                if (j == 0) {
                    const float pb = p.projb[r];
#pragma unroll
                    for (int s = 0; s < WL; ++s)
                        if (s < nw) p.dec[static_cast<size_t>(act[w0 + s]) * HD + r] = __fadd_rn(d[s], pb);
                }
            }
        }
        __syncthreads();
        const int n = misc[1];
        for (int k = tid; k < n; k += THREADS) hp[act[k]] ^= 1;
    };

    if (p.mode == DEC_JOINT) {   // p2_joint (csrc/decoder.c:78-88): logits of enc[0] with dec[0], every row out
        for (int i = tid; i < HD; i += THREADS) {
            xs_s[i] = relu_ref(__fadd_rn(p.enc[i], p.dec[i]));
        }
        __syncthreads();
        for (int r = grp; r < nrows; r += GROUPS) {
            float v[1];
            dot_rows<1>(head_s + r * HDP, xs_s, HDP, 1, j, v);
            if (j == 0) p.logits[r0 + r] = __fadd_rn(v[0], p.headb[r0 + r]);
        }
        return;
    }

    // the first prediction-network step (from zero state for a decode, csrc/decoder.c:112)
    lstm_layer(0);
    if (!grid_sync(p.bar_count, p.bar_gen, G, p.err, s_ok)) return;
    lstm_layer(1);
    if (!grid_sync(p.bar_count, p.bar_gen, G, p.err, s_ok)) return;
    projector();
    if (p.mode == DEC_STEP) return;   // p2_decoder_step: the new h is on side 1, c in place, dec written
    if (warp == 0) {
        int n = 0;
        for (int b0 = 0; b0 < B; b0 += 32) n = warp_append(b0 + lane < B && T_of(b0 + lane) > 0, b0 + lane, live, n);
        if (lane == 0) misc[2] = n;
    }
    if (!grid_sync(p.bar_count, p.bar_gen, G, p.err, s_ok)) return;

    int iter = 0;
    for (; iter < p.max_iters && misc[2] > 0; ++iter) {
        const int par = iter & 1, n_live = misc[2];
        Cand* cand = reinterpret_cast<Cand*>(p.cand) + static_cast<size_t>(par) * G * B;
        float* dur = p.dur + static_cast<size_t>(par) * B * NDUR;

        // ---- J: joint logits relu(enc[t] + dec) . head (csrc/decoder.c:78-88) for the CTA's rows ----
        for (int w0 = 0; w0 < n_live; w0 += WG) {
            const int nw = n_live - w0 < WG ? n_live - w0 : WG;
            __syncthreads();
            for (int i = tid; i < nw * (HD / 4); i += THREADS) {
                const int s = i / (HD / 4), k = i % (HD / 4), b = live[w0 + s];
                const float4 e = reinterpret_cast<const float4*>(
                    p.enc + (static_cast<size_t>(p.win_off[b]) + t_s[b]) * HD)[k];
                const float4 d = reinterpret_cast<const float4*>(p.dec + static_cast<size_t>(b) * HD)[k];
                float4 v;   // v > 0 ? v : 0, as the reference writes it (a -0 sum becomes +0)
                v.x = relu_ref(__fadd_rn(e.x, d.x));
                v.y = relu_ref(__fadd_rn(e.y, d.y));
                v.z = relu_ref(__fadd_rn(e.z, d.z));
                v.w = relu_ref(__fadd_rn(e.w, d.w));
                *reinterpret_cast<float4*>(xs_s + s * HDP + 4 * k) = v;
            }
            __syncthreads();
            for (int r = grp; r < nrows; r += GROUPS) {
                float v[WG];
                dot_rows<WG>(head_s + r * HDP, xs_s, HDP, nw, j, v);
                if (j == 0) {
                    const float hb = p.headb[r0 + r];
#pragma unroll
                    for (int s = 0; s < WG; ++s)
                        if (s < nw) logit_s[r * WG + s] = __fadd_rn(v[s], hb);
                }
            }
            __syncthreads();
            for (int s = tid; s < nw; s += THREADS) {   // the CTA's first maximum; the duration rows it owns
                const int b = live[w0 + s];
                Cand best{-INFINITY, NO_ROW};
                for (int r = 0; r < nrows; ++r) {
                    const int row = r0 + r;
                    const float v = logit_s[r * WG + s];
                    if (row < NVOCAB) {
                        if (best.i == NO_ROW || v > best.v) best = Cand{v, row};
                    } else {
                        dur[static_cast<size_t>(b) * NDUR + (row - NVOCAB)] = v;
                    }
                }
                cand[static_cast<size_t>(cta) * B + b] = best;
            }
        }
        if (!grid_sync(p.bar_count, p.bar_gen, G, p.err, s_ok)) return;

        // ---- A: the decisions of csrc/decoder.c:115-140, the same in every CTA; a warp per window ----
        for (int k = warp; k < n_live; k += WARPS) {
            const int b = live[k];
            float bv = -INFINITY;
            int bi = NO_ROW;
            for (int c = lane; c < G; c += 32) {
                const Cand x = cand[static_cast<size_t>(c) * B + b];
                if (beats(x.v, x.i, bv, bi)) { bv = x.v; bi = x.i; }
            }
#pragma unroll
            for (int off = 16; off; off >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                if (beats(ov, oi, bv, bi)) { bv = ov; bi = oi; }
            }
            if (lane == 0) {
                const float* dl = dur + static_cast<size_t>(b) * NDUR;
                int duration = 0;   // the durations are {0, 1, 2, 3, 4}: the argmax index itself
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
                            int* o = p.tokens + (static_cast<size_t>(P2CU_DEC_MAX_SYMBOLS) * p.win_off[b] + n) * 3;
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
        if (misc[1] > 0) {
            lstm_layer(0);
            if (!grid_sync(p.bar_count, p.bar_gen, G, p.err, s_ok)) return;
            lstm_layer(1);
            if (!grid_sync(p.bar_count, p.bar_gen, G, p.err, s_ok)) return;
            projector();
            if (!grid_sync(p.bar_count, p.bar_gen, G, p.err, s_ok)) return;
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
        const int* src = p.tokens + static_cast<size_t>(P2CU_DEC_MAX_SYMBOLS) * p.win_off[b] * 3;
        for (int i = lane; i < 3 * n; i += 32) p.tok_out[static_cast<size_t>(o) * 3 + i] = src[i];
    }
}

}  // namespace

int decoder_smem_bytes(int grid) {
    const int rows_max = (NLOG + grid - 1) / grid;
    return (rows_max * HDP + WG * HDP + rows_max * WG + WL * GROUPS) * 4 + (7 * MAXW + 4) * 4;
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
