// encoder_ops.h - launch interfaces of the FastConformer encoder's memory-bound ops (encoder_ops.cu). Internal to
// the library. Activations are row-major [rows][features]; a batch of windows is stacked along the rows and every
// op that looks across rows (convolutions over time, attention) stops at window edges, found through prefix tables
// of row offsets in device memory.
#pragma once
#include <cstdint>
#include <vector>
#include <cuda_runtime.h>
#include "gemm.h"

namespace p2cu {

// The reference's per-row int8 quantisation of dense rows [rows][D] (lda = D) into q / qscale, as quant_rows_launch;
// D = 1024 with 16-byte aligned rows takes one warp per row.
cudaError_t quant_rows_dense_launch(const float* x, int8_t* q, float* qscale, int rows, int D, cudaStream_t s);

// LayerNorm (eps 1e-5) of each row; into `out` (fp32, may alias x) or, with q != nullptr, quantised per row into
// int8 q [rows][D] with one scale per row (the reference's quantiser). With a fold (fold->nblk > 0), x is first
// completed by the K blocks of the GEMM that wrote it (KFold) and stored back, then normed.
cudaError_t ln_rows_launch(const float* x, int ldx, const float* gamma, const float* beta, float* out, int ldo,
                           int8_t* q, float* qscale, int rows, int D, cudaStream_t s, const KFold* fold = nullptr);

// Two LayerNorms in a row: x <- LN(x; g1, b1) in place, then LN(x; g2, b2) into out2 or quantised into q / qscale.
// With a fold, x is first completed by the K blocks of the GEMM that wrote it (KFold); only LN1 of it is stored.
cudaError_t ln2_rows_launch(float* x, int ldx, const float* g1, const float* b1, const float* g2, const float* b2,
                            float* out2, int ldo, int8_t* q, float* qscale, int rows, int D, cudaStream_t s,
                            const KFold* fold = nullptr);

// SiLU of each row, into `out` (fp32, may alias h) or quantised into q / qscale.
cudaError_t swish_rows_launch(const float* h, int ldh, float* out, int ldo, int8_t* q, float* qscale, int rows,
                              int len, cudaStream_t s);

// Elementwise SiLU of n values in place (p2_swish).
cudaError_t swish_launch(float* x, size_t n, cudaStream_t s);

// Plain softmax of each row in place (p2_softmax_rows).
cudaError_t softmax_rows_launch(float* x, int rows, int len, cudaStream_t s);

// GLU over the channel axis: gated[r][d] = pw1[r][d] * sigmoid(pw1[r][D + d]).
cudaError_t glu_rows_launch(const float* pw1, float* gated, int rows, int D, cudaStream_t s);

// Depthwise conv over time (kernel 9, padding 4 inside each window) + bias, then SiLU when `swish`; into fp32 `out`
// or quantised into q / qscale. row_off: n_win + 1 prefix offsets of the windows' rows (NULL: all rows are one
// window). b may be NULL (no bias).
cudaError_t dwconv_swish_launch(const float* gated, const float* w, const float* b, const int* row_off, int n_win,
                                float* out, int8_t* q, float* qscale, int rows, int D, cudaStream_t s,
                                bool swish = true);

// dst[r] = src[map[r]] for rows of `cols` floats.
cudaError_t gather_rows_launch(float* dst, const float* src, const int* map, int rows, int cols, cudaStream_t s);

// Subsampling, Conv2d(1 -> C, 3x3, stride 2, pad 1) + ReLU and then depthwise Conv2d(C, 3x3, stride 2, pad 1) + bias
// over each window, fused: mel [frames][W_in] -> [rows2][W2][C] (mel_off / h1_off / h2_off: the windows' row offsets
// in the mel, after the first convolution and after the second). W_in is 128.
cudaError_t sub_conv0_dw_launch(const float* mel, const int* mel_off, const int* h1_off, const int* h2_off, int n_win,
                                const float* w0, const float* b0, const float* w2, const float* b2, float* out,
                                int rows2, int W_in, int C, cudaStream_t s);

// Subsampling, depthwise Conv2d(C, 3x3, stride 2, pad 1) + bias over each window: [rows_in][W_in][C] ->
// [rows_out][W_out][C].
cudaError_t sub_dwconv_launch(const float* in, const int* in_off, const int* out_off, int n_win, const float* w,
                              const float* b, float* out, int rows_out, int W_in, int C, cudaStream_t s);

// [rows][W][C] -> [rows][C * W] (channel-major within a frame).
cudaError_t sub_flatten_launch(const float* in, float* out, int rows, int W, int C, cudaStream_t s);

// V (columns 2048 + 128 h .. of qkv [rows][3072]) of every window and head transposed into vt: the block of (window
// w, head h) starts at vt_off[w] + h * 128 * ldT and holds [128][ldT], ldT = T rounded up to a multiple of 4.
cudaError_t v_transpose_launch(const float* qkv, float* vt, const int* row_off, const long long* vt_off, int n_win,
                               int rows, cudaStream_t s);

// x[r][n] += b[n].
cudaError_t bias_rows_launch(float* x, const float* b, int rows, int N, cudaStream_t s);

// One SIMT fp32 GEMM problem of a group launch: C[m][n] = sum_k (A[m][k] + a_bias[k]) * B[k][n], one FMA chain
// per output in k order (the reference's fp32 sgemm). Offsets are in elements from the launch's base pointers.
struct GemmGroup {
    int M, N, K, tile0;
    long long a_off, b_off, c_off;
    int lda, ldb, ldc;
    int bias_off;   // offset into the launch's a_bias vector, or -1
};

// All groups in one launch; B is [k][n] (transB == 0) or [n][k] (transB == 1).
cudaError_t group_gemm_launch(const GemmGroup* groups, int n_groups, int total_tiles, const float* A, const float* B,
                              float* C, const float* a_bias, int transB, cudaStream_t s);
int group_gemm_tiles(int M, int N);

// Attention scores of every (window, head, query) row, in place in S_ac: x_j = (ac[i][j] + bd[i][T-1-i+j]) * scale,
// then softmax over j. srow_off: prefix offsets of the H*T rows per window; s_off / b_off: element offsets of each
// window's S_ac / S_bd blocks, whose rows are T and 2T - 1 floats rounded up to a multiple of 4 apart; Tw: frames per
// window.
cudaError_t attn_softmax_launch(float* s_ac, const float* s_bd, const int* srow_off, const long long* s_off,
                                const long long* b_off, const int* Tw, int n_win, int H, int rows, float scale,
                                cudaStream_t s);

// Fused relative-position attention for windows of at most ATT_MAXT frames: scores (content + shifted positional
// band), softmax and context in one kernel, output in the concatenated-heads layout attn [rows][1024]. qkv [rows][3072]
// (Q | K | V), P [2 Tmax - 1][1024] the projected positions of the longest window (a window of T frames uses rows
// Tmax - T .. Tmax + T - 2), tiles: (window, first query) of every 32-query tile.
constexpr int ATT_MAXT = 512;
int attn_fused_smem_bytes(int Tmax);
cudaError_t attn_fused_launch(const float* qkv, const float* P, const float* bias_u, const float* bias_v,
                              const int* row_off, const int2* tiles, int n_tiles, int Tmax, float scale, float* attn,
                              cudaStream_t s);

// The same attention on the tensor cores (attn_rel_tc.cu): one CTA per (128-query tile, head), the products in the
// three-part tf32 split, softmax in the kernel. qkv has `rows` rows (TMA reads past a window's rows, never past
// these); tiles: (window, first query) of every ATT_TC_QT-query tile; err: the device error word of the bounded
// waits. Returns a P2CU code.
constexpr int ATT_TC_QT = 128;
// One CTA's share of a launch (per head): window w, queries q0 .. q0 + 127, key chunks [c0, c1) of 64 keys; split
// `split` of `nsplit` of query tile `group`, whose splits are tiles first .. first + nsplit - 1.
struct AttnTile {
    int w, q0, c0, c1, split, nsplit, group, first;
};
// The tiles of a launch over windows of T[0 .. n_win) frames on a GPU of `sms` SMs: the key chunks split over up to
// four CTAs when the query tiles give fewer than half the SMs a CTA. Returns the tile count; *n_groups the query tiles.
int attn_rel_tc_plan(const int* T, int n_win, int sms, std::vector<AttnTile>& tiles, int* n_groups);
// Device bytes of the split parts of a launch of n_tiles tiles (used only when some tile has nsplit > 1), and the
// launch: parts and counters (n_groups x 8 ints, zero before the first launch; the merging CTA zeroes its own) may be
// null when no tile splits.
size_t attn_rel_tc_part_bytes(int n_tiles);
int attn_rel_tc_launch(const float* qkv, int rows, const float* P, const float* bias_u, const float* bias_v,
                       const int* row_off, const AttnTile* tiles, int n_tiles, int Tmax, float scale, float* attn,
                       void* parts, int* counters, uint32_t* err, cudaStream_t s);

}  // namespace p2cu
