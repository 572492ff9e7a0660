// fv_gemm.h - launch interface of the tcgen05 five-value / int8-table GEMM (fv_gemm.cu). Internal to the library.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace p2cu {

// How the epilogue turns int32 sums into fp32 (the reference's GEMM modes, csrc/blas.c:1316-1336).
enum : int { CM_INT8 = 0, CM_INT8W = 2, CM_Q8B = 8 };

// The B operand: five-value planes expanded to int8w codes, to the two int8-mode planes S and T, or an int8 table.
enum : int { KIND_TABLE = 0, KIND_ST = 1, KIND_CODES = 2 };

struct FvGemmParams {
    int M, N, K;
    float alpha;
    int beta_zero;            // 1: the first 1024-row K block stores into C; 0: every block accumulates into C
    int cmode;                // CM_*
    const float* a_scales;    // [M] per-row scales of the quantised A
    const float* lo;          // [N] five-value magnitudes (CM_INT8, CM_INT8W)
    const float* hi;          // [N]
    const float* scales;      // [N] int8-table column scales (CM_Q8B)
    float* C;
    int ldc;
    int ksplit;               // CTAs along K, one per 1024-row block; > 1 writes per-block f to the workspace slices
    int m_pad;                // rows per workspace slice (M rounded up to 128)
    uint32_t* err;            // device error word (timeouts), first error wins
    long long* trace;         // diagnostic builds only (-DP2CU_TRACE): event timestamps of CTA (0, 0), or null
};

// One launch of the GEMM kernel: tile width bn (64, 128, or 256 for KIND_CODES / KIND_TABLE); for the planes kinds
// b0 = signs [K, N/4] in bn/4 x 128 boxes and b1 = flags [K, N/8] in max(16, bn/8) x 128 boxes, for KIND_TABLE
// b0 = [K, N] in min(bn, 128) x 128 boxes with that many bytes of swizzle. a = int8 A [M, K] in 128 x 128 boxes,
// 128-byte swizzle. out = fp32 C [M, N] (ksplit == 1) or the workspace slices [ksplit * m_pad, N] (ksplit > 1),
// 32 x 128 boxes, 128-byte swizzle.
cudaError_t fv_gemm_launch(int bn, int kind, const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                           const CUtensorMap& out, const FvGemmParams& p, cudaStream_t stream);

// The persistent form of the same GEMM (fv_gemm_p.cu) for launches with many output tiles: same arguments and
// results, one CTA per SM walking the tiles with the epilogue of one tile overlapping the MMAs of the next.
cudaError_t fv_gemm_p_launch(int bn, int kind, const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                             const CUtensorMap& out, const FvGemmParams& p, cudaStream_t stream);
int fv_gemm_p_tiles(int M, int N, int bn, int ksplit);

// The CTA-pair form (fv_gemm_2sm.cu): 256 x 256 output tiles on clusters of two CTAs (tcgen05 cta_group::2), for
// KIND_TABLE and KIND_CODES with N % 256 == 0. The A and B maps are those of bn = 128 (each CTA loads a 128-column
// half of B); the output map's box is 32 x 32 (each epilogue warp stores its own 32-row blocks).
cudaError_t fv_gemm_2sm_launch(int kind, const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                               const CUtensorMap& out, const FvGemmParams& p, cudaStream_t stream);
int fv_gemm_2sm_tiles(int M, int N, int ksplit);
int fv_gemm_p_min_tiles();   // the SM count: below it every tile has an SM of its own anyway

// The same GEMM as a plain SIMT kernel (fv_gemm_simt.cu) for shapes the tensor-core kernels do not take (N % 128,
// K % 16, unaligned C): B from the planes (signs [K, N/4], flags [K, N/8]) or from `table` [K, ldb] (an int8 table, or
// the int8w code cache with ldb = N); no workspace, K blocks folded in registers.
cudaError_t fv_gemm_simt_launch(const int8_t* q, const uint8_t* signs, const uint8_t* flags, const int8_t* table,
                                int ldb, const FvGemmParams& p, cudaStream_t stream);

// The int8w GEMM with the weights in tensor memory (fv_gemm_t.cu), for few rows: 128 output columns x MT rows per
// CTA (MT = fv_gemm_t_rows(...), a multiple of 16 up to 128), one 1024-row K block per CTA. B comes as the value-index
// plane of p2cu_fv_pack_vindex (vindex, kchunks = ceil(K / 32) chunks of N x 16 bytes); a = int8 A [M, K] in
// 128 x MT boxes (128-byte swizzle). N % 128 == 0. ksplit > 1 writes f per block to ws slices [ksplit][m_pad][N] for
// fv_combine_launch.
struct FvGemmTParams {
    int M, N, K;
    float alpha;
    int beta_zero;
    const float* a_scales;
    const float* lo;
    const float* hi;
    const uint32_t* vindex;
    int kchunks;
    float* C;
    int ldc;
    float* ws;
    int ksplit;
    int m_pad;
    uint32_t* err;
    int trace_slot;   // diagnostic builds only (-DP2CU_TRACE): the launch's slot in the trace ring
};
// Rows per CTA for an M x N GEMM of ksplit K blocks on a GPU of `sms` SMs.
int fv_gemm_t_rows(int M, int N, int ksplit, int sms);
cudaError_t fv_gemm_t_launch(int mt, const CUtensorMap& a, const FvGemmTParams& p, cudaStream_t stream);
// The value-index plane of a five-value weight (p2cu_fv_pack_vindex): [ceil(K/32)][N][4] 32-bit words.
cudaError_t fv_vindex_launch(const uint8_t* signs, const uint8_t* flags, int K, int N, uint32_t* out,
                             cudaStream_t stream);

// C = fold of the workspace slices (fp32 f per 1024-row block) in block order, with the row scales.
cudaError_t fv_combine_launch(const float* f, int m_pad, int nblk, const float* a_scales, float alpha, int beta_zero,
                              float* C, int M, int N, int ldc, cudaStream_t stream);

}  // namespace p2cu
