// fv_common.cuh - device helpers shared by the five-value GEMM kernels (fv_gemm.cu, fv_gemm_p.cu): plane expansion
// into int8 operand bytes, clo, and the swizzled shared-memory offsets.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace p2cu {

// Byte masks from bits: byte p of the result is 0xFF when bit 7 of byte p of x is set. PTX prmt with the selector's
// sign bit set replicates the selected byte's top bit (the __byte_perm intrinsic only uses the low three bits).
__device__ __forceinline__ uint32_t msb_mask(uint32_t x) {
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, 0xBA98;" : "=r"(r) : "r"(x));
    return r;
}

// The planes of 32 columns of one K row in "column-transposed" words: word j holds, at byte p, column 8p + j of the
// group. x0, x1 are the 8 sign bytes of the columns and fw their 32 flag bits; u / v gather the sign bytes of
// columns 0-3, 8-11, 16-19, 24-27 / 4-7, 12-15, 20-23, 28-31, so for word j the 2-bit code of each column sits at
// bits 2 (j mod 4), 2 (j mod 4) + 1 of its byte and its flag at bit j of its byte of fw. The epilogue undoes the
// transposition with compile-time register indexing.
struct Planes32 {
    uint32_t u, v, fw;
    __device__ __forceinline__ void load(uint32_t x0, uint32_t x1, uint32_t f) {
        u = __byte_perm(x0, x1, 0x6420);
        v = __byte_perm(x0, x1, 0x7531);
        fw = f;
    }
    // Byte masks of word j: code 2 (+1), code 1 (0), and the magnitude flag.
    __device__ __forceinline__ void masks(int j, uint32_t& pos, uint32_t& zero, uint32_t& hi) const {
        const uint32_t src = j < 4 ? u : v;
        const int b = 2 * (j & 3);
        pos = msb_mask(src << (6 - b));    // bit b + 1 -> bit 7
        zero = msb_mask(src << (7 - b));   // bit b -> bit 7
        hi = msb_mask(fw << (7 - j));      // bit j -> bit 7
    }
};

// S = sign (+1 / 0 / -1) and T = sign * flag as int8 bytes.
__device__ __forceinline__ void expand_st(const Planes32& pl, uint32_t (&S)[8], uint32_t (&T)[8]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t pos, zero, hi;
        pl.masks(j, pos, zero, hi);
        // +1 = 0x01 (pos), 0 = 0x00 (zero), -1 = 0xFF (neither)
        const uint32_t s = (pos & 0x01010101u) | (~pos & ~zero);
        S[j] = s;
        T[j] = s & hi;
    }
}

// The int8w codes sign * (flag ? 127 : clo) with this thread's per-column clo bytes (same word layout).
__device__ __forceinline__ void expand_codes(const Planes32& pl, const uint32_t (&clo)[8], const uint32_t (&nclo)[8],
                                             uint32_t (&W)[8]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t pos, zero, hi;
        pl.masks(j, pos, zero, hi);
        const uint32_t mag = (hi & 0x7F7F7F7Fu) | (~hi & clo[j]);     // 127 or clo
        const uint32_t nmag = (hi & 0x81818181u) | (~hi & nclo[j]);   // -127 or -clo
        W[j] = (mag & pos) | (nmag & ~zero & ~pos);
    }
}

// clo = clamp(rint(127 * lo / hi), 0, 127), 0 when hi <= 0 (csrc/blas.c:1319-1324, IEEE division).
__device__ __forceinline__ int clo_of(float lo, float hi) {
    const int c = hi > 0.f ? __float2int_rn(__fdiv_rn(__fmul_rn(127.0f, lo), hi)) : 0;
    return c < 0 ? 0 : c > 127 ? 127 : c;
}

// Byte offset of (row k, 16-byte chunk c) in an MN-major atom column W bytes wide, 8-row swizzle atoms
// (128-byte mode: chunk ^= k mod 8; 64-byte mode: chunk ^= (k / 2) mod 4 - the address bits 7-8 of the row).
template <int W>
__device__ __forceinline__ uint32_t b_offset(int k, int c) {
    const int swz = W == 128 ? (k & 7) : ((k >> 1) & 3);
    return static_cast<uint32_t>((k >> 3) * (8 * W) + (k & 7) * W + ((c ^ swz) << 4));
}

// Byte offset of (row r, float4 chunk j) in a 128-row x 32-float staging tile with 128-byte swizzle.
__device__ __forceinline__ uint32_t out_offset(int r, int j) {
    return static_cast<uint32_t>(r * 128 + ((j ^ (r & 7)) << 4));
}

}  // namespace p2cu
