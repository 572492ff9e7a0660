// tf32_split.cuh - fp32 operands for the three-part tf32 tensor-core products (attn_tc.cu, attn_rel_tc.cu).
//
// Every operand value x becomes hi = x rounded to the tf32 grid and lo = x - hi (exact in fp32); a product of two
// operands is then hi*hi + hi*lo + lo*hi, three kind::tf32 MMAs into one fp32 accumulator, which keeps about the
// accuracy of an fp32 dot product (the dropped lo*lo term and the tf32 truncation of lo are near 2^-21 of a term).
// The operand tiles are K-major with 16 fp32 (64 bytes) per row and the 64-byte swizzle the MMA descriptors name.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace p2cu {

// x rounded to the tf32 grid (10 explicit mantissa bits, ties away from zero) and the exact remainder.
__device__ __forceinline__ void tf32_split(float x, float& hi, float& lo) {
    hi = __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
    lo = __fsub_rn(x, hi);
}

// Byte offset of (row r, 16-byte chunk c) in a K-major tile of 64-byte rows with the 64-byte swizzle (8-row groups
// of 512 bytes; chunk c of row r sits at chunk c ^ ((r >> 1) & 3)).
__device__ __forceinline__ uint32_t kmaj_off(int r, int c) {
    return static_cast<uint32_t>((r >> 3) * 512 + (r & 7) * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

// The four values of v split into the hi tile and the lo tile at the same offset.
__device__ __forceinline__ void store_split(uint8_t* hi_tile, uint8_t* lo_tile, uint32_t off, float4 v) {
    float4 h, l;
    tf32_split(v.x, h.x, l.x);
    tf32_split(v.y, h.y, l.y);
    tf32_split(v.z, h.z, l.z);
    tf32_split(v.w, h.w, l.w);
    *reinterpret_cast<float4*>(hi_tile + off) = h;
    *reinterpret_cast<float4*>(lo_tile + off) = l;
}

}  // namespace p2cu
