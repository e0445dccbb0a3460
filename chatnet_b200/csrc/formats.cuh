// formats.cuh -- GGUF block formats (Q4_0, Q4_K, Q6_K) on the device.
//
// Two kinds of decode live here:
//  * bit-exact scalar dequantization that follows the reference's rounding
//    order (DequantQ4_0.cs:28-58, DequantQ4K.cs:37-77, DequantQ6K.cs:37-88);
//  * register decode of packed nibbles straight into mma.sync A fragments
//    for the GEMVs.  Quantized integers are exact in fp16, so the tensor
//    core sees the same integer weights as the reference; block scales are
//    applied to the fp32 partial sums afterwards.
#pragma once

#include "cn_common.cuh"

namespace cn {

// ---- bit-exact scalar decode ------------------------------------------------

__device__ __forceinline__ float ld_half(const uint8_t* p) {
    return half_bits_to_float((uint16_t)(p[0] | (p[1] << 8)));
}

// DequantQ4K.DecodeScales (DequantQ4K.cs:218-241) for sub-block j.
__device__ __forceinline__ void q4k_scale_min(const uint8_t* q, int j, int& sc, int& m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// ---- GEMV fragment decode -------------------------------------------------
//
// mma.m16n8k16 k-slot permutation used by every format: lane (g, t) holds,
// for each 16-position k-step, positions 4t..4t+3 of that step as
//   A reg (row r, slots 2t,2t+1)   = half2(w[r][4t+0], w[r][4t+2])
//   A reg (row r, slots 2t+8,2t+9) = half2(w[r][4t+1], w[r][4t+3])
// and the activation fragments (built by the x-prep kernel) use the same
// mapping, so the dot product over the 16 positions is unchanged.

constexpr uint32_t kMagic = 0x64006400u;  // half2(1024, 1024)

// Low nibbles of bytes 0/2 and 1/3 of w as half2 (1024 + q).
__device__ __forceinline__ void nib_lo(uint32_t w, uint32_t& a02, uint32_t& a13) {
    a02 = lop3_and_or(w, 0x000F000Fu, kMagic);
    a13 = lop3_and_or(w >> 8, 0x000F000Fu, kMagic);
}
// High nibbles as half2 (1024 + 16 q).
__device__ __forceinline__ void nib_hi(uint32_t w, uint32_t& a02, uint32_t& a13) {
    a02 = lop3_and_or(w, 0x00F000F0u, kMagic);
    a13 = lop3_and_or(w >> 8, 0x00F000F0u, kMagic);
}

}  // namespace cn
