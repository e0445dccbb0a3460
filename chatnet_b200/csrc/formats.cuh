// formats.cuh -- GGUF block formats (Q4_0, Q4_K, Q6_K; Q4_1, Q5_0, Q5_1, Q8_0
// through the generic paths) on the device.
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

// Element j (0..31) of one 32-weight block of Q4_1, Q5_0, Q5_1 or Q8_0, with
// the reference's operation order (no fused multiply-add):
//   Q4_1  q * d + m, q the low (j < 16) or high nibble of byte j % 16
//                                          DequantQ4_1.cs:24-56 (d@0, m@2, qs@4)
//   Q5_0  (q5 - 16) * d, q5 = nibble | bit j of qh << 4
//                                          DequantQ5_0.cs:29-68 (d@0, qh@2, qs@6)
//   Q5_1  q5 * d + m                       DequantQ5_1.cs:30-69 (d@0, m@2, qh@4, qs@8)
//   Q8_0  (sbyte)q * d                     DequantQ8_0.cs:19-41 (d@0, qs@2)
// DequantIQ.IQ4NL_Table (DequantIQ.cs:29-33), the 16 levels of IQ4_NL / IQ4_XS.
__device__ __forceinline__ float iq4nl_level(int i) {
    const int8_t lv[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
    return (float)lv[i];
}

__device__ __forceinline__ float block32_elem(int type, const uint8_t* p, int j) {
    if (type == CN_TYPE_Q8_0) return __fmul_rn((float)(int8_t)p[2 + j], ld_half(p));
    if (type == CN_TYPE_IQ4_NL) {
        // scale * table[nibble] (DequantIQ.cs:45-76; d@0, qs@2 as Q4_0)
        const uint8_t byte = p[2 + (j & 15)];
        return __fmul_rn(ld_half(p), iq4nl_level(j < 16 ? (byte & 0x0F) : (byte >> 4)));
    }
    const int qs_off = type == CN_TYPE_Q4_1 ? 4 : type == CN_TYPE_Q5_0 ? 6 : 8;
    const uint8_t byte = p[qs_off + (j & 15)];
    int q = j < 16 ? (byte & 0x0F) : ((byte >> 4) & 0x0F);
    if (type != CN_TYPE_Q4_1) {
        const int qh_off = type == CN_TYPE_Q5_0 ? 2 : 4;
        const uint32_t qh = (uint32_t)p[qh_off] | ((uint32_t)p[qh_off + 1] << 8) | ((uint32_t)p[qh_off + 2] << 16) |
                            ((uint32_t)p[qh_off + 3] << 24);
        q |= (int)((qh >> j) & 1u) << 4;
    }
    if (type == CN_TYPE_Q5_0) return __fmul_rn((float)(q - 16), ld_half(p));
    return __fadd_rn(__fmul_rn((float)q, ld_half(p)), ld_half(p + 2));
}

// Element e (0..255) of one super-block of Q2_K, Q3_K, Q5_K, Q8_K or IQ4_XS,
// with the reference's operation order (no fused multiply-add):
//   Q2_K  d*(sc&15) * q2 - dmin*(sc>>4); element e: group e/128, 2-bit shift
//         2*((e/32)%4), half (e/16)%2, scale byte 8g + 2*shift + half, quant
//         byte 16 + 32g + 16*half + e%16        DequantQ2K.cs:32-88 (d@80, dmin@82)
//   Q3_K  d * sc * (q3 - 4), sc 6-bit - 32 (DecodeScales), q3 = 2 bits of
//         qs[e/4] | hmask bit e%8 of byte e/8 << 2
//                                              DequantQ3K.cs:35-70, :124-148 (d@108)
//   Q5_K  d*sc * q5 - dmin*m (scales as Q4_K), q5 = nibble | qh bit << 4
//                                              DequantQ5K.cs:36-90 (qh@16, qs@48)
//   Q8_K  (sbyte)q * d, d fp32                 DequantQ8K.cs:25-47
//   IQ4_XS d*sc * table[nibble], sc = ((byte 4+sub & 63) | 2 bits of the
//         uint16 at 2 << 6) - 32               DequantIQ.cs:143-180 (qs@8)
// and the reference's own simplified decodes of the importance-quantised
// types (no codebook grids; d, fp16 at byte 0, then):
//   IQ3_S   (d*sc) * q3, negated by sign bit e%8 of byte 98 + e/8; q3 = 2 bits
//           of qs[e/4] | qh bit e%8 of byte 66 + e/8 << 2; sc = 2 bits of
//           byte 130 + e/32 + 1                DequantIQ.cs:244-290
//           (the sign and scale bytes lie past the 110-byte block: the next
//           block's bytes inside a tensor, read as 0 from `end` on)
//   IQ3_XXS d * (q3 - 4), q3 = 3 bits 3(e%8) of the 24-bit group at 2 + 3(e/8)
//                                              DequantIQ.cs:364-398
//   IQ2_XS  (d*sc) * (q - 1), q = 2 bits of byte 2 + e/4; sc = nibble e/16%2
//           of byte 66 + e/32, - 8             DequantIQ.cs:456-495
//   IQ2_XXS d * (q - 1)                        DequantIQ.cs:568-597
//   IQ2_S   (d*sc) * q, sc = low nibble of byte 66 + e/16, + 1; elements 0-3
//           of each 16 negated by the high nibble's bits
//                                              DequantIQ.cs:656-695
//   IQ1_S   d, -d or 0: bit e%8 of qs byte 2 + e/8, else bit
//           4(e/8 % 2) + (e%8)/2 of qh byte 34 + e/16
//                                              DequantIQ.cs:767-805
//   IQ1_M   as IQ1_S times sc = 1 or 0.5 (bit (e/8)%8 of byte 50 + e/64)
//                                              DequantIQ.cs:869-912
__device__ __forceinline__ float iq_elem(int type, const uint8_t* p, int e, const uint8_t* end) {
    const float d = ld_half(p);
    if (type == CN_TYPE_IQ3_S) {
        const int sub = e >> 3, j = e & 7;
        const uint8_t* ps = p + 130 + (sub >> 2);
        const uint8_t* pg = p + 98 + sub;
        const int sc = (((ps < end ? *ps : 0) >> (2 * (sub & 3))) & 3) + 1;
        const int q3 = ((p[2 + (e >> 2)] >> (2 * (e & 3))) & 3) | (((p[66 + (e >> 3)] >> (e & 7)) & 1) << 2);
        const float v = __fmul_rn(__fmul_rn(d, (float)sc), (float)q3);
        return (((pg < end ? *pg : 0) >> j) & 1) ? -v : v;
    }
    if (type == CN_TYPE_IQ3_XXS) {
        const uint8_t* g = p + 2 + 3 * (e >> 3);
        const uint32_t packed = (uint32_t)g[0] | ((uint32_t)g[1] << 8) | ((uint32_t)g[2] << 16);
        return __fmul_rn(d, (float)((int)((packed >> (3 * (e & 7))) & 7u) - 4));
    }
    if (type == CN_TYPE_IQ2_XS || type == CN_TYPE_IQ2_XXS || type == CN_TYPE_IQ2_S) {
        const int sub = e >> 4, r = e & 15;
        const int q = (p[2 + 4 * sub + (r >> 2)] >> (2 * (r & 3))) & 3;
        if (type == CN_TYPE_IQ2_XXS) return __fmul_rn(d, (float)(q - 1));
        if (type == CN_TYPE_IQ2_XS) {
            const int sb = p[66 + (sub >> 1)];
            const int sc = ((sub & 1) ? ((sb >> 4) & 0x0F) : (sb & 0x0F)) - 8;
            return __fmul_rn(__fmul_rn(d, (float)sc), (float)(q - 1));
        }
        const int qh = p[66 + sub];
        const float v = __fmul_rn(__fmul_rn(d, (float)((qh & 0x0F) + 1)), (float)q);
        return (r < 4 && ((qh >> (4 + r)) & 1)) ? -v : v;
    }
    // IQ1_S, IQ1_M
    const int sub = e >> 3, j = e & 7;
    const int bit = (p[2 + sub] >> j) & 1;
    const int hbit = (p[34 + (sub >> 1)] >> (4 * (sub & 1) + (j >> 1))) & 1;
    float w = d;
    if (type == CN_TYPE_IQ1_M) w = __fmul_rn(d, ((p[50 + (sub >> 3)] >> (sub & 7)) & 1) ? 1.0f : 0.5f);
    return bit ? w : hbit ? -w : 0.0f;
}

// `end`: one past the last byte an IQ3_S decode may read (see above).
__device__ __forceinline__ float superblock_elem(int type, const uint8_t* p, int e, const uint8_t* end) {
    if (type == CN_TYPE_IQ2_XXS || type == CN_TYPE_IQ2_XS || type == CN_TYPE_IQ3_XXS || type == CN_TYPE_IQ1_S ||
        type == CN_TYPE_IQ3_S || type == CN_TYPE_IQ2_S || type == CN_TYPE_IQ1_M)
        return iq_elem(type, p, e, end);
    if (type == CN_TYPE_Q2_K) {
        const int g = e >> 7, si = (e >> 5) & 3, h = (e >> 4) & 1;
        const int sb = p[8 * g + 2 * si + h];
        const float dl = __fmul_rn(ld_half(p + 80), (float)(sb & 0x0F));
        const float ml = __fmul_rn(ld_half(p + 82), (float)((sb >> 4) & 0x0F));
        const int q = (p[16 + 32 * g + 16 * h + (e & 15)] >> (2 * si)) & 3;
        return __fsub_rn(__fmul_rn(dl, (float)q), ml);
    }
    if (type == CN_TYPE_Q3_K) {
        const int k = e >> 4;
        const uint8_t* sc8 = p + 96;
        int sc = k < 8 ? (sc8[k] & 0x0F) : ((sc8[k - 8] >> 4) & 0x0F);
        sc = (sc | (((sc8[8 + (k & 3)] >> (2 * (k >> 2))) & 3) << 4)) - 32;
        const int q3 = ((p[32 + (e >> 2)] >> (2 * (e & 3))) & 3) | (((p[e >> 3] >> (e & 7)) & 1) << 2);
        return __fmul_rn(__fmul_rn(ld_half(p + 108), (float)sc), (float)(q3 - 4));
    }
    if (type == CN_TYPE_Q5_K) {
        const int sub = e >> 5, j = e & 31;
        int sc, m;
        q4k_scale_min(p + 4, sub, sc, m);
        const float dsc = __fmul_rn(ld_half(p), (float)sc), dm = __fmul_rn(ld_half(p + 2), (float)m);
        const uint8_t byte = p[48 + 16 * sub + (j & 15)];
        const int q5 = (j < 16 ? (byte & 0x0F) : (byte >> 4)) | (((p[16 + (e >> 3)] >> (e & 7)) & 1) << 4);
        return __fsub_rn(__fmul_rn(dsc, (float)q5), dm);
    }
    if (type == CN_TYPE_Q8_K) {
        const uint32_t u = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
        return __fmul_rn((float)(int8_t)p[4 + e], __uint_as_float(u));
    }
    // IQ4_XS
    const int sub = e >> 5, j = e & 31;
    const int sh = p[2] | (p[3] << 8);
    const int sc = ((p[4 + sub] & 0x3F) | (((sh >> (2 * sub)) & 3) << 6)) - 32;
    const uint8_t byte = p[8 + 16 * sub + (j & 15)];
    return __fmul_rn(__fmul_rn(ld_half(p), (float)sc), iq4nl_level(j < 16 ? (byte & 0x0F) : (byte >> 4)));
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
