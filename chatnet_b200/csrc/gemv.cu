// gemv.cu -- fused dequant-GEMV for decode (batch 1..32), sm_100a.
//
// Replaces TensorMath.MatVecMulQ4_0 / MatVecMulQ6K / MatVecMulGeneric(Q4_K)
// (Tensors/TensorMath.cs:548-656) and the per-row DotProduct kernels
// (DequantQ4_0.cs:80-149, DequantQ4K.cs:89-163, DequantQ6K.cs:104-188).
//
// Design (HBM-bound at small batch):
//  * The packed GGUF rows stay untouched in HBM.  Each warp runs its own
//    TMA pipeline: lane 0 streams [16 rows x 256 positions] tiles of raw
//    blocks into shared memory (cp.async.bulk.tensor.2d, 8-byte elements,
//    zero-filled past the edges), kStages deep, tracked by mbarriers.
//  * Decode happens in registers: nibbles become fp16 integers with the
//    1024-magic LOP3 trick (exact), laid out directly as mma.m16n8k16 A
//    fragments.  The activation fragments come from a prep kernel that
//    splits x into fp16 hi + lo parts (x = hi + lo to ~2^-22 relative), so
//    the tensor-core product keeps fp32-level accuracy.  Batch columns
//    are interleaved (col 2b = hi of x_b, 2b+1 = lo of x_b): lane (g,t)
//    ends up owning batch t's result for rows g and g+8 with no shuffle.
//  * Block scales are applied in fp32 to the per-block mma results
//    (Q4_0: d per 32; Q4_K: d*sc per 32 minus dmin*m*sum(x); Q6_K: d*sc
//    per 16).
//  * Work is scheduled stream-K style: the (16-row tile, 256-position unit)
//    space is cut into equal contiguous ranges, one per resident warp.
//    Tiles shared by several warps are combined through scratch partials
//    by the last warp to arrive, in warp order (deterministic).
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "cn_common.cuh"
#include "cn_internal.h"
#include "formats.cuh"
#include "gemv_i8.cuh"
#include "gemv_tc.cuh"
#include "prep.cuh"

namespace cn {

// CTA shape: 8 consumer warps (16 rows each, one mma m-tile) and 1 producer
// warp that streams 128-row x 256-position units into a ring of stages.
constexpr int kCons = 8;
constexpr int kThreads = (kCons + 1) * 32;
constexpr int kTileRows = 16 * kCons;

template <int TYPE>
struct Fmt;
template <>
struct Fmt<CN_TYPE_Q4_0> {
    static constexpr int kBox = 144;  // bytes per row per unit (8 blocks of 18)
    __device__ static int box_x(int u) { return 18 * u; }  // uint64 elements
    __device__ static int offset(int) { return 0; }
};
// Q4_1 / Q5_0 / Q5_1: eight 20 / 22 / 24-byte blocks per row and unit
template <>
struct Fmt<CN_TYPE_Q4_1> {
    static constexpr int kBox = 160;
    __device__ static int box_x(int u) { return 20 * u; }
    __device__ static int offset(int) { return 0; }
};
template <>
struct Fmt<CN_TYPE_Q5_0> {
    static constexpr int kBox = 176;
    __device__ static int box_x(int u) { return 22 * u; }
    __device__ static int offset(int) { return 0; }
};
template <>
struct Fmt<CN_TYPE_Q5_1> {
    static constexpr int kBox = 192;
    __device__ static int box_x(int u) { return 24 * u; }
    __device__ static int offset(int) { return 0; }
};
template <>
struct Fmt<CN_TYPE_Q8_0> {
    static constexpr int kBox = 272;  // bytes per row per unit (8 blocks of 34)
    __device__ static int box_x(int u) { return 34 * u; }
    __device__ static int offset(int) { return 0; }
};
template <>
struct Fmt<CN_TYPE_Q5_K> {
    static constexpr int kBox = 176;  // one 176-byte super-block (qh@16, qs@48)
    __device__ static int box_x(int u) { return 22 * u; }
    __device__ static int offset(int) { return 0; }
};
template <>
struct Fmt<CN_TYPE_Q4_K> {
    static constexpr int kBox = 144;  // one 144-byte super-block
    __device__ static int box_x(int u) { return 18 * u; }
    __device__ static int offset(int) { return 0; }
};
template <>
struct Fmt<CN_TYPE_Q6_K> {
    // 210-byte super-blocks are only 2-byte aligned: load the 16-byte
    // aligned 240-byte window that covers super-block u and index into it.
    static constexpr int kBox = 240;
    __device__ static int box_x(int u) { return ((210 * u) >> 4) * 2; }
    __device__ static int offset(int u) { return (210 * u) & 15; }
};

// Shared-memory geometry of one (format, n-tiles) instantiation.
template <int TYPE, int NT>
struct Geo {
    static constexpr int kW = Fmt<TYPE>::kBox * kTileRows;             // raw blocks
    static constexpr int kXF = 8 * NT * 32 * 16;                        // B fragments
    static constexpr bool kKQ = TYPE == CN_TYPE_Q4_K || TYPE == CN_TYPE_Q5_K;  // scales and mins
    // chunk sums of x: the min terms of Q4_K / Q5_K and of Q4_1 / Q5_1
    static constexpr bool kMin = kKQ || TYPE == CN_TYPE_Q4_1 || TYPE == CN_TYPE_Q5_1;
    static constexpr int kXS = kMin ? 8 * NT * 4 * 4 : 0;
    static constexpr int kXI = NT * 4 * 4;                              // unit 2^-e per column
    static constexpr int kXIpad = (kXI + 127) / 128 * 128;
    static constexpr int kBytes = kW + kXF + kXS + kXI;                 // bytes landing per stage
    static constexpr int kStage = kW + kXF + kXS + kXIpad;              // multiple of 128
    static constexpr int kTable = kKQ ? kCons * 16 * 8 * 8 : 0;
    static constexpr int kFixed = kTable + 64 * 16;                     // table + barriers
    // Two CTAs per SM when three or more stages fit in half the SM's shared
    // memory; otherwise one CTA with up to six stages.
    static constexpr int kHalf = 113 * 1024;
    static constexpr int kFull = 225 * 1024;
    static constexpr int kS2 = (kHalf - kFixed) / kStage;
    static constexpr int kStages = kS2 >= 3 ? (kS2 > 4 ? 4 : kS2)
                                            : ((kFull - kFixed) / kStage > 6 ? 6 : (kFull - kFixed) / kStage);
    static constexpr int kMinCtas = kS2 >= 3 ? 2 : 1;
    static constexpr int kSmem = kFixed + kStages * kStage;
    // cluster split (batch 1-8): one slot of a CTA's sums, and the most
    // slots the leader can add past kSmem within the 227 KB a CTA may use
    static constexpr int kSlotB = kTileRows * NT * 4 * 4;
    static constexpr int kClusMax =
        NT > 2 ? 0 : ((227 * 1024 - kSmem) / kSlotB > 7 ? 7 : (227 * 1024 - kSmem) / kSlotB);
};

// Up to three matrices with the same input run as one launch (q/k/v,
// gate/up): their 128-row tiles are numbered one after another, matrix m
// owning tiles [toff[m], toff[m + 1]); nmat == 1 uses rows / y.
constexpr int kMaxGroup = 3;
struct GemvMaps {
    CUtensorMap m[kMaxGroup];
};

struct GemvArgs {
    int64_t rows;
    int nmat;
    int toff[kMaxGroup + 1];
    int64_t mrows[kMaxGroup];
    float* my[kMaxGroup];
    int units;  // 256-position units per row
    int tiles;  // 128-row tiles
    int batch;
    const uint4* xfrag;  // [chunk][nt][32 lanes]
    const float* xsum;   // [chunk][nt*4]
    const float* xinv;   // [unit][nt*4] 2^-e of each unit's activation scaling
    float* y;            // [batch][rows]
    float* partials;     // [2 * ctas][128 rows][nt*4] stream-K partial slots
    int* counters;       // [tiles * kCons]
    uint32_t* err;
    int csize;           // > 1: CTAs csize*k .. csize*k + csize-1 (one cluster) split tile k (cluster_finish_mma)
};

// 32-bit word at byte offset `off` of a 4-byte aligned shared row, where
// off % 4 is known at compile time (0 or 2).
template <int MIS>
__device__ __forceinline__ uint32_t word_at(const uint8_t* row, int off) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(row + (off & ~3));
    if constexpr (MIS == 0) return w[0];
    else return __byte_perm(w[0], w[1], 0x5432);
}

// 32-bit word at a 2-byte aligned address whose misalignment (0 or 2) is a
// compile-time constant.
template <int MIS>
__device__ __forceinline__ uint32_t word2(const uint8_t* p) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(p - MIS);
    if constexpr (MIS == 0) return w[0];
    else return __byte_perm(w[0], w[1], 0x5432);
}

// Exact float of an unsigned byte via the 2^23 magic (no I2F).
__device__ __forceinline__ float ubyte_f(uint32_t w, int k) {
    return __int_as_float(0x4B000000 | ((w >> (8 * k)) & 0xFF)) - 8388608.0f;
}
__device__ __forceinline__ float sbyte_f(uint32_t w, int k) {
    return (float)(int8_t)((w >> (8 * k)) & 0xFF);
}

__device__ __forceinline__ void fma2(float& a0, float& a1, float t0, float t1, float s) {
    // (a0, a1) += (t0, t1) * s with the packed fp32x2 FMA of sm_100
    uint64_t acc, tv, sv;
    asm("mov.b64 %0, {%1, %2};" : "=l"(acc) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(tv) : "f"(t0), "f"(t1));
    asm("mov.b64 %0, {%1, %1};" : "=l"(sv) : "f"(s));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(tv), "l"(sv));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(acc));
}

// Padding columns of the fragments are zero in shared memory, so every lane
// loads unconditionally (no divergence).
template <int NT>
__device__ __forceinline__ uint4 bfrag(const uint4* xf, int c, int nt, int lane, bool) {
    return xf[(c * NT + nt) * 32 + lane];
}

// ---- per-unit consumers (one warp, 16 rows) ----------------------------------

template <int NT>
__device__ __forceinline__ void unit_q4_0(const uint8_t* stw, const uint4* xf, int row0, int g,
                                          int t, int lane, const bool* live, float (&acc)[NT][4]) {
    const uint8_t* rg = stw + (row0 + g) * 144;
    const uint8_t* rh = rg + 8 * 144;
    const uint32_t k1032 = 0x64086408u;  // half2(1032, 1032)
    const uint32_t k1_16 = 0x2C002C00u;  // half2(1/16, 1/16)
    const uint32_t km72 = 0xD480D480u;   // half2(-72, -72)
#pragma unroll
    for (int b = 0; b < 8; b++) {
        float dg = half_bits_to_float(lds_u16(rg + 18 * b));
        float dh = half_bits_to_float(lds_u16(rh + 18 * b));
        uint32_t wg, wh;
        if (b & 1) {
            wg = word_at<0>(rg, 18 * b + 2 + 4 * t);
            wh = word_at<0>(rh, 18 * b + 2 + 4 * t);
        } else {
            wg = word_at<2>(rg, 18 * b + 2 + 4 * t);
            wh = word_at<2>(rh, 18 * b + 2 + 4 * t);
        }
        // (1024 + q) - 1032 = q - 8 and (1024 + 16q)/16 - 72 = q - 8, exact
        uint32_t a0[4], a1[4], p, q;
        nib_lo(wg, p, q);
        a0[0] = h2_sub(p, k1032);
        a0[2] = h2_sub(q, k1032);
        nib_lo(wh, p, q);
        a0[1] = h2_sub(p, k1032);
        a0[3] = h2_sub(q, k1032);
        nib_hi(wg, p, q);
        a1[0] = h2_fma(p, k1_16, km72);
        a1[2] = h2_fma(q, k1_16, km72);
        nib_hi(wh, p, q);
        a1[1] = h2_fma(p, k1_16, km72);
        a1[3] = h2_fma(q, k1_16, km72);
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            uint4 bx = bfrag<NT>(xf, b, nt, lane, live[nt]);
            float tmp[4];
            const float z[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t b0[2] = {bx.x, bx.y}, b1[2] = {bx.z, bx.w};
            mma_16816(tmp, a0, b0, z);
            mma_16816(tmp, a1, b1, tmp);
            fma2(acc[nt][0], acc[nt][1], tmp[0], tmp[1], dg);
            fma2(acc[nt][2], acc[nt][3], tmp[2], tmp[3], dh);
        }
    }
}

// Q4_1 (DequantQ4_1.cs:24-56, 134-171; d@0, m@2, qs@4), Q5_0
// (DequantQ5_0.cs:29-68, 77-114; d@0, qh@2, qs@6) and Q5_1 (DequantQ5_1.cs:
// 30-69, 78-119; d@0, m@2, qh@4, qs@8): Q4_0's nibble layout (byte i: low
// nibble = element i, high nibble = element 16 + i), Q5's fifth bit of
// element j at bit j of qh.  Each element enters the A fragment as the exact
// fp16 1024 + q (low nibbles) or 1024 + 16 q (high nibbles), the fifth bit
// ORed in at mantissa bit 4 or 8; one subtraction or FMA takes it to q (Q4_1,
// Q5_1) or q - 16 (Q5_0).  d scales the block's fp32 partial sums and m times
// the block's x sum (the chunk sums) joins the row, as the reference's
// blockSum * d + inputSum * m.
template <int TYPE>
struct B32 {
    static constexpr int kBpb = TYPE == CN_TYPE_Q4_1 ? 20 : TYPE == CN_TYPE_Q5_0 ? 22 : 24;
    static constexpr int kQs = TYPE == CN_TYPE_Q4_1 ? 4 : TYPE == CN_TYPE_Q5_0 ? 6 : 8;
    static constexpr int kQh = TYPE == CN_TYPE_Q5_0 ? 2 : 4;
    static constexpr bool kQ5 = TYPE != CN_TYPE_Q4_1, kM = TYPE != CN_TYPE_Q5_0;
};

// the fifth bits of elements e, e + 2 (of qh) at bits 0 and 16
__device__ __forceinline__ uint32_t qh_pair(uint32_t qh, int e) {
    return ((qh >> e) & 1u) | (((qh >> (e + 2)) & 1u) << 16);
}

template <int TYPE, int NT, int B>
__device__ __forceinline__ void block_b32(const uint8_t* rg, const uint8_t* rh, const uint4* xf, const float* xs,
                                          int t, int lane, const bool* live, float (&acc)[NT][4]) {
    using F = B32<TYPE>;
    constexpr int o = F::kBpb * B;
    constexpr uint32_t kLo = F::kM ? 0x64006400u : 0x64106410u;  // half2(1024) or half2(1040)
    constexpr uint32_t kHi = F::kM ? 0xD400D400u : 0xD500D500u;  // half2(-64) or half2(-80)
    const uint32_t k1_16 = 0x2C002C00u;                          // half2(1/16)
    const float dg = half_bits_to_float(lds_u16(rg + o)), dh = half_bits_to_float(lds_u16(rh + o));
    float mg = 0.f, mh = 0.f;
    if constexpr (F::kM) {
        mg = half_bits_to_float(lds_u16(rg + o + 2));
        mh = half_bits_to_float(lds_u16(rh + o + 2));
    }
    constexpr int qmis = (o + F::kQs) & 3;
    const uint32_t wg = word_at<qmis>(rg, o + F::kQs + 4 * t), wh = word_at<qmis>(rh, o + F::kQs + 4 * t);
    uint32_t a0[4], a1[4], p, q;
    nib_lo(wg, p, q);
    a0[0] = p;
    a0[2] = q;
    nib_lo(wh, p, q);
    a0[1] = p;
    a0[3] = q;
    nib_hi(wg, p, q);
    a1[0] = p;
    a1[2] = q;
    nib_hi(wh, p, q);
    a1[1] = p;
    a1[3] = q;
    if constexpr (F::kQ5) {
        constexpr int hmis = (o + F::kQh) & 3;
        const uint32_t qg = word_at<hmis>(rg, o + F::kQh), qhh = word_at<hmis>(rh, o + F::kQh);
        // low nibbles: elements 4t + {0, 2} in a0[0], 4t + {1, 3} in a0[2]
        a0[0] |= qh_pair(qg, 4 * t) << 4;
        a0[2] |= qh_pair(qg, 4 * t + 1) << 4;
        a0[1] |= qh_pair(qhh, 4 * t) << 4;
        a0[3] |= qh_pair(qhh, 4 * t + 1) << 4;
        // high nibbles: elements 16 + 4t + ...
        a1[0] |= qh_pair(qg, 16 + 4 * t) << 8;
        a1[2] |= qh_pair(qg, 16 + 4 * t + 1) << 8;
        a1[1] |= qh_pair(qhh, 16 + 4 * t) << 8;
        a1[3] |= qh_pair(qhh, 16 + 4 * t + 1) << 8;
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
        a0[k] = h2_sub(a0[k], kLo);
        a1[k] = h2_fma(a1[k], k1_16, kHi);
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        uint4 bx = bfrag<NT>(xf, B, nt, lane, live[nt]);
        float tmp[4];
        const float z[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t b0[2] = {bx.x, bx.y}, b1[2] = {bx.z, bx.w};
        mma_16816(tmp, a0, b0, z);
        mma_16816(tmp, a1, b1, tmp);
        if constexpr (F::kM) {
            const float X = xs[B * NT * 4 + nt * 4 + t];
            acc[nt][0] = fmaf(mg, X, acc[nt][0]);
            acc[nt][2] = fmaf(mh, X, acc[nt][2]);
        }
        fma2(acc[nt][0], acc[nt][1], tmp[0], tmp[1], dg);
        fma2(acc[nt][2], acc[nt][3], tmp[2], tmp[3], dh);
    }
}

template <int TYPE, int NT, int B = 0>
__device__ __forceinline__ void unit_b32(const uint8_t* stw, const uint4* xf, const float* xs, int row0, int g,
                                         int t, int lane, const bool* live, float (&acc)[NT][4]) {
    constexpr int RB = Fmt<TYPE>::kBox;
    const uint8_t* rg = stw + (row0 + g) * RB;
    block_b32<TYPE, NT, B>(rg, rg + 8 * RB, xf, xs, t, lane, live, acc);
    if constexpr (B < 7) unit_b32<TYPE, NT, B + 1>(stw, xf, xs, row0, g, t, lane, live, acc);
}

// Q8_0 (DequantQ8_0.cs:19-41; d@0, 32 int8 quants @2): each byte goes into
// the A fragment as the fp16 1024 + (q + 128) (byte ^ 0x80 under the 0x64
// exponent byte), minus 1152 = q, exact; d is applied to the fp32 partial
// sums per block, as for Q4_0.
__device__ __forceinline__ void s8_pairs(uint32_t w, uint32_t& a02, uint32_t& a13) {
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t k1152 = 0x64806480u;  // half2(1152, 1152)
    a02 = h2_sub(__byte_perm(u, 0x64646464u, 0x4240), k1152);
    a13 = h2_sub(__byte_perm(u, 0x64646464u, 0x4341), k1152);
}

template <int NT>
__device__ __forceinline__ void unit_q8_0(const uint8_t* stw, const uint4* xf, int row0, int g,
                                          int t, int lane, const bool* live, float (&acc)[NT][4]) {
    const uint8_t* rg = stw + (row0 + g) * 272;
    const uint8_t* rh = rg + 8 * 272;
#pragma unroll
    for (int b = 0; b < 8; b++) {
        const float dg = half_bits_to_float(lds_u16(rg + 34 * b));
        const float dh = half_bits_to_float(lds_u16(rh + 34 * b));
        // positions 4t..4t+3 (first k-step) and 16+4t..16+4t+3 (second)
        uint32_t wg0, wh0, wg1, wh1;
        if (b & 1) {
            wg0 = word_at<0>(rg, 34 * b + 2 + 4 * t);
            wh0 = word_at<0>(rh, 34 * b + 2 + 4 * t);
            wg1 = word_at<0>(rg, 34 * b + 18 + 4 * t);
            wh1 = word_at<0>(rh, 34 * b + 18 + 4 * t);
        } else {
            wg0 = word_at<2>(rg, 34 * b + 2 + 4 * t);
            wh0 = word_at<2>(rh, 34 * b + 2 + 4 * t);
            wg1 = word_at<2>(rg, 34 * b + 18 + 4 * t);
            wh1 = word_at<2>(rh, 34 * b + 18 + 4 * t);
        }
        uint32_t a0[4], a1[4];
        s8_pairs(wg0, a0[0], a0[2]);
        s8_pairs(wh0, a0[1], a0[3]);
        s8_pairs(wg1, a1[0], a1[2]);
        s8_pairs(wh1, a1[1], a1[3]);
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            uint4 bx = bfrag<NT>(xf, b, nt, lane, live[nt]);
            float tmp[4];
            const float z[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t b0[2] = {bx.x, bx.y}, b1[2] = {bx.z, bx.w};
            mma_16816(tmp, a0, b0, z);
            mma_16816(tmp, a1, b1, tmp);
            fma2(acc[nt][0], acc[nt][1], tmp[0], tmp[1], dg);
            fma2(acc[nt][2], acc[nt][3], tmp[2], tmp[3], dh);
        }
    }
}

// Q4_K.  Nibbles go into the A fragments as fp16 subnormals (bit pattern q,
// value q * 2^-24, exact), so decode is a mask per half2; 2^24 is folded
// into d*sc.  The per-(row, sub-block) scales d*sc*2^24 and dmin*m are
// decoded once per unit by the whole warp into a shared table.
// Q5_K (Q5 = true; DequantQ5K.cs:36-90): the same scales and mins at bytes
// 4..15, the 32 high bits of a sub-block at qh bytes 4j..4j+3 (bit e % 8 of
// byte e / 8 for element e) and its nibbles at 48 + 16j; each high bit goes
// into the fp16 subnormal at bit 4 (low k-step, value (q + 16 h) 2^-24) or
// bit 8 (high k-step, 16 (q + 16 h) 2^-24, the x fragments pre-scaled by 1/16).
template <int NT, bool Q5 = false>
__device__ __forceinline__ void unit_q4_k(const uint8_t* stw, const uint4* xf, const float* xs,
                                          float2* table, int row0, int g, int t, int lane,
                                          const bool* live, float (&acc)[NT][4]) {
    constexpr int RB = Q5 ? 176 : 144;  // bytes per row of a unit
    constexpr int QW = Q5 ? 12 : 4;     // first quant word of a row
    {
        // DecodeScales (DequantQ4K.cs:218-241) for row lane/2, sub-blocks
        // 4*(lane&1) .. +3, four 6-bit fields at a time
        const int r = lane >> 1, jh = lane & 1;
        const uint8_t* rp = stw + (row0 + r) * RB;
        const uint32_t* W = reinterpret_cast<const uint32_t*>(rp);
        float d = half_bits_to_float(lds_u16(rp)) * 16777216.0f;
        float dmin = half_bits_to_float(lds_u16(rp + 2));
        uint32_t w1 = W[1], w2 = W[2], w3 = W[3];
        const uint32_t sc_lo = w1 & 0x3F3F3F3Fu, m_lo = w2 & 0x3F3F3F3Fu;
        const uint32_t sc_hi = (w3 & 0x0F0F0F0Fu) | ((w1 >> 2) & 0x30303030u);
        const uint32_t m_hi = ((w3 >> 4) & 0x0F0F0F0Fu) | ((w2 >> 2) & 0x30303030u);
        const uint32_t sc = jh ? sc_hi : sc_lo, m = jh ? m_hi : m_lo;
#pragma unroll
        for (int k = 0; k < 4; k++)
            table[r * 8 + 4 * jh + k] = make_float2(d * ubyte_f(sc, k), dmin * ubyte_f(m, k));
    }
    __syncwarp();
    const uint8_t* rg = stw + (row0 + g) * RB;
    const uint8_t* rh = rg + 8 * RB;
    const uint32_t* Wg = reinterpret_cast<const uint32_t*>(rg);
    const uint32_t* Wh = reinterpret_cast<const uint32_t*>(rh);
    const uint32_t M = 0x000F000Fu, MH = 0x00F000F0u;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        uint32_t wg = Wg[QW + 4 * j + t], wh = Wh[QW + 4 * j + t];
        // low nibbles at bits 0-3 (value q * 2^-24), high nibbles left at
        // bits 4-7 (value 16 q * 2^-24); the high k-step's x fragments are
        // pre-scaled by 1/16, so both k-steps accumulate q * x * 2^-24.
        const uint32_t wg8 = wg >> 8, wh8 = wh >> 8;
        uint32_t a0[4], a1[4];
        a0[0] = wg & M;
        a0[1] = wh & M;
        a0[2] = wg8 & M;
        a0[3] = wh8 & M;
        a1[0] = wg & MH;
        a1[1] = wh & MH;
        a1[2] = wg8 & MH;
        a1[3] = wh8 & MH;
        if constexpr (Q5) {
            // high bits of positions 4t..4t+3 (low k-step) and 16+4t..16+4t+3
            const int sh4 = 4 * (t & 1);
            const uint32_t hg0 = (rg[16 + 4 * j + (t >> 1)] >> sh4) & 15u, hh0 = (rh[16 + 4 * j + (t >> 1)] >> sh4) & 15u;
            const uint32_t hg1 = (rg[18 + 4 * j + (t >> 1)] >> sh4) & 15u, hh1 = (rh[18 + 4 * j + (t >> 1)] >> sh4) & 15u;
            a0[0] |= ((hg0 & 1u) << 4) | ((hg0 & 4u) << 18);
            a0[1] |= ((hh0 & 1u) << 4) | ((hh0 & 4u) << 18);
            a0[2] |= ((hg0 & 2u) << 3) | ((hg0 & 8u) << 17);
            a0[3] |= ((hh0 & 2u) << 3) | ((hh0 & 8u) << 17);
            a1[0] |= ((hg1 & 1u) << 8) | ((hg1 & 4u) << 22);
            a1[1] |= ((hh1 & 1u) << 8) | ((hh1 & 4u) << 22);
            a1[2] |= ((hg1 & 2u) << 7) | ((hg1 & 8u) << 21);
            a1[3] |= ((hh1 & 2u) << 7) | ((hh1 & 8u) << 21);
        }
        const float2 sg = table[g * 8 + j], sh = table[(g + 8) * 8 + j];
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            uint4 bx = bfrag<NT>(xf, j, nt, lane, live[nt]);
            float X = xs[j * NT * 4 + nt * 4 + t];
            float tmp[4];
            const float z[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t b0[2] = {bx.x, bx.y}, b1[2] = {bx.z, bx.w};
            mma_16816(tmp, a0, b0, z);
            mma_16816(tmp, a1, b1, tmp);
            acc[nt][0] = fmaf(-sg.y, X, acc[nt][0]);
            acc[nt][2] = fmaf(-sh.y, X, acc[nt][2]);
            fma2(acc[nt][0], acc[nt][1], tmp[0], tmp[1], sg.x);
            fma2(acc[nt][2], acc[nt][3], tmp[2], tmp[3], sh.x);
        }
    }
    __syncwarp();  // the table is rebuilt by the next unit
}

// MIS = (210 u) mod 4: super-blocks of odd units start 2 bytes off a word.
template <int NT, int MIS>
__device__ __forceinline__ void unit_q6_k(const uint8_t* stw, const uint4* xf, int u, int row0,
                                          int g, int t, int lane, const bool* live,
                                          float (&acc)[NT][4]) {
    const int o = Fmt<CN_TYPE_Q6_K>::offset(u);
    const uint8_t* rg = stw + (row0 + g) * 240 + o;
    const uint8_t* rh = rg + 8 * 240;
    const uint32_t k1056 = 0x64206420u;  // half2(1056, 1056): (1024 + q) - 1056 = q - 32
    float dg = half_bits_to_float(lds_u16(rg + 208));
    float dh = half_bits_to_float(lds_u16(rh + 208));
    uint32_t scg[4], sch[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        scg[i] = word2<MIS>(rg + 192 + 4 * i);
        sch[i] = word2<MIS>(rh + 192 + 4 * i);
    }
#pragma unroll
    for (int h = 0; h < 2; h++) {
        uint32_t Ag[2], Bg[2], Hg[2], Ah[2], Bh[2], Hh[2];
#pragma unroll
        for (int j = 0; j < 2; j++) {
            Ag[j] = word2<MIS>(rg + 64 * h + 16 * j + 4 * t);
            Bg[j] = word2<MIS>(rg + 64 * h + 32 + 16 * j + 4 * t);
            Hg[j] = word2<MIS>(rg + 128 + 32 * h + 16 * j + 4 * t);
            Ah[j] = word2<MIS>(rh + 64 * h + 16 * j + 4 * t);
            Bh[j] = word2<MIS>(rh + 64 * h + 32 + 16 * j + 4 * t);
            Hh[j] = word2<MIS>(rh + 128 + 32 * h + 16 * j + 4 * t);
        }
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const int c = 4 * h + s;
            uint4 bxs[NT];
#pragma unroll
            for (int nt = 0; nt < NT; nt++) bxs[nt] = bfrag<NT>(xf, c, nt, lane, live[nt]);
#pragma unroll
            for (int j = 0; j < 2; j++) {
                // 6-bit quants of positions 4t..4t+3 of k-step (h, s, j)
                uint32_t qg, qh;
                if (s == 0) {
                    qg = (Ag[j] & 0x0F0F0F0Fu) | ((Hg[j] << 4) & 0x30303030u);
                    qh = (Ah[j] & 0x0F0F0F0Fu) | ((Hh[j] << 4) & 0x30303030u);
                } else if (s == 1) {
                    qg = (Bg[j] & 0x0F0F0F0Fu) | ((Hg[j] << 2) & 0x30303030u);
                    qh = (Bh[j] & 0x0F0F0F0Fu) | ((Hh[j] << 2) & 0x30303030u);
                } else if (s == 2) {
                    qg = ((Ag[j] >> 4) & 0x0F0F0F0Fu) | (Hg[j] & 0x30303030u);
                    qh = ((Ah[j] >> 4) & 0x0F0F0F0Fu) | (Hh[j] & 0x30303030u);
                } else {
                    qg = ((Bg[j] >> 4) & 0x0F0F0F0Fu) | ((Hg[j] >> 2) & 0x30303030u);
                    qh = ((Bh[j] >> 4) & 0x0F0F0F0Fu) | ((Hh[j] >> 2) & 0x30303030u);
                }
                uint32_t av[4];
                av[0] = h2_sub(__byte_perm(qg, 0x64646464u, 0x4240), k1056);
                av[2] = h2_sub(__byte_perm(qg, 0x64646464u, 0x4341), k1056);
                av[1] = h2_sub(__byte_perm(qh, 0x64646464u, 0x4240), k1056);
                av[3] = h2_sub(__byte_perm(qh, 0x64646464u, 0x4341), k1056);
                const int si = 8 * h + j + 2 * s;  // scale index (DequantQ6K.cs:61,73-76)
                const float sg = dg * sbyte_f(scg[si >> 2], si & 3);
                const float sh = dh * sbyte_f(sch[si >> 2], si & 3);
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    uint32_t bb[2];
                    if (j == 0) {
                        bb[0] = bxs[nt].x;
                        bb[1] = bxs[nt].y;
                    } else {
                        bb[0] = bxs[nt].z;
                        bb[1] = bxs[nt].w;
                    }
                    float tmp[4];
                    const float z[4] = {0.f, 0.f, 0.f, 0.f};
                    mma_16816(tmp, av, bb, z);
                    fma2(acc[nt][0], acc[nt][1], tmp[0], tmp[1], sg);
                    fma2(acc[nt][2], acc[nt][3], tmp[2], tmp[3], sh);
                }
            }
        }
    }
}

// ---- stream-K bookkeeping ---------------------------------------------------
//
// The (128-row tile, unit) space is linearised tile-major and cut into C
// equal contiguous ranges, one per CTA, with C = min(CTAs, total units) so
// every range is non-empty (idle CTAs, if any, come last).  A tile whose
// units all belong to one CTA is written directly; otherwise every
// contributing CTA stores its partial in slot 2*c + (tile is c's first tile
// ? 0 : 1), and for each 16-row sub-tile the last warp to arrive sums the
// slots in CTA order (deterministic) and resets that sub-tile's counter.

__device__ __forceinline__ int64_t range_start(int64_t total, int c, int C) {
    return total * c / C;
}

__device__ __forceinline__ int owner_of(int64_t v, int64_t total, int C) {
    int c = (int)((v * C) / total);
    while (c + 1 < C && range_start(total, c + 1, C) <= v) c++;
    while (c > 0 && range_start(total, c, C) > v) c--;
    return c;
}

// The matrix a tile belongs to: its index, its local tile number, rows and
// output.
__device__ __forceinline__ int tile_mat(const GemvArgs& a, int tile, int& local, int64_t& rows, float*& y) {
    if (a.nmat <= 1) {
        local = tile;
        rows = a.rows;
        y = a.y;
        return 0;
    }
    const int m = (a.nmat > 2 && tile >= a.toff[2]) ? 2 : (tile >= a.toff[1]) ? 1 : 0;
    local = tile - a.toff[m];
    rows = a.mrows[m];
    y = a.my[m];
    return m;
}

// Writes the tile's rows directly (the CTA computed all of its units).
template <int NT>
__device__ __forceinline__ void store_rows(const GemvArgs& a, int tile, int warp, int g, int t,
                                           float (&acc)[NT][4]) {
    int local;
    int64_t rows;
    float* y;
    tile_mat(a, tile, local, rows, y);
    const int64_t r0 = (int64_t)local * kTileRows + warp * 16 + g, r1 = r0 + 8;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        int b = nt * 4 + t;
        if (b < a.batch) {
            if (r0 < rows) y[(size_t)b * rows + r0] = acc[nt][0] + acc[nt][1];
            if (r1 < rows) y[(size_t)b * rows + r1] = acc[nt][2] + acc[nt][3];
        }
    }
}

// A tile shared by CTAs c_first..c_last: store this CTA's partial in its
// slot (0 for its first tile, 1 for its last), and let the last warp to
// arrive (per 16-row sub-tile) sum the slots in CTA order.
template <int NT>
__device__ void finish_shared(const GemvArgs& a, int tile, int warp, int cta, int my_slot,
                              int64_t total, int C, int g, int t, int lane, float (&acc)[NT][4]) {
    constexpr int BW = NT * 4;
    const int c_first = owner_of((int64_t)tile * a.units, total, C);
    const int c_last = owner_of((int64_t)(tile + 1) * a.units - 1, total, C);
    float* p = a.partials + ((size_t)(2 * cta + my_slot) * kTileRows + warp * 16) * BW;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        p[g * BW + nt * 4 + t] = acc[nt][0] + acc[nt][1];
        p[(g + 8) * BW + nt * 4 + t] = acc[nt][2] + acc[nt][3];
    }
    __threadfence();
    __syncwarp();
    int prev = 0;
    int* ctr = &a.counters[tile * kCons + warp];
    if (lane == 0) prev = atomicAdd(ctr, 1);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != c_last - c_first) return;
    __threadfence();
    // contributors: c_first's last tile (slot 1, unless the tile is also its
    // first), the middle CTAs (whole range inside the tile: slot 0), c_last's
    // first tile (slot 0)
    const float* src[8];
    int ns = 0;
    for (int c = c_first; c <= c_last && ns < 8; c++) {
        const int first_tile = (int)(range_start(total, c, C) / a.units);
        const int slot = 2 * c + (tile == first_tile ? 0 : 1);
        src[ns++] = a.partials + ((size_t)slot * kTileRows + warp * 16) * BW;
    }
    int local;
    int64_t rows;
    float* y;
    tile_mat(a, tile, local, rows, y);
    // each lane sums kE elements of the sub-tile; the loads of kBatchC
    // contributors are issued together (about 32 in flight per lane) rather
    // than one L2 round trip after another, and the sums run in CTA order
    constexpr int kE = 16 * BW / 32;
    constexpr int kBatchC = 32 / kE < 1 ? 1 : (32 / kE > 8 ? 8 : 32 / kE);
    float s[kE];
#pragma unroll
    for (int i = 0; i < kE; i++) s[i] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < 8; k0 += kBatchC) {
        if (k0 >= ns) break;
        float v[kBatchC][kE];
#pragma unroll
        for (int k = 0; k < kBatchC; k++)
#pragma unroll
            for (int i = 0; i < kE; i++) v[k][i] = k0 + k < ns ? __ldcg(src[k0 + k] + lane + 32 * i) : 0.f;
#pragma unroll
        for (int k = 0; k < kBatchC; k++)
#pragma unroll
            for (int i = 0; i < kE; i++)
                if (k0 + k < ns) s[i] += v[k][i];
    }
#pragma unroll
    for (int i = 0; i < kE; i++) {
        const int e = lane + 32 * i;
        const int row = e / BW, b = e % BW;
        const int64_t r = (int64_t)local * kTileRows + warp * 16 + row;
        if (b < a.batch && r < rows) y[(size_t)b * rows + r] = s[i];
    }
    if (lane == 0) atomicExch(ctr, 0);
}

// Cluster split (batch 1-8, the same number s = 2..8 of CTAs on every
// tile): the s CTAs of tile k form one cluster; rank j > 0 stores its sums
// into the leader's slot j - 1 (dynamic shared memory past the kernel's own
// layout) and each of its warps arrives on the leader's barrier with release
// semantics at cluster scope; the leader waits for all kCons (s - 1)
// arrivals (bounded) and adds the slots after its own sums in rank order --
// the stream-K order of finish_shared, without its L2 partials and counter.
template <int NT>
__device__ void cluster_finish_mma(const GemvArgs& a, int tile, int warp, int g, int t, int lane,
                                   float (&acc)[NT][4], uint32_t pbar, uint32_t pbuf, const float* slots) {
    constexpr int BW = NT * 4;
    constexpr uint32_t kSlot = kTileRows * BW * 4;  // bytes of one CTA's sums
    const int r0 = warp * 16 + g, r1 = r0 + 8;
    cluster_wait();
    const uint32_t rank = cluster_rank();
    if (rank != 0) {
        const uint32_t dst = map_rank(pbuf + (rank - 1) * kSlot, 0);
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const uint32_t c = (uint32_t)(nt * 4 + t) * 4u;
            asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst + (uint32_t)r0 * BW * 4 + c),
                         "f"(acc[nt][0] + acc[nt][1])
                         : "memory");
            asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst + (uint32_t)r1 * BW * 4 + c),
                         "f"(acc[nt][2] + acc[nt][3])
                         : "memory");
        }
        __syncwarp();
        if (lane == 0)
            asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(map_rank(pbar, 0))
                         : "memory");
        return;
    }
    if (!mbar_wait_cluster(pbar, 0)) {
        if (lane == 0) atomicOr(a.err, kErrTimeout);
        return;
    }
    int local;
    int64_t rows;
    float* y;
    tile_mat(a, tile, local, rows, y);
    const int64_t g0 = (int64_t)local * kTileRows + r0, g1 = g0 + 8;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const int b = nt * 4 + t;
        if (b >= a.batch) continue;
        float v0 = acc[nt][0] + acc[nt][1], v1 = acc[nt][2] + acc[nt][3];
#pragma unroll 1
        for (int j = 1; j < a.csize; j++) {
            v0 += slots[(j - 1) * kTileRows * BW + r0 * BW + b];
            v1 += slots[(j - 1) * kTileRows * BW + r1 * BW + b];
        }
        if (g0 < rows) y[(size_t)b * rows + g0] = v0;
        if (g1 < rows) y[(size_t)b * rows + g1] = v1;
    }
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---- the kernel ---------------------------------------------------------------

template <int TYPE, int NT>
__global__ void __launch_bounds__(kThreads, Geo<TYPE, NT>::kMinCtas)
    gemv_kernel(const __grid_constant__ GemvMaps maps, const GemvArgs a) {
    using G = Geo<TYPE, NT>;
    constexpr int S = G::kStages;
    // Dynamic shared memory starts at the CTA's shared window (no static
    // shared variables here), which is 1 KB aligned; every region below is
    // a multiple of 128 bytes, as TMA destinations need.
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* stages = smem;
    float2* table = reinterpret_cast<float2*>(smem + S * G::kStage);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * G::kStage + G::kTable);
    uint64_t* empty = full + S;
    // cluster split: the leader's barrier, and its slots past the layout above
    uint64_t* pbar_p = empty + S;
    static_assert(16 * G::kStages + 8 <= 64 * 16, "barrier slot");
    const bool clus = NT <= 2 && a.csize > 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCons);
        }
        if (clus) mbar_init(pbar_p, kCons * (a.csize - 1));
        fence_mbar_init();
    }
    __syncthreads();
    if (clus) cluster_arrive_relaxed();
    pdl_trigger();

    const int64_t total = (int64_t)a.tiles * a.units;
    const int C = (int)(total < (int64_t)gridDim.x ? total : (int64_t)gridDim.x);
    const int cta = blockIdx.x;
    if (cta >= C) {
        pdl_wait();
        return;
    }
    const int64_t v0 = range_start(total, cta, C), v1 = range_start(total, cta + 1, C);

    if (warp == kCons) {
        // producer: one lane streams raw blocks + activation fragments
        if (lane != 0) {
            pdl_wait();
            return;
        }
        const int nunits = (int)(v1 - v0);
        auto load_w = [&](uint8_t* st, int tile, int u, uint64_t* bar) {
            int local;
            int64_t rows;
            float* y;
            const int m = tile_mat(a, tile, local, rows, y);
            tma_load_2d(st, &maps.m[m], Fmt<TYPE>::box_x(u), local * kTileRows, bar);
        };
        // the weights depend on no earlier kernel: the first stages' weight
        // loads start before the wait for the kernel that writes the
        // activation fragments
        const int pre = nunits < S ? nunits : S;
        {
            int tile = (int)(v0 / a.units), u = (int)(v0 % a.units);
            for (int k = 0; k < pre; k++) {
                mbar_expect_tx(&full[k], G::kBytes);
                load_w(stages + k * G::kStage, tile, u, &full[k]);
                if (++u == a.units) {
                    u = 0;
                    tile++;
                }
            }
        }
        pdl_wait();
        int tile = (int)(v0 / a.units), u = (int)(v0 % a.units);
        int s = 0;
        uint32_t n = 0, phase = 0;
        for (; n < (uint32_t)nunits; n++) {
            if (n >= (uint32_t)S && !mbar_wait(&empty[s], phase ^ 1)) {
                atomicOr(a.err, kErrTimeout);
                for (uint32_t k = n - S; k < n; k++) mbar_wait(&full[k % S], (k / S) & 1);
                return;
            }
            uint8_t* st = stages + s * G::kStage;
            if (n >= (uint32_t)S) {
                mbar_expect_tx(&full[s], G::kBytes);
                load_w(st, tile, u, &full[s]);
            }
            bulk_g2s(st + G::kW, a.xfrag + (size_t)u * 8 * NT * 32, G::kXF, &full[s]);
            if constexpr (G::kXS > 0)
                bulk_g2s(st + G::kW + G::kXF, a.xsum + (size_t)u * 8 * NT * 4, G::kXS, &full[s]);
            bulk_g2s(st + G::kW + G::kXF + G::kXS, a.xinv + (size_t)u * NT * 4, G::kXI, &full[s]);
            if (++u == a.units) {
                u = 0;
                tile++;
            }
            if (++s == S) {
                s = 0;
                phase ^= 1;
            }
        }
        // let the last copies land before the CTA can retire
        for (uint32_t k = (n > (uint32_t)S ? n - S : 0); k < n; k++) mbar_wait(&full[k % S], (k / S) & 1);
        return;
    }

    pdl_wait();
    const int g = lane >> 2, t = lane & 3;
    bool live[NT];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) live[nt] = (nt * 4 + (g >> 1)) < a.batch;
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

    const int nunits = (int)(v1 - v0);
    int tile = (int)(v0 / a.units), u = (int)(v0 % a.units);
    const int tile0 = tile, u0 = u;
    int s = 0;
    uint32_t phase = 0;
    for (int n = 0; n < nunits; n++) {
        if (!mbar_wait(&full[s], phase)) {
            if (lane == 0) atomicOr(a.err, kErrTimeout);
            return;
        }
        const uint8_t* st = stages + s * G::kStage;
        const uint4* xf = reinterpret_cast<const uint4*>(st + G::kW);
        float au[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++) au[nt][0] = au[nt][1] = au[nt][2] = au[nt][3] = 0.f;
        if constexpr (TYPE == CN_TYPE_Q4_0) {
            unit_q4_0<NT>(st, xf, warp * 16, g, t, lane, live, au);
        } else if constexpr (TYPE == CN_TYPE_Q8_0) {
            unit_q8_0<NT>(st, xf, warp * 16, g, t, lane, live, au);
        } else if constexpr (TYPE == CN_TYPE_Q4_1 || TYPE == CN_TYPE_Q5_0 || TYPE == CN_TYPE_Q5_1) {
            const float* xs = reinterpret_cast<const float*>(st + G::kW + G::kXF);
            unit_b32<TYPE, NT>(st, xf, xs, warp * 16, g, t, lane, live, au);
        } else if constexpr (TYPE == CN_TYPE_Q4_K || TYPE == CN_TYPE_Q5_K) {
            const float* xs = reinterpret_cast<const float*>(st + G::kW + G::kXF);
            unit_q4_k<NT, TYPE == CN_TYPE_Q5_K>(st, xf, xs, table + warp * 128, warp * 16, g, t, lane, live, au);
        } else {
            if (u & 1) unit_q6_k<NT, 2>(st, xf, u, warp * 16, g, t, lane, live, au);
            else unit_q6_k<NT, 0>(st, xf, u, warp * 16, g, t, lane, live, au);
        }
        // undo the unit's activation scaling (exact power of two per column)
        const float* xi = reinterpret_cast<const float*>(st + G::kW + G::kXF + G::kXS);
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const float inv = xi[nt * 4 + t];
            fma2(acc[nt][0], acc[nt][1], au[nt][0], au[nt][1], inv);
            fma2(acc[nt][2], acc[nt][3], au[nt][2], au[nt][3], inv);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (u == a.units - 1 || n == nunits - 1) {
            // only the first and the last tile of the range can be shared
            const bool head_cut = (tile == tile0) && (u0 != 0);
            const bool tail_cut = (n == nunits - 1) && (u != a.units - 1);
            if constexpr (NT <= 2) {
                if (clus) {  // the range lies in one tile: this is its last unit
                    cluster_finish_mma<NT>(a, tile, warp, g, t, lane, acc, smem_u32(pbar_p), smem_u32(smem + G::kSmem),
                                           reinterpret_cast<const float*>(smem + G::kSmem));
                    break;
                }
            }
            if (head_cut || tail_cut)
                finish_shared<NT>(a, tile, warp, cta, tile == tile0 ? 0 : 1, total, C, g, t, lane, acc);
            else
                store_rows<NT>(a, tile, warp, g, t, acc);
#pragma unroll
            for (int nt = 0; nt < NT; nt++) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
        }
        if (++u == a.units) {
            u = 0;
            tile++;
        }
        if (++s == S) {
            s = 0;
            phase ^= 1;
        }
    }
}

// Standalone prep of any record form: one warp per (unit, batch row).
__global__ void xprep_kernel(const float* __restrict__ x, int K, int batch, PrepTarget pt) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int units = K / 256;
    const int64_t items = (int64_t)units * batch;
    const int64_t w0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t it = w0; it < items; it += nw) {
        const int u = (int)(it % units), b = (int)(it / units);
        const float* p = x + (size_t)b * K + (size_t)u * 256 + (lane >> 2) * 32 + 4 * (lane & 3);
        float4 a0 = *reinterpret_cast<const float4*>(p);
        float4 a1 = *reinterpret_cast<const float4*>(p + 16);
        const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        emit_any(pt, v, u, b, batch, lane);
    }
}

// Residual add fused with RMSNorm (TensorMath.Add, Tensors/TensorMath.cs:712-733;
// TensorMath.RmsNorm, Tensors/TensorMath.cs:97-165) and with the prep of the
// normalised row for the GEMV that reads it next.  Grid (units, rows): every
// CTA sums the squares of its whole row (x_in + delta, read from L2), then
// writes its own 256-value slice of x_out = x_in + delta (when delta is
// given) and of y = x * (1 / sqrt(sum(x^2)/n + eps)) * w, elementwise in the
// reference's order, and emits the slice's record.  x_out must not alias
// x_in (other CTAs still read x_in).  512 threads: under tensor parallelism
// the whole-row sum reads every rank's pairs of the row (512 KB at 8 ranks
// and dim 8192), and each pass of the loop is one round trip, so more
// threads mean fewer passes.
constexpr int kNormThreads = 512;
constexpr int kNormBatch = 4;  // float4 loads per thread in flight (one GPU)

// An exchange wait gives up at its time limit, or at once when an earlier
// wait of the step already gave up (the error word holds kErrTimeout): a rank
// that never arrives then costs one limit per step, not one per exchange.
__device__ __forceinline__ bool xchg_give_up(const XchgIn& xi, uint64_t t0) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) return true;
    return (*reinterpret_cast<volatile const uint32_t*>(xi.err) & kErrTimeout) != 0;
}

// Bounded wait of one thread for an exchange: every rank's flag must reach
// this use's sequence number; on timeout the error word is raised and the
// caller runs on (its results are then flagged garbage).
__device__ __forceinline__ uint32_t xchg_wait_dev(const XchgIn& xi) {
    const uint32_t seq = *xi.seq_base * xi.uses + xi.seq_add;
    const uint64_t t0 = globaltimer_ns();
    for (int p = 0; p < xi.size; p++) {
        for (;;) {
            uint32_t f;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(f) : "l"(xi.flags + p) : "memory");
            if ((int32_t)(f - seq) >= 0) break;
            if (xchg_give_up(xi, t0)) {
                atomicOr(xi.err, kErrTimeout);
                return seq;
            }
            __nanosleep(64);
        }
    }
    return seq;
}

__global__ void xchg_wait_kernel(XchgIn xi) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) xchg_wait_dev(xi);
}

// One element of the exchange's summed input (as ll_sum4).
__device__ __forceinline__ float ll_sum1(const XchgIn& xi, const uint64_t* base, size_t i, uint32_t seq,
                                         uint64_t t0) {
    uint64_t v[kMaxTp];
    for (;;) {
#pragma unroll
        for (int p = 0; p < kMaxTp; p++)
            if (p < xi.size)
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];"
                             : "=l"(v[p]) : "l"(base + p * xi.rank_stride + i) : "memory");
        bool ok = true;
#pragma unroll
        for (int p = 0; p < kMaxTp; p++)
            if (p < xi.size) ok = ok && (uint32_t)(v[p] >> 32) == seq;
        if (ok) break;
        if (xchg_give_up(xi, t0)) {
            atomicOr(xi.err, kErrTimeout);
            break;
        }
    }
    float d = __uint_as_float((uint32_t)v[0]);
#pragma unroll
    for (int p = 1; p < kMaxTp; p++)
        if (p < xi.size) d = __fadd_rn(d, __uint_as_float((uint32_t)v[p]));
    return d;
}

// The exchange's summed input at elements i..i+3 of a row (8-byte pairs;
// ranks added in rank order, so every rank computes the same bits).  All
// ranks' pairs are requested before any is checked, so the loads overlap;
// the batch is re-read until every sequence number matches (bounded).
__device__ __forceinline__ float4 ll_sum4(const XchgIn& xi, const uint64_t* base, size_t i, uint32_t seq,
                                          uint64_t t0) {
    uint64_t v[kMaxTp][4];
    for (;;) {
#pragma unroll
        for (int p = 0; p < kMaxTp; p++) {
            if (p < xi.size) {
                const uint64_t* q = base + p * xi.rank_stride + i;
                asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];"
                             : "=l"(v[p][0]), "=l"(v[p][1]) : "l"(q) : "memory");
                asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];"
                             : "=l"(v[p][2]), "=l"(v[p][3]) : "l"(q + 2) : "memory");
            }
        }
        bool ok = true;
#pragma unroll
        for (int p = 0; p < kMaxTp; p++)
            if (p < xi.size)
#pragma unroll
                for (int e = 0; e < 4; e++) ok = ok && (uint32_t)(v[p][e] >> 32) == seq;
        if (ok) break;
        if (xchg_give_up(xi, t0)) {
            atomicOr(xi.err, kErrTimeout);
            break;
        }
    }
    float4 s = make_float4(__uint_as_float((uint32_t)v[0][0]), __uint_as_float((uint32_t)v[0][1]),
                           __uint_as_float((uint32_t)v[0][2]), __uint_as_float((uint32_t)v[0][3]));
#pragma unroll
    for (int p = 1; p < kMaxTp; p++) {
        if (p < xi.size) {
            s.x = __fadd_rn(s.x, __uint_as_float((uint32_t)v[p][0]));
            s.y = __fadd_rn(s.y, __uint_as_float((uint32_t)v[p][1]));
            s.z = __fadd_rn(s.z, __uint_as_float((uint32_t)v[p][2]));
            s.w = __fadd_rn(s.w, __uint_as_float((uint32_t)v[p][3]));
        }
    }
    return s;
}

// The exchange's summed input at element i of row b (ranks added in rank
// order, so every rank computes the same bits).
__device__ __forceinline__ float4 xchg_sum4(const XchgIn& xi, const float* base, size_t off) {
    float4 s = __ldcg(reinterpret_cast<const float4*>(base + off));
    for (int p = 1; p < xi.size; p++) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(base + p * xi.rank_stride + off));
        s.x = __fadd_rn(s.x, v.x);
        s.y = __fadd_rn(s.y, v.y);
        s.z = __fadd_rn(s.z, v.z);
        s.w = __fadd_rn(s.w, v.w);
    }
    return s;
}

__global__ void __launch_bounds__(kNormThreads)
    add_norm_prep_kernel(const float* __restrict__ x_in, const float* __restrict__ delta,
                         float* __restrict__ x_out, const float* __restrict__ w, float* __restrict__ y,
                         int n, float eps, PrepTarget pt, XchgIn xi) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[kNormThreads / 32];
    __shared__ __align__(16) float vals[256];
    __shared__ uint32_t s_seq;
    const int u = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const float* xr = x_in + (size_t)b * n;
    const float* dr = delta ? delta + (size_t)b * n : nullptr;
    // tensor parallel: delta is the sum of every rank's partial (in rank order)
    const float* xbase = nullptr;
    const uint64_t* llbase = nullptr;
    uint32_t seq = 0;
    const uint64_t t0 = globaltimer_ns();
    if (xi.size > 1) {
        if (xi.ll) {
            seq = *xi.seq_base * xi.uses + xi.seq_add;
            llbase = reinterpret_cast<const uint64_t*>(xi.src) + (seq & 1u) * xi.parity_stride + (size_t)b * n;
        } else {
            if (tid == 0) s_seq = xchg_wait_dev(xi);
            __syncthreads();
            xbase = xi.src + (s_seq & 1u) * xi.parity_stride + (size_t)b * n;
        }
        dr = nullptr;
    }
    float ss = 0.f;
    const int i = u * 256 + tid;
    const bool mine = tid < 256 && i < n;  // this thread's output element
    float v_own = 0.f, w_own = 0.f;
    if (xi.size <= 1) {
        // one GPU: every load of a batch of up to kNormBatch float4 per
        // thread (and the thread's own element and weight) is issued before
        // the first is used, so the vector arrives in one round trip; the
        // sums keep the per-thread order of the loop below
        if (mine) {
            v_own = xr[i];
            if (dr) v_own = __fadd_rn(v_own, dr[i]);
            w_own = w[i];
        }
        for (int base = 4 * tid; base < n; base += kNormBatch * 4 * kNormThreads) {
            float4 xv[kNormBatch], dv[kNormBatch];
#pragma unroll
            for (int k = 0; k < kNormBatch; k++) {
                const int j = base + k * 4 * kNormThreads;
                if (j < n) {
                    xv[k] = *reinterpret_cast<const float4*>(xr + j);
                    dv[k] = dr ? *reinterpret_cast<const float4*>(dr + j) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int k = 0; k < kNormBatch; k++) {
                if (base + k * 4 * kNormThreads < n) {
                    float4 v = xv[k];
                    if (dr) {
                        v.x = __fadd_rn(v.x, dv[k].x);
                        v.y = __fadd_rn(v.y, dv[k].y);
                        v.z = __fadd_rn(v.z, dv[k].z);
                        v.w = __fadd_rn(v.w, dv[k].w);
                    }
                    ss = fmaf(v.x, v.x, ss);
                    ss = fmaf(v.y, v.y, ss);
                    ss = fmaf(v.z, v.z, ss);
                    ss = fmaf(v.w, v.w, ss);
                }
            }
        }
    } else {
        for (int j = 4 * tid; j < n; j += 4 * kNormThreads) {
            float4 v = *reinterpret_cast<const float4*>(xr + j);
            if (xbase || llbase) {
                const float4 d = llbase ? ll_sum4(xi, llbase, j, seq, t0) : xchg_sum4(xi, xbase, j);
                v.x = __fadd_rn(v.x, d.x);
                v.y = __fadd_rn(v.y, d.y);
                v.z = __fadd_rn(v.z, d.z);
                v.w = __fadd_rn(v.w, d.w);
            }
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int k = 0; k < kNormThreads / 32; k++) ss += red[k];
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    if (mine && xi.size <= 1) {
        if (dr) x_out[(size_t)b * n + i] = v_own;
        const float o = __fmul_rn(__fmul_rn(v_own, rms), w_own);
        y[(size_t)b * n + i] = o;
        vals[tid] = o;
    } else if (mine) {  // tensor parallel: the exchange's sum is the delta
        float v = xr[i];
        if (xbase || llbase) {
            float d;
            if (llbase) {
                d = ll_sum1(xi, llbase, i, seq, t0);
            } else {
                d = __ldcg(xbase + i);
                for (int p = 1; p < xi.size; p++) d = __fadd_rn(d, __ldcg(xbase + p * xi.rank_stride + i));
            }
            v = __fadd_rn(v, d);
            x_out[(size_t)b * n + i] = v;
        }
        const float o = __fmul_rn(__fmul_rn(v, rms), w[i]);
        y[(size_t)b * n + i] = o;
        vals[tid] = o;
    }
    if (pt.kind < 0) return;
    __syncthreads();
    if (tid < 32) {
        const int c = tid >> 2, t = tid & 3;
        const float4 a0 = *reinterpret_cast<const float4*>(vals + 32 * c + 4 * t);
        const float4 a1 = *reinterpret_cast<const float4*>(vals + 32 * c + 16 + 4 * t);
        const float v8[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        emit_any(pt, v8, u, b, (int)gridDim.y, tid);
    }
}

// The same fused residual add + RmsNorm + prep as one thread-block cluster
// of up to kNormCluster CTAs per batch row: CTA r of a row owns a contiguous
// range of the row's 256-position units, reads only its slice of x, of the
// delta and (tensor parallel) of every rank's exchange slots, and keeps the
// summed values in shared memory.  The CTAs' partial sums of squares are
// added through distributed shared memory (in CTA order, so every CTA and
// every rank gets the same rms), then each CTA writes its slice and its
// units' records.  Compared with add_norm_prep_kernel, which has every CTA
// read the whole row (under tensor parallelism every rank's whole row), the
// row is read once; used for tensor-parallel exchanges.
constexpr int kNormCluster = 8;
constexpr int kNormClThreads = 256;
constexpr int kNormClMaxVals = 4096;  // values a CTA holds: rows up to 8 x 4096 = 32768

__global__ void __launch_bounds__(kNormClThreads)
    add_norm_prep_cl_kernel(const float* __restrict__ x_in, const float* __restrict__ delta,
                            float* __restrict__ x_out, const float* __restrict__ w, float* __restrict__ y,
                            int n, float eps, PrepTarget pt, XchgIn xi) {
    pdl_trigger();
    pdl_wait();
    __shared__ __align__(16) float vals[kNormClMaxVals];
    __shared__ float red[kNormClThreads / 32];
    __shared__ float s_part;
    __shared__ uint32_t s_seq;
    const int C = (int)cluster_size(), r = (int)cluster_rank();
    const int b = blockIdx.y, tid = threadIdx.x;
    const int units = n / 256;
    const int u0 = units * r / C, u1 = units * (r + 1) / C;
    const int i0 = u0 * 256, i1 = u1 * 256;
    const float* xr = x_in + (size_t)b * n;
    const float* dr = delta ? delta + (size_t)b * n : nullptr;
    const float* xbase = nullptr;
    const uint64_t* llbase = nullptr;
    uint32_t seq = 0;
    const uint64_t t0 = globaltimer_ns();
    if (xi.size > 1) {
        if (xi.ll) {
            seq = *xi.seq_base * xi.uses + xi.seq_add;
            llbase = reinterpret_cast<const uint64_t*>(xi.src) + (seq & 1u) * xi.parity_stride + (size_t)b * n;
        } else {
            if (tid == 0) s_seq = xchg_wait_dev(xi);
            __syncthreads();
            xbase = xi.src + (s_seq & 1u) * xi.parity_stride + (size_t)b * n;
        }
        dr = nullptr;
    }
    const bool add = dr || xbase || llbase;
    float ss = 0.f;
    for (int i = i0 + 4 * tid; i < i1; i += 4 * kNormClThreads) {
        float4 v = *reinterpret_cast<const float4*>(xr + i);
        if (add) {
            const float4 d = llbase  ? ll_sum4(xi, llbase, i, seq, t0)
                             : xbase ? xchg_sum4(xi, xbase, i)
                                     : *reinterpret_cast<const float4*>(dr + i);
            v.x = __fadd_rn(v.x, d.x);
            v.y = __fadd_rn(v.y, d.y);
            v.z = __fadd_rn(v.z, d.z);
            v.w = __fadd_rn(v.w, d.w);
            *reinterpret_cast<float4*>(x_out + (size_t)b * n + i) = v;
        }
        *reinterpret_cast<float4*>(vals + (i - i0)) = v;
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < kNormClThreads / 32; i++) t += red[i];
        s_part = t;
    }
    cluster_arrive();  // s_part (and this CTA's values) are ready
    cluster_wait();
    float tot = 0.f;
    for (int c = 0; c < C; c++) tot += ld_peer_f32(&s_part, (uint32_t)c);
    cluster_arrive();  // done reading the peers' s_part (matched by the wait before exit)
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), eps)));
    for (int i = i0 + 4 * tid; i < i1; i += 4 * kNormClThreads) {
        float4 v = *reinterpret_cast<const float4*>(vals + (i - i0));
        const float4 g = *reinterpret_cast<const float4*>(w + i);
        v.x = __fmul_rn(__fmul_rn(v.x, rms), g.x);
        v.y = __fmul_rn(__fmul_rn(v.y, rms), g.y);
        v.z = __fmul_rn(__fmul_rn(v.z, rms), g.z);
        v.w = __fmul_rn(__fmul_rn(v.w, rms), g.w);
        *reinterpret_cast<float4*>(y + (size_t)b * n + i) = v;
        *reinterpret_cast<float4*>(vals + (i - i0)) = v;
    }
    if (pt.kind >= 0) {
        __syncthreads();
        const int lane = tid & 31;
        for (int u = u0 + (tid >> 5); u < u1; u += kNormClThreads / 32) {
            const int c = lane >> 2, t = lane & 3;
            const float* vu = vals + (u - u0) * 256;
            const float4 a0 = *reinterpret_cast<const float4*>(vu + 32 * c + 4 * t);
            const float4 a1 = *reinterpret_cast<const float4*>(vu + 32 * c + 16 + 4 * t);
            const float v8[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            emit_any(pt, v8, u, b, (int)gridDim.y, lane);
        }
    }
    cluster_wait();  // no CTA leaves while a peer may still read its s_part
}

// ---- generic (untiled) fallback -------------------------------------------------
//
// For shapes the TMA path cannot tile (row bytes not a multiple of 16, or K
// not a multiple of 256): one warp per (row, batch), exact block decode and
// fp32 FMAs.  Slow but shape-agnostic.
// end: one past the matrix's last byte (bounds IQ3_S's reads past a block).
__device__ float block_dot(int type, const uint8_t* row, int blk, const float* x, const uint8_t* end) {
    float s = 0.f;
    if (type == CN_TYPE_Q4_0) {
        const uint8_t* p = row + (size_t)blk * 18;
        float d = ld_half(p);
        const float* xb = x + (size_t)blk * 32;
        float bs = 0.f;
        for (int j = 0; j < 16; j++) {
            bs += (float)((p[2 + j] & 15) - 8) * xb[j];
            bs += (float)((p[2 + j] >> 4) - 8) * xb[j + 16];
        }
        s = bs * d;
    } else if (type == CN_TYPE_Q4_K) {
        const uint8_t* p = row + (size_t)blk * 144;
        float d = ld_half(p), dmin = ld_half(p + 2);
        const float* xb = x + (size_t)blk * 256;
        for (int j = 0; j < 8; j++) {
            int sc, m;
            q4k_scale_min(p + 4, j, sc, m);
            float dsc = d * (float)sc, dm = dmin * (float)m;
            for (int i = 0; i < 16; i++) {
                uint8_t v = p[16 + 16 * j + i];
                s += (dsc * (float)(v & 15) - dm) * xb[32 * j + i];
                s += (dsc * (float)(v >> 4) - dm) * xb[32 * j + 16 + i];
            }
        }
    } else if (type == CN_TYPE_Q6_K) {
        const uint8_t* p = row + (size_t)blk * 210;
        float d = ld_half(p + 208);
        const float* xb = x + (size_t)blk * 256;
        for (int h = 0; h < 2; h++) {
            const uint8_t* ql = p + 64 * h;
            const uint8_t* qh = p + 128 + 32 * h;
            const int8_t* sc = (const int8_t*)(p + 192);
            for (int l = 0; l < 32; l++) {
                int si = 8 * h + l / 16;
                int q1 = ((ql[l] & 15) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int q2 = ((ql[l + 32] & 15) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                const float* xh = xb + 128 * h;
                s += d * (float)sc[si] * (float)q1 * xh[l];
                s += d * (float)sc[si + 2] * (float)q2 * xh[l + 32];
                s += d * (float)sc[si + 4] * (float)q3 * xh[l + 64];
                s += d * (float)sc[si + 6] * (float)q4 * xh[l + 96];
            }
        }
    } else if (type == CN_TYPE_F32) {
        s = reinterpret_cast<const float*>(row)[blk] * x[blk];
    } else if (is_block32(type)) {
        const uint8_t* p = row + (size_t)blk * block32_bytes(type);
        const float* xb = x + (size_t)blk * 32;
        for (int j = 0; j < 32; j++) s = fmaf(block32_elem(type, p, j), xb[j], s);
    } else if (is_superblock(type)) {
        const uint8_t* p = row + (size_t)blk * superblock_bytes(type);
        const float* xb = x + (size_t)blk * 256;
        for (int e = 0; e < 256; e++) s = fmaf(superblock_elem(type, p, e, end), xb[e], s);
    } else if (type == CN_TYPE_F16) {
        s = ld_half(row + 2 * (size_t)blk) * x[blk];
    }
    return s;
}

__global__ void gemv_generic_kernel(int type, const uint8_t* __restrict__ w, int64_t rows, int cols,
                                    uint64_t rbytes, int blk_elems, const float* __restrict__ x,
                                    float* __restrict__ y, int batch) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int nblk = cols / blk_elems;
    for (int64_t wi = warp; wi < rows * batch; wi += nwarps) {
        int64_t r = wi % rows;
        int b = (int)(wi / rows);
        const uint8_t* row = w + (size_t)r * rbytes;
        const float* xb = x + (size_t)b * cols;
        float s = 0.f;
        for (int k = lane; k < nblk; k += 32) s += block_dot(type, row, k, xb, w + (size_t)rows * rbytes);
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) y[(size_t)b * rows + r] = s;
    }
}

// ---- host side ------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
    // initialised once, thread-safely (function-local static)
    static const EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<EncodeTiledFn>(p);
        return static_cast<EncodeTiledFn>(nullptr);
    }();
    return fn;
}

// Types whose tiled GEMV reads the chunk sums of x (their min terms).
static bool type_needs_xsum(int type) {
    return type == CN_TYPE_Q4_K || type == CN_TYPE_Q5_K || type == CN_TYPE_Q4_1 || type == CN_TYPE_Q5_1;
}

static int box_bytes(int type) {
    switch (type) {
        case CN_TYPE_Q4_0: return Fmt<CN_TYPE_Q4_0>::kBox;
        case CN_TYPE_Q8_0: return Fmt<CN_TYPE_Q8_0>::kBox;
        case CN_TYPE_Q4_K: return Fmt<CN_TYPE_Q4_K>::kBox;
        case CN_TYPE_Q5_K: return Fmt<CN_TYPE_Q5_K>::kBox;
        case CN_TYPE_Q4_1: return Fmt<CN_TYPE_Q4_1>::kBox;
        case CN_TYPE_Q5_0: return Fmt<CN_TYPE_Q5_0>::kBox;
        case CN_TYPE_Q5_1: return Fmt<CN_TYPE_Q5_1>::kBox;
        case CN_TYPE_Q6_K: return Fmt<CN_TYPE_Q6_K>::kBox;
        default: return 0;
    }
}

int encode_tiled_2d(CUtensorMapDataType dt, void* base, const cuuint64_t (&dims)[2],
                    const cuuint64_t (&strides)[1], const cuuint32_t (&box)[2],
                    CUtensorMapSwizzle swz, CUtensorMap* out) {
    EncodeTiledFn enc = get_encode();
    if (!enc) return set_error(CN_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(out, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(CN_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return CN_OK;
}

int encode_weight_map(int type, const void* d_w, int64_t rows, uint64_t rb, CUtensorMap* out) {
    int bx = box_bytes(type);
    if (bx == 0) return set_error(CN_ERR_UNSUPPORTED, "no tiled GEMV for type %d", type);
    if (rb % 16 != 0 || (reinterpret_cast<uintptr_t>(d_w) & 15) != 0 || rows <= 0)
        return set_error(CN_ERR_UNSUPPORTED, "weight layout not TMA-tileable");
    EncodeTiledFn enc = get_encode();
    if (!enc) return set_error(CN_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {rb / 8, (cuuint64_t)rows};
    cuuint64_t strides[1] = {rb};
    cuuint32_t box[2] = {(cuuint32_t)(bx / 8), (cuuint32_t)kTileRows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(d_w), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(CN_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return CN_OK;
}

template <int TYPE, int NT>
static int occupancy_ctas(cn_ctx* ctx) {
    static int cached[64] = {0};  // per device
    int dev = ctx->device & 63;
    if (cached[dev] <= 0) {
        auto k = gemv_kernel<TYPE, NT>;
        CN_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Geo<TYPE, NT>::kSmem + Geo<TYPE, NT>::kClusMax * Geo<TYPE, NT>::kSlotB));
        int n = 0;
        CN_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kThreads, Geo<TYPE, NT>::kSmem));
        cached[dev] = n > 0 ? n : 1;
    }
    return cached[dev];
}

static int pick_nt(int batch) { return batch <= 4 ? 1 : batch <= 8 ? 2 : batch <= 16 ? 4 : 8; }

static bool tileable(int type, int64_t cols, uint64_t rb) {
    return box_bytes(type) > 0 && cols % 256 == 0 && rb % 16 == 0;
}

int gemv_plan(cn_ctx* ctx, int type, int64_t rows, int64_t cols, int batch, bool tma,
              GemvPlan* p) {
    p->nt = pick_nt(batch);
    p->tma = tma;
    p->tiles = (int)((rows + kTileRows - 1) / kTileRows);
    p->units = (int)(cols / 256);
    p->path = kPathMma;
    if (!tma) return CN_OK;
    const int q4k_path = type == CN_TYPE_Q4_K ? gemv_q4k_path() : kPathMma;
    // batches 9-16 take the integer kernel's 16-sequence form (measured on B200
    // at batch 16: Llama-2-70B's 28672 x 8192 77 us against 84-92 us on the
    // fp16 kernel, 11008 x 4096 33.5 against 36.0 us; only a matrix of a few
    // units per SM does worse, 4096 x 4096 39.1 against 32.1 us -- kept on the
    // integer form so that a layer's q/k/v and gate/up still form one launch)
    if (q4k_path == kPathI8 && batch <= i8::kMaxNB) {
        p->path = kPathI8;
        p->tiles = (int)((rows + 127) / 128);
        p->ctas = gemv_i8_ctas(ctx->sms, p->tiles, p->units, batch);
        p->xfrag_bytes = gemv_i8_xbytes(cols, batch);
        p->xsum_bytes = 0;
        p->xinv_bytes = 0;
        p->partial_bytes = gemv_i8_partial_bytes(p->ctas);
        p->counters = (size_t)p->tiles * 8;  // one per 16-row sub-tile
        return gemv_i8_prepare();
    }
    if (q4k_path == kPathTc && batch <= tc::kMaxNB) {
        p->path = kPathTc;
        p->tiles = (int)((rows + tc::kRows - 1) / tc::kRows);
        p->ctas = gemv_tc_ctas(ctx->sms, p->tiles, p->units);
        p->xfrag_bytes = gemv_tc_xbytes(cols);
        p->xsum_bytes = 0;
        p->xinv_bytes = 0;
        p->partial_bytes = gemv_tc_partial_bytes(p->ctas);
        p->counters = (size_t)p->tiles;
        return gemv_tc_prepare();
    }
    int occ = 1;
#define CN_OCC(T)                                                  \
    switch (p->nt) {                                               \
        case 1: occ = occupancy_ctas<T, 1>(ctx); break;            \
        case 2: occ = occupancy_ctas<T, 2>(ctx); break;            \
        case 4: occ = occupancy_ctas<T, 4>(ctx); break;            \
        default: occ = occupancy_ctas<T, 8>(ctx); break;           \
    }
    if (type == CN_TYPE_Q4_0) { CN_OCC(CN_TYPE_Q4_0) }
    else if (type == CN_TYPE_Q8_0) { CN_OCC(CN_TYPE_Q8_0) }
    else if (type == CN_TYPE_Q4_K) { CN_OCC(CN_TYPE_Q4_K) }
    else if (type == CN_TYPE_Q5_K) { CN_OCC(CN_TYPE_Q5_K) }
    else if (type == CN_TYPE_Q4_1) { CN_OCC(CN_TYPE_Q4_1) }
    else if (type == CN_TYPE_Q5_0) { CN_OCC(CN_TYPE_Q5_0) }
    else if (type == CN_TYPE_Q5_1) { CN_OCC(CN_TYPE_Q5_1) }
    else { CN_OCC(CN_TYPE_Q6_K) }
#undef CN_OCC
    if (occ < 0) return occ;  // error code from the occupancy query
    // Stream-K grid: every resident CTA gets an equal share of the
    // (tile, unit) space, but at least 2 units each.
    const int64_t total = (int64_t)p->tiles * p->units;
    int min_units = 2;
#ifdef CHATNET_TUNING
    if (const char* e = getenv("CHATNET_MMA_MIN_UNITS")) min_units = atoi(e) > 0 ? atoi(e) : 2;
#endif
    int64_t want = total / min_units > 0 ? total / min_units : 1;
    // at most 8 CTAs may share a tile (the fix-up sums up to 8 partials):
    // ranges of at least units/7 units guarantee that
    const int64_t cap = (int64_t)p->tiles * 7 > 0 ? (int64_t)p->tiles * 7 : 1;
    if (want > cap) want = cap;
    int ctas = ctx->sms * occ;
    if (want < ctas) ctas = (int)want;
    // Whole tiles for short rows when there are enough tiles: one CTA per
    // 128-row tile of at most 16 units, none shared (a shared tile's fix-up --
    // partials, fence, counter, the last CTA's sum -- costs more there than
    // the extra CTAs gain).  Measured on B200 (prep + GEMV replayed from a
    // graph): Q4_0 5632 x 2048 (44 tiles) 11.9 -> 10.9 us, Q6_K 32000 x 4096
    // 35.0 -> 29.9 us, Q4_K 11008 x 4096 at batch 32 53.5 -> 42.2 us,
    // TinyLlama decode 621 -> 651 tok/s; long rows (Llama-2-70B's O and down
    // at batch 32) lose with whole tiles (611 -> 504 tok/s) and keep the split.
    int whole = 40;
#ifdef CHATNET_TUNING
    if (const char* e = getenv("CHATNET_MMA_WHOLE_TILES")) whole = atoi(e);
#endif
    if (whole > 0 && p->tiles >= whole && p->units <= 16 && p->tiles <= ctx->sms * occ) {
        ctas = p->tiles;
        // at batch 1-8, s = 2..4 CTAs per tile when all of them are resident
        // together, at least two units each: a cluster split (launch_tma),
        // whose fix-up costs little.  Measured on B200 (prep + GEMV, us):
        // Q4_0 5632 x 2048 10.7 -> 8.3 / 7.5 / 6.7 at s = 2 / 3 / 4 (7.7 at
        // s = 6), Q6_K 11008 x 4096 26.6 -> 17.9 / 17.8 at s = 2 / 3, and
        // TinyLlama decode 911 -> 987 / 1005 tok/s at s = 2 / 3 for its
        // 88-tile gate/up.
        int sp = (ctx->sms * occ) / p->tiles;
        if (sp > p->units / 2) sp = p->units / 2;
        if (sp > 4) sp = 4;
        if (p->nt <= 2 && sp >= 2) ctas = sp * p->tiles;
    }
    p->ctas = ctas;
    const int chunks = p->units * 8;
    p->xfrag_bytes = (size_t)chunks * p->nt * 32 * sizeof(uint4);
    p->xsum_bytes = type_needs_xsum(type) ? (size_t)chunks * p->nt * 4 * sizeof(float) : 0;
    p->xinv_bytes = (size_t)p->units * p->nt * 4 * sizeof(float);
    p->partial_bytes = (size_t)2 * ctas * kTileRows * p->nt * 4 * sizeof(float);
    p->counters = (size_t)p->tiles * kCons;
    return CN_OK;
}

// How many clusters of `cs` CTAs of gemv_kernel<TYPE, NT> fit on the device
// at once with cs - 1 slots (0 if the query fails); read once per device and
// size.
template <int TYPE, int NT>
static int cluster_fit_mma(int dev, int cs) {
    static std::mutex mu;
    static int n[64][9];
    static bool have[64][9] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (have[dev & 63][cs]) return n[dev & 63][cs];
    using G = Geo<TYPE, NT>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs * 64);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)G::kSmem + (size_t)(cs - 1) * G::kSlotB;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)cs;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, gemv_kernel<TYPE, NT>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        c = 0;
    }
    n[dev & 63][cs] = c;
    have[dev & 63][cs] = true;
    return c;
}

template <int TYPE, int NT>
static int launch_tma(cn_ctx* ctx, const GemvMaps* maps, const GemvPlan& p, GemvArgs a) {
    using G = Geo<TYPE, NT>;
    // the same number (2..8) of CTAs on every tile at batch 1-8, every
    // cluster resident at once: cluster split
    a.csize = 0;
    const int cs = p.ctas % p.tiles == 0 ? p.ctas / p.tiles : 0;
    if (NT <= 2 && cs >= 2 && cs - 1 <= G::kClusMax && cs <= p.units &&
        cluster_fit_mma<TYPE, NT>(ctx->device, cs) >= p.tiles) {
        a.csize = cs;
        CN_CUDA(launch_cluster_k(true, cs, gemv_kernel<TYPE, NT>, dim3(p.ctas), dim3(kThreads),
                                 (size_t)G::kSmem + (size_t)(cs - 1) * G::kSlotB, ctx->stream, *maps, a));
    } else {
        CN_CUDA(launch_k(true, gemv_kernel<TYPE, NT>, dim3(p.ctas), dim3(kThreads), (size_t)G::kSmem, ctx->stream,
                         *maps, a));
    }
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

int gemv_make(cn_ctx* ctx, int type, const void* d_w, int64_t rows, int64_t cols,
              const CUtensorMap* map, int batch, GemvOp* op, uint64_t rb) {
    CN_CHECK(type_supported(type), CN_ERR_UNSUPPORTED, "Unsupported weight quantization type: %d",
             type);
    CN_CHECK(d_w, CN_ERR_INVALID_ARG, "null weight pointer");
    CN_CHECK(rows > 0 && cols > 0 && batch > 0 && batch <= 32, CN_ERR_INVALID_ARG,
             "bad matvec shape rows=%lld cols=%lld batch=%d", (long long)rows, (long long)cols,
             batch);
    CN_CHECK(rows < (1ll << 31) && cols < (1ll << 31), CN_ERR_INVALID_ARG, "matvec too large");
    op->type = type;
    op->w = d_w;
    op->rows = rows;
    op->cols = cols;
    op->batch = batch;
    op->rb = rb ? rb : row_bytes(type, cols);
    CN_CHECK(op->rb >= row_bytes(type, cols), CN_ERR_INVALID_ARG, "row stride below the row's bytes");
    op->tma = tileable(type, cols, op->rb) && ((reinterpret_cast<uintptr_t>(d_w) & 15) == 0);
    if (op->tma) {
        if (map) op->map = *map;
        else if (encode_weight_map(type, d_w, rows, op->rb, &op->map) != CN_OK) op->tma = false;
    }
    if (!op->tma) {
        int blk = type == CN_TYPE_Q4_0 || is_block32(type) ? 32
                  : (type == CN_TYPE_Q4_K || type == CN_TYPE_Q6_K || is_superblock(type)) ? 256 : 1;
        CN_CHECK(cols % blk == 0, CN_ERR_INVALID_ARG, "inDim %lld not a multiple of %d",
                 (long long)cols, blk);
    }
    set_error(CN_OK, "");
    return gemv_plan(ctx, type, rows, cols, batch, op->tma, &op->plan);
}

float gemv_step1_scale(int type) { return type == CN_TYPE_Q4_K || type == CN_TYPE_Q5_K ? 0.0625f : 1.0f; }

int gemv_prep_kind(const GemvOp& op) {
    if (op.plan.path == kPathI8) return 3;
    if (op.plan.path == kPathTc) return 2;
    return type_needs_xsum(op.type) ? 1 : 0;
}

bool pdl_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("CHATNET_PDL");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

// Q4_K decode GEMVs run on the integer path unless CHATNET_GEMV names
// another family ("tc" or "mma"); read once per process.
int gemv_q4k_path() {
    static int path = -1;
    if (path < 0) {
        const char* e = getenv("CHATNET_GEMV");
        path = (e && strcmp(e, "tc") == 0) ? kPathTc : (e && strcmp(e, "mma") == 0) ? kPathMma : kPathI8;
    }
    return path;
}

PrepTarget prep_target(const GemvOp* op, const GemvBufs& b) {
    PrepTarget pt;
    if (!op || !op->tma) return pt;
    pt.kind = gemv_prep_kind(*op);
    pt.nt_count = op->plan.nt;
    pt.step1 = gemv_step1_scale(op->type);
    pt.xfrag = b.xfrag;
    pt.xsum = type_needs_xsum(op->type) ? b.xsum : nullptr;
    pt.xinv = b.xinv;
    return pt;
}

int gemv_prep(cudaStream_t st, int sms, const GemvOp& op, const float* d_x, const GemvBufs& b) {
    if (!op.tma) return CN_OK;
    CN_CHECK((reinterpret_cast<uintptr_t>(d_x) & 15) == 0, CN_ERR_INVALID_ARG,
             "x must be 16-byte aligned");
    const int64_t items = (int64_t)op.plan.units * op.batch;
    int blocks = (int)((items + 7) / 8);
    if (blocks > sms * 8) blocks = sms * 8;
    CN_CUDA(launch_k(true, xprep_kernel, dim3(blocks), dim3(256), 0, st, d_x, (int)op.cols, op.batch,
                     prep_target(&op, b)));
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

int add_norm_prep(cudaStream_t st, const float* x_in, const float* delta, float* x_out, const float* w,
                  float* y, int n, int rows, float eps, const GemvOp* op, const GemvBufs& b,
                  const XchgIn* xin) {
    const bool xch = xin && xin->size > 1;
    CN_CHECK(n % 4 == 0 && (reinterpret_cast<uintptr_t>(x_in) & 15) == 0 &&
                 (!delta || (reinterpret_cast<uintptr_t>(delta) & 15) == 0),
             CN_ERR_INVALID_ARG, "norm: dim must be a multiple of 4 and rows 16-byte aligned");
    CN_CHECK(!(delta || xch) || (x_out && x_out != x_in), CN_ERR_INVALID_ARG, "norm: x_out must not alias x_in");
    CN_CHECK(!xch || (xin->src && xin->flags && xin->seq_base && xin->err &&
                      (reinterpret_cast<uintptr_t>(xin->src) & 15) == 0 && xin->rank_stride % 4 == 0 &&
                      xin->parity_stride % 4 == 0),
             CN_ERR_INVALID_ARG, "norm: bad exchange input");
    PrepTarget pt = prep_target(op, b);
    if (pt.kind >= 0 && n % 256 != 0) pt.kind = -1;  // the GEMV preps for itself
    XchgIn xi;
    if (xch) xi = *xin;
    const int units = n / 256;
    // tensor parallel: the cluster form reads every rank's slots once per row
    // instead of once per CTA; on one GPU the plain form schedules sooner
    // behind a GEMV that holds whole SMs (a cluster needs free SMs in one GPC)
    if (xch && n % 256 == 0 && units >= 1 && (units + kNormCluster - 1) / kNormCluster * 256 <= kNormClMaxVals) {
        const int C = units < kNormCluster ? units : kNormCluster;
        CN_CUDA(launch_cluster_k(true, C, add_norm_prep_cl_kernel, dim3(C, rows), dim3(kNormClThreads), 0, st,
                                 x_in, delta, x_out, w, y, n, eps, pt, xi));
    } else {
        CN_CUDA(launch_k(true, add_norm_prep_kernel, dim3((n + 255) / 256, rows), dim3(kNormThreads), 0, st, x_in,
                         delta, x_out, w, y, n, eps, pt, xi));
    }
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

int xchg_wait(cudaStream_t st, const XchgIn& xin) {
    CN_CHECK(xin.size > 1 && !xin.ll && xin.flags && xin.seq_base && xin.err, CN_ERR_INVALID_ARG,
             "bad exchange");
    CN_CUDA(launch_k(true, xchg_wait_kernel, dim3(1), dim3(32), 0, st, xin));
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

int norm_prep(cudaStream_t st, const float* x, const float* w, float* y, int n, int rows,
              float eps, const GemvOp* op, const GemvBufs& b) {
    return add_norm_prep(st, x, nullptr, nullptr, w, y, n, rows, eps, op, b);
}

static int gemv_mma_launch(cn_ctx* ctx, cudaStream_t st, const GemvOp* ops, int n, const GemvPlan& p,
                           const GemvBufs& b, float* const* y);

int gemv_run(cn_ctx* ctx, cudaStream_t st, const GemvOp& op, const float* d_x, const GemvBufs& b,
             float* d_y, const XchgOut* xo) {
    CN_CHECK((reinterpret_cast<uintptr_t>(d_y) & 3) == 0, CN_ERR_INVALID_ARG, "y must be aligned");
    CN_CHECK(!xo || xo->size <= 1 || op.plan.path == kPathI8, CN_ERR_UNSUPPORTED,
             "tensor-parallel exchange needs the integer GEMV (Q4_K, batch <= 8)");
    if (!op.tma) {
        int blk = op.type == CN_TYPE_Q4_0 || is_block32(op.type) ? 32
                  : (op.type == CN_TYPE_Q4_K || op.type == CN_TYPE_Q6_K || is_superblock(op.type)) ? 256 : 1;
        int threads = 256;
        int64_t warps = op.rows * op.batch;
        int64_t blocks = (warps * 32 + threads - 1) / threads;
        if (blocks > ctx->sms * 16) blocks = ctx->sms * 16;
        CN_CUDA(launch_k(true, gemv_generic_kernel, dim3((unsigned)blocks), dim3(threads), 0, st,
            op.type, (const uint8_t*)op.w, op.rows, (int)op.cols, op.rb, blk, d_x, d_y, op.batch));
        CN_CUDA(cudaGetLastError());
        return CN_OK;
    }
    if (op.plan.path == kPathI8)
        return gemv_i8_run(st, ctx->dev_err, &op.map, op.rows, op.cols, op.batch, op.plan.ctas,
                           reinterpret_cast<const uint8_t*>(b.xfrag), b.partials, b.counters, d_y, xo);
    if (op.plan.path == kPathTc)
        return gemv_tc_run(st, ctx->dev_err, &op.map, op.rows, op.cols, op.batch, op.plan.ctas,
                           reinterpret_cast<const uint8_t*>(b.xfrag), b.partials, b.counters, d_y);
    return gemv_mma_launch(ctx, st, &op, 1, op.plan, b, &d_y);
}

// The fp16 mma.sync GEMV over n matrices of one type with the same input
// (one launch; n == 1: a single matrix).
static int gemv_mma_launch(cn_ctx* ctx, cudaStream_t st, const GemvOp* ops, int n, const GemvPlan& p,
                           const GemvBufs& b, float* const* y) {
    GemvArgs a = {};
    GemvMaps maps;
    a.nmat = n;
    int tiles = 0;
    for (int i = 0; i < kMaxGroup; i++) {
        const int mi = i < n ? i : n - 1;
        maps.m[i] = ops[mi].map;
        a.toff[i] = tiles;
        if (i < n) {
            a.mrows[i] = ops[i].rows;
            a.my[i] = y[i];
            tiles += (int)((ops[i].rows + kTileRows - 1) / kTileRows);
        }
    }
    a.toff[kMaxGroup] = tiles;
    CN_CHECK(tiles == p.tiles, CN_ERR_INVALID_ARG, "GEMV plan does not match its matrices");
    a.rows = ops[0].rows;
    a.y = y[0];
    a.units = p.units;
    a.tiles = p.tiles;
    a.batch = ops[0].batch;
    a.xfrag = b.xfrag;
    a.xsum = b.xsum;
    a.xinv = b.xinv;
    a.partials = b.partials;
    a.counters = b.counters;
    a.err = ctx->dev_err;
    cn_ctx tmp = *ctx;
    tmp.stream = st;
#define CN_DISPATCH(T)                                               \
    switch (p.nt) {                                                  \
        case 1: return launch_tma<T, 1>(&tmp, &maps, p, a);          \
        case 2: return launch_tma<T, 2>(&tmp, &maps, p, a);          \
        case 4: return launch_tma<T, 4>(&tmp, &maps, p, a);          \
        default: return launch_tma<T, 8>(&tmp, &maps, p, a);         \
    }
    const int type = ops[0].type;
    if (type == CN_TYPE_Q4_0) { CN_DISPATCH(CN_TYPE_Q4_0) }
    if (type == CN_TYPE_Q8_0) { CN_DISPATCH(CN_TYPE_Q8_0) }
    if (type == CN_TYPE_Q4_K) { CN_DISPATCH(CN_TYPE_Q4_K) }
    if (type == CN_TYPE_Q5_K) { CN_DISPATCH(CN_TYPE_Q5_K) }
    if (type == CN_TYPE_Q4_1) { CN_DISPATCH(CN_TYPE_Q4_1) }
    if (type == CN_TYPE_Q5_0) { CN_DISPATCH(CN_TYPE_Q5_0) }
    if (type == CN_TYPE_Q5_1) { CN_DISPATCH(CN_TYPE_Q5_1) }
    CN_DISPATCH(CN_TYPE_Q6_K)
#undef CN_DISPATCH
}

int gemv_group_make(cn_ctx* ctx, const GemvOp* ops, int n, GemvGroup* g) {
    CN_CHECK(n >= 1 && n <= 3, CN_ERR_INVALID_ARG, "a GEMV group has 1..3 members");
    int64_t rows = 0;
    const int path = ops[0].plan.path;
    for (int i = 0; i < n; i++) {
        const GemvOp& o = ops[i];
        if ((o.plan.path != kPathI8 && o.plan.path != kPathMma) || !o.tma || o.plan.path != path ||
            o.cols != ops[0].cols || o.batch != ops[0].batch || o.type != ops[0].type)
            return set_error(CN_ERR_UNSUPPORTED, "GEMVs cannot share a launch");
        g->ops[i] = o;
        rows += (o.rows + 127) / 128 * 128;
    }
    g->n = n;
    if (path == kPathMma) {
        // the fp16 kernel's stream-K plan over the concatenated row tiles
        int rc = gemv_plan(ctx, ops[0].type, rows, ops[0].cols, ops[0].batch, true, &g->plan);
        if (rc) return rc;
        CN_CHECK(g->plan.path == kPathMma, CN_ERR_UNSUPPORTED, "GEMVs cannot share a launch");
        return CN_OK;
    }
    GemvPlan p = ops[0].plan;
    p.tiles = (int)(rows / 128);
    p.ctas = gemv_i8_ctas(ctx->sms, p.tiles, p.units, ops[0].batch);
    p.partial_bytes = gemv_i8_partial_bytes(p.ctas);
    p.counters = (size_t)p.tiles * 8;
    g->plan = p;
    return CN_OK;
}

int gemv_group_run(cn_ctx* ctx, cudaStream_t st, const GemvGroup& g, const GemvBufs& b, float* const* y) {
    for (int i = 0; i < g.n; i++)
        CN_CHECK((reinterpret_cast<uintptr_t>(y[i]) & 3) == 0, CN_ERR_INVALID_ARG, "y must be aligned");
    if (g.plan.path == kPathMma) return gemv_mma_launch(ctx, st, g.ops, g.n, g.plan, b, y);
    const CUtensorMap* maps[3];
    int64_t rows[3];
    for (int i = 0; i < g.n; i++) {
        CN_CHECK((reinterpret_cast<uintptr_t>(y[i]) & 3) == 0, CN_ERR_INVALID_ARG, "y must be aligned");
        maps[i] = &g.ops[i].map;
        rows[i] = g.ops[i].rows;
    }
    return gemv_i8_run_group(st, ctx->dev_err, g.n, maps, rows, g.ops[0].cols, g.ops[0].batch, g.plan.ctas,
                             reinterpret_cast<const uint8_t*>(b.xfrag), b.partials, b.counters, y);
}

int gemv_reserve(const GemvPlan& p, GemvNeeds* n) {
    size_t x = p.xfrag_bytes, s = p.xsum_bytes, pa = p.partial_bytes, c = p.counters;
    if (p.xinv_bytes > n->xinv_bytes) n->xinv_bytes = p.xinv_bytes;
    if (x > n->xfrag_bytes) n->xfrag_bytes = x;
    if (s > n->xsum_bytes) n->xsum_bytes = s;
    if (pa > n->partial_bytes) n->partial_bytes = pa;
    if (c > n->counters) n->counters = c;
    return CN_OK;
}

// Grows the context's GEMV scratch to what `op` needs.
static int ctx_reserve(cn_ctx* ctx, const GemvOp& op) {
    if (!op.tma) return CN_OK;
    const GemvPlan& p = op.plan;
    int rc = ensure(&ctx->xfrag, &ctx->xfrag_bytes, p.xfrag_bytes, false);
    if (!rc && p.xsum_bytes) rc = ensure((void**)&ctx->xsum, &ctx->xsum_bytes, p.xsum_bytes, false);
    if (!rc) rc = ensure((void**)&ctx->partials, &ctx->partial_bytes, p.partial_bytes, false);
    if (!rc) rc = ensure((void**)&ctx->xinv, &ctx->xinv_bytes, p.xinv_bytes, false);
    if (!rc) {
        size_t cb = ctx->counter_count * sizeof(int);
        rc = ensure((void**)&ctx->counters, &cb, p.counters * sizeof(int), true);
        ctx->counter_count = cb / sizeof(int);
    }
    return rc;
}

static GemvBufs ctx_bufs(cn_ctx* ctx) {
    return GemvBufs{(uint4*)ctx->xfrag, ctx->xsum, ctx->partials, ctx->counters, ctx->xinv};
}

int gemv_launch(cn_ctx* ctx, int type, const void* d_w, int64_t rows, int64_t cols,
                const CUtensorMap* map, const float* d_x, float* d_y, int batch) {
    CN_CHECK((reinterpret_cast<uintptr_t>(d_x) & 15) == 0 && (reinterpret_cast<uintptr_t>(d_y) & 3) == 0,
             CN_ERR_INVALID_ARG, "x must be 16-byte aligned and y 4-byte aligned");
    GemvOp op;
    int rc = gemv_make(ctx, type, d_w, rows, cols, map, batch, &op);
    if (rc || (rc = ctx_reserve(ctx, op))) return rc;
    const GemvBufs b = ctx_bufs(ctx);
    rc = gemv_prep(ctx->stream, ctx->sms, op, d_x, b);
    if (rc) return rc;
    return gemv_run(ctx, ctx->stream, op, d_x, b, d_y);
}

int gemv_time(cn_ctx* ctx, const cn_tensor* const* ws, int n_w, const float* d_x, float* d_y, int batch,
              int launches, int reps, float* us_out, int* kernels_per_launch) {
    CN_CHECK(n_w >= 1 && launches >= 1 && reps >= 1, CN_ERR_INVALID_ARG, "bad timing request");
    CN_CHECK((reinterpret_cast<uintptr_t>(d_x) & 15) == 0 && (reinterpret_cast<uintptr_t>(d_y) & 3) == 0,
             CN_ERR_INVALID_ARG, "x must be 16-byte aligned and y 4-byte aligned");
    std::vector<GemvOp> ops(n_w);
    for (int i = 0; i < n_w; i++) {
        const cn_tensor* w = ws[i];
        CN_CHECK(w && w->ctx == ctx && w->rows == ws[0]->rows && w->cols == ws[0]->cols && w->type == ws[0]->type,
                 CN_ERR_INVALID_ARG, "timed matrices must share one shape and type on this context");
        int rc = gemv_make(ctx, w->type, w->d, w->rows, w->cols, w->has_map ? &w->map : nullptr, batch, &ops[i]);
        if (rc || (rc = ctx_reserve(ctx, ops[i]))) return rc;
    }
    const GemvBufs b = ctx_bufs(ctx);
    cudaStream_t s = ctx->stream;
    // one graph holds `launches` ops (prep + GEMV each) cycling through the
    // matrices, so no host launch gap lands inside the timed replays
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    CN_CUDA(cudaStreamSynchronize(s));
    CN_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    int rc = CN_OK;
    for (int i = 0; i < launches && !rc; i++) {
        rc = gemv_prep(s, ctx->sms, ops[i % n_w], d_x, b);
        if (!rc) rc = gemv_run(ctx, s, ops[i % n_w], d_x, b, d_y);
    }
    cudaError_t e = cudaStreamEndCapture(s, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_error(e, "cudaStreamEndCapture");
    e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_error(e, "cudaGraphInstantiate");
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    for (int r = 0; r < 2 && e == cudaSuccess; r++) e = cudaGraphLaunch(ge, s);  // warm-up
    for (int r = 0; r < reps && e == cudaSuccess; r++) {
        e = cudaEventRecord(e0, s);
        if (e == cudaSuccess) e = cudaGraphLaunch(ge, s);
        if (e == cudaSuccess) e = cudaEventRecord(e1, s);
        if (e == cudaSuccess) e = cudaEventSynchronize(e1);
        float ms = 0.f;
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
        us_out[r] = ms * 1000.f / launches;
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaGraphExecDestroy(ge);
    if (e != cudaSuccess) return cuda_error(e, "timed GEMV replays");
    if (kernels_per_launch) *kernels_per_launch = ops[0].tma ? 2 : 1;
    return CN_OK;
}

}  // namespace cn
