// matmul.cu -- prefill: Q4_0 / Q4_K dequant-matmul on the 5th-generation
// tensor cores (tcgen05, tensor memory, TMA).
//
// Y[m][n] (+)= sum_k X[m][k] * W[n][k] for M tokens in one pass: the batched
// form of TensorMath.MatVecMulQ4_0 / MatVecMulGeneric(Q4_K)
// (Tensors/TensorMath.cs:548-578, :624-656) with the weights of
// DequantQ4_0.Dequantize (Tensors/Quantization/DequantQ4_0.cs:28-58) or
// DequantQ4K.Dequantize (DequantQ4K.cs:37-77), which ChatNet runs as M
// sequential matvecs (InferenceEngine.cs:235-239).  Both formats store 256
// weights of a row in 144 bytes (8 Q4_0 blocks, or one Q4_K super-block), so
// the raw ring is the same; only the expansion differs.
//
//  * A tile is 128 weight rows x 128 tokens.  The kernel is persistent: one
//    CTA per SM walks the tiles (weight row tile-major, so the CTAs running
//    at the same time share weight tiles in L2), and its accumulator in
//    tensor memory is double-buffered, so the epilogue of one tile overlaps
//    the MMAs of the next.
//  * The weights are the MMA's A operand and live in tensor memory: eight
//    decode warps in two warpgroups (one weight row per thread, the thread's
//    lane of tensor memory; warpgroup g takes blocks 2g and 2g + 1 of the
//    four Q4_0 blocks of every 128-position stage) read the row's raw blocks
//    from a shared-memory ring that TMA fills with 128 rows x 144 bytes (8
//    blocks, 2 stages) at a time, expand them to fp16 ((q - 8) exact, times
//    d, one rounding) and write them to tensor memory with tcgen05.st.  The
//    expanded weights never touch shared memory.
//  * The activations (fp16, K-major) are the B operand: per stage two TMA
//    tiles of 128 tokens x 64 positions with 128-byte swizzle, in a 4-stage
//    ring.
//  * One thread issues tcgen05.mma kind::f16 (M=128, N=128, K=16; fp32
//    accumulator in tensor-memory columns [0, 128) or [128, 256)), eight per
//    stage, and commits each stage to the barrier that frees its A slot and
//    B stage, and each tile to the barrier that hands its accumulator on.
//    The decode warps and the TMA producer signal one barrier per stage (one
//    arrival per warp), so the issuing thread waits once per eight MMAs: its
//    barrier wait costs about as long as two N = 128 MMAs take, and the
//    test of the next stage's barrier is issued before this stage's MMAs.
//  * Four epilogue warps read the accumulator back (tcgen05.ld, one weight
//    row per thread, 32 tokens per load), release it, and store Y with
//    coalesced rows (optionally adding into Y, the residual stream).
//  * Up to three weight matrices with the same K share one launch (q/k/v,
//    gate/up): the tiles run over their row tiles.
// Every mbarrier wait is bounded.  A thread that gives up raises the error
// word and stops waiting (its control flow stays uniform; results are
// garbage and flagged).  The CTA still waits for its own copies and MMAs
// before it frees its tensor memory.
#include <math.h>
#include <string.h>

#include <cmath>
#include <mutex>

#include "cn_common.cuh"
#include "cn_internal.h"

namespace cn {
namespace mm {

constexpr int kRows = 128;               // weight rows per tile (MMA M, tensor-memory lanes)
constexpr int kNT = 128;                 // tokens per tile (MMA N)
constexpr int kKS = 128;                 // K positions per stage (two 128-byte swizzle rows)
constexpr int kStages = 4;
constexpr int kBHalf = kNT * 64 * 2;     // 16 KB: one swizzled tile of 64 positions
constexpr int kBStage = 2 * kBHalf;      // 32 KB of activations per stage
// Raw weight ring: one stage holds 256 positions of 128 rows -- 144 bytes
// per row for Q4_0 (8 blocks) and Q4_K (one super-block).  Q6_K's 210-byte
// super-blocks are only 2-byte aligned, so its stages hold the 16-byte
// aligned 240-byte window around each (as the decode GEMV loads them).
// Both rings take 92,160 bytes.
template <int WT>
struct RawGeo {
    static constexpr int kRow = WT == CN_TYPE_Q6_K ? 240 : 144;
    static constexpr int kBytes = kRow * 128;
    static constexpr int kStages = WT == CN_TYPE_Q6_K ? 3 : 5;
};
constexpr int kRawStages = 5;  // barriers reserved (the most any ring uses)
constexpr int kRawRing = 5 * 144 * 128;
static_assert(RawGeo<CN_TYPE_Q6_K>::kStages * RawGeo<CN_TYPE_Q6_K>::kBytes == kRawRing &&
                  RawGeo<CN_TYPE_Q4_K>::kStages * RawGeo<CN_TYPE_Q4_K>::kBytes == kRawRing,
              "raw rings");
constexpr int kDBufs = 2;                // accumulator buffers
constexpr int kRawOff = kStages * kBStage;
constexpr int kACols = kKS / 2;          // tensor-memory columns of one A stage (2 fp16 each)
constexpr int kACol = kDBufs * kNT;      // accumulator(s) first, the A ring after them
// The split (hi + lo) variant: every weight and activation is carried as an
// exact pair of fp16 halves and each k-step runs three MMAs (Whi Xhi, Whi Xlo,
// Wlo Xhi) into the same accumulator.  A stage then holds both activation
// halves (64 KB) and an A slot both weight halves (128 columns), so the ring
// has two stages; shared and tensor memory add up to the same totals.
template <bool SPLIT>
struct SGeo {
    static constexpr int kStages = SPLIT ? 2 : mm::kStages;
    static constexpr int kBStage = SPLIT ? 2 * mm::kBStage : mm::kBStage;
    static constexpr int kACols = SPLIT ? 2 * mm::kACols : mm::kACols;
};
static_assert(SGeo<true>::kStages * SGeo<true>::kBStage == kStages * kBStage &&
                  SGeo<true>::kStages * SGeo<true>::kACols == kStages * kACols,
              "split ring sizes");
constexpr int kTmemCols = 512;
constexpr int kDecode = 256;             // decode threads: warps 0-7
constexpr int kEpi = 128;                // epilogue threads: warps 8-11
constexpr int kDecodeWarps = kDecode / 32, kEpiWarps = kEpi / 32;  // barrier arrivals (one per warp)
constexpr int kThreads = kDecode + kEpi + 64;  // warp 12 TMA, warp 13 MMA
constexpr int kWarpEpi0 = 8, kWarpTma = 12, kWarpMma = 13;
constexpr int kBarOff = kRawOff + kRawRing;
constexpr int kSmem = kBarOff + 512 + 1024;  // barriers, and slack to align the ring to 1 KB
constexpr int kMaxMats = 3;
static_assert(kACol + kStages * kACols <= kTmemCols, "tensor memory plan");
static_assert(kRawOff % 1024 == 0 && RawGeo<CN_TYPE_Q6_K>::kBytes % 128 == 0 && kBarOff % 8 == 0,
              "ring alignment");

// TMA descriptors: the activations and each weight matrix (8-byte elements,
// rows x row bytes, boxes of 144 bytes x 128 rows, as for the decode GEMV).
struct Maps {
    CUtensorMap x;
    CUtensorMap xlo;  // split variant: the activations' low halves
    CUtensorMap w[kMaxMats];
};
static_assert(kSmem <= 227 * 1024, "shared memory");

// kind::f16 instruction descriptor: D f32 (bits 4-5 = 1), A and B f16
// (bits 7-9, 10-12 = 0), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kNT >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);

struct Args {
    int nmat;
    int toff[kMaxMats + 1];     // first row tile of each matrix; toff[nmat] = all row tiles
    const uint8_t* w[kMaxMats];
    int64_t rows[kMaxMats];
    float* y[kMaxMats];         // [M][ldy[m]]
    int64_t ldy[kMaxMats];
    int64_t rb;                 // bytes per weight row
    const float* xs;            // per-token factor of the result (x's inverse scale), or null
    float wscale[kMaxMats];     // split variant: power of two the weights are expanded at (2^E)
    float oscale[kMaxMats];     // factor of matrix m's results (2^-E; 1 outside the split variant)
    int M, K;                   // K % 256 == 0
    int accumulate;             // 1: Y += result, 0: Y = result
    int tok_tiles;              // token tiles of 128; tile t = row tile t / tok_tiles, token tile t % tok_tiles
    int tiles;                  // row tiles x token tiles
    uint32_t* err;
};

template <typename T>
__device__ __forceinline__ T pick(const T (&v)[kMaxMats], int m) {
    return m == 2 ? v[2] : m == 1 ? v[1] : v[0];
}

__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// Expands two consecutive Q4_0 blocks, the 36 bytes wd[0..8] (block 0: d
// at bytes 0-1, quants at 2-17; block 1: d at 18-19, quants at 20-35), into
// 64 fp16 weights in K order, two per word: o[c] holds positions 2c (low
// half) and 2c + 1.  Position j < 16 of a block is the low nibble of quant
// byte j, position 16 + j its high nibble; the value is fp16((q - 8) * d).
__device__ __forceinline__ void expand_q4_0_pair(const uint32_t (&wd)[9], uint32_t (&o)[32]) {
    constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024 in both halves
    constexpr uint32_t kBias = 0x64086408u;   // fp16 1032 = 1024 + 8
#pragma unroll
    for (int blk = 0; blk < 2; blk++) {
        uint32_t q[4], d;
        if (blk == 0) {
            d = wd[0] & 0xFFFFu;
#pragma unroll
            for (int i = 0; i < 4; i++) q[i] = __funnelshift_r(wd[i], wd[i + 1], 16);
        } else {
            d = wd[4] >> 16;
#pragma unroll
            for (int i = 0; i < 4; i++) q[i] = wd[5 + i];
        }
        const uint32_t d2 = d | (d << 16);
#pragma unroll
        for (int i = 0; i < 4; i++) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                // quant bytes 4i + 2h and 4i + 2h + 1 in the low byte of each half
                const uint32_t t = __byte_perm(q[i], 0u, h ? 0x4342u : 0x4140u);
                const uint32_t lo = lop3_and_or(t, 0x000F000Fu, kMagic);       // 1024 + q
                const uint32_t hi = lop3_and_or(t >> 4, 0x000F000Fu, kMagic);
                o[16 * blk + 2 * i + h] = h2_mul(h2_sub(lo, kBias), d2);      // (q - 8) exact, then * d
                o[16 * blk + 8 + 2 * i + h] = h2_mul(h2_sub(hi, kBias), d2);
            }
        }
    }
}

// Expands two Q4_K sub-blocks into 64 fp16 weights in K order (o[c] holds
// positions 2c, 2c + 1).  qw[0..3] and qw[4..7] are the sub-blocks' 16 quant
// bytes each (DequantQ4K.cs:59-71: position j < 16 is the low nibble of byte
// j, 16 + j its high nibble).  The weight d * sc * q - dmin * m is formed as
// fma(sc * q, d, -fp16(dmin * m)): q, sc * q (<= 945) and d are exact in
// fp16, so only the sub-block's minimum term and the result are rounded.
// d2: d in both halves; sc2/ndm2: the sub-blocks' sc and -dmin * m pairs.
__device__ __forceinline__ void expand_q4k_pair(const uint32_t (&qw)[8], uint32_t d2, const uint32_t (&sc2)[2],
                                                const uint32_t (&ndm2)[2], uint32_t (&o)[32]) {
    constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024 in both halves
#pragma unroll
    for (int blk = 0; blk < 2; blk++) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t t = __byte_perm(qw[4 * blk + i], 0u, h ? 0x4342u : 0x4140u);
                const uint32_t lo = h2_mul(h2_sub(lop3_and_or(t, 0x000F000Fu, kMagic), kMagic), sc2[blk]);
                const uint32_t hi = h2_mul(h2_sub(lop3_and_or(t >> 4, 0x000F000Fu, kMagic), kMagic), sc2[blk]);
                o[16 * blk + 2 * i + h] = h2_fma(lo, d2, ndm2[blk]);
                o[16 * blk + 8 + 2 * i + h] = h2_fma(hi, d2, ndm2[blk]);
            }
        }
    }
}

// Expands this thread's 64 positions of half h of a Q6_K super-block (sb:
// its first byte in shared memory, 2-byte aligned) into fp16, o[c] holding
// positions 2c, 2c + 1.  Position 32s + l of the half (DequantQ6K.cs:37-88)
// takes the low (s < 2) or high nibble of ql[64h + l + 32(s & 1)], bits 2s of
// qh[32h + l] and scale 8h + l/16 + 2s, and is (d * sc) * (q - 32) in fp32 --
// the reference's value -- rounded once to fp16.  Warpgroup wg holds s = 2wg,
// 2wg + 1: slice position j = ql byte 64h + j, nibble wg, qh bits 4wg + 2(j/32).
__device__ __forceinline__ void expand_q6k_half(const uint8_t* sb, int h, int wg, float d, uint32_t (&o)[32]) {
    uint32_t qh[8];
#pragma unroll
    for (int k = 0; k < 8; k++) qh[k] = lds_u32_a2(sb + 128 + 32 * h + 4 * k);
    float dsc[4];  // [j / 32][l / 16]
#pragma unroll
    for (int jj = 0; jj < 2; jj++)
#pragma unroll
        for (int ll = 0; ll < 2; ll++)
            dsc[2 * jj + ll] = __fmul_rn(d, (float)(int8_t)sb[192 + 8 * h + ll + 4 * wg + 2 * jj]);
#pragma unroll
    for (int k = 0; k < 16; k++) {
        const uint32_t w = lds_u32_a2(sb + 64 * h + 4 * k);
        const uint32_t nib = (wg ? (w >> 4) : w) & 0x0F0F0F0Fu;
        const int jj = k >> 3;
        const uint32_t hb = (qh[k & 7] >> (4 * wg + 2 * jj)) & 0x03030303u;
        const uint32_t q4 = nib | (hb << 4);
        const float t = dsc[2 * jj + ((k & 7) >> 2)];
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; e++) v[e] = __fmul_rn(t, (float)((int)((q4 >> (8 * e)) & 0xFFu) - 32));
        o[2 * k] = pack_half2(v[0], v[1]);
        o[2 * k + 1] = pack_half2(v[2], v[3]);
    }
}

// ---- split variant: each weight as an exact pair of fp16 halves ----------
// Weights are expanded at 2^E (ws), a power of two chosen per matrix so that
// its largest weight stays below 2^14; the epilogue multiplies by 2^-E.

// hi = fp16(w), lo = fp16(w - hi) for two fp32 weights, packed in pairs.
__device__ __forceinline__ void split_pair(float w0, float w1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(w0, w1);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = pack_half2(w0 - __low2float(h), w1 - __high2float(h));  // the differences are exact in fp32
}

// The four low (or high, sh = 4) nibbles of w as floats, exactly: the nibble
// becomes the low mantissa bits of 2^23.
__device__ __forceinline__ void nib4_f32(uint32_t w, int sh, float (&f)[4]) {
#pragma unroll
    for (int k = 0; k < 4; k++)
        f[k] = __uint_as_float(0x4B000000u | ((w >> (8 * k + sh)) & 15u)) - 8388608.0f;
}

// Q4_0, split: two blocks as expand_q4_0_pair lays them out.  With D = d * ws
// (11 significant bits) cut into Dhi (its top 7 bits) and Dlo = D - Dhi (the
// other 4), (q - 8) * Dhi needs at most 11 bits and (q - 8) * Dlo at most 8,
// so both fp16 products are exact and hi + lo is the weight (q - 8) * d * ws.
__device__ __forceinline__ void expand_q4_0_pair_split(const uint32_t (&wd)[9], float ws, uint32_t (&ohi)[32],
                                                       uint32_t (&olo)[32]) {
    constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024 in both halves
    constexpr uint32_t kBias = 0x64086408u;   // fp16 1032 = 1024 + 8
#pragma unroll
    for (int blk = 0; blk < 2; blk++) {
        uint32_t q[4], d;
        if (blk == 0) {
            d = wd[0] & 0xFFFFu;
#pragma unroll
            for (int i = 0; i < 4; i++) q[i] = __funnelshift_r(wd[i], wd[i + 1], 16);
        } else {
            d = wd[4] >> 16;
#pragma unroll
            for (int i = 0; i < 4; i++) q[i] = wd[5 + i];
        }
        const float D = half_bits_to_float((uint16_t)d) * ws;
        const float Dhi = __uint_as_float(__float_as_uint(D) & 0xFFFE0000u);
        const uint32_t dh2 = pack_half2(Dhi, Dhi), dl2 = pack_half2(D - Dhi, D - Dhi);
#pragma unroll
        for (int i = 0; i < 4; i++) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t t = __byte_perm(q[i], 0u, h ? 0x4342u : 0x4140u);
                const uint32_t lo = h2_sub(lop3_and_or(t, 0x000F000Fu, kMagic), kBias);  // q - 8, exact
                const uint32_t hi = h2_sub(lop3_and_or(t >> 4, 0x000F000Fu, kMagic), kBias);
                ohi[16 * blk + 2 * i + h] = h2_mul(lo, dh2);
                olo[16 * blk + 2 * i + h] = h2_mul(lo, dl2);
                ohi[16 * blk + 8 + 2 * i + h] = h2_mul(hi, dh2);
                olo[16 * blk + 8 + 2 * i + h] = h2_mul(hi, dl2);
            }
        }
    }
}

// Q4_K, split: two sub-blocks as expand_q4k_pair lays them out.  The weight is
// the reference's fp32 value (d*sc)*q - dmin*m (DequantQ4K.cs:59-71), here at
// 2^E: dsc = fp32(d*sc) * ws and dm = fp32(dmin*m) * ws per sub-block.
__device__ __forceinline__ void expand_q4k_pair_split(const uint32_t (&qw)[8], const float (&dsc)[2],
                                                      const float (&dm)[2], uint32_t (&ohi)[32],
                                                      uint32_t (&olo)[32]) {
#pragma unroll
    for (int blk = 0; blk < 2; blk++) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float fl[4], fh[4];
            nib4_f32(qw[4 * blk + i], 0, fl);
            nib4_f32(qw[4 * blk + i], 4, fh);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                split_pair(__fsub_rn(__fmul_rn(dsc[blk], fl[2 * h]), dm[blk]),
                           __fsub_rn(__fmul_rn(dsc[blk], fl[2 * h + 1]), dm[blk]), ohi[16 * blk + 2 * i + h],
                           olo[16 * blk + 2 * i + h]);
                split_pair(__fsub_rn(__fmul_rn(dsc[blk], fh[2 * h]), dm[blk]),
                           __fsub_rn(__fmul_rn(dsc[blk], fh[2 * h + 1]), dm[blk]), ohi[16 * blk + 8 + 2 * i + h],
                           olo[16 * blk + 8 + 2 * i + h]);
            }
        }
    }
}

// Q6_K, split: expand_q6k_half's positions, each the reference's fp32 value
// (d * sc) * (q - 32) at 2^E (d already multiplied by ws), as hi + lo.
__device__ __forceinline__ void expand_q6k_half_split(const uint8_t* sb, int h, int wg, float d, uint32_t (&ohi)[32],
                                                      uint32_t (&olo)[32]) {
    uint32_t qh[8];
#pragma unroll
    for (int k = 0; k < 8; k++) qh[k] = lds_u32_a2(sb + 128 + 32 * h + 4 * k);
    float dsc[4];
#pragma unroll
    for (int jj = 0; jj < 2; jj++)
#pragma unroll
        for (int ll = 0; ll < 2; ll++)
            dsc[2 * jj + ll] = __fmul_rn(d, (float)(int8_t)sb[192 + 8 * h + ll + 4 * wg + 2 * jj]);
#pragma unroll
    for (int k = 0; k < 16; k++) {
        const uint32_t w = lds_u32_a2(sb + 64 * h + 4 * k);
        const uint32_t nib = (wg ? (w >> 4) : w) & 0x0F0F0F0Fu;
        const int jj = k >> 3;
        const uint32_t hb = (qh[k & 7] >> (4 * wg + 2 * jj)) & 0x03030303u;
        const uint32_t q4 = nib | (hb << 4);
        const float t = dsc[2 * jj + ((k & 7) >> 2)];
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; e++) v[e] = __fmul_rn(t, (float)((int)((q4 >> (8 * e)) & 0xFFu) - 32));
        split_pair(v[0], v[1], ohi[2 * k], olo[2 * k]);
        split_pair(v[2], v[3], ohi[2 * k + 1], olo[2 * k + 1]);
    }
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
        "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
        "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
          "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
          "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem d] (+)= A[tmem a] x B[smem desc]^T; accumulate != 0 adds to old D.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

// Non-blocking test of a barrier phase (1 once the phase with this parity completed).
__device__ __forceinline__ uint32_t mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done;
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// Shared-memory descriptor of a K-major operand tile written by TMA with
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart (stride
// byte offset), leading byte offset 16 (unused by swizzled K-major layouts),
// descriptor version 1, layout type 2 (128-byte swizzle).  `addr` is the
// tile's shared address plus 32 bytes per 16 K positions already consumed.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           (1ull << 46) | (2ull << 61);
}

}  // namespace mm

template <int WT, bool SPLIT>
__global__ void __launch_bounds__(mm::kThreads, 1)
    matmul_q_kernel(const __grid_constant__ mm::Maps maps, const mm::Args a) {
    using RG = mm::RawGeo<WT>;
    using SG = mm::SGeo<SPLIT>;
    using namespace mm;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);  // A slot written and B stage landed
    uint64_t* empty = full + kStages;
    uint64_t* raw_full = empty + kStages;
    uint64_t* raw_empty = raw_full + kRawStages;
    uint64_t* dfull = raw_empty + kRawStages;  // [kDBufs] accumulator written
    uint64_t* dempty = dfull + kDBufs;         // [kDBufs] accumulator read back
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(dempty + kDBufs);
    const uint8_t* raw = smem + kRawOff;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nst = a.K / kKS;     // stages per tile
    const int nch = nst / 2;       // raw runs per tile
    // the tiles of this CTA: blockIdx.x, + gridDim.x, ...
    auto tile_mat = [&](int t, int& m, int64_t& row0, int& tok0) {
        const int rt = t / a.tok_tiles;
        m = a.nmat > 2 && rt >= a.toff[2] ? 2 : (a.nmat > 1 && rt >= a.toff[1] ? 1 : 0);
        row0 = (int64_t)(rt - (m == 2 ? a.toff[2] : m == 1 ? a.toff[1] : 0)) * kRows;
        tok0 = (t % a.tok_tiles) * kNT;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < SG::kStages; s++) {
            mbar_init(&full[s], kDecodeWarps + 1);  // the decode warps and the producer's expect_tx
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < kRawStages; s++) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], kDecodeWarps);
        }
        for (int d = 0; d < kDBufs; d++) {
            mbar_init(&dfull[d], 1);
            mbar_init(&dempty[d], kEpiWarps);
        }
        fence_mbar_init();
    }
    if (warp == kWarpMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_holder)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == kWarpTma) {
        // ---- producer (TMA): raw weight runs and activation stages ----
        if (lane == 0) {
            pdl_wait();  // X is the previous kernel's output
            int gs = 0, gc = 0;  // stages and runs issued so far (over all tiles)
            bool ok = true;
            for (int t = blockIdx.x; t < a.tiles && ok; t += gridDim.x) {
                int m, tok0;
                int64_t row0;
                tile_mat(t, m, row0, tok0);
                const CUtensorMap* wmap = m == 2 ? &maps.w[2] : m == 1 ? &maps.w[1] : &maps.w[0];
                for (int s = 0; s < nst; s++) {
                    if ((s & 1) == 0) {
                        const int rs = gc % RG::kStages;
                        if (gc >= RG::kStages &&
                            !mbar_wait(&raw_empty[rs], (uint32_t)((gc / RG::kStages) - 1) & 1)) {
                            atomicOr(a.err, kErrTimeout);
                            ok = false;
                            break;
                        }
                        // x in 8-byte elements: 18 per Q4 run; Q6_K: the 16-byte
                        // aligned start of super-block s / 2
                        const int x = WT == CN_TYPE_Q6_K ? ((210 * (s / 2)) >> 4) * 2 : 18 * (s / 2);
                        mbar_expect_tx(&raw_full[rs], RG::kBytes);
                        tma_load_2d(smem + kRawOff + rs * RG::kBytes, wmap, x, (int)row0, &raw_full[rs]);
                        gc++;
                    }
                    const int slot = gs % SG::kStages;
                    if (gs >= SG::kStages &&
                        !mbar_wait(&empty[slot], (uint32_t)((gs / SG::kStages) - 1) & 1)) {
                        atomicOr(a.err, kErrTimeout);
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&full[slot], SG::kBStage);
                    uint8_t* bst = smem + slot * SG::kBStage;
                    tma_load_2d(bst, &maps.x, s * kKS, tok0, &full[slot]);
                    tma_load_2d(bst + kBHalf, &maps.x, s * kKS + 64, tok0, &full[slot]);
                    if (SPLIT) {  // the low halves after the high ones
                        tma_load_2d(bst + 2 * kBHalf, &maps.xlo, s * kKS, tok0, &full[slot]);
                        tma_load_2d(bst + 3 * kBHalf, &maps.xlo, s * kKS + 64, tok0, &full[slot]);
                    }
                    gs++;
                }
            }
            // no copy may still be landing when the CTA exits
            for (int i = gs - SG::kStages < 0 ? 0 : gs - SG::kStages; i < gs; i++)
                mbar_wait(&full[i % SG::kStages], (uint32_t)(i / SG::kStages) & 1);
            for (int i = gc - RG::kStages < 0 ? 0 : gc - RG::kStages; i < gc; i++)
                mbar_wait(&raw_full[i % RG::kStages], (uint32_t)(i / RG::kStages) & 1);
        }
    } else if (warp == kWarpMma) {
        // ---- MMA issuer ----
        if (lane == 0) {
            int gs = 0, i = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < a.tiles && ok; t += gridDim.x, i++) {
                const int db = i % kDBufs;
                if (i >= kDBufs && !mbar_wait(&dempty[db], (uint32_t)((i / kDBufs) - 1) & 1)) {
                    atomicOr(a.err, kErrTimeout);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem + db * kNT;
                // the test of a stage's barrier is issued before the previous
                // stage's MMAs, so its latency hides behind their issue
                uint32_t ready = mbar_test(&full[gs % SG::kStages], (uint32_t)(gs / SG::kStages) & 1);
                for (int s = 0; s < nst; s++, gs++) {
                    const int slot = gs % SG::kStages;
                    const uint32_t ph = (uint32_t)(gs / SG::kStages) & 1;
                    if (!ready && !mbar_wait(&full[slot], ph)) {
                        atomicOr(a.err, kErrTimeout);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int ns = gs + 1;
                    ready = s + 1 < nst ? mbar_test(&full[ns % SG::kStages], (uint32_t)(ns / SG::kStages) & 1) : 0u;
                    const uint32_t b0 = smem_u32(smem + slot * SG::kBStage);
#pragma unroll
                    for (int kk = 0; kk < kKS / 16; kk++) {
                        const uint32_t a_hi = tmem + kACol + slot * SG::kACols + 8 * kk;
                        const uint64_t b_hi = desc_sw128(b0 + (kk / 4) * kBHalf + 32 * (kk % 4));
                        mma_f16(d_tmem, a_hi, b_hi, (s | kk) != 0);
                        if (SPLIT) {
                            // Whi Xlo and Wlo Xhi into the same accumulator (Wlo Xlo is
                            // below the pair's own rounding)
                            mma_f16(d_tmem, a_hi, desc_sw128(b0 + (2 + kk / 4) * kBHalf + 32 * (kk % 4)), 1u);
                            mma_f16(d_tmem, a_hi + kACols, b_hi, 1u);
                        }
                    }
                    mma_commit(&empty[slot]);
                }
                mma_commit(&dfull[db]);  // completes once every MMA issued above has
            }
        }
    } else if (warp >= kWarpEpi0) {
        // ---- epilogue: accumulator row r, 32 tokens per tensor-memory load ----
        const int r = threadIdx.x & (kRows - 1);
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        bool failed = false;
        pdl_wait();  // Y may be the previous kernel's data
        int i = 0;
        for (int t = blockIdx.x; t < a.tiles; t += gridDim.x, i++) {
            int m, tok0;
            int64_t row0;
            tile_mat(t, m, row0, tok0);
            const int db = i % kDBufs;
            if (!failed && !mbar_wait(&dfull[db], (uint32_t)(i / kDBufs) & 1)) {
                atomicOr(a.err, kErrTimeout);
                failed = true;
            }
            tc_fence_after();
            const int64_t row = row0 + r;
            const bool live = row < pick(a.rows, m);
            float* y = pick(a.y, m);
            const int64_t ldy = pick(a.ldy, m);
#pragma unroll 1
            for (int j = 0; j < kNT / 32; j++) {
                uint32_t v[32];
                tmem_ld32(tmem + lane_off + db * kNT + 32 * j, v);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (j == kNT / 32 - 1) {
                    // the accumulator is read (the warp-wide wait covers every
                    // lane's load): hand it back to the MMA issuer
                    tc_fence_before();
                    if (lane == 0) mbar_arrive(&dempty[db]);
                }
                if (a.xs || SPLIT) {
                    // undo token t's activation scaling and the split variant's
                    // weight scaling (both exact powers of two)
                    const int tk = tok0 + 32 * j + lane;
                    const float sc = (a.xs && tk < a.M ? a.xs[tk] : 1.f) * pick(a.oscale, m);
#pragma unroll
                    for (int u = 0; u < 32; u++)
                        v[u] = __float_as_uint(__uint_as_float(v[u]) * __shfl_sync(0xffffffffu, sc, u));
                }
                if (live) {
                    float* p = y + (size_t)(tok0 + 32 * j) * ldy + row;
                    const int nt = a.M - (tok0 + 32 * j);  // tokens of this chunk inside M
                    if (a.accumulate) {
                        // 16 loads in flight before the first store
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            float old[16];
#pragma unroll
                            for (int u = 0; u < 16; u++) old[u] = 16 * h + u < nt ? p[(size_t)(16 * h + u) * ldy] : 0.f;
#pragma unroll
                            for (int u = 0; u < 16; u++)
                                if (16 * h + u < nt) p[(size_t)(16 * h + u) * ldy] = old[u] + __uint_as_float(v[16 * h + u]);
                        }
                    } else {
#pragma unroll
                        for (int u = 0; u < 32; u++)
                            if (u < nt) p[(size_t)u * ldy] = __uint_as_float(v[u]);
                    }
                }
            }
        }
    } else {
        // ---- weight decode into tensor memory ----
        const int r = threadIdx.x & (kRows - 1);  // tile row == tensor-memory lane
        const int wg = threadIdx.x >> 7;          // blocks 2wg, 2wg + 1 of each stage
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        bool failed = false;
        int gs = 0, gc = 0;
        for (int t = blockIdx.x; t < a.tiles; t += gridDim.x) {
            int tmat, tok0_;
            int64_t row0_;
            tile_mat(t, tmat, row0_, tok0_);  // the tile's matrix (its split scale)
            for (int c = 0; c < nch; c++, gc++) {
                const int rs = gc % RG::kStages;
                if (!failed && !mbar_wait(&raw_full[rs], (uint32_t)(gc / RG::kStages) & 1)) {
                    atomicOr(a.err, kErrTimeout);
                    failed = true;
                }
                if (WT == CN_TYPE_Q6_K) {
                    // read in place (the window stays until both stages are
                    // expanded); d is the fp16 at byte 208 of the super-block
                    const uint8_t* sb = raw + rs * RG::kBytes + r * RG::kRow + ((210 * c) & 15);
                    const float d = half_bits_to_float(lds_u16(sb + 208));
#pragma unroll 1
                    for (int q = 0; q < 2; q++, gs++) {
                        const int slot = gs % SG::kStages;
                        if (gs >= SG::kStages && !failed &&
                            !mbar_wait(&empty[slot], (uint32_t)((gs / SG::kStages) - 1) & 1)) {
                            atomicOr(a.err, kErrTimeout);
                            failed = true;
                        }
                        tc_fence_after();
                        uint32_t o[32];
                        const uint32_t col = lane_base + kACol + slot * SG::kACols + 32 * wg;
                        if (SPLIT) {
                            uint32_t ol[32];
                            expand_q6k_half_split(sb, q, wg, d * pick(a.wscale, tmat), o, ol);
                            tmem_st32(col + kACols, ol);
                        } else {
                            expand_q6k_half(sb, q, wg, d, o);
                        }
                        tmem_st32(col, o);
                        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                        tc_fence_before();
                        if (lane == 0) mbar_arrive(&full[slot]);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&raw_empty[rs]);
                    continue;
                }
                // this thread's words of its row (rows past the matrix arrive as
                // zeros).  Q4_0: blocks 4q + 2wg, 4q + 2wg + 1 of stage q = words
                // 18q + 9wg .. 18q + 9wg + 8 of the row's 36.  Q4_K: the header
                // (words 0-3: d, dmin, packed scales) and sub-blocks 4q + 2wg,
                // 4q + 2wg + 1 = words 4 + 16q + 8wg .. +7.
                const uint32_t* row32 = reinterpret_cast<const uint32_t*>(raw + rs * RG::kBytes + r * RG::kRow);
                uint32_t cur[18];
                uint32_t d2 = 0, sc2[2][2], ndm2[2][2];  // Q4_K: d, [stage][sub-block] sc and -dmin * m
                float dscf[2][2], dmf[2][2];             // Q4_K split: fp32 d*sc and dmin*m at 2^E
                if (WT == CN_TYPE_Q4_0) {
#pragma unroll
                    for (int q = 0; q < 2; q++)
#pragma unroll
                        for (int k = 0; k < 9; k++) cur[9 * q + k] = row32[9 * wg + 18 * q + k];
                } else {
                    uint32_t hw[4];
#pragma unroll
                    for (int k = 0; k < 4; k++) hw[k] = row32[k];
#pragma unroll
                    for (int q = 0; q < 2; q++)
#pragma unroll
                        for (int k = 0; k < 8; k++) cur[8 * q + k] = row32[4 + 16 * q + 8 * wg + k];
                    // DequantQ4K.DecodeScales (DequantQ4K.cs:218-241) for this
                    // thread's four sub-blocks (byte b of the 12 scale bytes is
                    // byte b % 4 of word 1 + b / 4; stage 0 holds sub-blocks
                    // j < 4, stage 1 those >= 4), then sc and dmin * m
                    d2 = (hw[0] & 0xFFFFu) * 0x10001u;
                    const float dmin = half_bits_to_float((uint16_t)(hw[0] >> 16));
#pragma unroll
                    for (int q = 0; q < 2; q++)
#pragma unroll
                        for (int e = 0; e < 2; e++) {
                            const int sh = 8 * (2 * wg + e);  // byte j % 4 of a word
                            const int b0 = (int)(hw[1] >> sh) & 0xFF, b1 = (int)(hw[2] >> sh) & 0xFF;
                            int sc, mm_;
                            if (q == 0) {
                                sc = b0 & 63;
                                mm_ = b1 & 63;
                            } else {
                                const int b2 = (int)(hw[3] >> sh) & 0xFF;
                                sc = (b2 & 0xF) | ((b0 >> 6) << 4);
                                mm_ = (b2 >> 4) | ((b1 >> 6) << 4);
                            }
                            const float dm = __fmul_rn(dmin, (float)mm_);
                            sc2[q][e] = pack_half2((float)sc, (float)sc);
                            ndm2[q][e] = pack_half2(-dm, -dm);
                            if (SPLIT) {
                                const float ws = pick(a.wscale, tmat);
                                dscf[q][e] = __fmul_rn(half_bits_to_float((uint16_t)(hw[0] & 0xFFFFu)), (float)sc) * ws;
                                dmf[q][e] = dm * ws;
                            }
                        }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_empty[rs]);
#pragma unroll
                for (int q = 0; q < 2; q++, gs++) {
                    const int slot = gs % SG::kStages;
                    if (gs >= SG::kStages && !failed &&
                        !mbar_wait(&empty[slot], (uint32_t)((gs / SG::kStages) - 1) & 1)) {
                        atomicOr(a.err, kErrTimeout);
                        failed = true;
                    }
                    tc_fence_after();
                    uint32_t o[32];
                    const uint32_t col = lane_base + kACol + slot * SG::kACols + 32 * wg;
                    if (WT == CN_TYPE_Q4_0) {
                        uint32_t wd[9];
#pragma unroll
                        for (int k = 0; k < 9; k++) wd[k] = cur[9 * q + k];
                        if (SPLIT) {
                            uint32_t ol[32];
                            expand_q4_0_pair_split(wd, pick(a.wscale, tmat), o, ol);
                            tmem_st32(col + kACols, ol);
                        } else {
                            expand_q4_0_pair(wd, o);
                        }
                    } else {
                        uint32_t qw[8];
#pragma unroll
                        for (int k = 0; k < 8; k++) qw[k] = cur[8 * q + k];
                        if (SPLIT) {
                            uint32_t ol[32];
                            expand_q4k_pair_split(qw, dscf[q], dmf[q], o, ol);
                            tmem_st32(col + kACols, ol);
                        } else {
                            expand_q4k_pair(qw, d2, sc2[q], ndm2[q], o);
                        }
                    }
                    tmem_st32(col, o);
                    // warp-wide: every lane's stores of this stage are done
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    if (lane == 0) mbar_arrive(&full[slot]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

// ---- host side ------------------------------------------------------------------

int encode_act_map(const __half* x, int M, int64_t K, CUtensorMap* out) {
    CN_CHECK(K % mm::kKS == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && M >= 1,
             CN_ERR_UNSUPPORTED, "activation layout not TMA-tileable");
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)mm::kNT};  // one 128-byte swizzle row of fp16
    return encode_tiled_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, const_cast<__half*>(x), dims, strides,
                           box, CU_TENSOR_MAP_SWIZZLE_128B, out);
}

int matmul_quant(cudaStream_t st, uint32_t* err, int type, int nmat, const void* const* w,
                 const CUtensorMap* const* wmaps, const int64_t* rows, int64_t K, const __half* x, const float* xs,
                 int M, float* const* y, const int64_t* ldy, bool accumulate, const __half* xlo,
                 const float* wscale) {
    CN_CHECK(matmul_type_ok(type), CN_ERR_UNSUPPORTED, "matmul: weight type %d (Q4_0, Q4_K or Q6_K)", type);
    CN_CHECK(nmat >= 1 && nmat <= mm::kMaxMats && K > 0 && K % 256 == 0 && M >= 1, CN_ERR_INVALID_ARG,
             "matmul: bad shape (nmat %d, K %lld, M %d)", nmat, (long long)K, M);
    const bool split = xlo != nullptr;
    CN_CHECK(!split || wscale, CN_ERR_INVALID_ARG, "matmul: the split variant needs the weight scales");
    int dev = 0;
    CN_CUDA(cudaGetDevice(&dev));
    static std::mutex mu;
    static bool attr[64] = {false};
    static int sm_count[64] = {0};
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!attr[dev & 63]) {
#define CN_MM_ATTR(T, S) \
    CN_CUDA(cudaFuncSetAttribute(matmul_q_kernel<T, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, mm::kSmem));
            CN_MM_ATTR(CN_TYPE_Q4_0, false) CN_MM_ATTR(CN_TYPE_Q4_K, false) CN_MM_ATTR(CN_TYPE_Q6_K, false)
            CN_MM_ATTR(CN_TYPE_Q4_0, true) CN_MM_ATTR(CN_TYPE_Q4_K, true) CN_MM_ATTR(CN_TYPE_Q6_K, true)
#undef CN_MM_ATTR
            CN_CUDA(cudaDeviceGetAttribute(&sm_count[dev & 63], cudaDevAttrMultiProcessorCount, dev));
            attr[dev & 63] = true;
        }
    }
    const int sms = sm_count[dev & 63];
    mm::Args a = {};
    mm::Maps maps;
    a.nmat = nmat;
    int tiles = 0;
    for (int i = 0; i < mm::kMaxMats; i++) {
        const int mi = i < nmat ? i : nmat - 1;
        a.toff[i] = tiles;
        a.w[i] = static_cast<const uint8_t*>(w[mi]);
        if (wmaps && wmaps[mi]) {
            maps.w[i] = *wmaps[mi];
        } else {
            int rc = encode_weight_map(type, w[mi], rows[mi], row_bytes(type, K), &maps.w[i]);
            if (rc) return rc;
        }
        a.rows[i] = rows[mi];
        a.y[i] = y[mi];
        a.ldy[i] = ldy[mi];
        a.wscale[i] = split ? wscale[mi] : 1.f;
        a.oscale[i] = split ? 1.f / wscale[mi] : 1.f;  // exact: a power of two
        CN_CHECK(w[mi] && y[mi] && rows[mi] > 0 && ldy[mi] >= rows[mi], CN_ERR_INVALID_ARG,
                 "matmul: bad matrix %d", mi);
        CN_CHECK((reinterpret_cast<uintptr_t>(w[mi]) & 15) == 0, CN_ERR_UNSUPPORTED,
                 "matmul: weights not 16-byte aligned");
        if (i < nmat) tiles += (int)((rows[i] + mm::kRows - 1) / mm::kRows);
    }
    a.toff[nmat] = tiles;
    a.tok_tiles = (M + mm::kNT - 1) / mm::kNT;
    a.tiles = tiles * a.tok_tiles;
    a.rb = (int64_t)row_bytes(type, K);
    a.xs = xs;
    a.M = M;
    a.K = (int)K;
    a.accumulate = accumulate ? 1 : 0;
    a.err = err;
    int rc = encode_act_map(x, M, K, &maps.x);
    if (rc) return rc;
    if (split) {
        if ((rc = encode_act_map(xlo, M, K, &maps.xlo))) return rc;
    } else {
        maps.xlo = maps.x;
    }
    const dim3 grid(a.tiles < sms ? a.tiles : sms);  // persistent: one CTA per SM
#define CN_MM_LAUNCH(T)                                                                                         \
    CN_CUDA(split ? launch_k(false, matmul_q_kernel<T, true>, grid, dim3(mm::kThreads), (size_t)mm::kSmem, st, maps, a) \
                  : launch_k(false, matmul_q_kernel<T, false>, grid, dim3(mm::kThreads), (size_t)mm::kSmem, st, maps, a));
    if (type == CN_TYPE_Q4_0) {
        CN_MM_LAUNCH(CN_TYPE_Q4_0)
    } else if (type == CN_TYPE_Q4_K) {
        CN_MM_LAUNCH(CN_TYPE_Q4_K)
    } else {
        CN_MM_LAUNCH(CN_TYPE_Q6_K)
    }
#undef CN_MM_LAUNCH
    return CN_OK;
}

// Largest fp16 scale fields of a weight tensor's blocks: out[0] = max |d|,
// out[1] = max |dmin| (Q4_K), as float bits (non-negative floats order like
// their bit patterns).
__global__ void scale_max_kernel(int type, const uint8_t* __restrict__ w, int64_t nblocks, unsigned* out) {
    const int bpb = type == CN_TYPE_Q4_0 ? 18 : type == CN_TYPE_Q4_K ? 144 : 210;
    const int doff = type == CN_TYPE_Q6_K ? 208 : 0;
    unsigned m0 = 0, m1 = 0;
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nblocks; b += (int64_t)gridDim.x * blockDim.x) {
        const uint8_t* p = w + b * bpb;
        m0 = max(m0, __float_as_uint(fabsf(half_bits_to_float((uint16_t)(p[doff] | (p[doff + 1] << 8))))));
        if (type == CN_TYPE_Q4_K)
            m1 = max(m1, __float_as_uint(fabsf(half_bits_to_float((uint16_t)(p[2] | (p[3] << 8))))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        m0 = max(m0, __shfl_xor_sync(0xffffffffu, m0, o));
        m1 = max(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMax(out, m0);
        atomicMax(out + 1, m1);
    }
}

int matmul_split_scale(cn_tensor* t, cudaStream_t st, float* out) {
    CN_CHECK(t && out && matmul_type_ok(t->type), CN_ERR_INVALID_ARG, "split scale: bad tensor");
    if (t->split_scale > 0.f) {
        *out = t->split_scale;
        return CN_OK;
    }
    const int bpb = t->type == CN_TYPE_Q4_0 ? 18 : t->type == CN_TYPE_Q4_K ? 144 : 210;
    const int64_t nblocks = (int64_t)(t->bytes / bpb);
    unsigned* d = nullptr;
    CN_CUDA(cudaMalloc(&d, 2 * sizeof(unsigned)));
    unsigned h[2] = {0, 0};
    cudaError_t e = cudaMemsetAsync(d, 0, 2 * sizeof(unsigned), st);
    if (e == cudaSuccess) {
        int blocks = (int)((nblocks + 255) / 256);
        blocks = blocks < 1 ? 1 : blocks > 1024 ? 1024 : blocks;
        scale_max_kernel<<<blocks, 256, 0, st>>>(t->type, static_cast<const uint8_t*>(t->d), nblocks, d);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(h, d, sizeof(h), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaFree(d);
    if (e != cudaSuccess) return cuda_error(e, "split scale");
    float dmax, dminmax;
    memcpy(&dmax, &h[0], 4);
    memcpy(&dminmax, &h[1], 4);
    // the largest |weight| the format allows with these scales
    const double bound = t->type == CN_TYPE_Q4_0   ? 8.0 * dmax
                         : t->type == CN_TYPE_Q4_K ? 63.0 * 15.0 * dmax + 63.0 * dminmax
                                                   : 128.0 * 32.0 * dmax;
    int e2 = 0;
    if (bound > 0.0 && std::isfinite(bound)) {
        frexp(16384.0 / bound, &e2);  // 16384 / bound in [2^(e2-1), 2^e2)
        e2 -= 1;                      // bound * 2^e2 <= 2^14
        e2 = e2 < -100 ? -100 : e2 > 100 ? 100 : e2;
    }
    t->split_scale = (float)ldexp(1.0, e2);
    *out = t->split_scale;
    return CN_OK;
}

}  // namespace cn
