// gemv_tc.cuh -- shared pieces of the tensor-core (tcgen05) Q4_K GEMV:
// geometry of its activation-digit records and the warp routine that
// writes them (used by the standalone prep and by the fused RMSNorm prep).
#pragma once

#include <stdint.h>

namespace cn {
namespace tc {

constexpr int kRows = 128;   // rows per tile (MMA M)
constexpr int kN = 16;       // MMA N: digit columns, 3 per sequence
constexpr int kMaxNB = 5;    // sequences per call (3 * 5 <= 16)

// Activation record of one 256-position unit (one Q4_K super-block of x),
// for all sequences of the call:
//   [0, 4096)     digits: 8 sub-blocks j x 512 bytes, each a K-major B tile of
//                 16 columns x 32 positions in 8x16-byte core matrices:
//                 byte j*512 + (n/8)*256 + (k/16)*128 + (n%8)*16 + k%16
//                 holds column n at position 32j + k;
//   [4096, 4352)  xs: int32 [8 sub-blocks][8 slots], the sum of X over the
//                 sub-block for sequence b;
//   [4352, 4384)  inv: fp32 [8 slots], 2^-e of sequence b.
// X = rint(x * 2^e) = 65536 d2 + 256 d1 + d0 with balanced base-256 digits
// and e chosen per unit and sequence so |X| <= 2^22.  Sub-blocks share MMA
// accumulators: P = max(1, 16 / (3 * batch)) consecutive sub-blocks accumulate
// into one 16-column group, sub-block j owning columns
// 3 * batch * (j % P) + 3b + {0, 1, 2} (digits d2, d1, d0 of sequence b) of its
// tile; every other column of the tile is zero, so the group's sum keeps the
// sub-blocks apart (block-diagonal B).
constexpr int kDigB = 8 * 512;
constexpr int kXsOff = kDigB;
constexpr int kInvOff = kDigB + 8 * 8 * 4;
constexpr int kXReg = kInvOff + 8 * 4;  // 4384, a multiple of 16

__host__ __device__ constexpr int group_subblocks(int batch) {
    return 16 / (3 * batch) > 0 ? 16 / (3 * batch) : 1;
}

// One warp writes unit u of sequence b.  Lane (c = lane/4, t = lane%4) holds
// in v[0..3] positions 32c + 4t + 0..3 and in v[4..7] positions
// 32c + 16 + 4t + 0..3 (the layout of the mma.sync prep).  The warp with
// b == 0 also zeroes the columns no sequence uses.
__device__ __forceinline__ void emit_digits(const float (&v)[8], int u, int b, int batch,
                                            uint8_t* __restrict__ out, int lane) {
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) am = fmaxf(am, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    int e = 0;
    if (am > 0.f && am < INFINITY) e = 21 - ilogbf(am);
    e = e < -120 ? -120 : (e > 120 ? 120 : e);
    const float sc = ldexpf(1.0f, e);
    const int c = lane >> 2, t = lane & 3;
    uint8_t* reg = out + (size_t)u * kXReg;
    uint32_t dig[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
    int xsum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int X = __float2int_rn(v[i] * sc);
        xsum += X;
        const int d0 = ((X + 128) & 255) - 128;
        const int X1 = (X - d0) >> 8;
        const int d1 = ((X1 + 128) & 255) - 128;
        const int d2 = (X1 - d1) >> 8;
        const int w = i >> 2, sh = 8 * (i & 3);
        dig[0][w] |= (uint32_t)(d2 & 255) << sh;
        dig[1][w] |= (uint32_t)(d1 & 255) << sh;
        dig[2][w] |= (uint32_t)(d0 & 255) << sh;
    }
    const int c0 = 3 * batch * (c % group_subblocks(batch));  // this sub-block's first column
    uint8_t* base = reg + c * 512 + 4 * t;
#pragma unroll
    for (int d = 0; d < 3; d++) {
        const int n = c0 + 3 * b + d;
        uint8_t* p = base + (n >> 3) * 256 + (n & 7) * 16;
        *reinterpret_cast<uint32_t*>(p) = dig[d][0];        // positions 4t..4t+3
        *reinterpret_cast<uint32_t*>(p + 128) = dig[d][1];  // positions 16+4t..
    }
    if (b == 0) {
        for (int n = 0; n < kN; n++) {
            if (n >= c0 && n < c0 + 3 * batch) continue;
            uint8_t* p = base + (n >> 3) * 256 + (n & 7) * 16;
            *reinterpret_cast<uint32_t*>(p) = 0u;
            *reinterpret_cast<uint32_t*>(p + 128) = 0u;
        }
    }
    xsum += __shfl_xor_sync(0xffffffffu, xsum, 1);
    xsum += __shfl_xor_sync(0xffffffffu, xsum, 2);
    if (t == 0) reinterpret_cast<int*>(reg + kXsOff)[c * 8 + b] = xsum;
    if (lane == 0) reinterpret_cast<float*>(reg + kInvOff)[b] = ldexpf(1.0f, -e);
}

}  // namespace tc
}  // namespace cn
