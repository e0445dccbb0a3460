// gemv_i8.cuh -- activation records of the integer mma.sync GEMV (gemv_i8.cu)
// and the warp routine that writes them (standalone prep and fused RMSNorm).
#pragma once

#include <stdint.h>

namespace cn {
namespace i8 {

constexpr int kMaxNB = 16;  // sequences per call

// Activations enter the integer GEMV as exact integers: per 256-position
// unit u and sequence b, X = rint(x * 2^e) with e chosen so |X| <= 2^22, and
// X is split into balanced digits, each an int8 column of the MMA's B
// operand:
//   batch 1:  6 balanced base-15 digits d_i in [-7, 7], X = sum d_i 15^i,
//             column i (columns 6, 7 zero).  Quant byte 4t+i of a sub-block
//             holds the nibbles of positions p = 4t+i (low) and p' = 16+4t+i
//             (high).  The MMA's A operand takes the raw byte lo + 16 hi in
//             k-slot 4t+i (no unpacking) and lo in k-slot 16+4t+i; B holds
//             d(p') in k-slot 4t+i and 16 d(p) - d(p') (|.| <= 119) in k-slot
//             16+4t+i, so the lo * d(p') terms cancel and each column sums to
//             16 * sum_p q_p d_i(p).
//   batch >1: 3 base-256 digits, X = sum d_i 256^i, column 4b + i (column
//             4b + 3 zero).  Batches 9-16 use the 16-sequence form (8
//             n-tiles, columns of absent sequences zero).
// Record of unit u (rec_bytes(NT) bytes, NT = n-tiles of 8 columns):
//   [0, 2048 NT)      B fragments of m16n8k32: sub-block j, n-tile nt, lane L
//                     at ((j * NT + nt) * 32 + L) * 8: {b0, b1} = column
//                     nt*8 + L/4 at positions 32j + 4(L%4) + 0..3 and
//                     32j + 16 + 4(L%4) + 0..3;
//   [2048 NT, +32 S)  xsd: int8 [S sequences][4 digits k][8 sub-blocks j]:
//                     XS_j = sum of X over sub-block j = sum_k 256^k xsd[k][j]
//                     (balanced digits, so a dp4a against the row's packed
//                     6-bit mins gives sum_j m_j XS_j digit by digit);
//   [2048 NT+32 S, +4 S) inv: fp32 [S sequences], 2^-e (batch 1: 2^-e / 16,
//                     which undoes the digits' factor 16);
// S = rec_seqs(NT): 8, or 16 for the 8-n-tile form.
__host__ __device__ constexpr int n_tiles(int batch) {
    return batch == 1 ? 1 : batch <= 8 ? (4 * batch + 7) / 8 : 8;
}
__host__ __device__ constexpr int rec_seqs(int nt) { return nt <= 4 ? 8 : 16; }
__host__ __device__ constexpr int rec_bytes(int nt) { return 2048 * nt + 36 * rec_seqs(nt); }
__host__ __device__ constexpr int xs_off(int nt) { return 2048 * nt; }
__host__ __device__ constexpr int inv_off(int nt) { return 2048 * nt + 32 * rec_seqs(nt); }

// One warp writes unit u of sequence b.  Lane (c = lane/4, t = lane%4) holds
// in v[0..3] positions 32c + 4t + 0..3 and in v[4..7] positions
// 32c + 16 + 4t + 0..3.  The warp with b == 0 also writes the zero columns.
__device__ __forceinline__ void emit_i8(const float (&v)[8], int u, int b, int batch,
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
    const int NT = n_tiles(batch);
    uint8_t* reg = out + (size_t)u * rec_bytes(NT);
    int X[8], xsum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        X[i] = __float2int_rn(v[i] * sc);
        xsum += X[i];
    }
    // column n of this lane's sub-block c: word b0 (low-nibble positions) and b1
    // b0: k-slots 4t+0..3, b1: k-slots 16+4t+0..3 of column n
    auto put = [&](int n, uint32_t b0, uint32_t b1) {
        const int nt = n >> 3, L = (n & 7) * 4 + t;
        *reinterpret_cast<uint2*>(reg + ((size_t)(c * NT + nt) * 32 + L) * 8) = make_uint2(b0, b1);
    };
    if (batch == 1) {
        // balanced base-15 digits via plain ones: with the offset
        // 7 * (15^6 - 1) / 14 every X' = X + offset lies in [0, 15^6), its
        // base-15 digits u_i are in [0, 14], and d_i = u_i - 7 are the balanced
        // digits of X (|X| <= 2^22 < 5695312).  n / 15 = umulhi(n, 0x88888889) >> 3.
        uint32_t U[8];
#pragma unroll
        for (int k = 0; k < 8; k++) U[k] = (uint32_t)(X[k] + 5695312);
#pragma unroll
        for (int i = 0; i < 6; i++) {
            int d[8];
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const uint32_t q = __umulhi(U[k], 0x88888889u) >> 3;
                d[k] = (int)(U[k] - 15u * q) - 7;
                U[k] = q;
            }
            uint32_t w0 = 0, w1 = 0;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                w0 |= (uint32_t)(d[4 + k] & 255) << (8 * k);
                w1 |= (uint32_t)((16 * d[k] - d[4 + k]) & 255) << (8 * k);
            }
            put(i, w0, w1);
        }
        put(6, 0u, 0u);
        put(7, 0u, 0u);
    } else {
#pragma unroll
        for (int i = 0; i < 3; i++) {
            uint32_t w0 = 0, w1 = 0;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const int d = i < 2 ? ((X[k] + 128) & 255) - 128 : X[k];
                X[k] = (X[k] - d) >> 8;
                if (k < 4) w0 |= (uint32_t)(d & 255) << (8 * k);
                else w1 |= (uint32_t)(d & 255) << (8 * (k - 4));
            }
            put(4 * b + i, w0, w1);
        }
        put(4 * b + 3, 0u, 0u);
        if (b == 0)
            for (int n = 4 * batch; n < 8 * NT; n++) put(n, 0u, 0u);
    }
    xsum += __shfl_xor_sync(0xffffffffu, xsum, 1);
    xsum += __shfl_xor_sync(0xffffffffu, xsum, 2);
    if (t == 0) {
        int8_t* xd = reinterpret_cast<int8_t*>(reg + xs_off(NT)) + b * 32 + c;
#pragma unroll
        for (int k = 0; k < 3; k++) {
            const int d = ((xsum + 128) & 255) - 128;
            xd[8 * k] = (int8_t)d;
            xsum = (xsum - d) >> 8;
        }
        xd[24] = (int8_t)xsum;  // |sum| <= 2^27: the top digit is at most 8
    }
    if (lane == 0) reinterpret_cast<float*>(reg + inv_off(NT))[b] = ldexpf(1.0f, batch == 1 ? -e - 4 : -e);
}

}  // namespace i8
}  // namespace cn
