// prep.cuh -- the activation records the GEMV families read, and the warp
// routines that write them, for every kernel that produces a GEMV input
// (standalone prep, fused residual-add + RMSNorm, SiLU, attention).
#pragma once

#include <stdint.h>

#include "cn_internal.h"
#include "gemv_i8.cuh"
#include "gemv_tc.cuh"

namespace cn {

// ---- activation prep ----------------------------------------------------------
//
// The GEMVs read x as fp16 fragments.  Each 256-position unit u of each batch
// row b is scaled by its own power of two 2^e (max |x| over the unit lands in
// [2^14, 2^15)), which is exact and keeps the fp16 hi + lo split far from
// overflow and from subnormals whatever the activation range; the GEMV
// multiplies the unit's partial sums by xinv[u][b] = 2^-e.  Being unit-local,
// the conversion needs no reduction over the whole vector, so any kernel
// holding whole units can emit it (the standalone prep and the fused
// RMSNorm below).
//
// Layouts (nt_count n-tiles of 4 batch columns):
//   xfrag[c][nt][lane]: the four B-fragment registers lane (g, t) feeds the
//     two k-steps of chunk c; column g = hi (g even) or lo (g odd) part of
//     batch b = 4*nt + g/2; positions 4t+{0,2}, 4t+{1,3} of each 16-position
//     half, the second half multiplied by step1 (1/16 for Q4_K, else 1);
//   xsum[c][b]: fp32 sum of the scaled x over chunk c (Q4_K's dmin term);
//   xinv[u][b]: 2^-e.
// Columns of batch rows >= batch are never read back, so they are not written.

// One warp emits unit u of row b.  Lane (c = lane/4, t = lane%4) holds in
// v[0..3] positions 32c + 4t + 0..3 and in v[4..7] positions 32c + 16 + 4t + 0..3.
__device__ __forceinline__ void emit_unit(const float (&v)[8], int u, int b, int nt_count,
                                          float step1, uint4* __restrict__ xfrag,
                                          float* __restrict__ xsum, float* __restrict__ xinv,
                                          int lane) {
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) am = fmaxf(am, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    int e = 0;
    if (am > 0.f && am < INFINITY) e = 14 - ilogbf(am);
    e = e < -120 ? -120 : (e > 120 ? 120 : e);
    const float sc = ldexpf(1.0f, e), s1 = sc * step1;
    const int c = lane >> 2, t = lane & 3;
    const int nt = b >> 2, gh = 2 * (b & 3);
    float e8[8] = {v[0] * sc, v[2] * sc, v[1] * sc, v[3] * sc,
                   v[4] * s1, v[6] * s1, v[5] * s1, v[7] * s1};
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        __half2 h = __floats2half2_rn(e8[2 * k], e8[2 * k + 1]);
        float2 back = __half22float2(h);
        __half2 l = __floats2half2_rn(e8[2 * k] - back.x, e8[2 * k + 1] - back.y);
        hi[k] = *reinterpret_cast<uint32_t*>(&h);
        lo[k] = *reinterpret_cast<uint32_t*>(&l);
    }
    uint4* dst = xfrag + ((size_t)(8 * u + c) * nt_count + nt) * 32;
    dst[4 * gh + t] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    dst[4 * (gh + 1) + t] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    if (xsum) {
        float ps = ((v[0] * sc + v[1] * sc) + (v[2] * sc + v[3] * sc)) +
                   ((v[4] * sc + v[5] * sc) + (v[6] * sc + v[7] * sc));
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        if (t == 0) xsum[(size_t)(8 * u + c) * nt_count * 4 + b] = ps;
    }
    if (lane == 0) xinv[(size_t)u * nt_count * 4 + b] = ldexpf(1.0f, -e);
}

// Writes unit u of sequence b in whichever form pt names (see PrepTarget).
__device__ __forceinline__ void emit_any(const PrepTarget& pt, const float (&v)[8], int u, int b, int batch,
                                         int lane) {
    if (pt.kind == 3)
        i8::emit_i8(v, u, b, batch, reinterpret_cast<uint8_t*>(pt.xfrag), lane);
    else if (pt.kind == 2)
        tc::emit_digits(v, u, b, batch, reinterpret_cast<uint8_t*>(pt.xfrag), lane);
    else if (pt.kind >= 0)
        emit_unit(v, u, b, pt.nt_count, pt.step1, reinterpret_cast<uint4*>(pt.xfrag),
                  pt.kind == 1 ? pt.xsum : nullptr, pt.xinv, lane);
}

}  // namespace cn
