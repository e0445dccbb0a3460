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

#include "cn_common.cuh"
#include "cn_internal.h"
#include "formats.cuh"

namespace cn {

constexpr int kWarps = 4;  // warps per CTA, each an independent pipeline

template <int TYPE>
struct Fmt;
template <>
struct Fmt<CN_TYPE_Q4_0> {
    static constexpr int kBox = 144;  // bytes per row per unit (8 blocks)
    static constexpr int kStages = 8;
    __device__ static int box_x(int u) { return 18 * u; }  // uint64 elements
    __device__ static int offset(int) { return 0; }
};
template <>
struct Fmt<CN_TYPE_Q4_K> {
    static constexpr int kBox = 144;  // one super-block
    static constexpr int kStages = 8;
    __device__ static int box_x(int u) { return 18 * u; }
    __device__ static int offset(int) { return 0; }
};
template <>
struct Fmt<CN_TYPE_Q6_K> {
    // 210-byte super-blocks are only 2-byte aligned: load the 16-byte
    // aligned 240-byte window that covers super-block u and index into it.
    static constexpr int kBox = 240;
    static constexpr int kStages = 6;
    __device__ static int box_x(int u) { return ((210 * u) >> 4) * 2; }
    __device__ static int offset(int u) { return (210 * u) & 15; }
};

template <int TYPE>
constexpr int stage_bytes() {
    return Fmt<TYPE>::kBox * 16;
}
template <int TYPE>
constexpr int warp_smem() {
    return stage_bytes<TYPE>() * Fmt<TYPE>::kStages;
}
template <int TYPE>
constexpr int cta_smem() {
    return kWarps * warp_smem<TYPE>() + kWarps * Fmt<TYPE>::kStages * 8 + 1024;
}

struct GemvArgs {
    int64_t rows;
    int units;  // 256-position units per row
    int tiles;  // 16-row tiles
    int batch;
    const uint4* xfrag;  // [nt][chunks][32 lanes]
    const float* xsum;   // [batch][chunks]
    float* y;            // [batch][rows]
    float* partials;     // [2 * warps][16][nt*4] stream-K partial slots
    int* counters;       // [tiles]
    uint32_t* err;
};

// 32-bit word at byte offset `off` of a 4-byte aligned shared row, where
// off % 4 is known at compile time (0 or 2).
template <int MIS>
__device__ __forceinline__ uint32_t word_at(const uint8_t* row, int off) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(row + (off & ~3));
    if constexpr (MIS == 0) return w[0];
    else return __byte_perm(w[0], w[1], 0x5432);
}

__device__ __forceinline__ uint32_t word2(const uint8_t* p) {
    // p is 2-byte aligned; alignment known only at run time
    return lds_u32_a2(p);
}

// ---- per-unit consumers --------------------------------------------------

template <int NT>
__device__ __forceinline__ void unit_q4_0(const uint8_t* st, int u, int g, int t, int lane,
                                          const GemvArgs& a, int chunks, bool live[NT],
                                          float (&acc)[NT][4]) {
    const uint8_t* rg = st + g * 144;
    const uint8_t* rh = st + (g + 8) * 144;
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
        int c = u * 8 + b;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            uint4 bx = live[nt] ? __ldg(a.xfrag + ((size_t)nt * chunks + c) * 32 + lane)
                                : make_uint4(0, 0, 0, 0);
            float tmp[4];
            const float z[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t b0[2] = {bx.x, bx.y}, b1[2] = {bx.z, bx.w};
            mma_16816(tmp, a0, b0, z);
            mma_16816(tmp, a1, b1, tmp);
            acc[nt][0] = fmaf(tmp[0], dg, acc[nt][0]);
            acc[nt][1] = fmaf(tmp[1], dg, acc[nt][1]);
            acc[nt][2] = fmaf(tmp[2], dh, acc[nt][2]);
            acc[nt][3] = fmaf(tmp[3], dh, acc[nt][3]);
        }
    }
}

__device__ __forceinline__ float byte_f(uint32_t w, int k) { return (float)((w >> (8 * k)) & 0xFF); }

template <int NT>
__device__ __forceinline__ void unit_q4_k(const uint8_t* st, int u, int g, int t, int lane,
                                          const GemvArgs& a, int chunks, bool live[NT],
                                          float (&acc)[NT][4]) {
    const uint8_t* rg = st + g * 144;
    const uint8_t* rh = st + (g + 8) * 144;
    const uint32_t* Wg = reinterpret_cast<const uint32_t*>(rg);
    const uint32_t* Wh = reinterpret_cast<const uint32_t*>(rh);
    const uint32_t k1024 = 0x64006400u;
    const uint32_t k1_16 = 0x2C002C00u;
    const uint32_t km64 = 0xD400D400u;  // half2(-64, -64)
    float dg = half_bits_to_float(lds_u16(rg)), mg = half_bits_to_float(lds_u16(rg + 2));
    float dh = half_bits_to_float(lds_u16(rh)), mh = half_bits_to_float(lds_u16(rh + 2));
    // DecodeScales (DequantQ4K.cs:218-241), four bytes at a time
    uint32_t g0 = Wg[1], g1 = Wg[2], g2 = Wg[3];
    uint32_t h0 = Wh[1], h1 = Wh[2], h2 = Wh[3];
    uint32_t gsc[2] = {g0 & 0x3F3F3F3Fu, (g2 & 0x0F0F0F0Fu) | ((g0 >> 2) & 0x30303030u)};
    uint32_t gm[2] = {g1 & 0x3F3F3F3Fu, ((g2 >> 4) & 0x0F0F0F0Fu) | ((g1 >> 2) & 0x30303030u)};
    uint32_t hsc[2] = {h0 & 0x3F3F3F3Fu, (h2 & 0x0F0F0F0Fu) | ((h0 >> 2) & 0x30303030u)};
    uint32_t hm[2] = {h1 & 0x3F3F3F3Fu, ((h2 >> 4) & 0x0F0F0F0Fu) | ((h1 >> 2) & 0x30303030u)};
#pragma unroll
    for (int j = 0; j < 8; j++) {
        uint32_t wg = Wg[4 + 4 * j + t], wh = Wh[4 + 4 * j + t];
        uint32_t a0[4], a1[4], p, q;
        nib_lo(wg, p, q);
        a0[0] = h2_sub(p, k1024);
        a0[2] = h2_sub(q, k1024);
        nib_lo(wh, p, q);
        a0[1] = h2_sub(p, k1024);
        a0[3] = h2_sub(q, k1024);
        nib_hi(wg, p, q);
        a1[0] = h2_fma(p, k1_16, km64);
        a1[2] = h2_fma(q, k1_16, km64);
        nib_hi(wh, p, q);
        a1[1] = h2_fma(p, k1_16, km64);
        a1[3] = h2_fma(q, k1_16, km64);
        float dscg = dg * byte_f(gsc[j >> 2], j & 3), dmg = mg * byte_f(gm[j >> 2], j & 3);
        float dsch = dh * byte_f(hsc[j >> 2], j & 3), dmh = mh * byte_f(hm[j >> 2], j & 3);
        int c = u * 8 + j;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            uint4 bx = live[nt] ? __ldg(a.xfrag + ((size_t)nt * chunks + c) * 32 + lane)
                                : make_uint4(0, 0, 0, 0);
            int bidx = nt * 4 + t;
            float xs = bidx < a.batch ? __ldg(a.xsum + (size_t)bidx * chunks + c) : 0.f;
            float tmp[4];
            const float z[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t b0[2] = {bx.x, bx.y}, b1[2] = {bx.z, bx.w};
            mma_16816(tmp, a0, b0, z);
            mma_16816(tmp, a1, b1, tmp);
            acc[nt][0] = fmaf(tmp[0], dscg, fmaf(-dmg, xs, acc[nt][0]));
            acc[nt][1] = fmaf(tmp[1], dscg, acc[nt][1]);
            acc[nt][2] = fmaf(tmp[2], dsch, fmaf(-dmh, xs, acc[nt][2]));
            acc[nt][3] = fmaf(tmp[3], dsch, acc[nt][3]);
        }
    }
}

__device__ __forceinline__ float sbyte_f(uint32_t w, int k) {
    return (float)(int8_t)((w >> (8 * k)) & 0xFF);
}

template <int NT>
__device__ __forceinline__ void unit_q6_k(const uint8_t* st, int u, int g, int t, int lane,
                                          const GemvArgs& a, int chunks, bool live[NT],
                                          float (&acc)[NT][4]) {
    const int o = Fmt<CN_TYPE_Q6_K>::offset(u);
    const uint8_t* rg = st + g * 240 + o;
    const uint8_t* rh = st + (g + 8) * 240 + o;
    const uint32_t k1056 = 0x64206420u;  // half2(1056, 1056)
    float dg = half_bits_to_float(lds_u16(rg + 208));
    float dh = half_bits_to_float(lds_u16(rh + 208));
    uint32_t scg[4], sch[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        scg[i] = word2(rg + 192 + 4 * i);
        sch[i] = word2(rh + 192 + 4 * i);
    }
#pragma unroll
    for (int h = 0; h < 2; h++) {
        uint32_t Ag[2], Bg[2], Hg[2], Ah[2], Bh[2], Hh[2];
#pragma unroll
        for (int j = 0; j < 2; j++) {
            Ag[j] = word2(rg + 64 * h + 16 * j + 4 * t);
            Bg[j] = word2(rg + 64 * h + 32 + 16 * j + 4 * t);
            Hg[j] = word2(rg + 128 + 32 * h + 16 * j + 4 * t);
            Ah[j] = word2(rh + 64 * h + 16 * j + 4 * t);
            Bh[j] = word2(rh + 64 * h + 32 + 16 * j + 4 * t);
            Hh[j] = word2(rh + 128 + 32 * h + 16 * j + 4 * t);
        }
#pragma unroll
        for (int s = 0; s < 4; s++) {
            int c = u * 8 + 4 * h + s;
            uint4 bxs[NT];
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
                bxs[nt] = live[nt] ? __ldg(a.xfrag + ((size_t)nt * chunks + c) * 32 + lane)
                                   : make_uint4(0, 0, 0, 0);
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
                int si = 8 * h + j + 2 * s;  // scale index (DequantQ6K.cs:61,73-76)
                float sg = dg * sbyte_f(scg[si >> 2], si & 3);
                float sh = dh * sbyte_f(sch[si >> 2], si & 3);
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
                    acc[nt][0] = fmaf(tmp[0], sg, acc[nt][0]);
                    acc[nt][1] = fmaf(tmp[1], sg, acc[nt][1]);
                    acc[nt][2] = fmaf(tmp[2], sh, acc[nt][2]);
                    acc[nt][3] = fmaf(tmp[3], sh, acc[nt][3]);
                }
            }
        }
    }
}

// ---- stream-K bookkeeping ---------------------------------------------------
//
// The (tile, unit) space is linearised tile-major and cut into W equal
// contiguous ranges, one per warp.  A tile whose units all belong to one
// warp is written directly; otherwise every contributing warp stores its
// partial in slot 2*w + (tile is w's first tile ? 0 : 1), and the last of
// them to arrive sums the slots in warp order (deterministic) and resets
// the tile's counter for the next launch.

__device__ __forceinline__ int64_t range_start(int64_t total, int w, int W) {
    return total * w / W;
}

__device__ __forceinline__ int owner_of(int64_t v, int64_t total, int W) {
    int w = (int)((v * W) / total);
    while (w + 1 < W && range_start(total, w + 1, W) <= v) w++;
    while (w > 0 && range_start(total, w, W) > v) w--;
    return w;
}

template <int NT>
__device__ void finish_tile(const GemvArgs& a, int tile, int gw, int W, int64_t total, int g, int t,
                            int lane, float (&acc)[NT][4]) {
    const int64_t r0 = (int64_t)tile * 16 + g, r1 = r0 + 8;
    const int w_first = owner_of((int64_t)tile * a.units, total, W);
    const int w_last = owner_of((int64_t)(tile + 1) * a.units - 1, total, W);
    if (w_first == w_last) {
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            int b = nt * 4 + t;
            if (b < a.batch) {
                if (r0 < a.rows) a.y[(size_t)b * a.rows + r0] = acc[nt][0] + acc[nt][1];
                if (r1 < a.rows) a.y[(size_t)b * a.rows + r1] = acc[nt][2] + acc[nt][3];
            }
        }
        return;
    }
    constexpr int BW = NT * 4;
    auto slot = [&](int w) {
        int first_tile = (int)(range_start(total, w, W) / a.units);
        return 2 * w + (tile == first_tile ? 0 : 1);
    };
    float* p = a.partials + (size_t)slot(gw) * 16 * BW;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        p[g * BW + nt * 4 + t] = acc[nt][0] + acc[nt][1];
        p[(g + 8) * BW + nt * 4 + t] = acc[nt][2] + acc[nt][3];
    }
    __threadfence();
    __syncwarp();
    int prev = 0;
    if (lane == 0) prev = atomicAdd(&a.counters[tile], 1);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != w_last - w_first) return;
    // last arrival: reduce the contributors in warp order
    __threadfence();
    for (int e = lane; e < 16 * BW; e += 32) {
        float s = 0.f;
        for (int w = w_first; w <= w_last; w++)
            s += __ldcg(a.partials + (size_t)slot(w) * 16 * BW + e);
        int row = e / BW, b = e % BW;
        int64_t r = (int64_t)tile * 16 + row;
        if (b < a.batch && r < a.rows) a.y[(size_t)b * a.rows + r] = s;
    }
    if (lane == 0) atomicExch(&a.counters[tile], 0);
}

// ---- the kernel ---------------------------------------------------------------

template <int TYPE, int NT>
__global__ void __launch_bounds__(kWarps * 32)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap map, const GemvArgs a) {
    using F = Fmt<TYPE>;
    constexpr int S = F::kStages;
    constexpr int SB = stage_bytes<TYPE>();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    uint8_t* wsm = smem + warp * warp_smem<TYPE>();
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * warp_smem<TYPE>()) + warp * S;

    if (lane == 0) {
        for (int s = 0; s < S; s++) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    const int chunks = a.units * 8;
    const int64_t total = (int64_t)a.tiles * a.units;
    const int W = gridDim.x * kWarps;
    const int gw = blockIdx.x * kWarps + warp;
    const int64_t v0 = range_start(total, gw, W), v1 = range_start(total, gw + 1, W);
    bool live[NT];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) live[nt] = (nt * 4 + (g >> 1)) < a.batch;

    // lane 0 streams units v0..v1-1 into the stage ring
    int64_t pv = v0;
    auto issue = [&](int stage) {
        if (pv >= v1) return;
        int tile = (int)(pv / a.units), u = (int)(pv % a.units);
        mbar_expect_tx(&bars[stage], SB);
        tma_load_2d(wsm + stage * SB, &map, F::box_x(u), tile * 16, &bars[stage]);
        pv++;
    };
    if (lane == 0)
        for (int s = 0; s < S; s++) issue(s);

    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

    uint32_t n = 0;  // units consumed
    for (int64_t v = v0; v < v1; v++, n++) {
        const int stage = n % S;
        if (!mbar_wait(&bars[stage], (n / S) & 1)) {
            if (lane == 0) atomicOr(a.err, kErrTimeout);
            // let the copies already issued land (bounded) before leaving
            int64_t inflight = (v1 - v < S) ? (v1 - v) : S;
            for (int k = 1; k < inflight; k++) mbar_wait(&bars[(n + k) % S], ((n + k) / S) & 1);
            return;
        }
        const int tile = (int)(v / a.units), u = (int)(v % a.units);
        const uint8_t* st = wsm + stage * SB;
        if constexpr (TYPE == CN_TYPE_Q4_0) unit_q4_0<NT>(st, u, g, t, lane, a, chunks, live, acc);
        else if constexpr (TYPE == CN_TYPE_Q4_K) unit_q4_k<NT>(st, u, g, t, lane, a, chunks, live, acc);
        else unit_q6_k<NT>(st, u, g, t, lane, a, chunks, live, acc);
        __syncwarp();
        if (lane == 0) {
            fence_proxy_async();
            issue(stage);
        }
        if (u == a.units - 1 || v == v1 - 1) {
            finish_tile<NT>(a, tile, gw, W, total, g, t, lane, acc);
#pragma unroll
            for (int nt = 0; nt < NT; nt++) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
        }
    }
}

// ---- activation prep ----------------------------------------------------------
//
// xfrag[nt][c][lane] = the four B-fragment registers lane (g, t) feeds to
// the two k-steps of 32-position chunk c: column g = hi (g even) or lo
// (g odd) part of batch row 4*nt + g/2, positions 4t+{0,2}, 4t+{1,3} of
// each 16-position half.  xsum[b][c] = fp32 sum of x[b] over chunk c.
__global__ void xprep_kernel(const float* __restrict__ x, int K, int batch, int nt_count,
                             uint4* __restrict__ xfrag, float* __restrict__ xsum) {
    const int chunks = K / 32;
    const int64_t total = (int64_t)nt_count * chunks * 32;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int lane = (int)(i & 31);
        int64_t rest = i >> 5;
        int c = (int)(rest % chunks);
        int nt = (int)(rest / chunks);
        int g = lane >> 2, t = lane & 3;
        int b = nt * 4 + (g >> 1);
        uint4 out = make_uint4(0, 0, 0, 0);
        if (b < batch) {
            const float* xr = x + (size_t)b * K + (size_t)c * 32 + 4 * t;
            float4 v0 = *reinterpret_cast<const float4*>(xr);
            float4 v1 = *reinterpret_cast<const float4*>(xr + 16);
            float e[8] = {v0.x, v0.z, v0.y, v0.w, v1.x, v1.z, v1.y, v1.w};
            uint32_t r[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                float e0 = e[2 * k], e1 = e[2 * k + 1];
                __half2 h = __floats2half2_rn(e0, e1);
                if (g & 1) {  // lo part: the rounding residual of the hi part
                    float2 back = __half22float2(h);
                    h = __floats2half2_rn(e0 - back.x, e1 - back.y);
                }
                r[k] = *reinterpret_cast<uint32_t*>(&h);
            }
            out = make_uint4(r[0], r[1], r[2], r[3]);
        }
        xfrag[i] = out;
        if (xsum != nullptr && lane == 0 && nt == 0) {
            for (int bb = 0; bb < batch; bb++) {
                const float* xr = x + (size_t)bb * K + (size_t)c * 32;
                float s = 0.f;
                for (int k = 0; k < 32; k++) s += xr[k];
                xsum[(size_t)bb * chunks + c] = s;
            }
        }
    }
}

// ---- generic (untiled) fallback -------------------------------------------------
//
// For shapes the TMA path cannot tile (row bytes not a multiple of 16, or K
// not a multiple of 256): one warp per (row, batch), exact block decode and
// fp32 FMAs.  Slow but shape-agnostic.
__device__ float block_dot(int type, const uint8_t* row, int blk, const float* x) {
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
    } else if (type == CN_TYPE_F16) {
        s = ld_half(row + 2 * (size_t)blk) * x[blk];
    }
    return s;
}

__global__ void gemv_generic_kernel(int type, const uint8_t* __restrict__ w, int64_t rows, int cols,
                                    uint64_t rbytes, int blk_elems, const float* __restrict__ x,
                                    float* __restrict__ y, int batch) {
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
        for (int k = lane; k < nblk; k += 32) s += block_dot(type, row, k, xb);
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
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

static int box_bytes(int type) {
    switch (type) {
        case CN_TYPE_Q4_0: return Fmt<CN_TYPE_Q4_0>::kBox;
        case CN_TYPE_Q4_K: return Fmt<CN_TYPE_Q4_K>::kBox;
        case CN_TYPE_Q6_K: return Fmt<CN_TYPE_Q6_K>::kBox;
        default: return 0;
    }
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
    cuuint32_t box[2] = {(cuuint32_t)(bx / 8), 16};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(d_w), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(CN_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return CN_OK;
}

template <int TYPE, int NT>
static int occupancy_ctas(cn_ctx* ctx) {
    static int cached = -1;  // per instantiation (all B200s alike)
    if (cached < 0) {
        auto k = gemv_tma_kernel<TYPE, NT>;
        CN_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     cta_smem<TYPE>()));
        int n = 0;
        CN_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kWarps * 32, cta_smem<TYPE>()));
        cached = n > 0 ? n : 1;
    }
    return cached;
}

static int pick_nt(int batch) { return batch <= 4 ? 1 : batch <= 8 ? 2 : batch <= 16 ? 4 : 8; }

static bool tileable(int type, int64_t cols, uint64_t rb) {
    return box_bytes(type) > 0 && cols % 256 == 0 && rb % 16 == 0;
}

int gemv_plan(cn_ctx* ctx, int type, int64_t rows, int64_t cols, int batch, bool tma,
              GemvPlan* p) {
    p->nt = pick_nt(batch);
    p->tma = tma;
    p->tiles = (int)((rows + 15) / 16);
    p->units = (int)(cols / 256);
    if (!tma) return CN_OK;
    int occ = 1;
#define CN_OCC(T)                                                  \
    switch (p->nt) {                                               \
        case 1: occ = occupancy_ctas<T, 1>(ctx); break;            \
        case 2: occ = occupancy_ctas<T, 2>(ctx); break;            \
        case 4: occ = occupancy_ctas<T, 4>(ctx); break;            \
        default: occ = occupancy_ctas<T, 8>(ctx); break;           \
    }
    if (type == CN_TYPE_Q4_0) { CN_OCC(CN_TYPE_Q4_0) }
    else if (type == CN_TYPE_Q4_K) { CN_OCC(CN_TYPE_Q4_K) }
    else { CN_OCC(CN_TYPE_Q6_K) }
#undef CN_OCC
    if (occ < 0) return occ;  // error code from the occupancy query
    // Stream-K grid: every resident warp gets an equal share of the
    // (tile, unit) space, but at least 2 units each so short matrices do
    // not spread over warps that would only fill their pipelines.
    const int64_t total = (int64_t)p->tiles * p->units;
    int64_t want = (total / 2 + kWarps - 1) / kWarps;
    if (want < 1) want = 1;
    int ctas = ctx->sms * occ;
    if (want < ctas) ctas = (int)want;
    p->ctas = ctas;
    const int W = ctas * kWarps;
    const int chunks = p->units * 8;
    p->xfrag_bytes = (size_t)p->nt * chunks * 32 * sizeof(uint4);
    p->xsum_bytes = type == CN_TYPE_Q4_K ? (size_t)batch * chunks * sizeof(float) : 0;
    p->partial_bytes = (size_t)2 * W * 16 * p->nt * 4 * sizeof(float);
    p->counters = (size_t)p->tiles;
    return CN_OK;
}

template <int TYPE, int NT>
static int launch_tma(cn_ctx* ctx, const CUtensorMap* map, const GemvPlan& p, const GemvArgs& a) {
    auto k = gemv_tma_kernel<TYPE, NT>;
    k<<<p.ctas, kWarps * 32, cta_smem<TYPE>(), ctx->stream>>>(*map, a);
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

int gemv_launch(cn_ctx* ctx, int type, const void* d_w, int64_t rows, int64_t cols,
                const CUtensorMap* map, const float* d_x, float* d_y, int batch) {
    CN_CHECK(type_supported(type), CN_ERR_UNSUPPORTED, "Unsupported weight quantization type: %d",
             type);
    CN_CHECK(rows > 0 && cols > 0 && batch > 0 && batch <= 32, CN_ERR_INVALID_ARG,
             "bad matvec shape rows=%lld cols=%lld batch=%d", (long long)rows, (long long)cols,
             batch);
    CN_CHECK(rows < (1ll << 31) && cols < (1ll << 31), CN_ERR_INVALID_ARG, "matvec too large");
    CN_CHECK((reinterpret_cast<uintptr_t>(d_x) & 15) == 0 && (reinterpret_cast<uintptr_t>(d_y) & 3) == 0,
             CN_ERR_INVALID_ARG, "x must be 16-byte aligned and y 4-byte aligned");
    const uint64_t rb = row_bytes(type, cols);
    CUtensorMap local;
    bool tma = tileable(type, cols, rb) && ((reinterpret_cast<uintptr_t>(d_w) & 15) == 0);
    if (tma && map == nullptr) {
        if (encode_weight_map(type, d_w, rows, rb, &local) != CN_OK) tma = false;
        else map = &local;
    }
    if (!tma) {
        int blk = type == CN_TYPE_Q4_0 ? 32 : (type == CN_TYPE_Q4_K || type == CN_TYPE_Q6_K) ? 256 : 1;
        CN_CHECK(cols % blk == 0, CN_ERR_INVALID_ARG, "inDim %lld not a multiple of %d",
                 (long long)cols, blk);
        int threads = 256;
        int64_t warps = rows * batch;
        int64_t blocks = (warps * 32 + threads - 1) / threads;
        if (blocks > ctx->sms * 16) blocks = ctx->sms * 16;
        gemv_generic_kernel<<<(unsigned)blocks, threads, 0, ctx->stream>>>(
            type, (const uint8_t*)d_w, rows, (int)cols, rb, blk, d_x, d_y, batch);
        CN_CUDA(cudaGetLastError());
        return CN_OK;
    }
    GemvPlan p;
    int rc = gemv_plan(ctx, type, rows, cols, batch, true, &p);
    if (rc) return rc;
    rc = ensure(&ctx->xfrag, &ctx->xfrag_bytes, p.xfrag_bytes, false);
    if (rc) return rc;
    if (p.xsum_bytes) {
        rc = ensure((void**)&ctx->xsum, &ctx->xsum_bytes, p.xsum_bytes, false);
        if (rc) return rc;
    }
    if (p.partial_bytes) {
        rc = ensure((void**)&ctx->partials, &ctx->partial_bytes, p.partial_bytes, false);
        if (rc) return rc;
        size_t cb = ctx->counter_count * sizeof(int);
        rc = ensure((void**)&ctx->counters, &cb, p.counters * sizeof(int), true);
        if (rc) return rc;
        ctx->counter_count = cb / sizeof(int);
    }
    {
        const int chunks = p.units * 8;
        int64_t total = (int64_t)p.nt * chunks * 32;
        int threads = 256;
        int blocks = (int)((total + threads - 1) / threads);
        if (blocks > ctx->sms * 8) blocks = ctx->sms * 8;
        xprep_kernel<<<blocks, threads, 0, ctx->stream>>>(
            d_x, (int)cols, batch, p.nt, (uint4*)ctx->xfrag,
            type == CN_TYPE_Q4_K ? ctx->xsum : nullptr);
        CN_CUDA(cudaGetLastError());
    }
    GemvArgs a;
    a.rows = rows;
    a.units = p.units;
    a.tiles = p.tiles;
    a.batch = batch;
    a.xfrag = (const uint4*)ctx->xfrag;
    a.xsum = ctx->xsum;
    a.y = d_y;
    a.partials = ctx->partials;
    a.counters = ctx->counters;
    a.err = ctx->dev_err;
#define CN_DISPATCH(T)                                              \
    switch (p.nt) {                                                 \
        case 1: return launch_tma<T, 1>(ctx, map, p, a);            \
        case 2: return launch_tma<T, 2>(ctx, map, p, a);            \
        case 4: return launch_tma<T, 4>(ctx, map, p, a);            \
        default: return launch_tma<T, 8>(ctx, map, p, a);           \
    }
    if (type == CN_TYPE_Q4_0) { CN_DISPATCH(CN_TYPE_Q4_0) }
    if (type == CN_TYPE_Q4_K) { CN_DISPATCH(CN_TYPE_Q4_K) }
    CN_DISPATCH(CN_TYPE_Q6_K)
#undef CN_DISPATCH
}

}  // namespace cn
