// gemv_i8.cu -- Q4_K dequant-GEMV on integer mma.sync (m16n8k32, u8 x s8 ->
// s32), decode batch 1..8.
//
// Same contract as the other GEMVs (TensorMath.MatVecMulGeneric with
// DequantQ4K.DotProduct, Tensors/TensorMath.cs:624-656, DequantQ4K.cs:89-163).
// A decode GEMV streams every weight byte once and reuses it only for the
// batch's few columns, so the limit is instructions issued per weight, not
// math.  Here a weight costs about one instruction:
//
//  * A producer warp streams [128 rows x one 144-byte super-block] of raw
//    blocks per unit (2-D TMA) plus the unit's activation record (bulk copy,
//    gemv_i8.cuh) into a ring of shared-memory stages: at batch 1-2 one CTA
//    per SM with ~200 KB of stages (the deep instantiation), else 2-3 CTAs
//    per SM with 3-4 stages each.
//  * Eight consumer warps own 16 rows each.  One ldmatrix.x4 hands a warp the
//    quant words of two sub-blocks for its 16 rows, already in the A-fragment
//    layout of m16n8k32 (row g, bytes 4t..4t+3 of the sub-block's 16 bytes:
//    low nibbles = positions 4t+0..3, high nibbles = 16+4t+0..3).  One AND
//    (low nibbles) and one AND (batch 1: 16 * high nibble) or shift+AND
//    (high nibbles) per register give the u8 operand.
//  * Activations are exact integer digits (gemv_i8.cuh), so each MMA gives
//    the exact integer sum_i q_i X_i of a sub-block; its 6-bit scale is
//    applied with one integer multiply-add per accumulator.  Once per unit
//    and row the digits are recombined (fp32), and
//    d * sum - dmin * sum_j m_j XS_j, times 2^-e, joins the row's fp32 sum.
//  * Stream-K over (128-row tile, unit) as in gemv.cu, deterministic fix-up.
// Every mbarrier wait is bounded (error word, then uniform fall-through).
#include <stdlib.h>

#include <mutex>

#include "cn_common.cuh"
#include "cn_internal.h"
#include "gemv_i8.cuh"

namespace cn {

namespace i8 {

constexpr int kRows = 128;
constexpr int kRaw = 144 * kRows;  // raw Q4_K bytes per unit per tile
constexpr int kCons = 8;           // consumer warps, 16 rows each
constexpr int kMaxCluster = 8;     // most CTAs of one tile that meet in a cluster (portable size)

// Three CTAs per SM with three stages each when one n-tile of activation
// digits suffices (batch 1, 2), else two CTAs with four stages.  DEEP: one
// CTA per SM with ~200 KB of stages, for grids of at most one CTA per SM
// (short or few rows, e.g. tensor-parallel shards): the bytes one CTA keeps
// in flight, not the SM count, then bound the weight stream.
//
// DEEP == 2 is the deep pipeline with two groups of eight consumer warps
// that take alternate stages: a unit costs a group's warps a long latency
// chain (about a thousand cycles, which alone would hold an SM near 35 GB/s),
// so two units in flight keep the weight stream moving.  The groups' partial
// sums of a tile meet in shared memory at the tile's end.  Batch 1-2 uses it
// for every deep launch of up to 128 units per CTA (grouped_units).
template <int NB, int DEEP = 0>
struct Geo {
    static constexpr int NT = n_tiles(NB);
    static constexpr int kRec = (rec_bytes(NT) + 127) / 128 * 128;
    static constexpr int kStage = kRaw + kRec;
    static constexpr int kCtasPerSm = DEEP ? 1 : NT == 1 ? 3 : 2;
    static constexpr int kGroups = DEEP == 2 ? 2 : 1;
    static constexpr int kThreads = (kGroups * kCons + 1) * 32;
    static constexpr int kStages = (DEEP ? 200 * 1024 : NT == 1 ? 72 * 1024 : 110 * 1024) / kStage;
    static constexpr int kXchg = DEEP == 2 ? 2 * kCons * 32 * NT * 4 : 0;  // group partials, two buffers
    // the cluster form (batch 1-2): the other CTAs' sums of the shared tile
    static constexpr int kPair = DEEP && NB <= 2 ? (kMaxCluster - 1) * kRows * NB * 4 : 0;
    static constexpr int kSmem = kStages * kStage + 256 + kXchg + kPair;
    // full[kStages], empty[kStages] and the cluster barrier fit the 256-byte slot
    static_assert(16 * kStages + 8 <= 256, "barrier slot");
};
static_assert(Geo<1>::kStages >= 3 && Geo<3>::kStages >= 4 && Geo<8>::kStages >= 4 && Geo<16>::kStages >= 3,
              "pipeline depth");
static_assert(Geo<16, 1>::kSmem <= 227 * 1024 && Geo<16, 1>::kStages >= 5, "16-sequence deep pipeline");
static_assert(Geo<1, 1>::kStages >= 8 && Geo<8, 1>::kStages >= 7 && Geo<8, 1>::kSmem <= 227 * 1024,
              "deep pipeline depth");

// Up to kMaxMats weight matrices with the same inner dimension share one
// launch (and one activation record): their 128-row tiles are numbered one
// after another, matrix m owning tiles [toff[m], toff[m + 1]).
constexpr int kMaxMats = 3;
struct Maps {
    CUtensorMap m[kMaxMats];
};

struct Args {
    int units, tiles, batch, nmat;
    int toff[kMaxMats + 1];
    int64_t rows[kMaxMats];
    float* y[kMaxMats];   // [batch][rows[m]]
    const uint8_t* xrec;  // [unit][rec_bytes(NT)]
    float* partials;      // [2 * ctas][128][kMaxNB]
    int* counters;        // [tiles][kCons], zero on entry, left zero
    uint32_t* err;
    XchgOut xo;           // size > 1: outputs go to every rank (one matrix only)
    int csize;            // > 1: CTAs csize*k .. csize*k + csize-1 (one cluster) split tile k's units (cluster_finish)
};

// Stores output value (b, row) of matrix m: locally, or, in an exchange, into
// every rank's buffer (peer stores over NVLink).
__device__ __forceinline__ void store_out(const Args& a, float* y, int64_t rows, int b, int64_t row, float v,
                                          uint32_t seq) {
    if (a.xo.size <= 1) {
        y[(size_t)b * rows + row] = v;
        return;
    }
    const int64_t off = (seq & 1u) * a.xo.parity_stride + b * a.xo.dst_ld + a.xo.dst_row0 + row;
    if (a.xo.ll) {
        // value and sequence number in one 8-byte store: the pair is atomic
        const uint64_t pair = ((uint64_t)seq << 32) | __float_as_uint(v);
#pragma unroll
        for (int p = 0; p < kMaxTp; p++)
            if (p < a.xo.size)
                asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(reinterpret_cast<uint64_t*>(a.xo.dst[p]) + off),
                             "l"(pair)
                             : "memory");
        return;
    }
#pragma unroll
    for (int p = 0; p < kMaxTp; p++)
        if (p < a.xo.size) a.xo.dst[p][off] = v;
}

// matrix of a tile, its first row in that matrix, its row count and output
__device__ __forceinline__ int mat_of(const Args& a, int tile) {
    return (a.nmat > 2 && tile >= a.toff[2]) ? 2 : (a.nmat > 1 && tile >= a.toff[1]) ? 1 : 0;
}
__device__ __forceinline__ int64_t pick64(const int64_t (&v)[kMaxMats], int m) {
    return m == 2 ? v[2] : m == 1 ? v[1] : v[0];
}
__device__ __forceinline__ float* pickp(float* const (&v)[kMaxMats], int m) {
    return m == 2 ? v[2] : m == 1 ? v[1] : v[0];
}

__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

__device__ __forceinline__ void imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                     uint2 b) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y), "r"(0));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}
// byte k of w, zero-extended
__device__ __forceinline__ int byte_of(uint32_t w, int k) { return (int)__byte_perm(w, 0u, 0x4440u | k); }
// dot product of four u8 lanes of a with four s8 lanes of b, plus c
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ int64_t range_start(int64_t total, int c, int C) { return total * c / C; }
__device__ __forceinline__ int owner_of(int64_t v, int64_t total, int C) {
    int c = (int)((v * C) / total);
    while (c + 1 < C && range_start(total, c + 1, C) <= v) c++;
    while (c > 0 && range_start(total, c, C) > v) c--;
    return c;
}

// Which (row, sequence) pairs a consumer thread owns after the per-unit
// recombination: row (t & 1 ? g + 8 : g) of its warp's 16 and, per n-tile nt,
// sequence 2 nt + t / 2 (batch > 1) or sequence 0 for t < 2 (batch 1); -1
// past the call's batch (the 16-sequence form runs batches 9-16).
template <int NB>
__device__ __forceinline__ int owned_seq(int nt, int t, int batch) {
    const int b = NB == 1 ? (t < 2 ? 0 : -1) : 2 * nt + (t >> 1);
    return b < NB && b < batch ? b : -1;
}

// Stores the owned values of a finished 16-row sub-tile, or, for a tile
// several CTAs share, parks this warp's partials and lets the last warp to
// arrive (per 16-row sub-tile, so warps never wait for each other) add all
// contributors' partials in CTA order: deterministic.  r = the thread's row
// in the 128-row tile.
template <int NB>
__device__ void finish_subtile(const Args& a, int r, int t, int warp, int tile, int cta, int C,
                               int64_t total, bool shared_tile, int my_slot,
                               const float (&acc)[Geo<NB>::NT], uint32_t seq) {
    constexpr int NT = Geo<NB>::NT;
    const int m = mat_of(a, tile);
    const int64_t rows = pick64(a.rows, m);
    float* const y = pickp(a.y, m);
    const int64_t row = (int64_t)(tile - (m == 2 ? a.toff[2] : m == 1 ? a.toff[1] : 0)) * kRows + r;
    if (!shared_tile) {
        if (row < rows) {
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int b = owned_seq<NB>(nt, t, a.batch);
                if (b >= 0) store_out(a, y, rows, b, row, acc[nt], seq);
            }
        }
        return;
    }
    float* p = a.partials + ((size_t)(2 * cta + my_slot) * kRows + r) * kMaxNB;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const int b = owned_seq<NB>(nt, t, a.batch);
        if (b >= 0) p[b] = acc[nt];
    }
    // __syncwarp orders the lanes' partials before lane 0's release-acquire
    // increment; the last arrival's acquire orders every contributor's
    // partials before its reads
    __syncwarp();
    const int c_first = owner_of((int64_t)tile * a.units, total, C);
    const int c_last = owner_of((int64_t)(tile + 1) * a.units - 1, total, C);
    int* ctr = a.counters + tile * kCons + warp;
    int old = 0;
    if ((threadIdx.x & 31) == 0)
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(ctr) : "memory");
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != c_last - c_first) return;
    // Contributor c's partial of this tile sits in slot 2c (the tile is the
    // first of c's range) except for c_first when its range began in an
    // earlier tile (slot 2c + 1).  The loads of kBatchC contributors are
    // issued together (16-32 per thread), not one L2 round trip after
    // another (a tile shared by six CTAs at batch 16 took ~19 us that way);
    // the sums still run in CTA order.
    constexpr int kBatchC = NT >= 8 ? 2 : 4;
    const int first_slot = 2 * c_first + (range_start(total, c_first, C) < (int64_t)tile * a.units ? 1 : 0);
    const float* base = a.partials + (size_t)r * kMaxNB;
    float s[NT];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) s[nt] = 0.f;
    for (int c0 = c_first; c0 <= c_last; c0 += kBatchC) {
        float v[kBatchC][NT];
#pragma unroll
        for (int k = 0; k < kBatchC; k++) {
            const int c = c0 + k;
            const int slot = c == c_first ? first_slot : 2 * c;
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int b = owned_seq<NB>(nt, t, a.batch);
                v[k][nt] = (c <= c_last && b >= 0) ? __ldcg(base + (size_t)slot * kRows * kMaxNB + b) : 0.f;
            }
        }
#pragma unroll
        for (int k = 0; k < kBatchC; k++)
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
                if (c0 + k <= c_last) s[nt] += v[k][nt];
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const int b = owned_seq<NB>(nt, t, a.batch);
        if (b >= 0 && row < rows) store_out(a, y, rows, b, row, s[nt], seq);
    }
    __syncwarp();
    if ((threadIdx.x & 31) == 0) atomicExch(ctr, 0);
}

// ---- cluster splits -----------------------------------------------------------
//
// When a launch gives every 128-row tile the same number s (2..8) of CTAs
// (batch 1-2 grids of fewer tiles than SMs: Llama-2-70B's O and down with
// s = 2, tensor-parallel q/k/v shards with s up to 7), the s CTAs of a tile
// run as one cluster and meet in the leader's shared memory instead of the
// global fix-up above, whose release-acquire counter and L2 partials add
// ~3 us to the end of every CTA.  CTA s*k + j (cluster rank j) holds the
// j-th of s equal parts of tile k's units; each other CTA stores its owned
// sums into the leader's buffer slot j-1 (st.shared::cluster), and each of
// its warps then arrives, with release semantics at cluster scope, on the
// leader's barrier; the leader waits for all 8 (s - 1) arrivals (bounded),
// adds the slots to its own sums in rank order -- the stream-K order -- and
// stores.  Every thread of the cluster arrives on the cluster barrier at
// entry, and a warp waits on it before its first remote store, so the
// leader's shared memory is live; the leader stays resident until its
// barrier completes, so no remote store can land after it exits.
template <int NB>
__device__ void cluster_finish(const Args& a, int r, int t, int tile, const float (&acc)[Geo<NB>::NT],
                               uint32_t seq, uint32_t pbar, uint32_t pbuf) {
    static_assert(Geo<NB>::NT == 1, "cluster splits run batch 1-2");
    constexpr uint32_t kSlot = kRows * NB * 4;  // bytes of one CTA's sums
    const int b = owned_seq<NB>(0, t, a.batch);
    const uint32_t own = (uint32_t)(r * NB + (b < 0 ? 0 : b)) * 4u;
    cluster_wait();
    const uint32_t rank = cluster_rank();
    if (rank != 0) {
        if (b >= 0)
            asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(map_rank(pbuf + (rank - 1) * kSlot + own, 0)),
                         "f"(acc[0])
                         : "memory");
        __syncwarp();
        if ((threadIdx.x & 31) == 0)
            asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(map_rank(pbar, 0))
                         : "memory");
        return;
    }
    if (!mbar_wait_cluster(pbar, 0)) {
        atomicOr(a.err, kErrTimeout);
        return;
    }
    const int m = mat_of(a, tile);
    const int64_t rows = pick64(a.rows, m);
    const int64_t row = (int64_t)(tile - (m == 2 ? a.toff[2] : m == 1 ? a.toff[1] : 0)) * kRows + r;
    if (b < 0 || row >= rows) return;
    float v = acc[0];
    uint32_t p = pbuf + own;
#pragma unroll 1
    for (int j = 1; j < a.csize; j++, p += kSlot) v += lds_f32(p);
    store_out(a, pickp(a.y, m), rows, b, row, v, seq);
}

}  // namespace i8

template <int NB, int DEEP>
__global__ void __launch_bounds__(i8::Geo<NB, DEEP>::kThreads, i8::Geo<NB, DEEP>::kCtasPerSm)
    gemv_i8_q4k_kernel(const __grid_constant__ i8::Maps maps, const i8::Args a) {
    using namespace i8;
    using G = Geo<NB, DEEP>;
    constexpr int NT = G::NT;
    constexpr int kStages = G::kStages, kStage = G::kStage;
    constexpr int kRecB = rec_bytes(NT);
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStage);
    uint64_t* empty = full + kStages;
    float* xg = reinterpret_cast<float*>(smem + kStages * kStage + 256);  // [2][kCons][32][NT]
    // cluster pairs: the leader's barrier and its buffer of the partner's sums
    uint64_t* pbar_p = empty + kStages;
    const uint32_t pbar = smem_u32(pbar_p), pbuf = smem_u32(smem + kStages * kStage + 256 + G::kXchg);
    const bool pair = G::kPair != 0 && a.csize > 1;
    constexpr int kGroups = G::kGroups;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCons);
        }
        if (pair) mbar_init(pbar_p, kCons * (a.csize - 1));
        fence_mbar_init();
    }
    __syncthreads();
    if (pair) cluster_arrive_relaxed();
    pdl_trigger();

    const int64_t total = (int64_t)a.tiles * a.units;
    const int C = (int)(total < (int64_t)gridDim.x ? total : (int64_t)gridDim.x);
    const int cta = blockIdx.x;
    const int64_t v0 = cta < C ? range_start(total, cta, C) : 0;
    const int64_t v1 = cta < C ? range_start(total, cta + 1, C) : 0;
    const int nunits = (int)(v1 - v0);
    const int tile0 = cta < C ? (int)(v0 / a.units) : 0;
    const int u0 = cta < C ? (int)(v0 % a.units) : 0;

    if (warp == kGroups * kCons) {
        // ---- producer ----
        if (lane == 0) {
            // the weights depend on no earlier kernel: start the first
            // stages' loads, then wait for the kernel that writes the
            // activation records
            // raw blocks of unit u of global tile `tile` (its matrix's map, the
            // tile's rows within that matrix)
            auto load_raw = [&](uint8_t* dst, int tile, int u, uint64_t* bar) {
                const int m = mat_of(a, tile);
                const int lt = tile - (m == 2 ? a.toff[2] : m == 1 ? a.toff[1] : 0);
                tma_load_2d(dst, &maps.m[m], 18 * u, lt * kRows, bar);
            };
            const int pre = nunits < kStages ? nunits : kStages;
            {
                int tile = tile0, u = u0;
                for (int n = 0; n < pre; n++) {
                    mbar_expect_tx(&full[n], kRaw + kRecB);
                    load_raw(smem + n * kStage, tile, u, &full[n]);
                    if (++u == a.units) {
                        u = 0;
                        tile++;
                    }
                }
            }
            pdl_wait();
            int tile = tile0, u = u0, s = 0, issued = 0;
            uint32_t ph = 0;
            for (int n = 0; n < nunits; n++) {
                uint8_t* st = smem + s * kStage;
                if (n >= kStages) {
                    if (!mbar_wait_sleep(&empty[s], ph ^ 1)) {
                        atomicOr(a.err, kErrTimeout);
                        break;
                    }
                    mbar_expect_tx(&full[s], kRaw + kRecB);
                    load_raw(st, tile, u, &full[s]);
                }
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
                    "[%3];" ::"r"(smem_u32(st + kRaw)),
                    "l"(reinterpret_cast<uint64_t>(a.xrec + (size_t)u * kRecB)), "r"(kRecB),
                    "r"(smem_u32(&full[s]))
                    : "memory");
                issued = n + 1;
                if (++u == a.units) {
                    u = 0;
                    tile++;
                }
                if (++s == kStages) {
                    s = 0;
                    ph ^= 1;
                }
            }
            // no copy may still be landing when the CTA exits (the first
            // stages' weight loads were issued even if the loop stopped early)
            if (issued < pre) issued = pre;
            for (int n = issued - kStages < 0 ? 0 : issued - kStages; n < issued; n++)
                mbar_wait(&full[n % kStages], (uint32_t)(n / kStages) & 1);
        }
        return;
    }

    // ---- consumers ----
    pdl_wait();
    const uint32_t seq = a.xo.size > 1 ? *a.xo.seq_base * a.xo.uses + a.xo.seq_add : 0u;
    const int g = lane >> 2, t = lane & 3;
    const int cg = warp / kCons, cw = warp % kCons;  // consumer group, warp within it (16 rows each)
    const int row0 = 16 * cw + g, row1 = row0 + 8;
    const int r_own = (t & 1) ? row1 : row0;
    // ldmatrix.x2: lanes 0-7 address rows 0-7 of the warp's 16, lanes 8-15
    // rows 8-15 (lanes 16-31 repeat them), at the sub-block's quant bytes
    const uint32_t lds_off = (uint32_t)((16 * cw + (lane & 15)) * 144 + 16);
    // weights of this thread's two accumulator columns in the recombination
    // (batch 1: base 15, columns 2t and 2t+1 weigh 15^2t and 15^(2t+1))
    const float w_lo = NB == 1 ? (t == 0 ? 1.0f : t == 1 ? 225.0f : t == 2 ? 50625.0f : 11390625.0f)
                               : ldexpf(1.0f, 16 * (t & 1));
    const float w_hi = NB == 1 ? 15.0f * w_lo : ldexpf(1.0f, 16 * (t & 1) + 8);
    // weight of the min term (batch 1 sums carry the digits' factor 16)
    const float kMin = NB == 1 ? -16.0f : -1.0f;
    const uint32_t smem0 = smem_u32(smem);

    int n = 0, et = tile0, eu = u0, segi = 0;
    // this group's next stage and its phase: its units are cg, cg + kGroups, ...
    int s = cg;
    uint32_t ph = 0;
    bool ok = true;
    while (n < nunits) {
        // one tile segment of this CTA's range
        const int seg = min(nunits - n, a.units - eu);
        float acc[NT];
#pragma unroll
        for (int nt = 0; nt < NT; nt++) acc[nt] = 0.f;
        // group cg takes the range's units gn with gn % kGroups == cg
        for (int k = (kGroups - (n % kGroups) + cg) % kGroups; k < seg; k += kGroups) {
            if (ok && !mbar_wait_sleep(&full[s], ph)) {
                atomicOr(a.err, kErrTimeout);
                ok = false;
            }
            __syncwarp();
            const uint32_t st = smem0 + s * kStage;
            const uint32_t rec = st + kRaw;
            const uint4 h0 = lds128(st + row0 * 144);
            const uint4 h1 = lds128(st + row1 * 144);
            // DecodeScales (DequantQ4K.cs:218-241): the 8 six-bit scales of each row
            int sc0[8], sc1[8];
            {
                const uint32_t lo0 = h0.y & 0x3F3F3F3Fu, hi0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
                const uint32_t lo1 = h1.y & 0x3F3F3F3Fu, hi1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    sc0[q] = byte_of(lo0, q);
                    sc0[4 + q] = byte_of(hi0, q);
                    sc1[q] = byte_of(lo1, q);
                    sc1[4 + q] = byte_of(hi1, q);
                }
            }
            int S[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; nt++) S[nt][0] = S[nt][1] = S[nt][2] = S[nt][3] = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                // quant words of sub-block j, rows g and g+8: byte 4t+i holds
                // positions 4t+i (low nibble) and 16+4t+i (high nibble)
                uint32_t q0, q1;
                ldsm_x2(st + lds_off + 16 * j, q0, q1);
                // batch 1: k-slots 0-15 take the raw bytes, 16-31 the low
                // nibbles (gemv_i8.cuh); otherwise low, then high nibbles
                const uint32_t a0 = NB == 1 ? q0 : (q0 & 0x0F0F0F0Fu);
                const uint32_t a1 = NB == 1 ? q1 : (q1 & 0x0F0F0F0Fu);
                const uint32_t a2 = NB == 1 ? (q0 & 0x0F0F0F0Fu) : ((q0 >> 4) & 0x0F0F0F0Fu);
                const uint32_t a3 = NB == 1 ? (q1 & 0x0F0F0F0Fu) : ((q1 >> 4) & 0x0F0F0F0Fu);
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    const uint2 bf = lds64(rec + ((j * NT + nt) * 32 + lane) * 8);
                    int d[4];
                    imma(d, a0, a1, a2, a3, bf);
                    S[nt][0] += sc0[j] * d[0];
                    S[nt][1] += sc0[j] * d[1];
                    S[nt][2] += sc1[j] * d[2];
                    S[nt][3] += sc1[j] * d[3];
                }
            }
            // the owned row: d, dmin and its packed mins (DecodeScales)
            const uint4 ho = lds128(st + r_own * 144);
            const float dd = half_bits_to_float((uint16_t)(ho.x & 0xFFFF));
            const float dmin = half_bits_to_float((uint16_t)(ho.x >> 16));
            const uint32_t m_lo = ho.z & 0x3F3F3F3Fu;
            const uint32_t m_hi = ((ho.w >> 4) & 0x0F0F0F0Fu) | ((ho.z >> 2) & 0x30303030u);
            float mt[NT], iv[NT];
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int b = NB == 1 ? 0 : 2 * nt + (t >> 1);
                mt[nt] = 0.f;
                iv[nt] = 0.f;
                if (b < NB) {
                    // sum_j m_j XS_j, one base-256 digit of XS at a time
                    const uint4 xa = lds128(rec + xs_off(NT) + b * 32);
                    const uint4 xb = lds128(rec + xs_off(NT) + b * 32 + 16);
                    const int t0 = dp4a_us(m_hi, xa.y, dp4a_us(m_lo, xa.x, 0));
                    const int t1 = dp4a_us(m_hi, xa.w, dp4a_us(m_lo, xa.z, 0));
                    const int t2 = dp4a_us(m_hi, xb.y, dp4a_us(m_lo, xb.x, 0));
                    const int t3 = dp4a_us(m_hi, xb.w, dp4a_us(m_lo, xb.z, 0));
                    mt[nt] = fmaf((float)t3, 16777216.0f,
                                  fmaf((float)t2, 65536.0f, fmaf((float)t1, 256.0f, (float)t0)));
                    iv[nt] = lds_f32(rec + inv_off(NT) + 4 * b);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            s += kGroups;  // kGroups < kStages: at most one wrap
            if (s >= kStages) {
                s -= kStages;
                ph ^= 1;
            }
            // recombine the digits: this thread's two columns, then across the
            // threads that hold the same sequence (butterfly: keep the owned row)
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const float f0 = fmaf((float)S[nt][1], w_hi, (float)S[nt][0] * w_lo);
                const float f1 = fmaf((float)S[nt][3], w_hi, (float)S[nt][2] * w_lo);
                float v = ((t & 1) ? f1 : f0) + __shfl_xor_sync(0xffffffffu, (t & 1) ? f0 : f1, 1);
                if (NB == 1) v += __shfl_xor_sync(0xffffffffu, v, 2);
                acc[nt] = fmaf(fmaf(dd, v, kMin * dmin * mt[nt]), iv[nt], acc[nt]);
            }
        }
        n += seg;
        if (kGroups > 1) {
            // group 1's partial sums of the tile's rows go to group 0 (two
            // buffers by segment parity: a buffer is rewritten only after the
            // barrier of the next segment, which group 0 reaches once it has
            // read it)
            float* xb = xg + ((segi & 1) * kCons * 32 + cw * 32 + lane) * NT;
            if (cg == 1) {
#pragma unroll
                for (int nt = 0; nt < NT; nt++) xb[nt] = acc[nt];
            }
            asm volatile("bar.sync 2, %0;" ::"n"(kGroups * kCons * 32) : "memory");
            if (cg == 1) {
                et++;
                eu = 0;
                segi++;
                continue;
            }
#pragma unroll
            for (int nt = 0; nt < NT; nt++) acc[nt] += xb[nt];
        }
        const bool head_cut = (et == tile0) && (u0 != 0);
        const bool tail_cut = eu + seg != a.units;
        if constexpr (G::kPair != 0) {
            if (pair) {
                cluster_finish<NB>(a, r_own, t, et, acc, seq, pbar, pbuf);
                et++;
                eu = 0;
                segi++;
                continue;
            }
        }
        finish_subtile<NB>(a, r_own, t, cw, et, cta, C, total, head_cut || tail_cut, et == tile0 ? 0 : 1,
                           acc, seq);
        et++;
        eu = 0;
        segi++;
    }
    if (a.xo.size > 1 && !a.xo.ll) {
        // gather: once every CTA's peer stores are visible system-wide, the
        // last CTA raises this rank's flag on every rank
        // (the barrier orders every consumer's peer stores before thread 0's
        // system-scope release fence, which then covers them all; an
        // acquire-release fence is enough here and costs less than a
        // sequentially consistent one)
        asm volatile("bar.sync 1, %0;" ::"n"(kGroups * kCons * 32) : "memory");
        if (threadIdx.x == 0) {
            asm volatile("fence.acq_rel.sys;" ::: "memory");
            int old;
            asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(a.xo.done) : "memory");
            if (old == (int)gridDim.x - 1) {
                *a.xo.done = 0;
                asm volatile("fence.acq_rel.sys;" ::: "memory");
#pragma unroll
                for (int p = 0; p < kMaxTp; p++)
                    if (p < a.xo.size)
                        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.xo.flag[p]), "r"(seq) : "memory");
            }
        }
    }
}

// ---- host ---------------------------------------------------------------------------

// Grid-sizing knobs.  Builds with -DCHATNET_TUNING read three environment
// overrides for grid experiments (CHATNET_GEMV_CTAS: a fixed grid;
// CHATNET_GEMV_TILE_CAP: most CTAs sharing a tile; CHATNET_GEMV_MIN_UNITS:
// fewest units per CTA); product builds use the measured defaults.
#ifdef CHATNET_TUNING
static int env_int(const char* name, int fallback) {
    const char* e = getenv(name);
    return e ? atoi(e) : fallback;
}
#endif

// Fewest units a CTA should get (2): small GEMVs then use fewer, longer-running CTAs.
static int min_units_per_cta() {
#ifdef CHATNET_TUNING
    static const int v = env_int("CHATNET_GEMV_MIN_UNITS", 2) < 1 ? 1 : env_int("CHATNET_GEMV_MIN_UNITS", 2);
    return v;
#else
    return 2;
#endif
}

// A fixed most-CTAs-per-tile override (tuning builds), or -1.
static int tile_cap_env() {
#ifdef CHATNET_TUNING
    static const int v = getenv("CHATNET_GEMV_TILE_CAP") ? (env_int("CHATNET_GEMV_TILE_CAP", 1) < 1
                                                                ? 1 : env_int("CHATNET_GEMV_TILE_CAP", 1))
                                                          : -1;
    return v;
#else
    return -1;
#endif
}

// Most CTAs that share one tile for batches of two n-tiles or more: 7, but 1
// when a row has at most 16 units, where the split-K fix-up of a shared tile
// costs more than its extra parallelism saves.
static int tile_share_cap(int units) {
    const int v = tile_cap_env();
    if (v > 0) return v;
    return units <= 16 ? 1 : 7;
}

// Most units per CTA for the two-consumer-group form: 128 (tuning builds:
// CHATNET_GEMV_GROUPED_UNITS).  Measured on B200, Llama-2-70B decode step at
// batch 1 (three interleaved runs each): 9.957 ms per step with the groups
// only up to 16 units per CTA, 9.845 ms up to 32 (the q/k/v launch grouped
// too), 9.848 ms up to 128 (every launch of the step grouped), and the
// 28672 x 8192 GEMV alone 27.6 us -> 27.1 us.
static int grouped_units() {
#ifdef CHATNET_TUNING
    static const int v = env_int("CHATNET_GEMV_GROUPED_UNITS", 128);
    return v;
#else
    return 128;
#endif
}

int gemv_i8_ctas(int sms, int tiles, int units, int batch) {
    const int per_sm = i8::n_tiles(batch) == 1 ? i8::Geo<1>::kCtasPerSm : i8::Geo<8>::kCtasPerSm;
#ifdef CHATNET_TUNING
    if (const int v = env_int("CHATNET_GEMV_CTAS", 0); v > 0)  // experiments: a fixed grid
        return v < per_sm * sms ? v : per_sm * sms;
#endif
    const int64_t total = (int64_t)tiles * units;
    // One n-tile of activation digits (batch 1, 2): at most one CTA per SM,
    // which then runs the deep pipeline (gemv_i8_run_group).  With at least
    // as many tiles as SMs, one CTA per SM splits the units evenly; with
    // fewer, s CTAs per tile: the largest s <= 7 with tiles * s <= sms, and
    // for rows of at most 16 units also s <= 4 with at least two units per
    // CTA (such a grid runs as cluster splits, whose fix-up is cheap; the
    // global one cost more than the split saved there).  Measured on B200
    // (prep + GEMV replayed from a graph, batch 1, us), this grid against 444
    // three-stage CTAs: 57344x8192 50.6 vs 54.5, 10240x8192 15.6 vs 20.8,
    // 8192x28672 29.3 vs 39.6, 8192x3584 9.2 vs 19.7, 8192x1024 5.4 vs 9.0.
    if (i8::n_tiles(batch) == 1 && tile_cap_env() < 0) {
        if (tiles >= sms) return sms;
        int sh = sms / tiles;
        if (units <= 16) {
            if (sh > units / 2) sh = units / 2;
            if (sh > 4) sh = 4;
        }
        sh = sh < 1 ? 1 : sh > 7 ? 7 : sh;
        if (sh > units) sh = units;
        return tiles * sh;
    }
    // Four or more n-tiles (batch 7-16): one CTA per SM as well, the deep
    // pipeline.  Measured on B200, Llama-2-70B decode step: batch 8 19.76 ->
    // 18.37 ms, batch 16 35.21 -> 30.93 ms against two three-stage CTAs per
    // SM; batch 4 unchanged (12.85 / 12.76 ms), so it keeps the shared grid.
    if (i8::n_tiles(batch) >= 4 && tile_cap_env() < 0) return total < sms ? (int)total : sms;
    // otherwise every resident CTA, each at least min_units_per_cta() units
    // (but at least one CTA per SM); at most tile_share_cap() CTAs per tile
    int64_t want = total / min_units_per_cta();
    if (want < sms) want = total / 2 < sms ? total / 2 : sms;
    if (want < 1) want = 1;
    const int64_t cap = (int64_t)tiles * tile_share_cap(units);
    if (want > cap) want = cap;
    return per_sm * sms < want ? per_sm * sms : (int)want;
}

size_t gemv_i8_xbytes(int64_t cols, int batch) {
    return (size_t)(cols / 256) * i8::rec_bytes(i8::n_tiles(batch));
}
size_t gemv_i8_partial_bytes(int ctas) { return (size_t)2 * ctas * i8::kRows * i8::kMaxNB * sizeof(float); }

static int g_sms[64] = {0};

// How many clusters of `cs` CTAs of a deep batch-1/2 instantiation fit on
// the device at once (0 if the query fails); read once per device, form and
// size.
template <int NB, int DEEP>
static int cluster_fit(int dev, int cs) {
    static std::mutex mu;
    static int n[64][i8::kMaxCluster + 1];
    static bool have[64][i8::kMaxCluster + 1] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (have[dev & 63][cs]) return n[dev & 63][cs];
    using G = i8::Geo<NB, DEEP>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs * g_sms[dev & 63]);
    cfg.blockDim = dim3(G::kThreads);
    cfg.dynamicSmemBytes = G::kSmem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)cs;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, gemv_i8_q4k_kernel<NB, DEEP>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        c = 0;
    }
    n[dev & 63][cs] = c;
    have[dev & 63][cs] = true;
    return c;
}

int gemv_i8_prepare() {
    static std::mutex mu;  // callers may be several host threads (the no-alloc entry point has no context)
    static bool done[64] = {false};
    int dev = 0;
    CN_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if (done[dev & 63]) return CN_OK;
#define CN_ATTR(NB)                                                                                   \
    CN_CUDA(cudaFuncSetAttribute(gemv_i8_q4k_kernel<NB, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                                 i8::Geo<NB, 0>::kSmem));                                                 \
    CN_CUDA(cudaFuncSetAttribute(gemv_i8_q4k_kernel<NB, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                                 i8::Geo<NB, 1>::kSmem));
    CN_ATTR(1) CN_ATTR(2) CN_ATTR(3) CN_ATTR(4) CN_ATTR(5) CN_ATTR(6) CN_ATTR(7) CN_ATTR(8) CN_ATTR(16)
#undef CN_ATTR
    CN_CUDA(cudaFuncSetAttribute(gemv_i8_q4k_kernel<1, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 i8::Geo<1, 2>::kSmem));
    CN_CUDA(cudaFuncSetAttribute(gemv_i8_q4k_kernel<2, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 i8::Geo<2, 2>::kSmem));
    CN_CUDA(cudaDeviceGetAttribute(&g_sms[dev & 63], cudaDevAttrMultiProcessorCount, dev));
    done[dev & 63] = true;
    return CN_OK;
}

int gemv_i8_run_group(cudaStream_t st, uint32_t* err, int nmat, const CUtensorMap* const* maps,
                      const int64_t* rows, int64_t cols, int batch, int ctas, const uint8_t* xrec,
                      float* partials, int* counters, float* const* y, const XchgOut* xo) {
    CN_CHECK(batch >= 1 && batch <= i8::kMaxNB && cols % 256 == 0 && ctas > 0 && nmat >= 1 &&
                 nmat <= i8::kMaxMats,
             CN_ERR_INVALID_ARG, "integer GEMV: bad shape");
    CN_CHECK(!xo || xo->size <= 1 || (nmat == 1 && xo->size <= kMaxTp && (xo->ll || xo->done) && xo->seq_base),
             CN_ERR_INVALID_ARG, "integer GEMV: bad exchange");
    int rc = gemv_i8_prepare();
    if (rc) return rc;
    i8::Maps mp;
    i8::Args a;
    a.units = (int)(cols / 256);
    a.batch = batch;
    a.nmat = nmat;
    int tiles = 0;
    for (int m = 0; m < i8::kMaxMats; m++) {
        const int mm = m < nmat ? m : nmat - 1;
        mp.m[m] = *maps[mm];
        a.rows[m] = rows[mm];
        a.y[m] = y[mm];
        a.toff[m] = tiles;
        if (m < nmat) tiles += (int)((rows[m] + i8::kRows - 1) / i8::kRows);
    }
    a.toff[i8::kMaxMats] = tiles;
    a.tiles = tiles;
    a.xrec = xrec;
    a.partials = partials;
    a.counters = counters;
    a.err = err;
    if (xo) a.xo = *xo;
    int dev = 0;
    CN_CUDA(cudaGetDevice(&dev));
    const bool deep = ctas <= g_sms[dev & 63];  // one CTA per SM: the deep pipeline
    // batch 1-2, up to grouped_units() units per CTA: the deep pipeline with two consumer groups
    const bool grouped = deep && batch <= 2 && (int64_t)tiles * a.units <= (int64_t)grouped_units() * ctas;
    // the same number (2..8) of CTAs on every tile at batch 1-2, every
    // cluster resident at once: cluster splits
    a.csize = 0;
    const int cs = ctas % tiles == 0 ? ctas / tiles : 0;
    if (deep && batch <= 2 && cs >= 2 && cs <= i8::kMaxCluster && cs <= a.units &&
        (!xo || xo->size <= 1 || xo->ll)) {
        const int fit = grouped ? (batch == 1 ? cluster_fit<1, 2>(dev, cs) : cluster_fit<2, 2>(dev, cs))
                                : (batch == 1 ? cluster_fit<1, 1>(dev, cs) : cluster_fit<2, 1>(dev, cs));
        a.csize = fit >= tiles ? cs : 0;
    }
    if (a.csize) {
        if (grouped && batch == 1)
            CN_CUDA(launch_cluster_k(true, cs, gemv_i8_q4k_kernel<1, 2>, dim3(ctas),
                                     dim3(i8::Geo<1, 2>::kThreads), (size_t)i8::Geo<1, 2>::kSmem, st, mp, a));
        else if (grouped)
            CN_CUDA(launch_cluster_k(true, cs, gemv_i8_q4k_kernel<2, 2>, dim3(ctas),
                                     dim3(i8::Geo<2, 2>::kThreads), (size_t)i8::Geo<2, 2>::kSmem, st, mp, a));
        else if (batch == 1)
            CN_CUDA(launch_cluster_k(true, cs, gemv_i8_q4k_kernel<1, 1>, dim3(ctas),
                                     dim3(i8::Geo<1, 1>::kThreads), (size_t)i8::Geo<1, 1>::kSmem, st, mp, a));
        else
            CN_CUDA(launch_cluster_k(true, cs, gemv_i8_q4k_kernel<2, 1>, dim3(ctas),
                                     dim3(i8::Geo<2, 1>::kThreads), (size_t)i8::Geo<2, 1>::kSmem, st, mp, a));
        CN_CUDA(cudaGetLastError());
        return CN_OK;
    }
    if (grouped) {
        if (batch == 1)
            CN_CUDA(launch_k(true, gemv_i8_q4k_kernel<1, 2>, dim3(ctas), dim3(i8::Geo<1, 2>::kThreads),
                             (size_t)i8::Geo<1, 2>::kSmem, st, mp, a));
        else
            CN_CUDA(launch_k(true, gemv_i8_q4k_kernel<2, 2>, dim3(ctas), dim3(i8::Geo<2, 2>::kThreads),
                             (size_t)i8::Geo<2, 2>::kSmem, st, mp, a));
        CN_CUDA(cudaGetLastError());
        return CN_OK;
    }
    switch (batch) {
#define CN_I8(NB)                                                                                  \
    case NB:                                                                                       \
        if (deep)                                                                                  \
            CN_CUDA(launch_k(true, gemv_i8_q4k_kernel<NB, 1>, dim3(ctas), dim3(i8::Geo<NB, 1>::kThreads), \
                             (size_t)i8::Geo<NB, 1>::kSmem, st, mp, a));                           \
        else                                                                                       \
            CN_CUDA(launch_k(true, gemv_i8_q4k_kernel<NB, 0>, dim3(ctas), dim3(i8::Geo<NB, 0>::kThreads), \
                             (size_t)i8::Geo<NB, 0>::kSmem, st, mp, a));                           \
        break;
        CN_I8(1) CN_I8(2) CN_I8(3) CN_I8(4) CN_I8(5) CN_I8(6) CN_I8(7) CN_I8(8)
        default:  // batches 9-16: the 16-sequence form
            if (deep)
                CN_CUDA(launch_k(true, gemv_i8_q4k_kernel<16, 1>, dim3(ctas), dim3(i8::Geo<16, 1>::kThreads),
                                 (size_t)i8::Geo<16, 1>::kSmem, st, mp, a));
            else
                CN_CUDA(launch_k(true, gemv_i8_q4k_kernel<16, 0>, dim3(ctas), dim3(i8::Geo<16, 0>::kThreads),
                                 (size_t)i8::Geo<16, 0>::kSmem, st, mp, a));
            break;
#undef CN_I8
    }
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

int gemv_i8_run(cudaStream_t st, uint32_t* err, const CUtensorMap* map, int64_t rows, int64_t cols,
                int batch, int ctas, const uint8_t* xrec, float* partials, int* counters, float* y,
                const XchgOut* xo) {
    return gemv_i8_run_group(st, err, 1, &map, &rows, cols, batch, ctas, xrec, partials, counters, &y, xo);
}

}  // namespace cn
