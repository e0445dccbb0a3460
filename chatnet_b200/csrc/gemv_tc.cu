// gemv_tc.cu -- Q4_K dequant-GEMV on the 5th-generation tensor cores
// (tcgen05, tensor memory), decode batch 1..5.
//
// Same contract as the mma.sync GEMV in gemv.cu (TensorMath.MatVecMulGeneric
// with DequantQ4K.DotProduct, Tensors/TensorMath.cs:624-656,
// DequantQ4K.cs:89-163), different machine:
//
//  * A producer warp streams [128 rows x one 144-byte super-block] of raw
//    blocks per unit into one shared-memory ring (2-D TMA) and the unit's
//    activation record (gemv_tc.cuh) into another (bulk copy).
//  * Four decode warps own one weight row per thread.  A thread unpacks its
//    row's 128 quant bytes into 256 u8 values q (one AND, or shift and AND,
//    per 4 values) and writes them straight into tensor memory with
//    tcgen05.st: the A operand of the MMA, with no shared-memory round trip
//    for the expanded weights.  It parks the row's 16-byte block header for
//    the epilogue.
//  * One thread issues, per sub-block j of 32 positions, one tcgen05.mma
//    kind::i8 (u8 x s8 -> s32, M=128, N=16, K=32, A from tensor memory, B
//    from shared memory).  Up to five sub-blocks share one 16-column
//    accumulator through block-diagonal B tiles, so a unit needs only 32
//    accumulator columns at batch 1.
//  * Activations enter as exact integers X (|X| <= 2^22, three balanced
//    base-256 digit columns per sequence), so every sub-block sum
//    D_j = sum_i q_i X_i is exact.  Four epilogue warps (again one row per
//    thread) finish each unit: sum_j sc_j * D_j in int32 per digit,
//    recombined in int64, then d * that - dmin * sum_j m_j * sum_i X_i
//    (int64), times 2^-e.
//  * Tensor memory holds up to five units in flight (A and D per slot), so
//    decode, MMA and epilogue of different units overlap and the MMA round
//    trip is hidden.
//  * Work is split stream-K over (128-row tile, unit), one CTA per SM, with
//    the deterministic fix-up of shared tiles that gemv.cu uses.
// Every mbarrier wait is bounded.  A thread that gives up raises the error
// word and runs on without waiting (control flow stays uniform, the results
// are garbage and flagged); the CTA still waits for its own copies and MMAs
// and frees its tensor memory.
#include <mutex>

#include "cn_common.cuh"
#include "cn_internal.h"
#include "gemv_tc.cuh"

namespace cn {

namespace tc {

constexpr int kRaw = 144 * kRows;  // raw Q4_K bytes per unit per tile
constexpr int kRawStages = 9;
constexpr int kRec = (kXReg + 127) / 128 * 128;  // activation record slot
constexpr int kRecStages = 8;
constexpr int kHdr = kRows * 16;  // parked block headers of one unit
constexpr int kMaxSlots = 5;      // units in flight in tensor memory
constexpr int kThreads = 320;     // warps 0-3 decode, 4-7 epilogue, 8 producer, 9 MMA
constexpr int kTmemCols = 512;
constexpr int kRecOff = kRawStages * kRaw;
constexpr int kHdrOff = kRecOff + kRecStages * kRec;
constexpr int kBarOff = kHdrOff + kMaxSlots * kHdr;
constexpr int kSmem = kBarOff + 512;
static_assert(kRaw % 128 == 0 && kRec % 128 == 0 && kHdrOff % 16 == 0, "ring alignment");
static_assert(kSmem <= 227 * 1024, "shared memory");

// Tensor-memory plan for NB sequences: P sub-blocks per 16-column
// accumulator group, G groups (DC columns) per unit, K unit slots of
// 64 A columns + DC D columns.
template <int NB>
struct Plan {
    static constexpr int P = group_subblocks(NB);
    static constexpr int G = (8 + P - 1) / P;
    static constexpr int DC = 16 * G;
    static constexpr int K = kTmemCols / (64 + DC) < kMaxSlots ? kTmemCols / (64 + DC) : kMaxSlots;
    static constexpr int Acol(int k) { return 64 * k; }
    static constexpr int Dcol(int k) { return 64 * K + DC * k; }
    // first D column of sub-block j's sequence b
    static constexpr int col(int j, int b) { return 16 * (j / P) + 3 * NB * (j % P) + 3 * b; }
};
static_assert(Plan<1>::K == 5 && Plan<2>::K == 4 && Plan<5>::K == 2, "tensor memory plan");
static_assert(Plan<1>::Dcol(Plan<1>::K) <= kTmemCols && Plan<2>::Dcol(Plan<2>::K) <= kTmemCols &&
                  Plan<3>::Dcol(Plan<3>::K) <= kTmemCols, "tensor memory plan");

// kind::i8 instruction descriptor: D s32 (bits 4-5 = 2), A u8 (bits 7-9 = 0),
// B s8 (bits 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdesc =
    (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(kN >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
        : "memory");
}

// 32 consecutive 32-bit columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* v) {
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

__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem d] (+)= A[tmem a] x B[smem desc]^T; accumulate != 0 adds to old D.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}


__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory descriptor of one sub-block's B tile: K-major, no swizzle,
// core matrices of 8 rows x 16 bytes, the two 16-byte k-chunks 128 bytes
// apart (leading byte offset), the two 8-column groups 256 bytes apart
// (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t b_desc(const void* tile) {
    const uint64_t start = (smem_u32(tile) >> 4) & 0x3FFF;
    return start | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) | (1ull << 46);
}

struct Args {
    int64_t rows;
    int units, tiles, batch;
    const uint8_t* xdig;  // [unit][kXReg]
    float* y;             // [batch][rows]
    float* partials;      // [2 * ctas][128][8]
    int* counters;        // [tiles], zero on entry, left zero
    uint32_t* err;
};

__device__ __forceinline__ int64_t range_start(int64_t total, int c, int C) { return total * c / C; }
__device__ __forceinline__ int owner_of(int64_t v, int64_t total, int C) {
    int c = (int)((v * C) / total);
    while (c + 1 < C && range_start(total, c + 1, C) <= v) c++;
    while (c > 0 && range_start(total, c, C) > v) c--;
    return c;
}

__device__ __forceinline__ void bar_compute() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Stores a finished tile's rows, or, for a tile several CTAs share, parks
// this CTA's partial sums and lets the last arriving CTA add all partials in
// CTA order (deterministic).  Called by all 128 epilogue threads together
// (r = the thread's row in the tile).
template <int NB>
__device__ void finish_tile(const Args& a, int r, int tile, int cta, int C, int64_t total,
                            bool shared_tile, int my_slot, const float (&acc)[NB], int* bcast) {
    const int64_t row = (int64_t)tile * kRows + r;
    if (!shared_tile) {
        if (row < a.rows) {
#pragma unroll
            for (int b = 0; b < NB; b++) a.y[(size_t)b * a.rows + row] = acc[b];
        }
        return;
    }
    float* p = a.partials + ((size_t)(2 * cta + my_slot) * kRows + r) * 8;
#pragma unroll
    for (int b = 0; b < NB; b++) p[b] = acc[b];
    __threadfence();
    bar_compute();
    const int c_first = owner_of((int64_t)tile * a.units, total, C);
    const int c_last = owner_of((int64_t)(tile + 1) * a.units - 1, total, C);
    if (r == 0) *bcast = atomicAdd(&a.counters[tile], 1);
    bar_compute();
    if (*bcast != c_last - c_first) return;
    __threadfence();
    float s[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) s[b] = 0.f;
    // contributor c's partial sits in slot 2c, c_first's in 2c + 1 when its
    // range began in an earlier tile; four contributors' loads go out
    // together, the sums run in CTA order
    const int first_slot = 2 * c_first + (range_start(total, c_first, C) < (int64_t)tile * a.units ? 1 : 0);
    for (int c0 = c_first; c0 <= c_last; c0 += 4) {
        float v[4][NB];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int slot = c0 + k == c_first ? first_slot : 2 * (c0 + k);
            const float* q = a.partials + ((size_t)slot * kRows + r) * 8;
#pragma unroll
            for (int b = 0; b < NB; b++) v[k][b] = c0 + k <= c_last ? __ldcg(q + b) : 0.f;
        }
#pragma unroll
        for (int k = 0; k < 4; k++)
#pragma unroll
            for (int b = 0; b < NB; b++)
                if (c0 + k <= c_last) s[b] += v[k][b];
    }
    if (row < a.rows) {
#pragma unroll
        for (int b = 0; b < NB; b++) a.y[(size_t)b * a.rows + row] = s[b];
    }
    if (r == 0) atomicExch(&a.counters[tile], 0);
}

}  // namespace tc

template <int NB>
__global__ void __launch_bounds__(tc::kThreads, 1)
    gemv_tc_q4k_kernel(const __grid_constant__ CUtensorMap map, const tc::Args a) {
    using namespace tc;
    using PL = Plan<NB>;
    constexpr int K = PL::K;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* raw = smem;
    uint8_t* rec = smem + kRecOff;
    uint4* hdr = reinterpret_cast<uint4*>(smem + kHdrOff);
    uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem + kBarOff);
    uint64_t* raw_empty = raw_full + kRawStages;
    uint64_t* rec_full = raw_empty + kRawStages;
    uint64_t* rec_empty = rec_full + kRecStages;
    uint64_t* afull = rec_empty + kRecStages;  // [K] A and header of a slot written
    uint64_t* dfull = afull + kMaxSlots;       // [K] MMAs of a slot done
    uint64_t* sfree = dfull + kMaxSlots;       // [K] epilogue done with a slot
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sfree + kMaxSlots);
    int* bcast = reinterpret_cast<int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRawStages; s++) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], kRows);
        }
        for (int t = 0; t < kRecStages; t++) {
            mbar_init(&rec_full[t], 1);
            mbar_init(&rec_empty[t], kRows);
        }
        for (int k = 0; k < kMaxSlots; k++) {
            mbar_init(&afull[k], kRows);
            mbar_init(&dfull[k], 1);
            mbar_init(&sfree[k], kRows);
        }
        fence_mbar_init();
    }
    if (warp == 9) {
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

    const int64_t total = (int64_t)a.tiles * a.units;
    const int C = (int)(total < (int64_t)gridDim.x ? total : (int64_t)gridDim.x);
    const int cta = blockIdx.x;
    const int64_t v0 = cta < C ? range_start(total, cta, C) : 0;
    const int64_t v1 = cta < C ? range_start(total, cta + 1, C) : 0;
    const int nunits = (int)(v1 - v0);
    const int tile0 = cta < C ? (int)(v0 / a.units) : 0;
    const int u0 = cta < C ? (int)(v0 % a.units) : 0;

    if (warp == 8) {
        // ---- producer ----
        if (lane == 0) {
            int tile = tile0, u = u0, s = 0, t = 0, nraw = 0, nrec = 0;
            uint32_t ps = 0, pt = 0;
            for (int n = 0; n < nunits; n++) {
                if (n >= kRawStages && !mbar_wait(&raw_empty[s], ps ^ 1)) {
                    atomicOr(a.err, kErrTimeout);
                    break;
                }
                mbar_expect_tx(&raw_full[s], kRaw);
                tma_load_2d(raw + s * kRaw, &map, 18 * u, tile * kRows, &raw_full[s]);
                nraw = n + 1;
                if (n >= kRecStages && !mbar_wait(&rec_empty[t], pt ^ 1)) {
                    atomicOr(a.err, kErrTimeout);
                    break;
                }
                mbar_expect_tx(&rec_full[t], kXReg);
                bulk_g2s(rec + t * kRec, a.xdig + (size_t)u * kXReg, kXReg, &rec_full[t]);
                nrec = n + 1;
                if (++u == a.units) {
                    u = 0;
                    tile++;
                }
                if (++s == kRawStages) {
                    s = 0;
                    ps ^= 1;
                }
                if (++t == kRecStages) {
                    t = 0;
                    pt ^= 1;
                }
            }
            // no copy may still be landing when the CTA exits
            for (int n = nraw - kRawStages < 0 ? 0 : nraw - kRawStages; n < nraw; n++)
                mbar_wait(&raw_full[n % kRawStages], (uint32_t)(n / kRawStages) & 1);
            for (int n = nrec - kRecStages < 0 ? 0 : nrec - kRecStages; n < nrec; n++)
                mbar_wait(&rec_full[n % kRecStages], (uint32_t)(n / kRecStages) & 1);
        }
    } else if (warp == 9) {
        // ---- MMA issuer ----
        if (lane == 0) {
            int k = 0, t = 0, issued = 0;
            uint32_t pk = 0, pt = 0;
            for (int n = 0; n < nunits; n++) {
                if (!mbar_wait(&afull[k], pk) || !mbar_wait(&rec_full[t], pt)) {
                    atomicOr(a.err, kErrTimeout);
                    break;
                }
                tc_fence_after();
                const uint8_t* dig = rec + t * kRec;
#pragma unroll
                for (int j = 0; j < 8; j++)
                    mma_i8(tmem + PL::Dcol(k) + 16 * (j / PL::P), tmem + PL::Acol(k) + 8 * j,
                           b_desc(dig + j * 512), (uint32_t)(j % PL::P));
                mma_commit(&dfull[k]);
                issued = n + 1;
                if (++k == K) {
                    k = 0;
                    pk ^= 1;
                }
                if (++t == kRecStages) {
                    t = 0;
                    pt ^= 1;
                }
            }
            // the last commit covers every MMA issued before it
            if (issued > 0) mbar_wait(&dfull[(issued - 1) % K], (uint32_t)((issued - 1) / K) & 1);
        }
    } else if (warp < 4) {
        // ---- decode warps: thread r owns row r of each tile ----
        const int r = threadIdx.x;
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        int s = 0, k = 0;
        uint32_t ps = 0, pk = 0;
        bool ok = true;
        for (int n = 0; n < nunits; n++) {
            if (ok && !mbar_wait(&raw_full[s], ps)) ok = false;
            // slot k is free once the epilogue of unit n - K is done with it
            if (ok && n >= K && !mbar_wait(&sfree[k], pk ^ 1)) ok = false;
            if (!ok) atomicOr(a.err, kErrTimeout);
            __syncwarp();
            tc_fence_after();
            const uint4* row = reinterpret_cast<const uint4*>(raw + s * kRaw + r * 144);
            uint4 q[9];
#pragma unroll
            for (int i = 0; i < 9; i++) q[i] = row[i];
            hdr[k * kRows + r] = q[0];
            const uint32_t abase = tmem + lane_base + PL::Acol(k);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                // sub-block j: bytes 16j..16j+15 of qs; low nibbles are
                // positions 32j + 0..15, high nibbles 32j + 16..31
                const uint4 w = q[1 + j];
                uint32_t v[8];
                v[0] = w.x & 0x0F0F0F0Fu;
                v[1] = w.y & 0x0F0F0F0Fu;
                v[2] = w.z & 0x0F0F0F0Fu;
                v[3] = w.w & 0x0F0F0F0Fu;
                v[4] = (w.x >> 4) & 0x0F0F0F0Fu;
                v[5] = (w.y >> 4) & 0x0F0F0F0Fu;
                v[6] = (w.z >> 4) & 0x0F0F0F0Fu;
                v[7] = (w.w >> 4) & 0x0F0F0F0Fu;
                tmem_st8(abase + 8 * j, v);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&afull[k]);
            mbar_arrive(&raw_empty[s]);
            if (++s == kRawStages) {
                s = 0;
                ps ^= 1;
            }
            if (++k == K) {
                k = 0;
                pk ^= 1;
            }
        }
    } else {
        // ---- epilogue warps: thread r owns row r (tensor-memory lane r) ----
        const int r = threadIdx.x - 128;
        const uint32_t lane_base = (uint32_t)((warp - 4) * 32) << 16;
        float acc[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) acc[b] = 0.f;
        int k = 0, t = 0, et = tile0, eu = u0;
        uint32_t pk = 0, pt = 0;
        bool ok = true;
        for (int n = 0; n < nunits; n++) {
            if (ok && !mbar_wait(&afull[k], pk)) ok = false;
            if (ok && !mbar_wait(&rec_full[t], pt)) ok = false;
            if (ok && !mbar_wait(&dfull[k], pk)) ok = false;
            if (!ok) atomicOr(a.err, kErrTimeout);
            __syncwarp();
            tc_fence_after();
            // the unit's accumulators: DC columns in chunks of 32
            constexpr int CH = PL::DC / 32 > 0 ? PL::DC / 32 : 1;
            uint32_t dv[CH][32];
            if (CH <= 2) {
#pragma unroll
                for (int c = 0; c < CH; c++) tmem_ld32(tmem + lane_base + PL::Dcol(k) + 32 * c, dv[c]);
                tmem_wait_ld();
            }
            // block header: d, dmin, DecodeScales (DequantQ4K.cs:218-241)
            const uint4 h = hdr[k * kRows + r];
            const float d = half_bits_to_float((uint16_t)(h.x & 0xFFFF));
            const float dmin = half_bits_to_float((uint16_t)(h.x >> 16));
            const uint32_t sc_lo = h.y & 0x3F3F3F3Fu;
            const uint32_t sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
            const uint32_t m_lo = h.z & 0x3F3F3F3Fu;
            const uint32_t m_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
            const uint8_t* rc = rec + t * kRec;
            const int* xs = reinterpret_cast<const int*>(rc + kXsOff);
            const float* inv = reinterpret_cast<const float*>(rc + kInvOff);
            if (CH > 2) {
#pragma unroll
                for (int c = 0; c < 2; c++) tmem_ld32(tmem + lane_base + PL::Dcol(k) + 32 * c, dv[c]);
                tmem_wait_ld();
            }
            int S0[NB], S1[NB], S2[NB];
#pragma unroll
            for (int b = 0; b < NB; b++) S0[b] = S1[b] = S2[b] = 0;
#pragma unroll
            for (int half = 0; half < (CH > 2 ? 2 : 1); half++) {
                if (half == 1) {
#pragma unroll
                    for (int c = 2; c < CH; c++)
                        tmem_ld32(tmem + lane_base + PL::Dcol(k) + 32 * c, dv[c]);
                    tmem_wait_ld();
                }
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int c0 = PL::col(j, 0);
                    if ((CH > 2) && ((c0 / 32 >= 2) != (half == 1))) continue;
                    const int sc = (int)(((j < 4 ? sc_lo : sc_hi) >> (8 * (j & 3))) & 0xFF);
#pragma unroll
                    for (int b = 0; b < NB; b++) {
                        const int cc = PL::col(j, b);
                        S2[b] += sc * (int)dv[(cc + 0) / 32][(cc + 0) % 32];
                        S1[b] += sc * (int)dv[(cc + 1) / 32][(cc + 1) % 32];
                        S0[b] += sc * (int)dv[(cc + 2) / 32][(cc + 2) % 32];
                    }
                }
            }
#pragma unroll
            for (int b = 0; b < NB; b++) {
                long long mt = 0;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int mj = (int)(((j < 4 ? m_lo : m_hi) >> (8 * (j & 3))) & 0xFF);
                    mt += (long long)mj * xs[j * 8 + b];
                }
                const long long vi = (long long)S2[b] * 65536 + (long long)S1[b] * 256 + S0[b];
                const float tb = fmaf(d, (float)vi, -(dmin * (float)mt));
                acc[b] = fmaf(tb, inv[b], acc[b]);
            }
            tc_fence_before();
            mbar_arrive(&sfree[k]);
            mbar_arrive(&rec_empty[t]);
            if (++k == K) {
                k = 0;
                pk ^= 1;
            }
            if (++t == kRecStages) {
                t = 0;
                pt ^= 1;
            }
            // unit n ends a tile, or this CTA's range
            if (eu == a.units - 1 || n == nunits - 1) {
                const bool head_cut = (et == tile0) && (u0 != 0);
                const bool tail_cut = (n == nunits - 1) && (eu != a.units - 1);
                finish_tile<NB>(a, r, et, cta, C, total, head_cut || tail_cut, et == tile0 ? 0 : 1, acc,
                                bcast);
#pragma unroll
                for (int b = 0; b < NB; b++) acc[b] = 0.f;
            }
            if (++eu == a.units) {
                eu = 0;
                et++;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                     : "memory");
    }
}

// ---- host ---------------------------------------------------------------------------

int gemv_tc_ctas(int sms, int tiles, int units) {
    // every CTA takes at least 2 units; at most 8 CTAs share a tile (ranges
    // of at least units/7 units guarantee that)
    const int64_t total = (int64_t)tiles * units;
    int64_t want = total / 2 > 0 ? total / 2 : 1;
    const int64_t cap = (int64_t)tiles * 7;
    if (want > cap) want = cap;
    return sms < want ? sms : (int)want;
}

size_t gemv_tc_xbytes(int64_t cols) { return (size_t)(cols / 256) * tc::kXReg; }
size_t gemv_tc_partial_bytes(int ctas) { return (size_t)2 * ctas * tc::kRows * 8 * sizeof(float); }

// Sets the kernels' shared-memory limit on the current device (once per
// device; call outside any stream capture).
int gemv_tc_prepare() {
    static std::mutex mu;  // callers may be several host threads (the no-alloc entry point has no context)
    static bool done[64] = {false};
    int dev = 0;
    CN_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if (done[dev & 63]) return CN_OK;
    CN_CUDA(cudaFuncSetAttribute(gemv_tc_q4k_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kSmem));
    CN_CUDA(cudaFuncSetAttribute(gemv_tc_q4k_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kSmem));
    CN_CUDA(cudaFuncSetAttribute(gemv_tc_q4k_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kSmem));
    CN_CUDA(cudaFuncSetAttribute(gemv_tc_q4k_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kSmem));
    CN_CUDA(cudaFuncSetAttribute(gemv_tc_q4k_kernel<5>, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kSmem));
    done[dev & 63] = true;
    return CN_OK;
}

int gemv_tc_run(cudaStream_t st, uint32_t* err, const CUtensorMap* map, int64_t rows, int64_t cols,
                int batch, int ctas, const uint8_t* xdig, float* partials, int* counters, float* y) {
    CN_CHECK(batch >= 1 && batch <= tc::kMaxNB && cols % 256 == 0 && ctas > 0, CN_ERR_INVALID_ARG,
             "tensor-core GEMV: bad shape");
    int rc = gemv_tc_prepare();
    if (rc) return rc;
    tc::Args a;
    a.rows = rows;
    a.units = (int)(cols / 256);
    a.tiles = (int)((rows + tc::kRows - 1) / tc::kRows);
    a.batch = batch;
    a.xdig = xdig;
    a.y = y;
    a.partials = partials;
    a.counters = counters;
    a.err = err;
    switch (batch) {
#define CN_TC(NB) \
    case NB: gemv_tc_q4k_kernel<NB><<<ctas, tc::kThreads, tc::kSmem, st>>>(*map, a); break;
        CN_TC(1)
        CN_TC(2)
        CN_TC(3)
        CN_TC(4)
        CN_TC(5)
#undef CN_TC
    }
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

}  // namespace cn
