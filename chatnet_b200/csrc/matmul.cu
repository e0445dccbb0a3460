// matmul.cu -- prefill: Q4_0 dequant-matmul on the 5th-generation tensor
// cores (tcgen05, tensor memory, TMA).
//
// Y[m][n] (+)= sum_k X[m][k] * W[n][k] for M tokens in one pass: the batched
// form of TensorMath.MatVecMulQ4_0 (Tensors/TensorMath.cs:548-578) with the
// weights of DequantQ4_0.Dequantize (Tensors/Quantization/DequantQ4_0.cs:28-58),
// which ChatNet runs as M sequential matvecs (InferenceEngine.cs:235-239).
//
//  * A tile is 128 weight rows x 256 tokens.  The weights are the MMA's A
//    operand and live in tensor memory: eight decode warps in two
//    warpgroups (one weight row per thread, the thread's lane of tensor
//    memory; warpgroup g takes block g of the two Q4_0 blocks of every
//    64-position stage) read the row's raw blocks from a shared-memory ring
//    that TMA fills with 128 rows x 144 bytes (8 blocks, 4 stages) at a time,
//    expand their block to 32 fp16 values ((q - 8) exact, times d, one
//    rounding) and write them to tensor memory with tcgen05.st.  The
//    expanded weights never touch shared memory.
//  * The activations (fp16, K-major) are the B operand: TMA tiles of 256
//    tokens x 64 positions with 128-byte swizzle in a 5-stage ring.
//  * One thread issues tcgen05.mma kind::f16 (M=128, N=256, K=16; fp32
//    accumulator in tensor-memory columns 0-255), four per 64-position stage,
//    and commits each stage to the barrier that frees its A slot and B stage.
//  * The decode warps then read the accumulator back (tcgen05.ld, one weight
//    row per thread, 32 tokens per load; warpgroup g takes tokens
//    128g..128g+127) and store Y with coalesced rows, optionally adding into
//    Y (the residual stream).
//  * Up to three weight matrices with the same K share one launch (q/k/v,
//    gate/up): grid.x runs over their row tiles, grid.y over token tiles.
// Every mbarrier wait is bounded.  A thread that gives up raises the error
// word and stops waiting (its control flow stays uniform; results are
// garbage and flagged).  The CTA still waits for its own copies and MMAs
// before it frees its tensor memory.
#include "cn_common.cuh"
#include "cn_internal.h"

namespace cn {
namespace mm {

constexpr int kRows = 128;               // weight rows per tile (MMA M, tensor-memory lanes)
constexpr int kNT = 256;                 // tokens per tile (MMA N)
constexpr int kKS = 64;                  // K positions per stage (one 128-byte swizzle row)
constexpr int kStages = 5;
constexpr int kBStage = kNT * kKS * 2;   // 32 KB of activations per stage
constexpr int kRaw = 144 * kRows;        // raw Q4_0 bytes of 8 blocks x 128 rows (4 stages)
constexpr int kRawStages = 3;
constexpr int kRawOff = kStages * kBStage;
constexpr int kACols = kKS / 2;          // tensor-memory columns of one A stage (2 fp16 each)
constexpr int kACol = kNT;               // accumulator in columns [0, 256), A ring after it
constexpr int kTmemCols = 512;
constexpr int kDecode = 256;             // decode + epilogue threads: warps 0-7
constexpr int kThreads = kDecode + 64;   // warp 8 TMA, warp 9 MMA
constexpr int kWarpTma = 8, kWarpMma = 9;
constexpr int kBarOff = kRawOff + kRawStages * kRaw;
constexpr int kSmem = kBarOff + 256 + 1024;  // barriers, and slack to align the ring to 1 KB
constexpr int kMaxMats = 3;
static_assert(kACol + kStages * kACols <= kTmemCols, "tensor memory plan");
static_assert(kRawOff % 1024 == 0 && kRaw % 128 == 0 && kBarOff % 8 == 0, "ring alignment");

// TMA descriptors: the activations and each weight matrix (8-byte elements,
// rows x row bytes, boxes of 144 bytes x 128 rows, as for the decode GEMV).
struct Maps {
    CUtensorMap x;
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
    int64_t rb;                 // bytes per weight row (K / 32 * 18)
    int M, K;                   // K % 256 == 0
    int accumulate;             // 1: Y += result, 0: Y = result
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

// Expands one Q4_0 block into 32 fp16 weights in K order, two per word: o[c]
// holds positions 2c (low half) and 2c + 1.  wd holds the five 4-byte words
// the block touches in a pair of blocks (36 bytes, 4-byte aligned): for
// BLK 0 bytes 0-19 (d at 0-1, quants at 2-17), for BLK 1 bytes 16-35 (d at
// 18-19, quants at 20-35).  Position j < 16 of a block is the low nibble of
// quant byte j, position 16 + j its high nibble; the value is
// fp16((q - 8) * d).
template <int BLK>
__device__ __forceinline__ void expand_q4_0(const uint32_t (&wd)[5], uint32_t (&o)[16]) {
    constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024 in both halves
    constexpr uint32_t kBias = 0x64086408u;   // fp16 1032 = 1024 + 8
    uint32_t q[4], d;
    if (BLK == 0) {
        d = wd[0] & 0xFFFFu;
#pragma unroll
        for (int i = 0; i < 4; i++) q[i] = __funnelshift_r(wd[i], wd[i + 1], 16);
    } else {
        d = wd[0] >> 16;
#pragma unroll
        for (int i = 0; i < 4; i++) q[i] = wd[1 + i];
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
            o[2 * i + h] = h2_mul(h2_sub(lo, kBias), d2);                  // (q - 8) exact, then * d
            o[8 + 2 * i + h] = h2_mul(h2_sub(hi, kBias), d2);
        }
    }
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15])
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

__global__ void __launch_bounds__(mm::kThreads, 1)
    matmul_q4_0_kernel(const __grid_constant__ mm::Maps maps, const mm::Args a) {
    using namespace mm;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* full_b = reinterpret_cast<uint64_t*>(smem + kBarOff);
    uint64_t* full_a = full_b + kStages;
    uint64_t* empty = full_a + kStages;
    uint64_t* dfull = empty + kStages;
    uint64_t* raw_full = dfull + 1;
    uint64_t* raw_empty = raw_full + kRawStages;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(raw_empty + kRawStages);
    const uint8_t* raw = smem + kRawOff;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x;
    const int m = a.nmat > 2 && tile >= a.toff[2] ? 2 : (a.nmat > 1 && tile >= a.toff[1] ? 1 : 0);
    const int64_t row0 = (int64_t)(tile - (m == 2 ? a.toff[2] : m == 1 ? a.toff[1] : 0)) * kRows;
    const int tok0 = blockIdx.y * kNT;
    const int nst = a.K / kKS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full_b[s], 1);
            mbar_init(&full_a[s], kDecode);
            mbar_init(&empty[s], 1);
        }
        mbar_init(dfull, 1);
        for (int s = 0; s < kRawStages; s++) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], kDecode);
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
            const CUtensorMap* wmap = m == 2 ? &maps.w[2] : m == 1 ? &maps.w[1] : &maps.w[0];
            const int nch = nst / 4;
            // the weights depend on no earlier kernel: the first runs go out
            // before the wait for the activations
            const int pre = nch < kRawStages ? nch : kRawStages;
            for (int c = 0; c < pre; c++) {
                mbar_expect_tx(&raw_full[c], kRaw);
                tma_load_2d(smem + kRawOff + c * kRaw, wmap, 18 * c, (int)row0, &raw_full[c]);
            }
            pdl_wait();  // X is the previous kernel's output
            int issued = 0, raw_issued = pre;
            for (int s = 0; s < nst; s++) {
                const int c = s / 4;
                if ((s & 3) == 0 && c >= kRawStages) {
                    // run c reuses the slot of run c - kRawStages once every decode thread left it
                    const int rs = c % kRawStages;
                    if (!mbar_wait(&raw_empty[rs], (uint32_t)((c / kRawStages) - 1) & 1)) {
                        atomicOr(a.err, kErrTimeout);
                        break;
                    }
                    mbar_expect_tx(&raw_full[rs], kRaw);
                    tma_load_2d(smem + kRawOff + rs * kRaw, wmap, 18 * c, (int)row0, &raw_full[rs]);
                    raw_issued = c + 1;
                }
                const int slot = s % kStages;
                if (s >= kStages && !mbar_wait(&empty[slot], (uint32_t)((s / kStages) - 1) & 1)) {
                    atomicOr(a.err, kErrTimeout);
                    break;
                }
                mbar_expect_tx(&full_b[slot], kBStage);
                tma_load_2d(smem + slot * kBStage, &maps.x, s * kKS, tok0, &full_b[slot]);
                issued = s + 1;
            }
            // no copy may still be landing when the CTA exits
            for (int s = issued - kStages < 0 ? 0 : issued - kStages; s < issued; s++)
                mbar_wait(&full_b[s % kStages], (uint32_t)(s / kStages) & 1);
            for (int c = raw_issued - kRawStages < 0 ? 0 : raw_issued - kRawStages; c < raw_issued; c++)
                mbar_wait(&raw_full[c % kRawStages], (uint32_t)(c / kRawStages) & 1);
        }
    } else if (warp == kWarpMma) {
        // ---- MMA issuer ----
        if (lane == 0) {
            for (int s = 0; s < nst; s++) {
                const int slot = s % kStages;
                const uint32_t ph = (uint32_t)(s / kStages) & 1;
                if (!mbar_wait(&full_b[slot], ph) || !mbar_wait(&full_a[slot], ph)) {
                    atomicOr(a.err, kErrTimeout);
                    break;
                }
                tc_fence_after();
                const uint32_t b0 = smem_u32(smem + slot * kBStage);
#pragma unroll
                for (int kk = 0; kk < kKS / 16; kk++)
                    mma_f16(tmem, tmem + kACol + slot * kACols + 8 * kk, desc_sw128(b0 + 32 * kk),
                            (s | kk) != 0);
                mma_commit(&empty[slot]);
            }
            mma_commit(dfull);  // completes once every MMA issued above has
        }
    } else {
        // ---- weight decode into tensor memory, then the epilogue ----
        const int r = threadIdx.x & (kRows - 1);  // tile row == tensor-memory lane
        const int wg = threadIdx.x >> 7;          // which block of each stage, which token half
        const int64_t row = row0 + r;
        const int64_t nrows = pick(a.rows, m);
        const bool live = row < nrows;  // rows past the matrix arrive as zeros (TMA fill)
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const int nch = nst / 4;  // 144-byte runs of 8 blocks (256 positions, 4 stages)
        bool failed = false;
        for (int c = 0; c < nch; c++) {
            const int rs = c % kRawStages;
            if (!failed && !mbar_wait(&raw_full[rs], (uint32_t)(c / kRawStages) & 1)) {
                atomicOr(a.err, kErrTimeout);
                failed = true;
            }
            // this thread's words of its row: block wg of stage q = words
            // 9q + 4wg .. 9q + 4wg + 4 of the row's 36
            const uint32_t* src = reinterpret_cast<const uint32_t*>(raw + rs * kRaw + r * 144) + 4 * wg;
            uint32_t cur[20];
#pragma unroll
            for (int q = 0; q < 4; q++)
#pragma unroll
                for (int k = 0; k < 5; k++) cur[5 * q + k] = src[9 * q + k];
            mbar_arrive(&raw_empty[rs]);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int s = 4 * c + q, slot = s % kStages;
                if (s >= kStages && !failed &&
                    !mbar_wait(&empty[slot], (uint32_t)((s / kStages) - 1) & 1)) {
                    atomicOr(a.err, kErrTimeout);
                    failed = true;
                }
                tc_fence_after();
                uint32_t wd[5], o[16];
#pragma unroll
                for (int k = 0; k < 5; k++) wd[k] = cur[5 * q + k];
                if (wg == 0)
                    expand_q4_0<0>(wd, o);
                else
                    expand_q4_0<1>(wd, o);
                tmem_st16(lane_base + kACol + slot * kACols + 16 * wg, o);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                mbar_arrive(&full_a[slot]);
            }
        }

        // epilogue: accumulator row r, 32 tokens per tensor-memory load
        if (!failed && !mbar_wait(dfull, 0)) {
            atomicOr(a.err, kErrTimeout);
            failed = true;
        }
        tc_fence_after();
        pdl_wait();  // Y may be the previous kernel's data
        float* y = pick(a.y, m);
        const int64_t ldy = pick(a.ldy, m);
#pragma unroll 1
        for (int jj = 0; jj < kNT / 64; jj++) {
            const int j = (kNT / 64) * wg + jj;  // this warpgroup's half of the tokens
            uint32_t v[32];
            tmem_ld32(lane_base + 32 * j, v);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (live) {
                float* p = y + (size_t)(tok0 + 32 * j) * ldy + row;
                const int nt = a.M - (tok0 + 32 * j);  // tokens of this chunk inside M
                if (a.accumulate) {
                    // 16 loads in flight before the first store
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        float old[16];
#pragma unroll
                        for (int t = 0; t < 16; t++) old[t] = 16 * h + t < nt ? p[(size_t)(16 * h + t) * ldy] : 0.f;
#pragma unroll
                        for (int t = 0; t < 16; t++)
                            if (16 * h + t < nt) p[(size_t)(16 * h + t) * ldy] = old[t] + __uint_as_float(v[16 * h + t]);
                    }
                } else {
#pragma unroll
                    for (int t = 0; t < 32; t++)
                        if (t < nt) p[(size_t)t * ldy] = __uint_as_float(v[t]);
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

// fp32 -> fp16 rows (the activation operand of the matmul).
__global__ void to_half_kernel(const float* __restrict__ x, __half* __restrict__ y, int64_t n4) {
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float4 v = reinterpret_cast<const float4*>(x)[i];
        uint2 o;
        o.x = pack_half2(v.x, v.y);
        o.y = pack_half2(v.z, v.w);
        reinterpret_cast<uint2*>(y)[i] = o;
    }
}

// ---- host side ------------------------------------------------------------------

int encode_act_map(const __half* x, int M, int64_t K, CUtensorMap* out) {
    CN_CHECK(K % mm::kKS == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && M >= 1,
             CN_ERR_UNSUPPORTED, "activation layout not TMA-tileable");
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {(cuuint32_t)mm::kKS, (cuuint32_t)mm::kNT};
    return encode_tiled_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, const_cast<__half*>(x), dims, strides,
                           box, CU_TENSOR_MAP_SWIZZLE_128B, out);
}

int to_half(cudaStream_t st, const float* x, __half* y, int64_t n) {
    CN_CHECK(n % 4 == 0, CN_ERR_INVALID_ARG, "fp16 conversion needs a multiple of 4 values");
    const int64_t n4 = n / 4;
    const int blocks = (int)((n4 + 255) / 256 < 4096 ? (n4 + 255) / 256 : 4096);
    CN_CUDA(launch_k(false, to_half_kernel, dim3(blocks > 0 ? blocks : 1), dim3(256), 0, st, x, y, n4));
    return CN_OK;
}

int matmul_q4_0(cudaStream_t st, uint32_t* err, int nmat, const void* const* w, const CUtensorMap* const* wmaps,
                const int64_t* rows, int64_t K, const __half* x, int M, float* const* y, const int64_t* ldy,
                bool accumulate) {
    CN_CHECK(nmat >= 1 && nmat <= mm::kMaxMats && K > 0 && K % 256 == 0 && M >= 1, CN_ERR_INVALID_ARG,
             "matmul: bad shape (nmat %d, K %lld, M %d)", nmat, (long long)K, M);
    static bool attr = false;
    if (!attr) {
        CN_CUDA(cudaFuncSetAttribute(matmul_q4_0_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     mm::kSmem));
        attr = true;
    }
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
            int rc = encode_weight_map(CN_TYPE_Q4_0, w[mi], rows[mi], (uint64_t)(K / 32 * 18), &maps.w[i]);
            if (rc) return rc;
        }
        a.rows[i] = rows[mi];
        a.y[i] = y[mi];
        a.ldy[i] = ldy[mi];
        CN_CHECK(w[mi] && y[mi] && rows[mi] > 0 && ldy[mi] >= rows[mi], CN_ERR_INVALID_ARG,
                 "matmul: bad matrix %d", mi);
        CN_CHECK((reinterpret_cast<uintptr_t>(w[mi]) & 15) == 0, CN_ERR_UNSUPPORTED,
                 "matmul: weights not 16-byte aligned");
        if (i < nmat) tiles += (int)((rows[i] + mm::kRows - 1) / mm::kRows);
    }
    a.toff[nmat] = tiles;
    a.rb = K / 32 * 18;
    a.M = M;
    a.K = (int)K;
    a.accumulate = accumulate ? 1 : 0;
    a.err = err;
    int rc = encode_act_map(x, M, K, &maps.x);
    if (rc) return rc;
    const dim3 grid(tiles, (M + mm::kNT - 1) / mm::kNT);
    CN_CUDA(launch_k(false, matmul_q4_0_kernel, grid, dim3(mm::kThreads), (size_t)mm::kSmem, st, maps, a));
    return CN_OK;
}

}  // namespace cn
