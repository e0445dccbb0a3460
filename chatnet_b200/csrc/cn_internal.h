// cn_internal.h -- context / tensor structs and internal launchers.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "chatnet_cuda.h"

struct cn_ctx {
    int device = 0;
    int sms = 0;
    cudaStream_t stream = nullptr;
    uint32_t* dev_err = nullptr;  // device error word (cn::kErr* bits)

    // GEMV scratch: activation fragments, per-chunk sums, split-K partials
    // and the per-tile arrival counters (self-resetting, zeroed at alloc).
    void* xfrag = nullptr;
    size_t xfrag_bytes = 0;
    float* xsum = nullptr;
    size_t xsum_bytes = 0;
    float* partials = nullptr;
    size_t partial_bytes = 0;
    int* counters = nullptr;
    size_t counter_count = 0;
    float* xinv = nullptr;
    size_t xinv_bytes = 0;

    // fp16 copy of the prefill matmul's activations
    void* xhalf = nullptr;
    size_t xhalf_bytes = 0;

    // device sampler scratch (sample.cu)
    void* samp = nullptr;
    size_t samp_bytes = 0;

    // staging for the host-pointer entry points
    void* dstage = nullptr;
    size_t dstage_bytes = 0;
    void* hstage = nullptr;  // pinned
    size_t hstage_bytes = 0;
};

// A tensor-parallel rank's exchange state (tp.cu).  `buf` (IPC-exported)
// holds [flags: kMaxTp uint32, padded to 256 B][slots: 2 parities x size ranks
// x max_batch x dim {fp32, seq} pairs][logits: max_batch x vocab fp32]; peer[p] is rank
// p's buf mapped into this process (peer[rank] == buf).
struct cn_tp {
    cn_ctx* ctx = nullptr;
    int rank = 0, size = 1, max_batch = 1;
    int64_t dim = 0, vocab = 0;
    uint8_t* buf = nullptr;
    size_t bytes = 0, slots_off = 256, logits_off = 0;
    void* peer[8] = {};
    bool connected = false;
    uint32_t* step = nullptr;  // step counter (bumped once per decode step)
    int* done = nullptr;       // GEMV completion counters [16]
};

struct cn_tensor {
    cn_ctx* ctx = nullptr;
    int type = 0;
    int64_t rows = 0, cols = 0;
    uint64_t bytes = 0, row_bytes = 0;
    void* d = nullptr;
    bool owns = true;
    bool has_map = false;
    CUtensorMap map;
    float split_scale = 0.f;  // matmul_split_scale's cached result (0: not yet computed)
};

namespace cn {

uint64_t row_bytes(int type, int64_t cols);
// The 32-weight block codecs decoded through the generic paths (formats.cuh).
__host__ __device__ inline bool is_block32(int type) {
    return type == CN_TYPE_Q4_1 || type == CN_TYPE_Q5_0 || type == CN_TYPE_Q5_1 || type == CN_TYPE_Q8_0 ||
           type == CN_TYPE_IQ4_NL;
}
__host__ __device__ inline int block32_bytes(int type) {
    return type == CN_TYPE_Q4_1 ? 20 : type == CN_TYPE_Q5_0 ? 22 : type == CN_TYPE_Q5_1 ? 24
           : type == CN_TYPE_IQ4_NL ? 18 : 34;
}
// The 256-weight super-block codecs decoded through the generic paths.
__host__ __device__ inline bool is_superblock(int type) {
    return type == CN_TYPE_Q2_K || type == CN_TYPE_Q3_K || type == CN_TYPE_Q5_K || type == CN_TYPE_Q8_K ||
           type == CN_TYPE_IQ4_XS || type == CN_TYPE_IQ2_XXS || type == CN_TYPE_IQ2_XS || type == CN_TYPE_IQ3_XXS ||
           type == CN_TYPE_IQ1_S || type == CN_TYPE_IQ3_S || type == CN_TYPE_IQ2_S || type == CN_TYPE_IQ1_M;
}
// GgufTensorInfo.ByteSize (GgufTensorInfo.cs:30-114) per 256 elements.
__host__ __device__ inline int superblock_bytes(int type) {
    switch (type) {
        case CN_TYPE_Q2_K: return 84;
        case CN_TYPE_Q3_K: return 110;
        case CN_TYPE_Q5_K: return 176;
        case CN_TYPE_Q8_K: return 292;
        case CN_TYPE_IQ2_XXS: return 66;
        case CN_TYPE_IQ2_XS: return 74;
        case CN_TYPE_IQ3_XXS: return 98;
        case CN_TYPE_IQ1_S: return 50;
        case CN_TYPE_IQ3_S: return 110;
        case CN_TYPE_IQ2_S: return 82;
        case CN_TYPE_IQ1_M: return 56;
        default: return 136;  // IQ4_XS
    }
}
bool type_supported(int type);

int ensure(void** p, size_t* have, size_t need, bool zero);

// TemperatureSampler.Sample on device logits [batch][vocab] (sample.cu).
int sample_launch(cn_ctx* ctx, const float* d_logits, int vocab, int batch, float temperature, int top_k,
                  float top_p, const float* r_host, int* tokens_host);

// Encodes the TMA descriptor a GEMV uses for a [rows][row_bytes] weight
// matrix, or returns CN_ERR_UNSUPPORTED if the layout cannot be tiled
// (row_bytes not a multiple of 16, or unaligned base).
int encode_weight_map(int type, const void* d_w, int64_t rows, uint64_t row_bytes,
                      CUtensorMap* out);

// Encodes a 2-D tiled TMA descriptor (zero fill out of bounds, no interleave).
int encode_tiled_2d(CUtensorMapDataType dt, void* base, const cuuint64_t (&dims)[2],
                    const cuuint64_t (&strides)[1], const cuuint32_t (&box)[2],
                    CUtensorMapSwizzle swz, CUtensorMap* out);

// Prefill dequant-matmul (matmul.cu): y[i][t][r] (+)= dot(W_i[r], x[t]) for
// M tokens and nmat <= 3 matrices of one weight type (Q4_0, Q4_K, or Q6_K
// with row bytes a multiple of 16) with the
// same K (K % 256 == 0); x is fp16 [M][K] (16-byte aligned), y[i] fp32
// [M][ldy[i]].  Token t's results are multiplied by xs[t] (x's inverse row
// scale) when xs is not null.  wmaps[i] may be null (the weight map is then
// encoded per call).
int matmul_quant(cudaStream_t st, uint32_t* err, int type, int nmat, const void* const* w,
                 const CUtensorMap* const* wmaps, const int64_t* rows, int64_t K, const __half* x, const float* xs,
                 int M, float* const* y, const int64_t* ldy, bool accumulate, const __half* xlo = nullptr,
                 const float* wscale = nullptr);
// Split variant of matmul_quant (xlo != null): x carries its low halves in
// xlo (fp16(x - fp16(x)), same layout), the weights are expanded at the
// powers of two wscale[i] (matmul_split_scale) as exact hi + lo fp16 pairs, and
// each k-step runs three MMAs; near-fp32 accuracy at about three times the MMA
// work.
// The power of two 2^E a tensor's weights are expanded at in the split
// variant (largest possible |weight| * 2^E <= 2^14), computed on first use
// with a reduction over its blocks' scales (synchronises the stream) and
// cached in the tensor.
int matmul_split_scale(cn_tensor* t, cudaStream_t st, float* out);
inline bool matmul_type_ok(int type) {
    return type == CN_TYPE_Q4_0 || type == CN_TYPE_Q4_K || type == CN_TYPE_Q6_K;
}
// M rows of n fp32 values -> fp16 rows scaled by a power of two each, the
// inverses in inv[M] (prefill.cu); n % 4 == 0, x and y 16-byte aligned.
int to_half_rows(cudaStream_t st, const float* x, __half* y, float* inv, int n, int M);

// Prefill kernels around the matmul (prefill.cu).  With ylo, the norm also
// writes each value's fp16 rounding residual (the split matmul's low halves).
int prefill_norm(cudaStream_t st, const float* x, const float* w, __half* y, float* inv, int n, int M,
                 float eps, __half* ylo = nullptr);
int prefill_silu(cudaStream_t st, const float* g, const float* u, __half* h, float* inv, int n, int M,
                 __half* hlo = nullptr, int gelu = 0);
// RoPE of the M prompt tokens' q (in place) and k, k/v into the cache and
// their fp16 copies into kh/vh [M][kvdim] (with kl/vl, also k's and v's fp16
// residuals).
int prefill_rope(cudaStream_t st, float* q, const float* k, const float* v, const float2* rope, int pos0, int M,
                 int qdim, int kvdim, int hd, void* kcache, void* vcache, int64_t cache_off, bool kv_f16, __half* kh,
                 __half* vh, __half* kl = nullptr, __half* vl = nullptr, int neox = 0);
// Causal prefill attention; split: q, k (and, for fp32 caches, v) as hi + lo
// fp16 pairs (kl / vl: k's and v's residuals, needed for fp32 caches), and
// the output's residuals into out_lo when given.
int prefill_attention(cudaStream_t st, const float* q, int q_stride, const void* kcache,
                      const void* vcache, bool kv_f16, int64_t cache_off, int n_heads, int n_kv,
                      int hd, int M, int pos0, const __half* kh, const __half* vh, __half* out, int out_stride,
                      bool split = false, const __half* kl = nullptr, const __half* vl = nullptr,
                      __half* out_lo = nullptr);

// Scratch requirements of one GEMV call.
struct GemvPlan {
    int nt = 1;       // n-tiles of 4 batch columns
    int tiles = 0;    // 16-row tiles
    int units = 0;    // 256-position k units
    int ctas = 0;
    bool tma = false;
    // Kernel family: kPathMma (fp16 mma.sync, gemv.cu), kPathI8 (integer
    // mma.sync, gemv_i8.cu: Q4_K at batch 1..8), kPathTc (tcgen05,
    // gemv_tc.cu: Q4_K at batch 1..5, opt-in).  The integer and tcgen05
    // paths use 128-row tiles and keep activation records in the xfrag
    // buffer (no xsum / xinv).
    int path = 0;
    size_t xfrag_bytes = 0, xsum_bytes = 0, xinv_bytes = 0, partial_bytes = 0, counters = 0;
};
enum { kPathMma = 0, kPathTc = 1, kPathI8 = 2 };
int gemv_plan(cn_ctx* ctx, int type, int64_t rows, int64_t cols, int batch, bool tma,
              GemvPlan* plan);

// A GEMV bound to one weight matrix and batch size.
struct GemvOp {
    int type = 0;
    const void* w = nullptr;
    int64_t rows = 0, cols = 0;
    uint64_t rb = 0;
    int batch = 1;
    bool tma = false;
    CUtensorMap map;
    GemvPlan plan;
};

// Scratch a GEMV reads and writes (owned by the caller; one GEMV at a time
// per set of buffers; the counters must start zeroed and are left zeroed).
struct GemvBufs {
    uint4* xfrag;
    float* xsum;
    float* partials;
    int* counters;
    float* xinv;  // [units][nt*4] per-unit 2^-e written by the prep
};

// Where and in which form a kernel that produces a GEMV's input also
// writes that input's activation record: kind -1 none, 0 fp16 fragments,
// 1 fp16 fragments + chunk sums (Q4_K), 2 tcgen05 digit records, 3 integer
// records (gemv_prep_kind).
struct PrepTarget {
    int kind = -1;
    int nt_count = 1;
    float step1 = 1.0f;
    void* xfrag = nullptr;
    float* xsum = nullptr;
    float* xinv = nullptr;
};

// Tensor-parallel exchange, producer side: a GEMV whose output is a partial
// sum (O and down split along their input) or a slice (lm_head rows) stores
// every output value into each rank's buffer over NVLink.  Two forms:
//  * ll = 1 (residual partial sums): each value travels with its use's
//    sequence number in one 8-byte store {value bits, seq}, so a consumer
//    that reads the pair sees a value exactly when its sequence number
//    matches; no fence, counter or flag.  Destination (b, row) on rank p:
//    8-byte element dst[p] + parity * parity_stride + b * dst_ld + dst_row0 + row.
//  * ll = 0 (lm_head slices): plain fp32 stores at the same index; when all
//    the GEMV's CTAs are done the last one raises its flag on every rank.
// parity = seq & 1, seq = *seq_base * uses + seq_add.
constexpr int kMaxTp = 8;
struct XchgOut {
    int size = 1, rank = 0;
    float* dst[kMaxTp] = {};
    int64_t parity_stride = 0, dst_ld = 0, dst_row0 = 0;
    uint32_t* flag[kMaxTp] = {};  // &flags[rank] on each rank
    const uint32_t* seq_base = nullptr;
    uint32_t uses = 1, seq_add = 0;
    int* done = nullptr;  // completion counter, zero on entry, left zero
    int ll = 0;
};
// Consumer side: the summed input is sum_p src[parity * parity_stride +
// p * rank_stride + ...], in 8-byte {value, seq} elements read until their
// seq matches (ll = 1), or fp32 after every flags[p] >= seq (ll = 0).
struct XchgIn {
    int size = 1;
    const float* src = nullptr;
    int64_t parity_stride = 0, rank_stride = 0;
    const uint32_t* flags = nullptr;
    const uint32_t* seq_base = nullptr;
    uint32_t uses = 1, seq_add = 0;
    uint32_t* err = nullptr;
    int ll = 0;
};

struct GemvNeeds {
    size_t xfrag_bytes = 0, xsum_bytes = 0, xinv_bytes = 0, partial_bytes = 0, counters = 0;
};

// rb: the matrix's row stride in bytes (0: packed rows, row_bytes(type, cols)).
int gemv_make(cn_ctx* ctx, int type, const void* d_w, int64_t rows, int64_t cols,
              const CUtensorMap* map, int batch, GemvOp* op, uint64_t rb = 0);
// Converts x [batch][cols] into the GEMV's activation fragments (TMA path).
int gemv_prep(cudaStream_t st, int sms, const GemvOp& op, const float* d_x, const GemvBufs& b);
// Runs the GEMV on prepped fragments (TMA path) or on x directly (generic).
int gemv_run(cn_ctx* ctx, cudaStream_t st, const GemvOp& op, const float* d_x, const GemvBufs& b,
             float* d_y, const XchgOut* xo = nullptr);
int gemv_reserve(const GemvPlan& p, GemvNeeds* n);
// RMSNorm of `rows` rows of n values into y, and, when op is a tiled GEMV,
// its activation records for op in b (one kernel).
int norm_prep(cudaStream_t st, const float* x, const float* w, float* y, int n, int rows,
              float eps, const GemvOp* op, const GemvBufs& b);
// Same after a residual add: x_out = x_in + delta (x_out must not alias
// x_in), then y = RMSNorm(x_out) * w and op's records.
int add_norm_prep(cudaStream_t st, const float* x_in, const float* delta, float* x_out, const float* w,
                  float* y, int n, int rows, float eps, const GemvOp* op, const GemvBufs& b,
                  const XchgIn* xin = nullptr);
// Waits (bounded) until every rank's flag reached this use's sequence number.
int xchg_wait(cudaStream_t st, const XchgIn& xin);
// The record target of op in b (kind -1 when op reads plain fp32).
PrepTarget prep_target(const GemvOp* op, const GemvBufs& b);
float gemv_step1_scale(int type);
// Which activation form a GEMV reads: 0 plain fragments, 1 Q4_K fragments
// (pre-scaled second k-step + chunk sums), 2 tensor-core digit records,
// 3 integer-GEMV records.
int gemv_prep_kind(const GemvOp& op);

// Kernel family the environment selects for Q4_K decode GEMVs:
// CHATNET_GEMV=i8 (default), tc or mma.
int gemv_q4k_path();

// integer mma.sync Q4_K GEMV (gemv_i8.cu)
int gemv_i8_ctas(int sms, int tiles, int units, int batch);
size_t gemv_i8_xbytes(int64_t cols, int batch);
size_t gemv_i8_partial_bytes(int ctas);
int gemv_i8_prepare();
int gemv_i8_run(cudaStream_t st, uint32_t* err, const CUtensorMap* map, int64_t rows, int64_t cols,
                int batch, int ctas, const uint8_t* xrec, float* partials, int* counters, float* y,
                const XchgOut* xo = nullptr);
int gemv_i8_run_group(cudaStream_t st, uint32_t* err, int nmat, const CUtensorMap* const* maps,
                      const int64_t* rows, int64_t cols, int batch, int ctas, const uint8_t* xrec,
                      float* partials, int* counters, float* const* y, const XchgOut* xo = nullptr);

// Several GEMVs that read the same activations (same inner dimension and
// batch and weight type, all on the integer path or all on the fp16 one)
// run as one launch: q/k/v, gate/up.
struct GemvGroup {
    int n = 0;
    GemvOp ops[3];
    GemvPlan plan;  // of the concatenated rows
};
// Fails with CN_ERR_UNSUPPORTED when the ops cannot share a launch.
int gemv_group_make(cn_ctx* ctx, const GemvOp* ops, int n, GemvGroup* g);
int gemv_group_run(cn_ctx* ctx, cudaStream_t st, const GemvGroup& g, const GemvBufs& b, float* const* y);

// tensor-core Q4_K GEMV (gemv_tc.cu)
int gemv_tc_ctas(int sms, int tiles, int units);
size_t gemv_tc_xbytes(int64_t cols);
size_t gemv_tc_partial_bytes(int ctas);
int gemv_tc_prepare();
int gemv_tc_run(cudaStream_t st, uint32_t* err, const CUtensorMap* map, int64_t rows, int64_t cols,
                int batch, int ctas, const uint8_t* xdig, float* partials, int* counters, float* y);

// Enqueues x-prep + GEMV on ctx->stream using the ctx's scratch.  `map` may
// be null (encoded on the fly when possible, else the generic kernel runs).
int gemv_launch(cn_ctx* ctx, int type, const void* d_w, int64_t rows, int64_t cols,
                const CUtensorMap* map, const float* d_x, float* d_y, int batch);
// Times `launches` GEMVs (prep + GEMV each) cycling through ws[0..n_w) from
// one CUDA graph, replayed `reps` times: us_out[r] = replay r's mean per launch.
int gemv_time(cn_ctx* ctx, const cn_tensor* const* ws, int n_w, const float* d_x, float* d_y, int batch,
              int launches, int reps, float* us_out, int* kernels_per_launch);

// tensor-parallel exchange descriptors (tp.cu); uses = exchanges per step
int tp_step_launch(const cn_tp* tp, cudaStream_t s);
XchgOut tp_reduce_out(const cn_tp* tp, uint32_t uses, uint32_t use, int done_index);
XchgIn tp_reduce_in(const cn_tp* tp, uint32_t uses, uint32_t use, uint32_t* err);
// The lm_head all-gather's completion (flags) for xchg_wait.
XchgIn tp_gather_in(const cn_tp* tp, uint32_t uses, uint32_t use, uint32_t* err);
XchgOut tp_gather_out(const cn_tp* tp, int64_t local_rows, uint32_t uses, uint32_t use, int done_index);
float* tp_logits(const cn_tp* tp);

// d_end: one past the tensor's last byte, when d_blocks starts inside a
// larger tensor (IQ3_S reads past a block; null: the range's own end).
int dequant_launch(int type, const void* d_blocks, float* d_out, int64_t n, cudaStream_t s,
                   const void* d_end = nullptr);
int synth_launch(int type, int64_t rows, int64_t cols, uint64_t seed, int dist, void* d_out,
                 cudaStream_t s);
// Region [row0, row0 + nrows) x [col0, col0 + ncols) of the rows x cols tensor
// that synth_launch would generate (columns in whole blocks).
int synth_slice_launch(int type, int64_t rows, int64_t cols, int64_t row0, int64_t nrows, int64_t col0,
                       int64_t ncols, uint64_t seed, int dist, void* d_out, cudaStream_t s);

}  // namespace cn
