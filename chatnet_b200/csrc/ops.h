// ops.h -- launchers of the decode-step kernels (ops.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cn_internal.h"

namespace cn {

struct AttnPlan {
    int splits = 0, chunk = 0;
    bool mma = false;  // tensor-core kernel (fp16 cache, kv_mul <= 8, head_dim 64 or 128)
    size_t part_floats = 0, smem = 0;
};

// RoPE and the KV-cache store done inside the tensor-core attention kernel
// (fp16 cache): q and the new k row are rotated as they are loaded, and the
// split that holds position pos writes the new k and v rows to the cache.
struct RopeIn {
    const float* k = nullptr;      // [batch][kv_stride] new k rows (not rotated)
    const float* v = nullptr;      // [batch][kv_stride] new v rows
    const float2* rope = nullptr;  // [ctx][hd/2] (cos, sin)
    int kv_stride = 0;
    int on = 0;
    int neox = 0;  // split-half pairs (ApplyRoPENeox)
};

struct AttnArgs {
    const float* q;  // [batch][q_stride] (rotated)
    const void* kcache;
    const void* vcache;
    const int* pos_dev;
    int pos_host;
    int batch, n_heads, n_kv, hd, q_stride;
    int64_t cache_seq_stride, cache_layer_off;
    int kv_f16, ctx_len;
    float* part;     // scratch: AttnPlan::part_floats
    int* counters;   // [batch][n_kv], zero on entry, left zero
    float* out;      // [batch][out_stride]
    int out_stride;
    PrepTarget prep;  // the O projection's records (kind -1: none)
    RopeIn rope;      // on: q not yet rotated, the new k/v rows not yet in the cache
};

int launch_rmsnorm(const float* x, const float* w, float* y, int n, int rows, float eps,
                   cudaStream_t s);
int attention_plan(int n_heads, int n_kv, int hd, int max_seq, int batch, int sms, bool kv_f16, AttnPlan* p);
// Sets the kernels' shared-memory limit for plan p (call before any capture).
int attention_prepare(const AttnPlan& p);
int launch_attention(const AttnArgs& a, const AttnPlan& p, cudaStream_t s);
int launch_silu_mul(float* gate, const float* up, int64_t n, cudaStream_t s, int gelu = 0);
// dst[i] = src[i] + c
int launch_add_scalar(float* dst, const float* src, float c, int64_t n, cudaStream_t s);
// gate = silu(gate) * up for `batch` rows of n values, plus the records of
// the GEMV that reads the result (falls back to launch_silu_mul when pt has
// no record form or n is not a multiple of 256).
int launch_silu_prep(float* gate, const float* up, int n, int batch, const PrepTarget& pt, cudaStream_t s,
                     int gelu = 0);
int launch_add(float* a, const float* b, int64_t n, cudaStream_t s);
int launch_embed(int type, const void* emb, uint64_t row_bytes, const int* tokens, int vocab,
                 int dim, int batch, float* x, uint32_t* err, cudaStream_t s);
int launch_argmax(const float* logits, int n, int batch, int* out, cudaStream_t s);

}  // namespace cn
