// sample.cu -- TemperatureSampler.Sample (Samplers/TemperatureSampler.cs:33-113)
// on the device, so a decode loop need not copy the logits back.
//
// Per sequence, one CTA of 1024 threads:
//   1. p = logit * (1 / temperature), max, exp(p - max), sum, p * (1 / sum):
//      TensorMath.Softmax's passes (Tensors/TensorMath.cs:177-241); the sum
//      runs as a tree instead of left to right, which moves probabilities by
//      fp32 rounding only;
//   2. the top-k entries in descending order (ties: the lower index first),
//      one block-wide argmax per entry, stopping as soon as the running sum
//      reaches top_p (nothing past that cut-off matters: the reference's
//      nucleus loop breaks there) or k entries are out;
//   3. thread 0: renormalise the kept entries and return the first whose
//      running sum exceeds r, in the reference's order and arithmetic.
// r is the caller's Random.NextDouble() draw, so the host keeps the
// reference's random stream.  temperature <= 0 is the greedy argmax (first
// index of the maximum, as TemperatureSampler.ArgMax).
#include <float.h>

#include "cn_common.cuh"
#include "cn_internal.h"

namespace cn {

namespace {

constexpr int kSampThreads = 1024;

// (value, index) pair order: larger value first, then the lower index.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

// Block-wide best pair; every thread gets it.  sv/si hold 32 entries.
__device__ __forceinline__ void block_best(float& v, int& i, float* sv, int* si) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
    __syncthreads();  // sv/si may still be read from the previous round
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = v;
        si[threadIdx.x >> 5] = i;
    }
    __syncthreads();
    v = sv[0];
    i = si[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++)
        if (better(sv[w], si[w], v, i)) {
            v = sv[w];
            i = si[w];
        }
}

__device__ __forceinline__ float block_sum_f(float v, float* sv) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sv[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += sv[w];
    return s;
}

// This thread's best (probability, index) among entries not yet taken
// (taken entries hold -1).
__device__ __forceinline__ void local_best(const float* p, int n, float& bv, int& bi) {
    bv = -FLT_MAX;
    bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = p[i];
        if (v >= 0.f && better(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
}

}  // namespace

__global__ void __launch_bounds__(kSampThreads)
    sample_kernel(const float* __restrict__ logits, int n, int greedy, float inv_temp, int k, float top_p,
                  const float* __restrict__ r, float* __restrict__ probs, float* __restrict__ sel_p,
                  int* __restrict__ sel_i, int* __restrict__ out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ int s_done;
    const int b = blockIdx.x;
    const float* lg = logits + (size_t)b * n;
    float* p = probs + (size_t)b * n;
    float* sp = sel_p + (size_t)b * n;
    int* sx = sel_i + (size_t)b * n;

    if (greedy) {
        float bv = -FLT_MAX;
        int bi = 0x7fffffff;
        for (int i = threadIdx.x; i < n; i += blockDim.x)
            if (better(lg[i], i, bv, bi)) {
                bv = lg[i];
                bi = i;
            }
        block_best(bv, bi, sv, si);
        if (threadIdx.x == 0) out[b] = bi < n ? bi : 0;
        return;
    }

    // softmax of logit * (1 / temperature)
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = lg[i] * inv_temp;
        p[i] = v;
        mx = fmaxf(mx, v);
    }
    {
        float m = mx;
        int dummy = 0;
        block_best(m, dummy, sv, si);  // (ties of the index are irrelevant here)
        mx = m;
    }
    float part = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(p[i] - mx);
        p[i] = e;
        part += e;
    }
    const float sum = block_sum_f(part, sv);
    if (sum > 0.f) {
        const float inv = 1.0f / sum;
        for (int i = threadIdx.x; i < n; i += blockDim.x) p[i] *= inv;
    }
    __syncthreads();

    // top-k in descending order, up to the nucleus cut-off
    float bv;
    int bi;
    local_best(p, n, bv, bi);
    float cumulative = 0.f;  // thread 0's
    int count = 0;
    for (;;) {
        float v = bv;
        int i = bi;
        block_best(v, i, sv, si);
        if (threadIdx.x == 0) {
            const bool ok = i < n;  // a pair exists (n >= 1 entries remain)
            if (ok) {
                sp[count] = v;
                sx[count] = i;
                count++;
                cumulative += v;
            }
            s_done = !ok || cumulative >= top_p || count >= k;
        }
        if (i < n && (i % (int)blockDim.x) == (int)threadIdx.x) {
            p[i] = -1.f;  // taken
            local_best(p, n, bv, bi);
        }
        __syncthreads();
        if (s_done) break;
    }

    if (threadIdx.x == 0) {
        // renormalise the kept entries, then the first whose running sum
        // exceeds r (TemperatureSampler.cs:80-108)
        const int cutoff = count;
        float s = 0.f;
        for (int j = 0; j < cutoff; j++) s += sp[j];
        const float inv = 1.0f / s;
        float acc = 0.f;
        int tok = cutoff > 0 ? sx[cutoff - 1] : 0;
        for (int j = 0; j < cutoff; j++) {
            acc += sp[j] * inv;
            if (r[b] < acc) {
                tok = sx[j];
                break;
            }
        }
        out[b] = tok;
    }
}

int sample_launch(cn_ctx* ctx, const float* d_logits, int vocab, int batch, float temperature, int top_k,
                  float top_p, const float* r_host, int* tokens_host) {
    CN_CHECK(ctx && d_logits && tokens_host, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(vocab >= 1 && batch >= 1, CN_ERR_INVALID_ARG, "bad vocab %d / batch %d", vocab, batch);
    const bool greedy = !(temperature > 0.f);
    CN_CHECK(greedy || (top_k >= 1 && r_host), CN_ERR_INVALID_ARG, "sampling needs top_k >= 1 and r");
    const int k = top_k < vocab ? top_k : vocab;
    // scratch: probabilities, kept values, kept indices [batch][vocab]; r, tokens [batch]
    const size_t nv = (size_t)batch * vocab;
    const size_t need = nv * 4 * 3 + (size_t)batch * 8 + 64;
    int rc = ensure(&ctx->samp, &ctx->samp_bytes, need, false);
    if (rc) return rc;
    float* probs = static_cast<float*>(ctx->samp);
    float* sel_p = probs + nv;
    int* sel_i = reinterpret_cast<int*>(sel_p + nv);
    float* d_r = reinterpret_cast<float*>(sel_i + nv);
    int* d_out = reinterpret_cast<int*>(d_r + batch);
    cudaStream_t s = ctx->stream;
    if (!greedy) CN_CUDA(cudaMemcpyAsync(d_r, r_host, (size_t)batch * 4, cudaMemcpyHostToDevice, s));
    const float inv_temp = greedy ? 1.f : 1.0f / temperature;
    sample_kernel<<<batch, kSampThreads, 0, s>>>(d_logits, vocab, greedy ? 1 : 0, inv_temp, k, top_p, d_r, probs,
                                                 sel_p, sel_i, d_out);
    CN_CUDA(cudaGetLastError());
    CN_CUDA(cudaMemcpyAsync(tokens_host, d_out, (size_t)batch * 4, cudaMemcpyDeviceToHost, s));
    CN_CUDA(cudaStreamSynchronize(s));
    return CN_OK;
}

}  // namespace cn

int cn_sample_dev(cn_ctx* ctx, const float* d_logits, int vocab, int batch, float temperature, int top_k,
                  float top_p, const float* r_host, int* tokens_host) {
    if (ctx) cudaSetDevice(ctx->device);
    return cn::sample_launch(ctx, d_logits, vocab, batch, temperature, top_k, top_p, r_host, tokens_host);
}
