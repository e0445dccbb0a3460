// prefill.cu -- the kernels around the prefill matmul (matmul.cu) when a
// prompt of M tokens runs through the decoder at once:
//
//   norm_half_kernel      TensorMath.RmsNorm (Tensors/TensorMath.cs:97-165), one
//                         token per CTA, output rounded to fp16 for the matmul
//   silu_half_kernel      TensorMath.SiluElementwiseMul (TensorMath.cs:253-286),
//                         output rounded to fp16 for the down projection
//   attn_prefill_kernel   LlamaModel.ComputeAttention + TensorMath.Softmax
//                         (Models/Llama/LlamaModel.cs:241-346, TensorMath.cs:177-241)
//                         for M queries at positions pos0..pos0+M-1 with causal
//                         masking: flash attention on mma.sync m16n8k16 (fp16
//                         operands, fp32 scores, online softmax in fp32)
//
// ChatNet itself feeds a prompt one token at a time (InferenceEngine.cs:235-239);
// these kernels compute the same per-token results in one pass.
#include <float.h>

#include "cn_common.cuh"
#include "cn_internal.h"

namespace cn {

namespace {

__device__ __forceinline__ float pf_warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

}  // namespace

// y[t] = fp16(RmsNorm(x[t]) * w), the reference's operation order.
__global__ void norm_half_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                 __half* __restrict__ y, int n, float eps) {
    __shared__ float red[32];
    const float* xr = x + (size_t)blockIdx.x * n;
    __half* yr = y + (size_t)blockIdx.x * n;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    ss = pf_warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) tot += red[i];
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        yr[i] = __float2half_rn(__fmul_rn(__fmul_rn(xr[i], rms), w[i]));
}

// h = fp16(g / (1 + exp(-g)) * u).
__global__ void silu_half_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                 __half* __restrict__ h, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float x = g[i];
        const float s = __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
        h[i] = __float2half_rn(__fmul_rn(s, u[i]));
    }
}

__global__ void positions_kernel(int* __restrict__ pos, int n, int pos0) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) pos[i] = pos0 + i;
}

// Causal attention for M queries of one sequence.  CTA = (64-query block,
// head); warp w owns queries 16w..16w+15 of the block.  Keys of the sequence
// are read from the cache (fp32 or fp16) in blocks of 64 and converted to
// fp16 in shared memory; query t (position pos0 + t) sees keys 0..pos0+t.
constexpr int kPfQ = 64;   // queries per CTA
constexpr int kPfK = 64;   // keys per block
constexpr int kPfThreads = 128;

template <int HD>
__global__ void __launch_bounds__(kPfThreads)
    attn_prefill_kernel(const float* __restrict__ q, int q_stride, const void* __restrict__ kcache,
                        const void* __restrict__ vcache, int kv_f16, int64_t cache_off, int kvdim,
                        int n_heads, int n_kv, int M, int pos0, float scale_log2,
                        __half* __restrict__ out, int out_stride) {
    constexpr int RS = HD + 8;  // halves per shared row (16-byte pad: conflict-free ldmatrix)
    constexpr int NT = HD / 8;  // 8-wide column tiles of the output
    constexpr int KS = HD / 16; // k-steps of Q K^T
    extern __shared__ __align__(16) uint8_t pf_smem[];
    __half* Qs = reinterpret_cast<__half*>(pf_smem);
    __half* Ks = Qs + kPfQ * RS;
    __half* Vs = Ks + kPfK * RS;
    const int qb = blockIdx.x, h = blockIdx.y;
    const int kh = h / (n_heads / n_kv);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int t0 = qb * kPfQ;

    // queries -> fp16
    constexpr int C4 = HD / 4;
    for (int i = tid; i < kPfQ * C4; i += kPfThreads) {
        const int r = i / C4, c = i % C4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t0 + r < M) v = *reinterpret_cast<const float4*>(q + (size_t)(t0 + r) * q_stride + h * HD + 4 * c);
        uint2 o;
        o.x = pack_half2(v.x, v.y);
        o.y = pack_half2(v.z, v.w);
        *reinterpret_cast<uint2*>(Qs + r * RS + 4 * c) = o;
    }
    __syncthreads();
    uint32_t qf[KS][4];
    {
        const int r = 16 * warp + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
        for (int ks = 0; ks < KS; ks++)
            ldsm_x4(smem_u32(Qs + r * RS + 16 * ks + 8 * (lane >> 4)), qf[ks]);
    }

    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float mrow[2] = {-FLT_MAX, -FLT_MAX}, lrow[2] = {0.f, 0.f};
    const int qpos[2] = {pos0 + t0 + 16 * warp + g, pos0 + t0 + 16 * warp + g + 8};
    const int last = pos0 + min(t0 + kPfQ, M) - 1;  // the block's last query position
    const int nkb = last / kPfK + 1;

    for (int kb = 0; kb < nkb; kb++) {
        const int p0 = kb * kPfK;
        __syncthreads();  // previous block's K/V no longer read
        constexpr int C8 = HD / 8;
        for (int i = tid; i < kPfK * C8; i += kPfThreads) {
            const int r = i / C8, c = i % C8;
            const int p = p0 + r;
            uint4 kv[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
            if (p <= last) {
                const int64_t e = cache_off + (int64_t)p * kvdim + kh * HD + 8 * c;
#pragma unroll
                for (int w = 0; w < 2; w++) {
                    const void* base = w == 0 ? kcache : vcache;
                    if (kv_f16) {
                        kv[w] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(base) + e);
                    } else {
                        const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + e);
                        const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + e + 4);
                        kv[w] = make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y),
                                           pack_half2(b.z, b.w));
                    }
                }
            }
            *reinterpret_cast<uint4*>(Ks + r * RS + 8 * c) = kv[0];
            *reinterpret_cast<uint4*>(Vs + r * RS + 8 * c) = kv[1];
        }
        __syncthreads();

        // S = Q K^T for this warp's 16 queries x 64 keys
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KS; ks++) {
#pragma unroll
            for (int jp = 0; jp < 4; jp++) {  // two 8-key tiles per ldmatrix.x4
                uint32_t b[4];
                const int key = 16 * jp + (lane & 7) + 8 * (lane >> 4);
                ldsm_x4(smem_u32(Ks + key * RS + 16 * ks + 8 * ((lane >> 3) & 1)), b);
                const uint32_t b0[2] = {b[0], b[1]}, b1[2] = {b[2], b[3]};
                mma_16816(s[2 * jp], qf[ks], b0, s[2 * jp]);
                mma_16816(s[2 * jp + 1], qf[ks], b1, s[2 * jp + 1]);
            }
        }
        // scale (log2 domain), causal mask, online softmax
        float mnew[2] = {mrow[0], mrow[1]};
#pragma unroll
        for (int j = 0; j < 8; j++) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int key = p0 + 8 * j + 2 * t4 + (e & 1);
                const int hr = e >> 1;
                float v = s[j][e] * scale_log2;
                if (key > qpos[hr]) v = -FLT_MAX;
                s[j][e] = v;
                mnew[hr] = fmaxf(mnew[hr], v);
            }
        }
        float alpha[2];
#pragma unroll
        for (int hr = 0; hr < 2; hr++) {
            mnew[hr] = fmaxf(mnew[hr], __shfl_xor_sync(0xffffffffu, mnew[hr], 1));
            mnew[hr] = fmaxf(mnew[hr], __shfl_xor_sync(0xffffffffu, mnew[hr], 2));
            alpha[hr] = exp2f(mrow[hr] - mnew[hr]);
            mrow[hr] = mnew[hr];
        }
        float rs[2] = {0.f, 0.f};
        uint32_t pa[4][4];  // P as A fragments, one per 16-key step
#pragma unroll
        for (int j = 0; j < 8; j++) {
            float pv[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int hr = e >> 1;
                pv[e] = s[j][e] == -FLT_MAX ? 0.f : exp2f(s[j][e] - mrow[hr]);
                rs[hr] += pv[e];
            }
            pa[j >> 1][(j & 1) * 2 + 0] = pack_half2(pv[0], pv[1]);
            pa[j >> 1][(j & 1) * 2 + 1] = pack_half2(pv[2], pv[3]);
        }
#pragma unroll
        for (int hr = 0; hr < 2; hr++) lrow[hr] = lrow[hr] * alpha[hr] + rs[hr];
#pragma unroll
        for (int j = 0; j < NT; j++) {
            o[j][0] *= alpha[0];
            o[j][1] *= alpha[0];
            o[j][2] *= alpha[1];
            o[j][3] *= alpha[1];
        }
        // O += P V; A fragment order: (row g, keys 2t..), (row g+8, keys 2t..),
        // (row g, keys 8+2t..), (row g+8, keys 8+2t..)
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            const uint32_t a[4] = {pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3]};
#pragma unroll
            for (int jp = 0; jp < NT / 2; jp++) {
                uint32_t b[4];
                const int key = 16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1);
                ldsm_x4_t(smem_u32(Vs + key * RS + 16 * jp + 8 * (lane >> 4)), b);
                const uint32_t b0[2] = {b[0], b[1]}, b1[2] = {b[2], b[3]};
                mma_16816(o[2 * jp], a, b0, o[2 * jp]);
                mma_16816(o[2 * jp + 1], a, b1, o[2 * jp + 1]);
            }
        }
    }

    // normalise and store
#pragma unroll
    for (int hr = 0; hr < 2; hr++) {
        lrow[hr] += __shfl_xor_sync(0xffffffffu, lrow[hr], 1);
        lrow[hr] += __shfl_xor_sync(0xffffffffu, lrow[hr], 2);
    }
#pragma unroll
    for (int hr = 0; hr < 2; hr++) {
        const int tq = t0 + 16 * warp + g + 8 * hr;
        if (tq >= M) continue;
        const float inv = lrow[hr] > 0.f ? 1.0f / lrow[hr] : 0.f;
        __half* orow = out + (size_t)tq * out_stride + h * HD;
#pragma unroll
        for (int j = 0; j < NT; j++)
            *reinterpret_cast<uint32_t*>(orow + 8 * j + 2 * t4) =
                pack_half2(o[j][2 * hr] * inv, o[j][2 * hr + 1] * inv);
    }
}

// ---- host side ------------------------------------------------------------------

int prefill_positions(cudaStream_t st, int* pos_dev, int n, int pos0) {
    CN_CUDA(launch_k(false, positions_kernel, dim3((n + 255) / 256), dim3(256), 0, st, pos_dev, n, pos0));
    return CN_OK;
}

int prefill_norm(cudaStream_t st, const float* x, const float* w, __half* y, int n, int M, float eps) {
    CN_CUDA(launch_k(false, norm_half_kernel, dim3(M), dim3(256), 0, st, x, w, y, n, eps));
    return CN_OK;
}

int prefill_silu(cudaStream_t st, const float* g, const float* u, __half* h, int64_t n) {
    const int64_t blocks = (n + 255) / 256 < 8192 ? (n + 255) / 256 : 8192;
    CN_CUDA(launch_k(false, silu_half_kernel, dim3((unsigned)blocks), dim3(256), 0, st, g, u, h, n));
    return CN_OK;
}

int prefill_attention(cudaStream_t st, const float* q, int q_stride, const void* kcache,
                      const void* vcache, bool kv_f16, int64_t cache_off, int n_heads, int n_kv,
                      int hd, int M, int pos0, __half* out, int out_stride) {
    CN_CHECK(hd == 64 || hd == 128, CN_ERR_UNSUPPORTED, "prefill attention: head_dim %d", hd);
    CN_CHECK(n_kv > 0 && n_heads % n_kv == 0 && M >= 1 && pos0 >= 0, CN_ERR_INVALID_ARG,
             "prefill attention: bad arguments");
    CN_CHECK(q_stride % 4 == 0 && out_stride % 2 == 0, CN_ERR_INVALID_ARG, "prefill attention: strides");
    const int RS = hd + 8;
    const size_t smem = (size_t)(kPfQ + 2 * kPfK) * RS * sizeof(__half);
    const float scale_log2 = 1.4426950408889634f / sqrtf((float)hd);
    const dim3 grid((M + kPfQ - 1) / kPfQ, n_heads);
    const int kvdim = n_kv * hd;
    if (hd == 128) {
        static bool attr = false;
        if (!attr) {
            CN_CUDA(cudaFuncSetAttribute(attn_prefill_kernel<128>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            attr = true;
        }
        CN_CUDA(launch_k(false, attn_prefill_kernel<128>, grid, dim3(kPfThreads), smem, st, q, q_stride,
                         kcache, vcache, kv_f16 ? 1 : 0, cache_off, kvdim, n_heads, n_kv, M, pos0,
                         scale_log2, out, out_stride));
    } else {
        CN_CUDA(launch_k(false, attn_prefill_kernel<64>, grid, dim3(kPfThreads), smem, st, q, q_stride,
                         kcache, vcache, kv_f16 ? 1 : 0, cache_off, kvdim, n_heads, n_kv, M, pos0,
                         scale_log2, out, out_stride));
    }
    return CN_OK;
}

}  // namespace cn
