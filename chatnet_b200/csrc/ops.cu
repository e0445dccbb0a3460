// ops.cu -- the decode-step kernels around the GEMVs.
//
//   rmsnorm_kernel     TensorMath.RmsNorm            (Tensors/TensorMath.cs:97-165)
//   attn_split_kernel  LlamaModel.ComputeAttention + TensorMath.Softmax
//                      (LlamaModel.cs:241-346, TensorMath.cs:177-241), split over
//                      the context (flash-decoding); the last split CTA of each
//                      (sequence, kv head) merges the splits.  Both attention
//                      kernels also apply TensorMath.ApplyRoPE to q and the
//                      new k row and store the new k/v rows in the cache
//                      (TensorMath.cs:408-458, Models/Llama/LlamaModel.cs:146-153)
//   silu_mul_kernel    TensorMath.SiluElementwiseMul (TensorMath.cs:253-286)
//   add_kernel         TensorMath.Add                (TensorMath.cs:712-733)
//   embed_kernel       LlamaModel.LoadEmbedding      (LlamaModel.cs:365-394)
//   argmax_kernel      GreedySampler.Sample          (Samplers/GreedySampler.cs:13-26)
//
// Elementwise arithmetic uses the reference's operation order with explicit
// round-to-nearest intrinsics; reductions (sums of squares, dot products,
// softmax sums) run in a different order than the C# loops, which changes
// results only at the level of fp32 rounding.
#include <stdlib.h>
#include <float.h>

#include "cn_common.cuh"
#include "cn_internal.h"
#include "formats.cuh"
#include "ops.h"
#include "prep.cuh"

namespace cn {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum; `red` holds one float per warp.  All threads get the sum.
__device__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float s = 0.f;
    for (int i = 0; i < nw; i++) s += red[i];
    return s;
}
__device__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float m = -FLT_MAX;
    for (int i = 0; i < nw; i++) m = fmaxf(m, red[i]);
    return m;
}

// ---- RMSNorm: y = x * (1 / sqrt(sum(x^2)/n + eps)) * w, one CTA per row ----

__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                               float* __restrict__ y, int n, float eps) {
    __shared__ float red[32];
    const float* xr = x + (size_t)blockIdx.x * n;
    float* yr = y + (size_t)blockIdx.x * n;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    ss = block_sum(ss, red);
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        yr[i] = __fmul_rn(__fmul_rn(xr[i], rms), w[i]);
}

// ---- RoPE (interleaved pairs) on q and k, then k and v into the cache ---------
//
// cos/sin come from a host-built table [ctx][head_dim/2] computed exactly as
// ApplyRoPE does (theta = pos * exp(i * (1/hd) * -ln(base)), libm cos/sin),
// so the rotation factors are bit-identical to the reference's.

// ---- attention: split-K over positions, then combine ----------------------------
//
// CTA (split s, kv head kh, sequence b) handles positions [p0, p1) of
// 0..pos for the kv_mul query heads that share kv head kh (GQA: head h uses
// kv head h / kv_mul, LlamaModel.cs:265).  It writes, per query head, the
// local max m, sum l = sum exp(score - m) and o = sum exp(score - m) v to
// scratch; the combine kernel merges the splits:
//   out = sum_s exp(m_s - M) o_s / sum_s exp(m_s - M) l_s.
// This equals Softmax followed by the weighted V sum up to fp32 rounding.

constexpr int kAttnThreads = 256;

// 16 bytes global -> shared; src_bytes 0 writes zeros
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
                 : "memory");
}

constexpr int kMaxKvMul = 16;
constexpr int kMaxHd = 256;

// K/V element widths, loaded 16 bytes at a time.
template <typename KV>
struct KvVec;
template <>
struct KvVec<float> {
    static constexpr int kPer16 = 4;
    __device__ static float from_float(float v) { return v; }
    __device__ static void to_float(const uint4& v, float* out) {
        out[0] = __uint_as_float(v.x);
        out[1] = __uint_as_float(v.y);
        out[2] = __uint_as_float(v.z);
        out[3] = __uint_as_float(v.w);
    }
};
template <>
struct KvVec<__half> {
    static constexpr int kPer16 = 8;
    __device__ static __half from_float(float v) { return __float2half_rn(v); }
    __device__ static void to_float(const uint4& v, float* out) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            out[2 * i] = f.x;
            out[2 * i + 1] = f.y;
        }
    }
};

// Shared-memory layout of one attention CTA (floats unless noted):
//   qs   [kv_mul][hd + 4]        the kv_mul query heads (fp32), padded rows
//   ks   [chunk][hd + pad] (KV)  K rows of the chunk, padded by 16 bytes
//   vs   [chunk][hd] (KV)        V rows of the chunk
//   sc   [kv_mul][chunk]         scores, then exp(score - max)
//   red  [64]
template <typename KV>
__host__ __device__ constexpr int attn_krow(int hd) {
    return hd + 16 / (int)sizeof(KV);  // elements per padded K row
}

// Tail of both attention kernels: counts this split in for (b, kv head) and,
// in the last split to arrive, merges all splits of the group's heads, writes
// the attention output and, when pt names a record form, the O projection's
// records.  `sm` is the CTA's dynamic shared memory (reused), s_last a shared
// int.  Called by every thread of the CTA.
__device__ __forceinline__ void attn_finish(float* __restrict__ pr_base, int splits, int prow, int hd, int kv_mul, int n_kv,
                            int b, int kh, int* __restrict__ counters, float* __restrict__ out,
                            int out_stride, const PrepTarget& pt, float* sm, int* s_last) {
    // The last split of (b, kv head) to finish merges all splits (the
    // barrier orders the CTA's partials before thread 0's release; the last
    // arrival's acquire, then the barrier, orders everyone's partials before
    // the merge reads them).
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = blockDim.x >> 5;
    __syncthreads();
    if (tid == 0) {
        int old;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                     : "=r"(old)
                     : "l"(counters + b * n_kv + kh)
                     : "memory");
        *s_last = old == splits - 1;
    }
    __syncthreads();
    if (!*s_last) return;

    // Merge (LlamaModel.cs:241-346, TensorMath.cs:177-241, split form):
    // w_s = exp(m_s - M), out[d] = sum_s w_s o_s[d] * (1 / sum_s w_s l_s).
    float* wsm = sm;                                    // [kv_mul][splits]
    float* linv = wsm + ((kv_mul * splits + 3) & ~3);  // [kv_mul]
    float* obuf = linv + ((kv_mul + 3) & ~3);           // [kv_mul * hd], 16-byte aligned
    for (int g = warp; g < kv_mul; g += nwarp) {
        const float* pr = pr_base + (size_t)g * splits * prow;
        if (splits <= 32) {
            // one split per lane: its m and l in one L2 round trip
            const bool has = lane < splits;
            const float m = has ? __ldcg(pr + (size_t)lane * prow + hd) : -FLT_MAX;
            const float l = has ? __ldcg(pr + (size_t)lane * prow + hd + 1) : 0.f;
            const float M = warp_max(m);
            const float w = m > -FLT_MAX ? expf(m - M) : 0.f;
            if (has) wsm[g * splits + lane] = w;
            const float lsum = warp_sum(w * l);
            if (lane == 0) linv[g] = 1.0f / lsum;
            continue;
        }
        float M = -FLT_MAX;
        for (int t = lane; t < splits; t += 32) M = fmaxf(M, __ldcg(pr + (size_t)t * prow + hd));
        M = warp_max(M);
        float lsum = 0.f;
        for (int t = lane; t < splits; t += 32) {
            const float m = __ldcg(pr + (size_t)t * prow + hd);
            const float w = m > -FLT_MAX ? expf(m - M) : 0.f;
            wsm[g * splits + t] = w;
            lsum += w * __ldcg(pr + (size_t)t * prow + hd + 1);
        }
        lsum = warp_sum(lsum);
        if (lane == 0) linv[g] = 1.0f / lsum;
    }
    __syncthreads();
    for (int e = tid; e < kv_mul * (hd / 4); e += blockDim.x) {
        const int g = e / (hd / 4), d = (e % (hd / 4)) * 4;
        const float* pr = pr_base + (size_t)g * splits * prow + d;
        const float* wr = wsm + g * splits;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        int t = 0;
        for (; t + 16 <= splits; t += 16) {  // sixteen independent loads in flight
            float4 v[16];
#pragma unroll
            for (int k = 0; k < 16; k++) v[k] = __ldcg(reinterpret_cast<const float4*>(pr + (size_t)(t + k) * prow));
#pragma unroll
            for (int k = 0; k < 16; k++) {
                const float w = wr[t + k];
                o.x = fmaf(w, v[k].x, o.x);
                o.y = fmaf(w, v[k].y, o.y);
                o.z = fmaf(w, v[k].z, o.z);
                o.w = fmaf(w, v[k].w, o.w);
            }
        }
        for (; t + 4 <= splits; t += 4) {  // four independent loads in flight
            float4 v[4];
#pragma unroll
            for (int k = 0; k < 4; k++) v[k] = __ldcg(reinterpret_cast<const float4*>(pr + (size_t)(t + k) * prow));
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float w = wr[t + k];
                o.x = fmaf(w, v[k].x, o.x);
                o.y = fmaf(w, v[k].y, o.y);
                o.z = fmaf(w, v[k].z, o.z);
                o.w = fmaf(w, v[k].w, o.w);
            }
        }
        for (; t < splits; t++) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(pr + (size_t)t * prow));
            const float w = wr[t];
            o.x = fmaf(w, v.x, o.x);
            o.y = fmaf(w, v.y, o.y);
            o.z = fmaf(w, v.z, o.z);
            o.w = fmaf(w, v.w, o.w);
        }
        const float li = linv[g];
        o = make_float4(o.x * li, o.y * li, o.z * li, o.w * li);
        *reinterpret_cast<float4*>(out + (size_t)b * out_stride + (kh * kv_mul + g) * hd + d) = o;
        *reinterpret_cast<float4*>(obuf + g * hd + d) = o;
    }
    if (tid == 0) counters[b * n_kv + kh] = 0;
    // the O projection's records: this group's kv_mul * hd outputs are whole
    // 256-position units (the host passes a record target only then)
    if (pt.kind < 0) return;
    __syncthreads();
    const int units = kv_mul * hd / 256;
    for (int w = warp; w < units; w += nwarp) {
        const int c = lane >> 2, t4 = lane & 3;
        const float* src = obuf + w * 256 + 32 * c + 4 * t4;
        const float4 a0 = *reinterpret_cast<const float4*>(src);
        const float4 a1 = *reinterpret_cast<const float4*>(src + 16);
        const float v8[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        emit_any(pt, v8, kh * units + w, b, (int)gridDim.z, lane);
    }
}

template <typename KV>
__global__ void __launch_bounds__(kAttnThreads)
    attn_split_kernel(const float* __restrict__ q, const KV* __restrict__ kcache,
                      const KV* __restrict__ vcache, const int* __restrict__ pos_dev, int pos_host,
                      int n_heads, int n_kv, int hd, int q_stride, int64_t cache_seq_stride,
                      int64_t cache_layer_off, int ctx_len, int splits, int chunk, float scale,
                      float* __restrict__ part /* [b][head][split][hd + 4] */, int* __restrict__ counters,
                      float* __restrict__ out, int out_stride, PrepTarget pt, RopeIn ri) {
    pdl_trigger();
    // Cache rows below the current position were written by earlier steps:
    // their copies start before the wait for the q/k/v kernel; the row at the
    // current position (this step's k/v, rotated and stored here when ri.on)
    // and q come after it.
    extern __shared__ __align__(16) float sm[];
    __shared__ int s_last;
    const int s = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
    const int kv_mul = n_heads / n_kv;
    const int prow = hd + 4;  // floats per partial row: o[hd], m, l, pad
    int pos = pos_dev ? pos_dev[b] : pos_host;
    if (pos < 0 || pos >= ctx_len) pos = -1;  // rejected upstream; read nothing
    const int seq = pos + 1;
    const int p0 = s * chunk;
    const int L = max(0, min(seq, p0 + chunk) - p0);
    const int qrow = hd + 4;
    const int krow = attn_krow<KV>(hd);
    float* qs = sm;
    KV* ks = reinterpret_cast<KV*>(qs + kv_mul * qrow);
    KV* vs = ks + chunk * krow;
    float* sc = reinterpret_cast<float*>(vs + chunk * hd);
    const int tid = threadIdx.x;
    const int kvdim = n_kv * hd;
    const int lane = tid & 31, warp = tid >> 5, nwarp = blockDim.x >> 5;
    float* pr_base = part + ((size_t)b * n_heads + kh * kv_mul) * splits * prow;

    if (L == 0) {  // nothing of this split is inside 0..pos: an empty partial
        pdl_wait();
        for (int e = tid; e < kv_mul * prow; e += blockDim.x) {
            const int g = e / prow, d = e % prow;
            pr_base[((size_t)g * splits + s) * prow + d] = d == hd ? -FLT_MAX : 0.f;
        }
    } else {
        // the K / V rows of the chunk (16-byte copies); the current row last
        constexpr int P16 = KvVec<KV>::kPer16;
        const int vec_per_row = hd / P16;
        KV* kbase = const_cast<KV*>(kcache) + (int64_t)b * cache_seq_stride + cache_layer_off + kh * hd;
        KV* vbase = const_cast<KV*>(vcache) + (int64_t)b * cache_seq_stride + cache_layer_off + kh * hd;
        const int r_new = pos - p0;
        for (int i = tid; i < L * vec_per_row; i += blockDim.x) {
            const int r = i / vec_per_row, c = i % vec_per_row;
            if (r == r_new) continue;
            const int64_t g = (int64_t)(p0 + r) * kvdim + c * P16;
            cp_async16(smem_u32(ks + r * krow + c * P16), kbase + g, 16);
            cp_async16(smem_u32(vs + r * hd + c * P16), vbase + g, 16);
        }
        pdl_wait();
        if (!ri.on && r_new >= 0 && r_new < L) {
            for (int c = tid; c < vec_per_row; c += blockDim.x) {
                const int64_t g = (int64_t)pos * kvdim + c * P16;
                cp_async16(smem_u32(ks + r_new * krow + c * P16), kbase + g, 16);
                cp_async16(smem_u32(vs + r_new * hd + c * P16), vbase + g, 16);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        const float2* tab = ri.on ? ri.rope + (size_t)pos * (hd / 2) : nullptr;
        if (ri.on && r_new >= 0 && r_new < L) {
            // TensorMath.ApplyRoPE on the new k row, then k and v into the
            // cache (rotation with explicit _rn products, pairs per ri.neox)
            const float* kr = ri.k + (size_t)b * ri.kv_stride + kh * hd;
            const float* vr = ri.v + (size_t)b * ri.kv_stride + kh * hd;
            KV* kw = kbase + (int64_t)pos * kvdim;
            KV* vw = vbase + (int64_t)pos * kvdim;
            for (int p = tid; p < hd / 2; p += blockDim.x) {
                const float2 cs = tab[p];
                const int ia = ri.neox ? p : 2 * p, ib = ri.neox ? p + hd / 2 : 2 * p + 1;
                const float x0 = kr[ia], x1 = kr[ib];
                const KV k0 = KvVec<KV>::from_float(__fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y)));
                const KV k1 = KvVec<KV>::from_float(__fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x)));
                ks[r_new * krow + ia] = k0;
                ks[r_new * krow + ib] = k1;
                kw[ia] = k0;
                kw[ib] = k1;
                const KV v0 = KvVec<KV>::from_float(vr[2 * p]), v1 = KvVec<KV>::from_float(vr[2 * p + 1]);
                vs[r_new * hd + 2 * p] = v0;
                vs[r_new * hd + 2 * p + 1] = v1;
                vw[2 * p] = v0;
                vw[2 * p + 1] = v1;
            }
        }
        // q of the group's heads (fp32), rotated here when ri.on
        for (int i = tid; i < kv_mul * (hd / 2); i += blockDim.x) {
            const int gi = i / (hd / 2), p = i % (hd / 2);
            const int ia = ri.on && ri.neox ? p : 2 * p, ib = ri.on && ri.neox ? p + hd / 2 : 2 * p + 1;
            const float* qr = q + (size_t)b * q_stride + (kh * kv_mul + gi) * hd;
            float v0 = qr[ia], v1 = qr[ib];
            if (ri.on) {
                const float2 cs = tab[p];
                const float r0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
                const float r1 = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
                v0 = r0;
                v1 = r1;
            }
            qs[gi * qrow + ia] = v0;
            qs[gi * qrow + ib] = v1;
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        // scores: one (position, head) dot product per thread-iteration
        for (int e = tid; e < L * kv_mul; e += blockDim.x) {
            const int p = e / kv_mul, g = e % kv_mul;
            const KV* kr = ks + p * krow;
            const float* qr = qs + g * qrow;
            float acc = 0.f;
            for (int d = 0; d < hd; d += P16) {
                float kf[P16];
                KvVec<KV>::to_float(*reinterpret_cast<const uint4*>(kr + d), kf);
#pragma unroll
                for (int j = 0; j < P16; j++) acc = fmaf(qr[d + j], kf[j], acc);
            }
            sc[g * chunk + p] = __fmul_rn(acc, scale);
        }
        __syncthreads();
        // softmax statistics per head: warp w handles heads w, w + nwarp, ...
        for (int g = warp; g < kv_mul; g += nwarp) {
            float m = -FLT_MAX;
            for (int p = lane; p < L; p += 32) m = fmaxf(m, sc[g * chunk + p]);
            m = warp_max(m);
            float l = 0.f;
            for (int p = lane; p < L; p += 32) {
                float ev = expf(sc[g * chunk + p] - m);
                sc[g * chunk + p] = ev;
                l += ev;
            }
            l = warp_sum(l);
            if (lane == 0) {
                float* pr = pr_base + ((size_t)g * splits + s) * prow;
                pr[hd] = m;
                pr[hd + 1] = l;
            }
        }
        __syncthreads();
        // o[g][d] = sum_p e[g][p] v[p][d], four consecutive d per thread
        for (int e = tid; e < kv_mul * (hd / 4); e += blockDim.x) {
            const int g = e / (hd / 4), d = (e % (hd / 4)) * 4;
            const float* er = sc + g * chunk;
            float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
            for (int p = 0; p < L; p++) {
                const float w = er[p];
                const KV* vr = vs + p * hd + d;
                float v4[4];
                if constexpr (sizeof(KV) == 2) {
                    float2 a = __half22float2(*reinterpret_cast<const __half2*>(vr));
                    float2 c = __half22float2(*reinterpret_cast<const __half2*>(vr + 2));
                    v4[0] = a.x; v4[1] = a.y; v4[2] = c.x; v4[3] = c.y;
                } else {
                    float4 f = *reinterpret_cast<const float4*>(vr);
                    v4[0] = f.x; v4[1] = f.y; v4[2] = f.z; v4[3] = f.w;
                }
                o0 = fmaf(w, v4[0], o0);
                o1 = fmaf(w, v4[1], o1);
                o2 = fmaf(w, v4[2], o2);
                o3 = fmaf(w, v4[3], o3);
            }
            *reinterpret_cast<float4*>(pr_base + ((size_t)g * splits + s) * prow + d) = make_float4(o0, o1, o2, o3);
        }
    }

    attn_finish(pr_base, splits, prow, hd, kv_mul, n_kv, b, kh, counters, out, out_stride, pt, sm, &s_last);
}

// ---- attention on the tensor cores (fp16 KV cache) -----------------------------
//
// Same math as attn_split_kernel for an fp16 cache with kv_mul <= 8 query heads
// per kv head and head_dim 64 or 128, but the two contractions run on
// mma.sync m16n8k16 (fp16 in, fp32 accumulate).  A CTA takes CHUNK positions
// (16 per warp, CHUNK / 16 warps) of one (sequence, kv head):
//   * K / V rows arrive by cp.async into padded shared rows (zero-filled past
//     the current position);
//   * the A operand of Q K^T stacks the kv_mul query heads twice: rows 0-7
//     hold fp16(q), rows 8-15 fp16(q - fp16(q)), so D row g + D row g + 8 is
//     the score at fp32-level accuracy (K is exact in fp16);
//   * the score fragments become, in registers, the A operand of P V, again
//     split into hi and lo halves; V comes in through ldmatrix.trans;
//   * the warps' partial outputs and exp-sums are added in shared memory and
//     the split is merged by attn_finish.
// The loads of cache rows below the current position are issued before the
// programmatic-launch wait, so they overlap the q/k/v GEMV.
constexpr int kMmaChunkMax = 128;

__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm4_trans(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ uint32_t half2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

template <int HD, int CHUNK>
__global__ void __launch_bounds__(2 * CHUNK)
    attn_mma_kernel(const float* __restrict__ q, const __half* __restrict__ kcache,
                    const __half* __restrict__ vcache, const int* __restrict__ pos_dev, int pos_host,
                    int n_heads, int n_kv, int q_stride, int64_t cache_seq_stride, int64_t cache_layer_off,
                    int ctx_len, int splits, float scale, float* __restrict__ part, int* __restrict__ counters,
                    float* __restrict__ out, int out_stride, PrepTarget pt, RopeIn ri) {
    pdl_trigger();
    // Cache rows below the current position were written by earlier steps,
    // so their copies start before the wait for the q/k/v kernel; the row at
    // the current position, q and everything written here come after it.
    constexpr int NW = CHUNK / 16, NT = 32 * NW;  // 16 positions per warp
    static_assert(CHUNK % 16 == 0 && CHUNK <= kMmaChunkMax, "chunk");
    constexpr int RS = HD + 8;  // halves per shared row (16-byte pad against bank conflicts)
    extern __shared__ __align__(16) float sm[];
    __shared__ int s_last;
    __shared__ float mx[NW][8], ls[NW][8];
    const int s = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
    const int kv_mul = n_heads / n_kv;
    const int prow = HD + 4;
    int pos = pos_dev ? pos_dev[b] : pos_host;
    if (pos < 0 || pos >= ctx_len) pos = -1;  // rejected upstream; read nothing
    const int seq = pos + 1;
    const int p0 = s * CHUNK;
    const int L = max(0, min(seq, p0 + CHUNK) - p0);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    float* pr_base = part + ((size_t)b * n_heads + kh * kv_mul) * splits * prow;
    __half* Ks = reinterpret_cast<__half*>(sm);
    __half* Vs = Ks + CHUNK * RS;
    __half* Qs = Vs + CHUNK * RS;  // [16][RS]

    if (L == 0) {  // nothing of this split is inside 0..pos: an empty partial
        pdl_wait();
        for (int e = tid; e < kv_mul * prow; e += blockDim.x) {
            const int gi = e / prow, d = e % prow;
            pr_base[((size_t)gi * splits + s) * prow + d] = d == HD ? -FLT_MAX : 0.f;
        }
    } else {
        const int kvdim = n_kv * HD;
        const __half* kbase = kcache + (int64_t)b * cache_seq_stride + cache_layer_off + kh * HD;
        const __half* vbase = vcache + (int64_t)b * cache_seq_stride + cache_layer_off + kh * HD;
        constexpr int CPR = HD / 8;  // 16-byte chunks per row
        // row pos of the cache: this step's k/v (written here with ri.on, or
        // by the preceding kernel otherwise)
        const int r_new = pos - p0;
        for (int i = tid; i < CHUNK * CPR; i += NT) {
            const int r = i / CPR, c = i % CPR;
            if (r == r_new) continue;  // after the wait (no zero fill racing it)
            const bool in = r < L;
            const int64_t go = (int64_t)(p0 + (in ? r : 0)) * kvdim + c * 8;
            cp_async16(smem_u32(Ks + r * RS + c * 8), kbase + go, in ? 16 : 0);
            cp_async16(smem_u32(Vs + r * RS + c * 8), vbase + go, in ? 16 : 0);
        }
        pdl_wait();
        if (!ri.on && r_new >= 0 && r_new < L) {
            for (int c = tid; c < CPR; c += NT) {
                const int64_t go = (int64_t)pos * kvdim + c * 8;
                cp_async16(smem_u32(Ks + r_new * RS + c * 8), kbase + go, 16);
                cp_async16(smem_u32(Vs + r_new * RS + c * 8), vbase + go, 16);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        if (ri.on && r_new >= 0 && r_new < L) {
            // TensorMath.ApplyRoPE on the new k row, then k and v into the cache
            // (the same arithmetic as attn_split_kernel's)
            const float2* tab = ri.rope + (size_t)pos * (HD / 2);
            const float* kr = ri.k + (size_t)b * ri.kv_stride + kh * HD;
            const float* vr = ri.v + (size_t)b * ri.kv_stride + kh * HD;
            __half* kw = const_cast<__half*>(kbase) + (int64_t)pos * kvdim;
            __half* vw = const_cast<__half*>(vbase) + (int64_t)pos * kvdim;
            for (int p = tid; p < HD / 2; p += NT) {
                const float2 cs = tab[p];
                const int ia = ri.neox ? p : 2 * p, ib = ri.neox ? p + HD / 2 : 2 * p + 1;
                const float x0 = kr[ia], x1 = kr[ib];
                const __half h0 = __float2half_rn(__fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y)));
                const __half h1 = __float2half_rn(__fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x)));
                Ks[r_new * RS + ia] = h0;
                Ks[r_new * RS + ib] = h1;
                kw[ia] = h0;
                kw[ib] = h1;
                const __half v0 = __float2half_rn(vr[2 * p]), v1 = __float2half_rn(vr[2 * p + 1]);
                Vs[r_new * RS + 2 * p] = v0;
                Vs[r_new * RS + 2 * p + 1] = v1;
                vw[2 * p] = v0;
                vw[2 * p + 1] = v1;
            }
        }
        // query heads: fp16 hi in rows 0-7, the fp16 remainder in rows 8-15
        // (rotated here when ri.on)
        for (int i = tid; i < 8 * HD / 2; i += NT) {
            const int gi = i / (HD / 2), p = i % (HD / 2);
            // the pair's elements: (2p, 2p + 1), or (p, p + HD/2) for split-half RoPE
            const int ia = ri.on && ri.neox ? p : 2 * p, ib = ri.on && ri.neox ? p + HD / 2 : 2 * p + 1;
            float v0 = 0.f, v1 = 0.f;
            if (gi < kv_mul) {
                const float* qr = q + (size_t)b * q_stride + (kh * kv_mul + gi) * HD;
                v0 = qr[ia];
                v1 = qr[ib];
                if (ri.on) {
                    const float2 cs = ri.rope[(size_t)pos * (HD / 2) + p];
                    const float r0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
                    const float r1 = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
                    v0 = r0;
                    v1 = r1;
                }
            }
            const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
            Qs[gi * RS + ia] = h0;
            Qs[gi * RS + ib] = h1;
            Qs[(8 + gi) * RS + ia] = __float2half_rn(v0 - __half2float(h0));
            Qs[(8 + gi) * RS + ib] = __float2half_rn(v1 - __half2float(h1));
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();

        // S = Q K^T for this warp's 16 positions (two n-tiles of 8)
        const uint32_t qaddr = smem_u32(Qs) + (uint32_t)(((lane & 7) + 8 * ((lane >> 3) & 1)) * RS + 8 * (lane >> 4)) * 2;
        const uint32_t kaddr =
            smem_u32(Ks) + (uint32_t)((16 * warp + (lane & 7) + 8 * (lane >> 4)) * RS + 8 * ((lane >> 3) & 1)) * 2;
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int ks = 0; ks < HD / 16; ks++) {
            uint32_t a[4], kb[4];
            ldsm4(qaddr + ks * 32, a);
            ldsm4(kaddr + ks * 32, kb);
            mma_16816(acc[0], a, kb, acc[0]);
            mma_16816(acc[1], a, kb + 2, acc[1]);
        }
        // scores of head g at positions 16 warp + 8 nt + 2t + e; softmax
        // statistics over the CTA's positions
        float sc[2][2];
        float m = -FLT_MAX;
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int pl = 16 * warp + 8 * nt + 2 * t + e;
                const float v = pl < L ? __fmul_rn(acc[nt][e] + acc[nt][2 + e], scale) : -FLT_MAX;
                sc[nt][e] = v;
                m = fmaxf(m, v);
            }
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        if (t == 0) mx[warp][g] = m;
        __syncthreads();
        float M = mx[0][g];
#pragma unroll
        for (int w = 1; w < NW; w++) M = fmaxf(M, mx[w][g]);
        float pe[2][2], l = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                pe[nt][e] = sc[nt][e] > -FLT_MAX ? expf(sc[nt][e] - M) : 0.f;
                l += pe[nt][e];
            }
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        if (t == 0) ls[warp][g] = l;

        // O = P V: A = P (rows 0-7 fp16(p), rows 8-15 the remainder), k =
        // this warp's 16 positions, n = head dims in tiles of 8
        uint32_t pa[4];
        {
            const __half2 h0 = __floats2half2_rn(pe[0][0], pe[0][1]);
            const __half2 h1 = __floats2half2_rn(pe[1][0], pe[1][1]);
            const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
            pa[0] = half2_bits(h0);
            pa[1] = half2_bits(__floats2half2_rn(pe[0][0] - f0.x, pe[0][1] - f0.y));
            pa[2] = half2_bits(h1);
            pa[3] = half2_bits(__floats2half2_rn(pe[1][0] - f1.x, pe[1][1] - f1.y));
        }
        const uint32_t vaddr =
            smem_u32(Vs) + (uint32_t)((16 * warp + (lane & 7) + 8 * ((lane >> 3) & 1)) * RS + 8 * (lane >> 4)) * 2;
        float o[HD / 8][4];
#pragma unroll
        for (int n = 0; n < HD / 8; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
#pragma unroll
        for (int n = 0; n < HD / 8; n += 2) {
            uint32_t vb[4];
            ldsm4_trans(vaddr + n * 16, vb);
            mma_16816(o[n], pa, vb, o[n]);
            mma_16816(o[n + 1], pa, vb + 2, o[n + 1]);
        }
        // sum the warps' outputs (the K rows are no longer read: every warp
        // passed the barrier after its scores)
        float* ob = reinterpret_cast<float*>(Ks);  // [NW warps][8 heads][HD]
#pragma unroll
        for (int n = 0; n < HD / 8; n++)
            *reinterpret_cast<float2*>(ob + (warp * 8 + g) * HD + 8 * n + 2 * t) =
                make_float2(o[n][0] + o[n][2], o[n][1] + o[n][3]);
        __syncthreads();
        for (int i = tid; i < kv_mul * HD; i += NT) {
            const int gi = i / HD, d = i % HD;
            float sum = 0.f;
#pragma unroll
            for (int w = 0; w < NW; w++) sum += ob[(w * 8 + gi) * HD + d];
            pr_base[((size_t)gi * splits + s) * prow + d] = sum;
        }
        if (tid < kv_mul) {
            float Mh = mx[0][tid], lh = 0.f;
#pragma unroll
            for (int w = 1; w < NW; w++) Mh = fmaxf(Mh, mx[w][tid]);
#pragma unroll
            for (int w = 0; w < NW; w++) lh += ls[w][tid];
            pr_base[((size_t)tid * splits + s) * prow + HD] = Mh;
            pr_base[((size_t)tid * splits + s) * prow + HD + 1] = lh;
        }
    }
    attn_finish(pr_base, splits, prow, HD, kv_mul, n_kv, b, kh, counters, out, out_stride, pt, sm, &s_last);
}

// ---- elementwise -----------------------------------------------------------------

__global__ void silu_mul_kernel(float* __restrict__ gate, const float* __restrict__ up, int64_t n, int gelu) {
    pdl_trigger();
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        gate[i] = act_mul(gate[i], up[i], gelu);
}

// SiluElementwiseMul fused with the prep of its output: one warp per
// (256-position unit, row); the lanes hold the values in the record layout.
__global__ void silu_prep_kernel(float* __restrict__ gate, const float* __restrict__ up, int n, int batch,
                                 PrepTarget pt, int gelu) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int units = n / 256;
    const int64_t items = (int64_t)units * batch;
    const int64_t w0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t it = w0; it < items; it += nw) {
        const int u = (int)(it % units), b = (int)(it / units);
        const size_t off = (size_t)b * n + (size_t)u * 256 + (lane >> 2) * 32 + 4 * (lane & 3);
        float v[8];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            float4 g4 = *reinterpret_cast<const float4*>(gate + off + 16 * h);
            const float4 u4 = *reinterpret_cast<const float4*>(up + off + 16 * h);
            float* gv = reinterpret_cast<float*>(&g4);
            const float* uv = reinterpret_cast<const float*>(&u4);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                gv[k] = act_mul(gv[k], uv[k], gelu);
                v[4 * h + k] = gv[k];
            }
            *reinterpret_cast<float4*>(gate + off + 16 * h) = g4;
        }
        emit_any(pt, v, u, b, batch, lane);
    }
}

__global__ void add_scalar_kernel(float* __restrict__ dst, const float* __restrict__ src, float c, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __fadd_rn(src[i], c);
}

__global__ void add_kernel(float* __restrict__ a, const float* __restrict__ b, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        a[i] = __fadd_rn(a[i], b[i]);
}

// ---- embedding: dequantize row tokens[b] of token_embd (bit-exact) -----------------

__global__ void embed_kernel(int type, const uint8_t* __restrict__ emb, uint64_t row_bytes,
                             const int* __restrict__ tokens, int vocab, int dim,
                             float* __restrict__ x, uint32_t* err) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.y;
    const int tok = tokens[b];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(err, kErrBadArg);
        return;
    }
    const uint8_t* row = emb + (size_t)tok * row_bytes;
    float* out = x + (size_t)b * dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) {
        float v;
        if (type == CN_TYPE_Q4_0) {
            const uint8_t* p = row + (i / 32) * 18;
            int j = i % 32;
            int q = j < 16 ? (p[2 + j] & 0x0F) : ((p[2 + j - 16] >> 4) & 0x0F);
            v = __fmul_rn((float)(q - 8), ld_half(p));
        } else if (type == CN_TYPE_Q4_K) {
            const uint8_t* p = row + (i / 256) * 144;
            int w = i % 256, sub = w / 32, j = w % 32;
            int sc, m;
            q4k_scale_min(p + 4, sub, sc, m);
            float dsc = __fmul_rn(ld_half(p), (float)sc), dm = __fmul_rn(ld_half(p + 2), (float)m);
            uint8_t byte = p[16 + sub * 16 + (j & 15)];
            int q = j < 16 ? (byte & 0x0F) : ((byte >> 4) & 0x0F);
            v = __fsub_rn(__fmul_rn(dsc, (float)q), dm);
        } else if (type == CN_TYPE_Q6_K) {
            const uint8_t* p = row + (i / 256) * 210;
            int w = i % 256, half = w / 128, r = w % 128, s = r / 32, l = r % 32;
            const uint8_t* ql = p + half * 64;
            const uint8_t* qh = p + 128 + half * 32;
            int lo = (s & 1) ? ql[l + 32] : ql[l];
            lo = (s >> 1) ? (lo >> 4) : (lo & 0x0F);
            int q = (lo | (((qh[l] >> (2 * s)) & 3) << 4)) - 32;
            int si = half * 8 + l / 16 + 2 * s;
            v = __fmul_rn(__fmul_rn(ld_half(p + 208), (float)(int8_t)p[192 + si]), (float)q);
        } else if (is_block32(type)) {
            v = block32_elem(type, row + (i / 32) * block32_bytes(type), i % 32);
        } else if (is_superblock(type)) {
            v = superblock_elem(type, row + (i / 256) * superblock_bytes(type), i % 256, row + row_bytes);
        } else if (type == CN_TYPE_F16) {
            v = ld_half(row + 2 * i);
        } else {
            v = reinterpret_cast<const float*>(row)[i];
        }
        out[i] = v;
    }
}

// ---- argmax: first index of the maximum (strict > in the scan) ---------------------

__global__ void argmax_kernel(const float* __restrict__ logits, int n, int* __restrict__ out) {
    pdl_trigger();
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    const float* l = logits + (size_t)blockIdx.x * n;
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = l[i];
        if (v > bv || (v == bv && i < bi)) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) {
        sv[w] = bv;
        si[w] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); k++)
            if (sv[k] > bv || (sv[k] == bv && si[k] < bi)) {
                bv = sv[k];
                bi = si[k];
            }
        out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
    }
}

// ---- launchers -----------------------------------------------------------------------

static int grid_1d(int64_t n, int threads, int cap) {
    int64_t g = (n + threads - 1) / threads;
    if (g < 1) g = 1;
    if (g > cap) g = cap;
    return (int)g;
}

int launch_rmsnorm(const float* x, const float* w, float* y, int n, int rows, float eps,
                   cudaStream_t s) {
    rmsnorm_kernel<<<rows, 256, 0, s>>>(x, w, y, n, eps);
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

static bool attn_use_mma(int n_heads, int n_kv, int hd, bool kv_f16) {
    return kv_f16 && n_heads / n_kv <= 8 && (hd == 64 || hd == 128);
}

using AttnMmaFn = void (*)(const float*, const __half*, const __half*, const int*, int, int, int, int, int64_t,
                           int64_t, int, int, float, float*, int*, float*, int, PrepTarget, RopeIn);
static AttnMmaFn attn_mma_fn(int hd, int chunk) {
#ifdef CHATNET_TUNING
    if (chunk == 32) return hd == 64 ? attn_mma_kernel<64, 32> : attn_mma_kernel<128, 32>;
    if (chunk == 64) return hd == 64 ? attn_mma_kernel<64, 64> : attn_mma_kernel<128, 64>;
#endif
    (void)chunk;
    return hd == 64 ? attn_mma_kernel<64, 128> : attn_mma_kernel<128, 128>;
}

// Positions per tensor-core attention CTA: 128.  Smaller chunks (tuning
// builds: CHATNET_ATTN_CHUNK=32 or 64) give more, smaller CTAs that fit
// beside the q/k/v GEMV's, but measured on B200 in the Llama-2-70B decode
// step (batch 1, position 2047) they cost more than they save: 9.95 ms per
// step with 128, 10.33 ms with 64, 11.69 ms with 32.
static int attn_mma_chunk() {
#ifdef CHATNET_TUNING
    if (const char* e = getenv("CHATNET_ATTN_CHUNK")) {
        const int v = atoi(e);
        if (v == 32 || v == 64 || v == 128) return v;
    }
#endif
    return kMmaChunkMax;
}

int attention_plan(int n_heads, int n_kv, int hd, int max_seq, int batch, int sms, bool kv_f16, AttnPlan* p) {
    CN_CHECK(n_kv > 0 && n_heads % n_kv == 0, CN_ERR_INVALID_ARG, "n_heads %% n_kv_heads != 0");
    CN_CHECK(n_heads / n_kv <= kMaxKvMul, CN_ERR_UNSUPPORTED, "kv_mul > %d", kMaxKvMul);
    CN_CHECK(hd <= kMaxHd && hd % 8 == 0, CN_ERR_UNSUPPORTED, "head_dim %d (needs a multiple of 8)", hd);
    const int kv_mul = n_heads / n_kv;
    p->mma = attn_use_mma(n_heads, n_kv, hd, kv_f16);
    int chunk;
    if (p->mma) {
        chunk = attn_mma_chunk();
    } else {
        // about one CTA per SM in total, chunks of 32..128 positions (the
        // merge then reads few partials per (sequence, kv head))
        const int want = (sms + batch * n_kv - 1) / (batch * n_kv);
        chunk = (max_seq + want - 1) / want;
        chunk = (chunk + 31) / 32 * 32;
        if (chunk < 32) chunk = 32;
        if (chunk > 128) chunk = 128;
    }
    p->chunk = chunk;
    p->splits = (max_seq + chunk - 1) / chunk;
    p->part_floats = (size_t)batch * n_heads * p->splits * (hd + 4);
    // worst case over both cache types (fp32 rows are the wider ones)
    const size_t q_bytes = (size_t)kv_mul * (hd + 4) * 4;
    const size_t kv_bytes = (size_t)chunk * (attn_krow<float>(hd) + hd) * 4;
    size_t smem = q_bytes + kv_bytes + (size_t)kv_mul * chunk * 4;
    const size_t mma_smem = (size_t)(2 * chunk + 16) * (hd + 8) * 2;
    const size_t merge_smem =
        (((size_t)kv_mul * p->splits + 3) / 4 * 4 + ((kv_mul + 3) & ~3) + (size_t)kv_mul * hd) * 4;
    if (p->mma) smem = mma_smem;
    p->smem = smem > merge_smem ? smem : merge_smem;
    return CN_OK;
}

int attention_prepare(const AttnPlan& p) {
    CN_CUDA(cudaFuncSetAttribute(attn_split_kernel<__half>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem));
    CN_CUDA(cudaFuncSetAttribute(attn_split_kernel<float>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem));
    if (p.mma)
        for (int hd : {64, 128})
            CN_CUDA(cudaFuncSetAttribute(attn_mma_fn(hd, p.chunk), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)p.smem));
    return CN_OK;
}

int launch_attention(const AttnArgs& a, const AttnPlan& p, cudaStream_t s) {
    dim3 grid(p.splits, a.n_kv, a.batch);
    CN_CHECK(!a.rope.on || (a.rope.k && a.rope.v && a.rope.rope), CN_ERR_INVALID_ARG,
             "attention: RoPE fusion needs the new k/v rows and the table");
    const float scale = 1.0f / sqrtf((float)a.hd);
    CN_CHECK(a.out_stride % 4 == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(a.part) & 15) == 0,
             CN_ERR_INVALID_ARG, "attention: output rows and scratch must be 16-byte aligned");
    PrepTarget pt = a.prep;
    if ((a.n_heads / a.n_kv) * a.hd % 256 != 0 || a.out_stride % 4 != 0) pt.kind = -1;
    if (p.mma) {
        CN_CHECK(a.kv_f16 && attn_use_mma(a.n_heads, a.n_kv, a.hd, true) && p.chunk == attn_mma_chunk(),
                 CN_ERR_INVALID_ARG, "attention plan does not match the call");
        CN_CUDA(launch_k(true, attn_mma_fn(a.hd, p.chunk), grid, dim3(2 * p.chunk), p.smem, s, a.q, (const __half*)a.kcache,
                         (const __half*)a.vcache, a.pos_dev, a.pos_host, a.n_heads, a.n_kv, a.q_stride,
                         a.cache_seq_stride, a.cache_layer_off, a.ctx_len, p.splits, scale, a.part,
                         a.counters, a.out, a.out_stride, pt, a.rope));
    } else if (a.kv_f16) {
        CN_CUDA(launch_k(true, attn_split_kernel<__half>, grid, dim3(kAttnThreads), p.smem, s,
            a.q, (const __half*)a.kcache, (const __half*)a.vcache, a.pos_dev, a.pos_host, a.n_heads,
            a.n_kv, a.hd, a.q_stride, a.cache_seq_stride, a.cache_layer_off, a.ctx_len, p.splits,
            p.chunk, scale, a.part, a.counters, a.out, a.out_stride, pt, a.rope));
    } else {
        CN_CUDA(launch_k(true, attn_split_kernel<float>, grid, dim3(kAttnThreads), p.smem, s,
            a.q, (const float*)a.kcache, (const float*)a.vcache, a.pos_dev, a.pos_host, a.n_heads,
            a.n_kv, a.hd, a.q_stride, a.cache_seq_stride, a.cache_layer_off, a.ctx_len, p.splits,
            p.chunk, scale, a.part, a.counters, a.out, a.out_stride, pt, a.rope));
    }
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

int launch_silu_mul(float* gate, const float* up, int64_t n, cudaStream_t s, int gelu) {
    CN_CUDA(launch_k(true, silu_mul_kernel, dim3(grid_1d(n, 256, 148 * 8)), dim3(256), 0, s, gate, up, n, gelu));
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

int launch_silu_prep(float* gate, const float* up, int n, int batch, const PrepTarget& pt, cudaStream_t s,
                     int gelu) {
    if (pt.kind < 0 || n % 256 != 0) return launch_silu_mul(gate, up, (int64_t)n * batch, s, gelu);
    const int64_t items = (int64_t)(n / 256) * batch;
    CN_CUDA(launch_k(true, silu_prep_kernel, dim3((unsigned)((items + 7) / 8)), dim3(256), 0, s, gate, up, n,
                     batch, pt, gelu));
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

int launch_add_scalar(float* dst, const float* src, float c, int64_t n, cudaStream_t s) {
    add_scalar_kernel<<<grid_1d(n, 256, 148 * 8), 256, 0, s>>>(dst, src, c, n);
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

int launch_add(float* a, const float* b, int64_t n, cudaStream_t s) {
    add_kernel<<<grid_1d(n, 256, 148 * 8), 256, 0, s>>>(a, b, n);
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

int launch_embed(int type, const void* emb, uint64_t row_bytes, const int* tokens, int vocab,
                 int dim, int batch, float* x, uint32_t* err, cudaStream_t s) {
    CN_CUDA(launch_k(true, embed_kernel, dim3(grid_1d(dim, 256, 32), batch), dim3(256), 0, s, type,
                     (const uint8_t*)emb, row_bytes, tokens, vocab, dim, x, err));
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

int launch_argmax(const float* logits, int n, int batch, int* out, cudaStream_t s) {
    CN_CUDA(launch_k(true, argmax_kernel, dim3(batch), dim3(1024), 0, s, logits, n, out));
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

}  // namespace cn
