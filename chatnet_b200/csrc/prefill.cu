// prefill.cu -- the kernels around the prefill matmul (matmul.cu) when a
// prompt of M tokens runs through the decoder at once:
//
//   norm_half_kernel      TensorMath.RmsNorm (Tensors/TensorMath.cs:97-165), one
//                         token per CTA, output rounded to fp16 for the matmul
//   silu_half_kernel      TensorMath.SiluElementwiseMul (TensorMath.cs:253-286),
//                         one token per CTA, output rounded to fp16 for the
//                         down projection
//
// Both scale each token's row by a power of two before rounding to fp16
// (row_pow2_scale) and leave the inverse in inv[t]; the matmul multiplies
// token t's results by it, so activations of any magnitude keep fp16's
// relative precision (SwiGLU products of synthetic weights exceed 65504).
//   attn_prefill_kernel   LlamaModel.ComputeAttention + TensorMath.Softmax
//                         (Models/Llama/LlamaModel.cs:241-346, TensorMath.cs:177-241)
//                         for M queries at positions pos0..pos0+M-1 with causal
//                         masking: flash attention on mma.sync m16n8k16 (fp16
//                         operands, fp32 scores, online softmax in fp32)
//
// ChatNet itself feeds a prompt one token at a time (InferenceEngine.cs:235-239);
// these kernels compute the same per-token results in one pass.
#include <float.h>

#include <mutex>

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

// y[t] = fp16(s_t * RmsNorm(x[t]) * w), the reference's operation order, and
// inv[t] = 1 / s_t; n % 4 == 0.  s_t comes from rms * max|x * w|, the row's
// largest output up to rounding.
__global__ void norm_half_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                 __half* __restrict__ y, float* __restrict__ inv, int n, float eps,
                                 __half* __restrict__ ylo) {
    __shared__ float red[32];
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)blockIdx.x * n);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    uint2* yr = reinterpret_cast<uint2*>(y + (size_t)blockIdx.x * n);
    const int n4 = n / 4;
    float ss = 0.f, xw = 0.f;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const float4 v = xr[i], g = w4[i];
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
        xw = fmaxf(xw, absmax4(make_float4(v.x * g.x, v.y * g.y, v.z * g.z, v.w * g.w)));
    }
    ss = pf_warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) tot += red[i];
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), eps)));
    float sc, iv;
    row_pow2_scale(block_absmax(xw, red) * rms, sc, iv);
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const float4 v = xr[i], g = w4[i];
        const float f0 = __fmul_rn(__fmul_rn(v.x, rms), g.x) * sc, f1 = __fmul_rn(__fmul_rn(v.y, rms), g.y) * sc;
        const float f2 = __fmul_rn(__fmul_rn(v.z, rms), g.z) * sc, f3 = __fmul_rn(__fmul_rn(v.w, rms), g.w) * sc;
        uint2 o;
        o.x = pack_half2(f0, f1);
        o.y = pack_half2(f2, f3);
        yr[i] = o;
        if (ylo) {  // the rounding residuals: y + ylo carries the value to ~2^-22
            const __half2 h01 = *reinterpret_cast<const __half2*>(&o.x), h23 = *reinterpret_cast<const __half2*>(&o.y);
            reinterpret_cast<uint2*>(ylo + (size_t)blockIdx.x * n)[i] =
                make_uint2(pack_half2(f0 - __low2float(h01), f1 - __high2float(h01)),
                           pack_half2(f2 - __low2float(h23), f3 - __high2float(h23)));
        }
    }
    if (threadIdx.x == 0) inv[blockIdx.x] = iv;
}

// h[t] = fp16(s_t * act(g) * u) for token t's row of n values (act: SiLU, or
// GELU with gelu set) and inv[t] = 1 / s_t; n % 4 == 0.  s_t comes from
// max(max(|g|, 0.2785) * |u|), a bound on the row's largest output for both:
// silu(g), gelu(g) <= g for g >= 0, |silu(g)| < 0.2785 and |gelu(g)| < 0.17
// for g < 0.  The second pass re-reads g and u (cache hits).
__global__ void silu_half_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                 __half* __restrict__ h, float* __restrict__ inv, int n, __half* __restrict__ hlo,
                                 int gelu) {
    __shared__ float red[32];
    const size_t base = (size_t)blockIdx.x * n;
    const float4* g4 = reinterpret_cast<const float4*>(g + base);
    const float4* u4 = reinterpret_cast<const float4*>(u + base);
    uint2* h2 = reinterpret_cast<uint2*>(h + base);
    const int n4 = n / 4;
    constexpr float kNegMax = 0.2785f;
    float bound = 0.f;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const float4 a = g4[i], b = u4[i];
        bound = fmaxf(bound, absmax4(make_float4(fmaxf(fabsf(a.x), kNegMax) * b.x, fmaxf(fabsf(a.y), kNegMax) * b.y,
                                                 fmaxf(fabsf(a.z), kNegMax) * b.z, fmaxf(fabsf(a.w), kNegMax) * b.w)));
    }
    float sc, iv;
    row_pow2_scale(block_absmax(bound, red), sc, iv);
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const float4 a = g4[i], b = u4[i];
        const float f0 = act_mul(a.x, b.x, gelu) * sc, f1 = act_mul(a.y, b.y, gelu) * sc;
        const float f2 = act_mul(a.z, b.z, gelu) * sc, f3 = act_mul(a.w, b.w, gelu) * sc;
        const uint2 o = make_uint2(pack_half2(f0, f1), pack_half2(f2, f3));
        h2[i] = o;
        if (hlo) {
            const __half2 h01 = *reinterpret_cast<const __half2*>(&o.x), h23 = *reinterpret_cast<const __half2*>(&o.y);
            reinterpret_cast<uint2*>(hlo + base)[i] =
                make_uint2(pack_half2(f0 - __low2float(h01), f1 - __high2float(h01)),
                           pack_half2(f2 - __low2float(h23), f3 - __high2float(h23)));
        }
    }
    if (threadIdx.x == 0) inv[blockIdx.x] = iv;
}

// fp16(s_t * x[t]) for M rows of n values (the activation operand of
// cn_matmul) and inv[t] = 1 / s_t; n % 4 == 0.
__global__ void half_rows_kernel(const float* __restrict__ x, __half* __restrict__ y, float* __restrict__ inv,
                                 int n) {
    __shared__ float red[32];
    pdl_wait();
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)blockIdx.x * n);
    uint2* yr = reinterpret_cast<uint2*>(y + (size_t)blockIdx.x * n);
    const int n4 = n / 4;
    float amax = 0.f;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) amax = fmaxf(amax, absmax4(xr[i]));
    float sc, iv;
    row_pow2_scale(block_absmax(amax, red), sc, iv);
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const float4 v = xr[i];
        yr[i] = make_uint2(pack_half2(v.x * sc, v.y * sc), pack_half2(v.z * sc, v.w * sc));
    }
    if (threadIdx.x == 0) inv[blockIdx.x] = iv;
}

// TensorMath.ApplyRoPE (interleaved pairs) on the q and k rows of the n prompt
// tokens (token t at position pos0 + t), then k and v into the cache, with
// the decode attention kernels' arithmetic.  Also leaves fp16 copies of the new k and v
// rows in kh/vh [n][kvdim] for the attention kernel.  One CTA per token, four
// values per thread.
__global__ void rope_prefill_kernel(float* __restrict__ q, const float* __restrict__ k,
                                    const float* __restrict__ v, const float2* __restrict__ rope, int pos0,
                                    int qdim, int kvdim, int hd, void* kcache, void* vcache, int64_t cache_off,
                                    int kv_f16, __half* __restrict__ kh, __half* __restrict__ vh,
                                    __half* __restrict__ kl, __half* __restrict__ vl, int neox) {
    const int t = blockIdx.x, pos = pos0 + t;
    const float4* tab = reinterpret_cast<const float4*>(rope + (size_t)pos * (hd / 2));  // two pairs per float4
    const int hd4 = hd / 4;
    float4* q4 = reinterpret_cast<float4*>(q + (size_t)t * qdim);
    const float4* k4 = reinterpret_cast<const float4*>(k + (size_t)t * kvdim);
    const float4* v4 = reinterpret_cast<const float4*>(v + (size_t)t * kvdim);
    const int64_t base = cache_off + (int64_t)pos * kvdim;
    auto rot = [](float4 x, float4 cs) {
        float4 r;
        r.x = __fsub_rn(__fmul_rn(x.x, cs.x), __fmul_rn(x.y, cs.y));
        r.y = __fadd_rn(__fmul_rn(x.x, cs.y), __fmul_rn(x.y, cs.x));
        r.z = __fsub_rn(__fmul_rn(x.z, cs.z), __fmul_rn(x.w, cs.w));
        r.w = __fadd_rn(__fmul_rn(x.z, cs.w), __fmul_rn(x.w, cs.z));
        return r;
    };
    // split-half RoPE (ApplyRoPENeox): element e of a head's first half pairs
    // with e + hd/2 and uses table entry e (the same table)
    const int half = hd / 2;
    const float2* tab2 = rope + (size_t)pos * half;
    auto rot_pairs = [](float4 a, float4 b, const float2* cs, float4& ra, float4& rb) {
        const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
        float r0[4], r1[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            r0[e] = __fsub_rn(__fmul_rn(av[e], cs[e].x), __fmul_rn(bv[e], cs[e].y));
            r1[e] = __fadd_rn(__fmul_rn(av[e], cs[e].y), __fmul_rn(bv[e], cs[e].x));
        }
        ra = make_float4(r0[0], r0[1], r0[2], r0[3]);
        rb = make_float4(r1[0], r1[1], r1[2], r1[3]);
    };
    if (neox) {
        const int hq = half / 4;  // float4 chunks per half head
        for (int i = threadIdx.x; i < (qdim / hd) * hq; i += blockDim.x) {
            float* a = q + (size_t)t * qdim + (i / hq) * hd + 4 * (i % hq);
            float4 ra, rb;
            rot_pairs(*reinterpret_cast<float4*>(a), *reinterpret_cast<float4*>(a + half), tab2 + 4 * (i % hq), ra, rb);
            *reinterpret_cast<float4*>(a) = ra;
            *reinterpret_cast<float4*>(a + half) = rb;
        }
    } else {
        for (int i = threadIdx.x; i < qdim / 4; i += blockDim.x) q4[i] = rot(q4[i], tab[i % hd4]);
    }
    for (int i = threadIdx.x; i < kvdim / 4; i += blockDim.x) {
        float4 kr;
        if (neox) {  // this chunk's elements and their partners in the other half
            const int o = (4 * i) % hd;
            const float* hb = k + (size_t)t * kvdim + (4 * i - o);
            float4 ra, rb;
            const int p = o < half ? o : o - half;
            rot_pairs(*reinterpret_cast<const float4*>(hb + p), *reinterpret_cast<const float4*>(hb + p + half),
                      tab2 + p, ra, rb);
            kr = o < half ? ra : rb;
        } else {
            kr = rot(k4[i], tab[i % hd4]);
        }
        const float4 vv = v4[i];
        const uint2 kp = make_uint2(pack_half2(kr.x, kr.y), pack_half2(kr.z, kr.w));
        const uint2 vp = make_uint2(pack_half2(vv.x, vv.y), pack_half2(vv.z, vv.w));
        if (kv_f16) {
            reinterpret_cast<uint2*>(reinterpret_cast<__half*>(kcache) + base)[i] = kp;
            reinterpret_cast<uint2*>(reinterpret_cast<__half*>(vcache) + base)[i] = vp;
        } else {
            reinterpret_cast<float4*>(reinterpret_cast<float*>(kcache) + base)[i] = kr;
            reinterpret_cast<float4*>(reinterpret_cast<float*>(vcache) + base)[i] = vv;
        }
        reinterpret_cast<uint2*>(kh + (size_t)t * kvdim)[i] = kp;
        reinterpret_cast<uint2*>(vh + (size_t)t * kvdim)[i] = vp;
        if (kl) {  // k's and v's rounding residuals (fp32 caches: the attention splits them)
            const __half2 a = *reinterpret_cast<const __half2*>(&kp.x), b = *reinterpret_cast<const __half2*>(&kp.y);
            reinterpret_cast<uint2*>(kl + (size_t)t * kvdim)[i] =
                make_uint2(pack_half2(kr.x - __low2float(a), kr.y - __high2float(a)),
                           pack_half2(kr.z - __low2float(b), kr.w - __high2float(b)));
            const __half2 c = *reinterpret_cast<const __half2*>(&vp.x), d = *reinterpret_cast<const __half2*>(&vp.y);
            reinterpret_cast<uint2*>(vl + (size_t)t * kvdim)[i] =
                make_uint2(pack_half2(vv.x - __low2float(c), vv.y - __high2float(c)),
                           pack_half2(vv.z - __low2float(d), vv.w - __high2float(d)));
        }
    }
}

// Causal attention for M queries of one sequence.  CTA = (64-query block,
// head), heaviest blocks first; warp w owns queries 16w..16w+15 of the block.
// Keys come in blocks of 64, double-buffered: positions of this prompt
// (>= pos0) from the fp16 copies kh/vh with cp.async, earlier positions from
// the cache (fp32 or fp16, converted in registers).  Query t (position
// pos0 + t) sees keys 0..pos0+t.
constexpr int kPfQ = 64;   // queries per CTA
constexpr int kPfK = 64;   // keys per block
constexpr int kPfThreads = 128;

__device__ __forceinline__ void pf_cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// Loads keys/values p0..p0+63 of kv head kh into Ks/Vs (and, when KLs is
// not null, the keys' fp16 rounding residuals into KLs): positions of this
// prompt (>= pos0) from the fp16 copies with cp.async, earlier ones from the
// cache (converted in registers), positions past `last` as zeros.
template <int HD>
__device__ __forceinline__ void pf_load_kv(__half* Ks, __half* Vs, __half* KLs, __half* VLs, int p0, int last,
                                           int pos0, int kh, const void* kcache, const void* vcache, int kv_f16,
                                           int64_t cache_off, int kvdim, const __half* kh16, const __half* vh16,
                                           const __half* kl16, const __half* vl16) {
    constexpr int RS = HD + 8, C8 = HD / 8;
    for (int i = threadIdx.x; i < kPfK * C8; i += kPfThreads) {
        const int r = i / C8, c = i % C8;
        const int p = p0 + r;
        __half* kd = Ks + r * RS + 8 * c;
        __half* vd = Vs + r * RS + 8 * c;
        __half* ld = KLs ? KLs + r * RS + 8 * c : nullptr;
        __half* lv = VLs ? VLs + r * RS + 8 * c : nullptr;
        if (p > last) {
            *reinterpret_cast<uint4*>(kd) = make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4*>(vd) = make_uint4(0u, 0u, 0u, 0u);
            if (ld) *reinterpret_cast<uint4*>(ld) = make_uint4(0u, 0u, 0u, 0u);
            if (lv) *reinterpret_cast<uint4*>(lv) = make_uint4(0u, 0u, 0u, 0u);
        } else if (p >= pos0) {
            const size_t e = (size_t)(p - pos0) * kvdim + kh * HD + 8 * c;
            pf_cp_async16(smem_u32(kd), kh16 + e);
            pf_cp_async16(smem_u32(vd), vh16 + e);
            if (ld) pf_cp_async16(smem_u32(ld), kl16 + e);
            if (lv) pf_cp_async16(smem_u32(lv), vl16 + e);
        } else {
            const int64_t e = cache_off + (int64_t)p * kvdim + kh * HD + 8 * c;
#pragma unroll
            for (int w = 0; w < 2; w++) {
                const void* base = w == 0 ? kcache : vcache;
                uint4 u;
                if (kv_f16) {
                    u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(base) + e);
                    __half* lo = w == 0 ? ld : lv;
                    if (lo) *reinterpret_cast<uint4*>(lo) = make_uint4(0u, 0u, 0u, 0u);  // exact already
                } else {
                    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + e);
                    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + e + 4);
                    u = make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y),
                                   pack_half2(b.z, b.w));
                    __half* lo = w == 0 ? ld : lv;
                    if (lo) {
                        const __half2* h = reinterpret_cast<const __half2*>(&u);
                        *reinterpret_cast<uint4*>(lo) = make_uint4(
                            pack_half2(a.x - __low2float(h[0]), a.y - __high2float(h[0])),
                            pack_half2(a.z - __low2float(h[1]), a.w - __high2float(h[1])),
                            pack_half2(b.x - __low2float(h[2]), b.y - __high2float(h[2])),
                            pack_half2(b.z - __low2float(h[3]), b.w - __high2float(h[3])));
                    }
                }
                *reinterpret_cast<uint4*>(w == 0 ? kd : vd) = u;
            }
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// SPLIT: the scores use q and k as exact pairs of fp16 halves, S = Qhi Khi +
// Qlo Khi + Qhi Klo (fp32 accumulation), so they carry near-fp32 precision
// into a peaked softmax; Klo is read only for fp32 caches (kl16 / klo on),
// since an fp16 cache holds its keys exactly.  Shared memory holds Q (and
// Qlo), two K, two V (and two Klo) blocks.
template <int HD, bool SPLIT>
__global__ void __launch_bounds__(kPfThreads)
    attn_prefill_kernel(const float* __restrict__ q, int q_stride, const void* __restrict__ kcache,
                        const void* __restrict__ vcache, int kv_f16, int64_t cache_off, int kvdim,
                        int n_heads, int n_kv, int M, int pos0, float scale_log2,
                        const __half* __restrict__ kh16, const __half* __restrict__ vh16,
                        __half* __restrict__ out, int out_stride, const __half* __restrict__ kl16,
                        const __half* __restrict__ vl16, int klo, __half* __restrict__ out_lo) {
    constexpr int RS = HD + 8;  // halves per shared row (16-byte pad: conflict-free ldmatrix)
    constexpr int NT = HD / 8;  // 8-wide column tiles of the output
    constexpr int KS = HD / 16; // k-steps of Q K^T
    constexpr int QR = SPLIT ? 2 * kPfQ : kPfQ;  // rows of Q (and Qlo)
    extern __shared__ __align__(16) uint8_t pf_smem[];
    __half* Qs = reinterpret_cast<__half*>(pf_smem);
    __half* Qls = Qs + kPfQ * RS;
    auto Kb = [&](int i) { return Qs + (QR + i * kPfK) * RS; };
    auto Vb = [&](int i) { return Qs + (QR + (2 + i) * kPfK) * RS; };
    auto KLb = [&](int i) { return (SPLIT && klo) ? Qs + (QR + (4 + i) * kPfK) * RS : (__half*)nullptr; };
    auto VLb = [&](int i) { return (SPLIT && klo) ? Qs + (QR + (6 + i) * kPfK) * RS : (__half*)nullptr; };
    const int qb = gridDim.x - 1 - blockIdx.x, h = blockIdx.y;
    const int kh = h / (n_heads / n_kv);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int t0 = qb * kPfQ;
    const int last = pos0 + min(t0 + kPfQ, M) - 1;  // the block's last query position
    const int nkb = last / kPfK + 1;

    pf_load_kv<HD>(Kb(0), Vb(0), KLb(0), VLb(0), 0, last, pos0, kh, kcache, vcache, kv_f16, cache_off, kvdim, kh16,
                   vh16, kl16, vl16);
    // queries -> fp16 (and their residuals)
    constexpr int C4 = HD / 4;
    for (int i = tid; i < kPfQ * C4; i += kPfThreads) {
        const int r = i / C4, c = i % C4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t0 + r < M) v = *reinterpret_cast<const float4*>(q + (size_t)(t0 + r) * q_stride + h * HD + 4 * c);
        uint2 o;
        o.x = pack_half2(v.x, v.y);
        o.y = pack_half2(v.z, v.w);
        *reinterpret_cast<uint2*>(Qs + r * RS + 4 * c) = o;
        if (SPLIT) {
            const __half2 a = *reinterpret_cast<const __half2*>(&o.x), b = *reinterpret_cast<const __half2*>(&o.y);
            *reinterpret_cast<uint2*>(Qls + r * RS + 4 * c) =
                make_uint2(pack_half2(v.x - __low2float(a), v.y - __high2float(a)),
                           pack_half2(v.z - __low2float(b), v.w - __high2float(b)));
        }
    }
    __syncthreads();
    uint32_t qf[KS][4], qlf[SPLIT ? KS : 1][4];
    {
        const int r = 16 * warp + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
        for (int ks = 0; ks < KS; ks++) {
            ldsm_x4(smem_u32(Qs + r * RS + 16 * ks + 8 * (lane >> 4)), qf[ks]);
            if (SPLIT) ldsm_x4(smem_u32(Qls + r * RS + 16 * ks + 8 * (lane >> 4)), qlf[SPLIT ? ks : 0]);
        }
    }

    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float mrow[2] = {-FLT_MAX, -FLT_MAX}, lrow[2] = {0.f, 0.f};
    const int qpos[2] = {pos0 + t0 + 16 * warp + g, pos0 + t0 + 16 * warp + g + 8};

    for (int kb = 0; kb < nkb; kb++) {
        const int p0 = kb * kPfK;
        __half* Ks = Kb(kb & 1);
        __half* Vs = Vb(kb & 1);
        __half* KLs = KLb(kb & 1);
        __half* VLs = VLb(kb & 1);
        if (kb + 1 < nkb) {
            // the other buffer was last read in block kb - 1 (barrier at its end)
            pf_load_kv<HD>(Kb((kb + 1) & 1), Vb((kb + 1) & 1), KLb((kb + 1) & 1), VLb((kb + 1) & 1), p0 + kPfK, last,
                           pos0, kh, kcache, vcache, kv_f16, cache_off, kvdim, kh16, vh16, kl16, vl16);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
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
                const int koff = key * RS + 16 * ks + 8 * ((lane >> 3) & 1);
                ldsm_x4(smem_u32(Ks + koff), b);
                const uint32_t b0[2] = {b[0], b[1]}, b1[2] = {b[2], b[3]};
                mma_16816(s[2 * jp], qf[ks], b0, s[2 * jp]);
                mma_16816(s[2 * jp + 1], qf[ks], b1, s[2 * jp + 1]);
                if (SPLIT) {
                    mma_16816(s[2 * jp], qlf[SPLIT ? ks : 0], b0, s[2 * jp]);
                    mma_16816(s[2 * jp + 1], qlf[SPLIT ? ks : 0], b1, s[2 * jp + 1]);
                    if (KLs) {
                        uint32_t bl[4];
                        ldsm_x4(smem_u32(KLs + koff), bl);
                        const uint32_t l0[2] = {bl[0], bl[1]}, l1[2] = {bl[2], bl[3]};
                        mma_16816(s[2 * jp], qf[ks], l0, s[2 * jp]);
                        mma_16816(s[2 * jp + 1], qf[ks], l1, s[2 * jp + 1]);
                    }
                }
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
                // rounded to fp16 here, so the normaliser sums exactly the
                // weights P V uses (a common offset of the V rows then passes
                // through unscaled)
                pv[e] = s[j][e] == -FLT_MAX ? 0.f : __half2float(__float2half_rn(exp2f(s[j][e] - mrow[hr])));
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
                const int voff = key * RS + 16 * jp + 8 * (lane >> 4);
                ldsm_x4_t(smem_u32(Vs + voff), b);
                const uint32_t b0[2] = {b[0], b[1]}, b1[2] = {b[2], b[3]};
                mma_16816(o[2 * jp], a, b0, o[2 * jp]);
                mma_16816(o[2 * jp + 1], a, b1, o[2 * jp + 1]);
                if (SPLIT && VLs) {  // fp32 cache: V's residuals as well
                    uint32_t bl[4];
                    ldsm_x4_t(smem_u32(VLs + voff), bl);
                    const uint32_t l0[2] = {bl[0], bl[1]}, l1[2] = {bl[2], bl[3]};
                    mma_16816(o[2 * jp], a, l0, o[2 * jp]);
                    mma_16816(o[2 * jp + 1], a, l1, o[2 * jp + 1]);
                }
            }
        }
        __syncthreads();  // this block's K/V no longer read: its buffer may be refilled
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
        for (int j = 0; j < NT; j++) {
            const float f0 = o[j][2 * hr] * inv, f1 = o[j][2 * hr + 1] * inv;
            const uint32_t hv = pack_half2(f0, f1);
            *reinterpret_cast<uint32_t*>(orow + 8 * j + 2 * t4) = hv;
            if (SPLIT && out_lo) {  // the O projection's low halves
                const __half2 hh = *reinterpret_cast<const __half2*>(&hv);
                *reinterpret_cast<uint32_t*>(out_lo + (size_t)tq * out_stride + h * HD + 8 * j + 2 * t4) =
                    pack_half2(f0 - __low2float(hh), f1 - __high2float(hh));
            }
        }
    }
}

// ---- host side ------------------------------------------------------------------

int prefill_norm(cudaStream_t st, const float* x, const float* w, __half* y, float* inv, int n, int M,
                 float eps, __half* ylo) {
    CN_CHECK(n % 4 == 0 && M >= 1, CN_ERR_INVALID_ARG, "prefill norm: shapes");
    CN_CUDA(launch_k(false, norm_half_kernel, dim3(M), dim3(256), 0, st, x, w, y, inv, n, eps, ylo));
    return CN_OK;
}

int prefill_silu(cudaStream_t st, const float* g, const float* u, __half* h, float* inv, int n, int M,
                 __half* hlo, int gelu) {
    CN_CHECK(n % 4 == 0 && M >= 1, CN_ERR_INVALID_ARG, "prefill silu: shapes");
    CN_CUDA(launch_k(false, silu_half_kernel, dim3(M), dim3(256), 0, st, g, u, h, inv, n, hlo, gelu));
    return CN_OK;
}

int to_half_rows(cudaStream_t st, const float* x, __half* y, float* inv, int n, int M) {
    CN_CHECK(n % 4 == 0 && M >= 1, CN_ERR_INVALID_ARG, "fp16 rows: shapes");
    CN_CUDA(launch_k(false, half_rows_kernel, dim3(M), dim3(256), 0, st, x, y, inv, n));
    return CN_OK;
}

int prefill_rope(cudaStream_t st, float* q, const float* k, const float* v, const float2* rope, int pos0, int M,
                 int qdim, int kvdim, int hd, void* kcache, void* vcache, int64_t cache_off, bool kv_f16, __half* kh,
                 __half* vh, __half* kl, __half* vl, int neox) {
    CN_CHECK(hd % 8 == 0 && qdim % 4 == 0 && kvdim % 4 == 0, CN_ERR_INVALID_ARG, "prefill rope: shapes");
    CN_CHECK(!kl == !vl, CN_ERR_INVALID_ARG, "prefill rope: k and v residuals go together");
    CN_CUDA(launch_k(false, rope_prefill_kernel, dim3(M), dim3(256), 0, st, q, k, v, rope, pos0, qdim, kvdim, hd,
                     kcache, vcache, cache_off, kv_f16 ? 1 : 0, kh, vh, kl, vl, neox));
    return CN_OK;
}

// Shared memory of attn_prefill_kernel: Q [+ Qlo], 2 K, 2 V [+ 2 Klo, 2 Vlo] blocks.
static size_t attn_smem(int hd, bool split, bool klo) {
    const int rows = kPfQ * (split ? 2 : 1) + kPfK * (4 + (split && klo ? 4 : 0));
    return (size_t)rows * (hd + 8) * sizeof(__half);
}

int prefill_attention(cudaStream_t st, const float* q, int q_stride, const void* kcache,
                      const void* vcache, bool kv_f16, int64_t cache_off, int n_heads, int n_kv,
                      int hd, int M, int pos0, const __half* kh, const __half* vh, __half* out, int out_stride,
                      bool split, const __half* kl, const __half* vl, __half* out_lo) {
    CN_CHECK(hd == 64 || hd == 128, CN_ERR_UNSUPPORTED, "prefill attention: head_dim %d", hd);
    CN_CHECK(n_kv > 0 && n_heads % n_kv == 0 && M >= 1 && pos0 >= 0, CN_ERR_INVALID_ARG,
             "prefill attention: bad arguments");
    CN_CHECK(q_stride % 4 == 0 && out_stride % 2 == 0, CN_ERR_INVALID_ARG, "prefill attention: strides");
    CN_CHECK(!split || kv_f16 || (kl && vl), CN_ERR_INVALID_ARG,
             "prefill attention: the split form on an fp32 cache needs k's and v's residuals");
    const bool klo = split && !kv_f16;
    const size_t smem = attn_smem(hd, split, klo);
    {
        int dev = 0;
        CN_CUDA(cudaGetDevice(&dev));
        static std::mutex mu;
        static bool attr[64] = {false};
        std::lock_guard<std::mutex> lock(mu);
        if (!attr[dev & 63]) {
            // the largest layout of each instantiation
            const int f128 = (int)attn_smem(128, false, false), s128 = (int)attn_smem(128, true, true);
            const int f64 = (int)attn_smem(64, false, false), s64 = (int)attn_smem(64, true, true);
            CN_CUDA(cudaFuncSetAttribute(attn_prefill_kernel<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, f128));
            CN_CUDA(cudaFuncSetAttribute(attn_prefill_kernel<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, s128));
            CN_CUDA(cudaFuncSetAttribute(attn_prefill_kernel<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, f64));
            CN_CUDA(cudaFuncSetAttribute(attn_prefill_kernel<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, s64));
            attr[dev & 63] = true;
        }
    }
    const float scale_log2 = 1.4426950408889634f / sqrtf((float)hd);
    const dim3 grid((M + kPfQ - 1) / kPfQ, n_heads);
    const int kvdim = n_kv * hd;
    const int kf = kv_f16 ? 1 : 0, klo_i = klo ? 1 : 0;
#define CN_PF_ATTN(HD, S)                                                                                          \
    CN_CUDA(launch_k(false, attn_prefill_kernel<HD, S>, grid, dim3(kPfThreads), smem, st, q, q_stride, kcache, vcache, \
                     kf, cache_off, kvdim, n_heads, n_kv, M, pos0, scale_log2, kh, vh, out, out_stride, kl, vl, klo_i, \
                     out_lo));
    if (hd == 128) {
        if (split) { CN_PF_ATTN(128, true) } else { CN_PF_ATTN(128, false) }
    } else {
        if (split) { CN_PF_ATTN(64, true) } else { CN_PF_ATTN(64, false) }
    }
#undef CN_PF_ATTN
    return CN_OK;
}

}  // namespace cn
