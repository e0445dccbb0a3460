// cn_common.cuh -- shared device helpers for libchatnet_cuda (sm_100a).
//
// Error plumbing, fp16 bit tricks, and thin inline-PTX wrappers for the
// Blackwell primitives the kernels use: mbarrier, TMA tensor loads
// (cp.async.bulk.tensor, never with .multicast), and the mma.sync tensor
// instruction used by the decode GEMVs.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "chatnet_cuda.h"

namespace cn {

// ---------------------------------------------------------------------------
// host-side error reporting (thread-local message, status codes)
// ---------------------------------------------------------------------------
int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);

#define CN_CUDA(call)                                   \
    do {                                                \
        cudaError_t _e = (call);                        \
        if (_e != cudaSuccess) return cn::cuda_error(_e, #call); \
    } while (0)

#define CN_CHECK(cond, code, ...)                               \
    do {                                                        \
        if (!(cond)) return cn::set_error((code), __VA_ARGS__); \
    } while (0)

// Bound on mbarrier / flag polls.  try_wait suspends the thread for a
// hardware time slice per call, so 1<<22 polls is far beyond any TMA load;
// hitting it means the pipeline is broken, and the kernel raises the
// context's error word instead of spinning forever.
constexpr uint32_t kSpinLimit = 1u << 22;

// Device error word bits (written with atomicOr into ctx->dev_err).
enum : uint32_t { kErrTimeout = 1u, kErrBadArg = 2u };

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// Programmatic dependent launch.  A kernel launched with launch_k(pdl = true)
// may start while the previous kernel in the stream is still running: it
// calls pdl_trigger() early (letting its own successor start) and pdl_wait()
// before it touches anything the previous kernel writes or reads; pdl_wait
// returns once that kernel has completed and its memory is visible.  Both
// are no-ops in a kernel launched without the attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Returns true once the phase with the given parity has completed, false if
// the poll bound ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    uint32_t addr = smem_u32(bar);
    for (uint32_t i = 0; i < kSpinLimit; i++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// 2-D TMA tile load into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Like mbar_wait, but each poll may suspend the thread until the phase
// completes (up to ~20 us), so a waiting warp issues few instructions; gives
// up after kWaitLimitNs of wall-clock time.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity) {
    const uint32_t addr = smem_u32(bar);
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity), "r"(20000u)
            : "memory");
        if (done) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// Thread-block clusters (more below): the relaxed arrival on the cluster
// barrier (every thread of the cluster arrives once; a wait returns once all
// have), the address of a shared-memory offset in another CTA of the
// cluster, and a bounded wait on a local mbarrier that other CTAs arrive on.
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
// address of the same shared-memory offset in cluster CTA `rank`
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// bounded wait on a local barrier whose arrivals come from other CTAs of the cluster
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t addr, uint32_t parity) {
    uint32_t done;
    uint64_t t0 = 0;
    for (;;) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if (!t0) t0 = globaltimer_ns();
        else if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// D = A * B + C, m16n8k16, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float* d, const uint32_t* a, const uint32_t* b,
                                          const float* c) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "f"(c[0]),
          "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
    // (a & mask) | orv in one LOP3
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));
    return r;
}

__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// A row's fp16 scaling: the power of two s with amax * s in [2^14, 2^15)
// (clamped to 2^-126..2^126; s = 1 when amax is 0, inf or NaN) and inv = 1/s.
// fp16 then holds the row's largest value well inside its range, and
// multiplying a product by inv is exact.
__device__ __forceinline__ void row_pow2_scale(float amax, float& s, float& inv) {
    const int eb = (int)((__float_as_uint(amax) >> 23) & 0xFFu);  // amax in [2^(eb-127), 2^(eb-126))
    if (!(amax > 0.f) || eb == 255) {
        s = inv = 1.f;
        return;
    }
    int k = 141 - (eb > 0 ? eb : 1);
    k = k < -126 ? -126 : k > 126 ? 126 : k;
    s = __uint_as_float((uint32_t)(k + 127) << 23);
    inv = __uint_as_float((uint32_t)(127 - k) << 23);
}

// Largest of the non-negative v over the block (every thread gets it); red holds 32 floats.
__device__ __forceinline__ float block_absmax(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();  // red may still be read from an earlier reduction
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) m = fmaxf(m, red[i]);
    return m;
}

__device__ __forceinline__ float absmax4(float4 v) {
    return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

// Loads a 32-bit word from shared memory at a 2-byte aligned address.
__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t* p) {
    const int mis = (int)(reinterpret_cast<uintptr_t>(p) & 3);
    // pointer arithmetic (not an integer round trip) keeps the address space
    const uint32_t* w = reinterpret_cast<const uint32_t*>(p - mis);
    if (mis == 0) return w[0];
    return __byte_perm(w[0], w[1], 0x5432);
}

__device__ __forceinline__ uint16_t lds_u16(const uint8_t* p) {
    return *reinterpret_cast<const uint16_t*>(p);
}

// Whether step kernels use programmatic dependent launch (on unless the
// environment sets CHATNET_PDL=0; read once).
bool pdl_enabled();

// Launches kernel<<<grid, block, smem, st>>>(args...), with programmatic
// stream serialization when pdl is set (the kernel must then follow the
// pdl_wait contract above).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// The FFN activation times up, with the reference's operation order:
// SiluElementwiseMul (TensorMath.cs:253-286) g / (1 + exp(-g)) * u, or
// GeluElementwiseMul (TensorMath.cs:294-333)
// 0.5 g (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3))) * u, each evaluated left to
// right with one rounding per operation.
__device__ __forceinline__ float act_mul(float g, float u, int gelu) {
    if (!gelu) return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
    const float c3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, g), g), g);
    const float t = tanhf(__fmul_rn(0.7978845608028654f, __fadd_rn(g, c3)));
    return __fmul_rn(__fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, t)), u);
}

// launch_k with a thread-block cluster of cluster_x CTAs along x (grid.x a
// multiple of it).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_cluster_k(bool pdl, int cluster_x, void (*kernel)(KArgs...), dim3 grid, dim3 block,
                                    size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)cluster_x;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl && pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Thread-block clusters: this CTA's rank, the cluster's size, a peer CTA's
// copy of a shared variable, and the split cluster barrier.
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ float ld_peer_f32(const float* local, uint32_t rank) {
    uint32_t a, v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
    return __uint_as_float(v);
}
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

}  // namespace cn
