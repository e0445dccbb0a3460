// noalloc.cu -- the fused dequant-GEMV for callers that cannot allocate
// device memory.
//
// Some hosts own all device memory themselves: a runtime that hands this
// library only pre-registered buffers, code running under a strict memory
// budget or a pool that forbids cudaMalloc/cudaFree after start-up, or a
// host that must not trigger the implicit device synchronisation cudaFree
// causes.  cn_matvec_dev cannot serve them: its context grows scratch
// buffers with cudaMalloc on demand.  cn_matvec_noalloc_dev runs the same
// kernels but takes every scratch byte (activation fragments, per-unit
// scales, stream-K partials and tile counters, the device error word) from
// one fixed array compiled into the library.
//
// Costs and limits, stated for users:
//  * The array, kNoAllocScratchBytes (4 MiB), exists on every GPU that
//    loads the library, for the life of the process.
//  * A call whose scratch would not fit is rejected with CN_ERR_INVALID_ARG
//    before anything is launched.  With batch 1..4 the array fits inner
//    dimensions beyond 100k (every shape of the benchmark configs), with
//    batch 5..8 up to about 45k; batches above 8 need more than it holds.
//  * All calls share the array and it keeps the previous call's contents,
//    so calls whose GPU work overlaps (different streams, or several host
//    threads) race with each other; serialise them.  Each call clears the
//    parts that must start at zero (tile counters, error word) on its stream.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    outside any stream capture.  The address is remembered per device
//    together with the unique id of the CUDA context it was looked up in, so
//    a host that resets the device (cudaDeviceReset) and keeps using the
//    library gets a fresh lookup on its next call (again outside a capture).
//  * The call only enqueues work and does not wait for it, so a kernel that
//    gives up waiting (bounded mbarrier polls) cannot be reported by the call
//    itself: its bit stays in the array's first word.  cn_matvec_noalloc_status
//    waits for the stream, reads and clears that word, and returns
//    CN_ERR_TIMEOUT if it was set -- again without allocating.
#include <mutex>

#include "cn_common.cuh"
#include "cn_internal.h"

namespace cn {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

// The scratch itself.  In host code this name is only a handle: its device
// address comes from cudaGetSymbolAddress, per device.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
struct Slot {
    unsigned long long ctx_id = 0;  // the CUDA context the address belongs to (0: none yet)
    void* addr = nullptr;
};
Slot g_slot[kMaxDevices];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current CUDA context (the device's
// primary context, which the runtime made current); ids are never reused
// within a process, so a reset device shows up as a new id.
int current_ctx_id(unsigned long long* id) {
    static CtxGetCurrentFn get_cur = nullptr;
    static CtxGetIdFn get_id = nullptr;
    if (!get_cur || !get_id) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_cur = reinterpret_cast<CtxGetCurrentFn>(p);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(p);
        CN_CHECK(get_cur && get_id, CN_ERR_CUDA, "driver entry points cuCtxGetCurrent/cuCtxGetId not found");
    }
    CUcontext c = nullptr;
    CN_CHECK(get_cur(&c) == CUDA_SUCCESS && c, CN_ERR_CUDA, "no current CUDA context");
    CN_CHECK(get_id(c, id) == CUDA_SUCCESS, CN_ERR_CUDA, "cuCtxGetId failed");
    return CN_OK;
}

int scratch_address(int device, uint8_t** out) {
    CN_CHECK(device >= 0 && device < kMaxDevices, CN_ERR_INVALID_ARG, "device %d out of range", device);
    std::lock_guard<std::mutex> lock(g_mu);
    // before the runtime's first use of the device no context is current yet;
    // the lookup below creates it
    unsigned long long id = 0;
    const bool have_id = current_ctx_id(&id) == CN_OK;
    Slot& s = g_slot[device];
    if (!have_id || !s.addr || s.ctx_id != id) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
        int rc = current_ctx_id(&id);
        if (rc) return rc;
        s.addr = p;
        s.ctx_id = id;
    }
    *out = static_cast<uint8_t*>(s.addr);
    return CN_OK;
}

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }
}  // namespace

}  // namespace cn

using namespace cn;

extern "C" int cn_matvec_noalloc_dev(int type, const void* d_w, int out_dim, int in_dim,
                                     const float* d_x, float* d_y, int batch, void* stream) {
    CN_CHECK(d_w && d_x && d_y, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK((reinterpret_cast<uintptr_t>(d_x) & 15) == 0 && (reinterpret_cast<uintptr_t>(d_y) & 3) == 0,
             CN_ERR_INVALID_ARG, "x must be 16-byte aligned and y 4-byte aligned");
    int device = 0;
    CN_CUDA(cudaGetDevice(&device));
    uint8_t* base = nullptr;
    int rc = scratch_address(device, &base);
    if (rc) return rc;

    // a stack context: this device, the caller's stream, the error word at
    // the start of the array; nothing here allocates
    cn_ctx c;
    c.device = device;
    CN_CUDA(cudaDeviceGetAttribute(&c.sms, cudaDevAttrMultiProcessorCount, device));
    c.stream = static_cast<cudaStream_t>(stream);
    c.dev_err = reinterpret_cast<uint32_t*>(base);

    GemvOp op;
    rc = gemv_make(&c, type, d_w, out_dim, in_dim, nullptr, batch, &op);
    if (rc) return rc;

    // carve the array: [error word][counters][xinv][xsum][xfrag][partials]
    const GemvPlan& p = op.plan;
    size_t off = 256;
    const size_t counters_off = off;
    off += align256(op.tma ? p.counters * sizeof(int) : 0);
    const size_t xinv_off = off;
    off += align256(op.tma ? p.xinv_bytes : 0);
    const size_t xsum_off = off;
    off += align256(op.tma ? p.xsum_bytes : 0);
    const size_t xfrag_off = off;
    off += align256(op.tma ? p.xfrag_bytes : 0);
    const size_t part_off = off;
    off += align256(op.tma ? p.partial_bytes : 0);
    CN_CHECK(off <= kNoAllocScratchBytes, CN_ERR_INVALID_ARG,
             "matvec [%d x %d] batch %d needs %zu bytes of scratch; the no-alloc entry point "
             "has %zu (use cn_matvec_dev, or a smaller batch or inner dimension)",
             out_dim, in_dim, batch, off, kNoAllocScratchBytes);

    // what must start at zero: the error word and the stream-K tile counters
    CN_CUDA(cudaMemsetAsync(base, 0, counters_off + (op.tma ? p.counters * sizeof(int) : 0),
                            c.stream));
    GemvBufs b;
    b.counters = reinterpret_cast<int*>(base + counters_off);
    b.xinv = reinterpret_cast<float*>(base + xinv_off);
    b.xsum = reinterpret_cast<float*>(base + xsum_off);
    b.xfrag = reinterpret_cast<uint4*>(base + xfrag_off);
    b.partials = reinterpret_cast<float*>(base + part_off);
    rc = gemv_prep(c.stream, c.sms, op, d_x, b);
    if (rc) return rc;
    return gemv_run(&c, c.stream, op, d_x, b, d_y);
}

extern "C" int cn_matvec_noalloc_status(void* stream) {
    int device = 0;
    CN_CUDA(cudaGetDevice(&device));
    uint8_t* base = nullptr;
    int rc = scratch_address(device, &base);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint32_t word = 0;
    CN_CUDA(cudaMemcpyAsync(&word, base, sizeof(word), cudaMemcpyDeviceToHost, s));
    CN_CUDA(cudaStreamSynchronize(s));
    if (word == 0) return CN_OK;
    CN_CUDA(cudaMemsetAsync(base, 0, sizeof(word), s));
    CN_CUDA(cudaStreamSynchronize(s));
    if (word & kErrTimeout)
        return set_error(CN_ERR_TIMEOUT, "a no-alloc GEMV gave up waiting (device error word 0x%x)", word);
    return set_error(CN_ERR_INVALID_ARG, "a no-alloc GEMV rejected its arguments (device error word 0x%x)", word);
}
