// capi.cu -- the C ABI of libchatnet_cuda (declared in include/chatnet_cuda.h).
//
// Every entry point validates its arguments on the host before touching the
// device, returns a status code, and records a message retrievable with
// cn_last_error().  Nothing throws across the boundary.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <new>

#include "cn_common.cuh"
#include "cn_internal.h"
#include "synth.cuh"

namespace cn {

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_error(cudaError_t e, const char* what) {
    int code = (e == cudaErrorMemoryAllocation) ? CN_ERR_OOM : CN_ERR_CUDA;
    return set_error(code, "%s: %s", what, cudaGetErrorString(e));
}

bool type_supported(int type) {
    return type == CN_TYPE_Q4_0 || type == CN_TYPE_Q4_K || type == CN_TYPE_Q6_K ||
           type == CN_TYPE_F32 || type == CN_TYPE_F16 || is_block32(type) || is_superblock(type);
}

uint64_t row_bytes(int type, int64_t cols) { return cn_byte_size(type, (uint64_t)cols); }

int ensure(void** p, size_t* have, size_t need, bool zero) {
    if (need <= *have && *p) return CN_OK;
    size_t cap = need < 4096 ? 4096 : need;
    cap = (cap + 4095) & ~size_t(4095);
    if (*p) {
        // the old buffer may still be read by queued work
        CN_CUDA(cudaDeviceSynchronize());
        CN_CUDA(cudaFree(*p));
        *p = nullptr;
        *have = 0;
    }
    void* q = nullptr;
    CN_CUDA(cudaMalloc(&q, cap));
    if (zero) CN_CUDA(cudaMemset(q, 0, cap));
    *p = q;
    *have = cap;
    return CN_OK;
}

static int check_dev_err(cn_ctx* ctx) {
    uint32_t e = 0;
    CN_CUDA(cudaMemcpy(&e, ctx->dev_err, 4, cudaMemcpyDeviceToHost));
    if (e == 0) return CN_OK;
    CN_CUDA(cudaMemset(ctx->dev_err, 0, 4));
    // a kernel that gave up may have left stream-K tile counters raised
    if (ctx->counters) CN_CUDA(cudaMemset(ctx->counters, 0, ctx->counter_count * sizeof(int)));
    if (e & kErrTimeout)
        return set_error(CN_ERR_TIMEOUT, "a kernel gave up waiting (device error word 0x%x)", e);
    return set_error(CN_ERR_INVALID_ARG, "a kernel rejected its arguments (device error word 0x%x)",
                     e);
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace cn

using namespace cn;

extern "C" {

int cn_abi_version(void) { return CN_ABI_VERSION; }

const char* cn_last_error(void) { return g_err; }

uint64_t cn_byte_size(int type, uint64_t elements) {
    switch (type) {
        case CN_TYPE_F32: return elements * 4;
        case CN_TYPE_F16: return elements * 2;
        case CN_TYPE_Q4_0: return (elements + 31) / 32 * 18;
        case CN_TYPE_Q4_1: return (elements + 31) / 32 * 20;
        case CN_TYPE_Q5_0: return (elements + 31) / 32 * 22;
        case CN_TYPE_Q5_1: return (elements + 31) / 32 * 24;
        case CN_TYPE_Q8_0: return (elements + 31) / 32 * 34;
        case CN_TYPE_Q4_K: return (elements + 255) / 256 * 144;
        case CN_TYPE_Q6_K: return (elements + 255) / 256 * 210;
        case CN_TYPE_IQ4_NL: return (elements + 31) / 32 * 18;
        case CN_TYPE_Q2_K:
        case CN_TYPE_Q3_K:
        case CN_TYPE_Q5_K:
        case CN_TYPE_Q8_K:
        case CN_TYPE_IQ4_XS:
        case CN_TYPE_IQ2_XXS:
        case CN_TYPE_IQ2_XS:
        case CN_TYPE_IQ3_XXS:
        case CN_TYPE_IQ1_S:
        case CN_TYPE_IQ3_S:
        case CN_TYPE_IQ2_S:
        case CN_TYPE_IQ1_M: return (elements + 255) / 256 * superblock_bytes(type);
        default: return 0;
    }
}

int cn_device_count(int* out_count) {
    CN_CHECK(out_count, CN_ERR_INVALID_ARG, "null out_count");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        *out_count = 0;
        return cuda_error(e, "cudaGetDeviceCount");
    }
    *out_count = n;
    return CN_OK;
}

int cn_create(int device, cn_ctx** out) {
    CN_CHECK(out, CN_ERR_INVALID_ARG, "null out");
    *out = nullptr;
    int n = 0;
    CN_CUDA(cudaGetDeviceCount(&n));
    CN_CHECK(device >= 0 && device < n, CN_ERR_INVALID_ARG, "device %d out of range (%d devices)",
             device, n);
    CN_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    CN_CUDA(cudaGetDeviceProperties(&prop, device));
    CN_CHECK(prop.major == 10, CN_ERR_UNSUPPORTED,
             "libchatnet_cuda is built for sm_100a (B200); device %d is sm_%d%d", device,
             prop.major, prop.minor);
    cn_ctx* c = new (std::nothrow) cn_ctx();
    CN_CHECK(c, CN_ERR_OOM, "host allocation failed");
    c->device = device;
    c->sms = prop.multiProcessorCount;
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&c->dev_err, 256);
    if (e == cudaSuccess) e = cudaMemset(c->dev_err, 0, 256);
    if (e != cudaSuccess) {
        if (c->stream) cudaStreamDestroy(c->stream);
        delete c;
        return cuda_error(e, "cn_create");
    }
    *out = c;
    return CN_OK;
}

int cn_destroy(cn_ctx* ctx) {
    if (!ctx) return CN_OK;
    DeviceGuard dg(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->xfrag);
    cudaFree(ctx->xsum);
    cudaFree(ctx->partials);
    cudaFree(ctx->counters);
    cudaFree(ctx->xinv);
    cudaFree(ctx->dstage);
    cudaFree(ctx->xhalf);
    cudaFree(ctx->samp);
    cudaFreeHost(ctx->hstage);
    cudaFree(ctx->dev_err);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return CN_OK;
}

void* cn_ctx_stream(cn_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

int cn_synchronize(cn_ctx* ctx) {
    CN_CHECK(ctx, CN_ERR_INVALID_ARG, "null ctx");
    DeviceGuard dg(ctx->device);
    CN_CUDA(cudaStreamSynchronize(ctx->stream));
    return check_dev_err(ctx);
}

// ---- tensors ----------------------------------------------------------------

static int tensor_alloc(cn_ctx* ctx, int type, int64_t rows, int64_t cols, cn_tensor** out) {
    CN_CHECK(ctx && out, CN_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    CN_CHECK(type_supported(type), CN_ERR_UNSUPPORTED, "Unsupported weight quantization type: %d",
             type);
    CN_CHECK(rows > 0 && cols > 0, CN_ERR_INVALID_ARG, "bad shape [%lld, %lld]", (long long)rows,
             (long long)cols);
    // the kernels index rows and columns with 32-bit ints
    CN_CHECK(rows < (1ll << 31) && cols < (1ll << 31), CN_ERR_INVALID_ARG,
             "shape [%lld, %lld]: rows and columns must be below 2^31", (long long)rows, (long long)cols);
    cn_tensor* t = new (std::nothrow) cn_tensor();
    CN_CHECK(t, CN_ERR_OOM, "host allocation failed");
    t->ctx = ctx;
    t->type = type;
    t->rows = rows;
    t->cols = cols;
    t->row_bytes = row_bytes(type, cols);
    t->bytes = t->row_bytes * (uint64_t)rows;
    cudaError_t e = cudaMalloc(&t->d, t->bytes);
    if (e != cudaSuccess) {
        delete t;
        return cuda_error(e, "cudaMalloc(tensor)");
    }
    if (encode_weight_map(type, t->d, rows, t->row_bytes, &t->map) == CN_OK && cols % 256 == 0)
        t->has_map = true;
    set_error(CN_OK, "");
    *out = t;
    return CN_OK;
}

int cn_tensor_upload(cn_ctx* ctx, const void* host_blocks, uint64_t bytes, int type, int64_t rows,
                     int64_t cols, cn_tensor** out) {
    CN_CHECK(ctx && host_blocks && out, CN_ERR_INVALID_ARG, "null argument");
    DeviceGuard dg(ctx->device);
    uint64_t want = 0;
    CN_CHECK(!__builtin_mul_overflow(row_bytes(type, cols), (uint64_t)(rows > 0 ? rows : 0), &want),
             CN_ERR_INVALID_ARG, "tensor [%lld, %lld] is too large", (long long)rows, (long long)cols);
    CN_CHECK(!type_supported(type) || bytes == want, CN_ERR_INVALID_ARG,
             "tensor bytes %llu != rows * ByteSize(cols) = %llu", (unsigned long long)bytes,
             (unsigned long long)want);
    cn_tensor* t = nullptr;
    int rc = tensor_alloc(ctx, type, rows, cols, &t);
    if (rc) return rc;
    cudaError_t e = cudaMemcpy(t->d, host_blocks, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(t->d);
        delete t;
        return cuda_error(e, "cudaMemcpy(upload)");
    }
    *out = t;
    return CN_OK;
}

int cn_tensor_upload_slice(cn_ctx* ctx, const void* host_blocks, uint64_t bytes, int type, int64_t rows,
                           int64_t cols, int64_t row0, int64_t nrows, int64_t col0, int64_t ncols,
                           cn_tensor** out) {
    CN_CHECK(ctx && host_blocks && out, CN_ERR_INVALID_ARG, "null argument");
    DeviceGuard dg(ctx->device);
    CN_CHECK(type_supported(type), CN_ERR_UNSUPPORTED, "Unsupported weight quantization type: %d", type);
    CN_CHECK(rows > 0 && cols > 0 && row0 >= 0 && nrows > 0 && row0 + nrows <= rows && col0 >= 0 && ncols > 0 &&
                 col0 + ncols <= cols,
             CN_ERR_INVALID_ARG, "slice [%lld+%lld, %lld+%lld] outside [%lld, %lld]", (long long)row0,
             (long long)nrows, (long long)col0, (long long)ncols, (long long)rows, (long long)cols);
    const int64_t blk = type == CN_TYPE_F32 || type == CN_TYPE_F16 ? 1
                        : (type == CN_TYPE_Q4_0 || is_block32(type)) ? 32 : 256;
    CN_CHECK(col0 % blk == 0 && ncols % blk == 0, CN_ERR_INVALID_ARG,
             "column slice must cover whole %lld-weight blocks", (long long)blk);
    const uint64_t rb = row_bytes(type, cols);
    uint64_t want = 0;
    CN_CHECK(!__builtin_mul_overflow(rb, (uint64_t)rows, &want) && bytes == want, CN_ERR_INVALID_ARG,
             "tensor bytes %llu != rows * ByteSize(cols) = %llu", (unsigned long long)bytes,
             (unsigned long long)want);
    const uint64_t off = row_bytes(type, col0);  // the slice's first byte within a row
    cn_tensor* t = nullptr;
    int rc = tensor_alloc(ctx, type, nrows, ncols, &t);
    if (rc) return rc;
    const uint8_t* src = static_cast<const uint8_t*>(host_blocks) + (uint64_t)row0 * rb + off;
    cudaError_t e = cudaMemcpy2D(t->d, t->row_bytes, src, rb, t->row_bytes, (size_t)nrows, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(t->d);
        delete t;
        return cuda_error(e, "cudaMemcpy2D(upload slice)");
    }
    *out = t;
    return CN_OK;
}

int cn_tensor_synth(cn_ctx* ctx, int type, int64_t rows, int64_t cols, uint64_t seed, int dist,
                    cn_tensor** out) {
    CN_CHECK(ctx && out, CN_ERR_INVALID_ARG, "null argument");
    DeviceGuard dg(ctx->device);
    cn_tensor* t = nullptr;
    int rc = tensor_alloc(ctx, type, rows, cols, &t);
    if (rc) return rc;
    rc = synth_launch(type, rows, cols, seed, dist, t->d, ctx->stream);
    if (rc == CN_OK) {
        cudaError_t e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) rc = cuda_error(e, "synth");
    }
    if (rc) {
        cudaFree(t->d);
        delete t;
        return rc;
    }
    *out = t;
    return CN_OK;
}

int cn_tensor_synth_slice(cn_ctx* ctx, int type, int64_t rows, int64_t cols, int64_t row0, int64_t nrows,
                          int64_t col0, int64_t ncols, uint64_t seed, int dist, cn_tensor** out) {
    CN_CHECK(ctx && out, CN_ERR_INVALID_ARG, "null argument");
    DeviceGuard dg(ctx->device);
    cn_tensor* t = nullptr;
    int rc = tensor_alloc(ctx, type, nrows, ncols, &t);
    if (rc) return rc;
    rc = synth_slice_launch(type, rows, cols, row0, nrows, col0, ncols, seed, dist, t->d, ctx->stream);
    if (rc == CN_OK) {
        cudaError_t e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) rc = cuda_error(e, "synth");
    }
    if (rc) {
        cudaFree(t->d);
        delete t;
        return rc;
    }
    *out = t;
    return CN_OK;
}

int cn_tensor_download(const cn_tensor* t, void* host, uint64_t bytes) {
    CN_CHECK(t && host, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(bytes == t->bytes, CN_ERR_INVALID_ARG, "download size %llu != tensor size %llu",
             (unsigned long long)bytes, (unsigned long long)t->bytes);
    DeviceGuard dg(t->ctx->device);
    CN_CUDA(cudaStreamSynchronize(t->ctx->stream));
    CN_CUDA(cudaMemcpy(host, t->d, bytes, cudaMemcpyDeviceToHost));
    return CN_OK;
}

int cn_tensor_free(cn_tensor* t) {
    if (!t) return CN_OK;
    DeviceGuard dg(t->ctx->device);
    cudaStreamSynchronize(t->ctx->stream);
    if (t->owns) cudaFree(t->d);
    delete t;
    return CN_OK;
}

const void* cn_tensor_device_ptr(const cn_tensor* t) { return t ? t->d : nullptr; }
uint64_t cn_tensor_bytes(const cn_tensor* t) { return t ? t->bytes : 0; }

// ---- synthetic inputs (host) -------------------------------------------------

uint64_t cn_synth_seed(int config_id, const char* name) {
    uint64_t h = 0xcbf29ce484222325ull;  // FNV-1a 64
    for (const char* p = name ? name : ""; *p; p++) {
        h ^= (uint8_t)*p;
        h *= 0x100000001b3ull;
    }
    return synth::mix64(h ^ ((uint64_t)(uint32_t)config_id * synth::kGolden));
}

int cn_synth_fill(int type, int64_t rows, int64_t cols, uint64_t seed, int dist, void* host,
                  uint64_t bytes) {
    CN_CHECK(host, CN_ERR_INVALID_ARG, "null host buffer");
    CN_CHECK(rows >= 0 && cols >= 0, CN_ERR_INVALID_ARG, "negative shape");
    CN_CHECK(type_supported(type), CN_ERR_UNSUPPORTED, "no generator for type %d", type);
    uint64_t want = row_bytes(type, cols) * (uint64_t)rows;
    CN_CHECK(bytes == want, CN_ERR_INVALID_ARG, "buffer bytes %llu != %llu",
             (unsigned long long)bytes, (unsigned long long)want);
    uint8_t* out = static_cast<uint8_t*>(host);
    const int64_t n = rows * cols;
    switch (type) {
        case CN_TYPE_Q4_0:
            CN_CHECK(dist == CN_DIST_CFG0_Q4_0 && cols % 32 == 0, CN_ERR_INVALID_ARG,
                     "bad Q4_0 request");
            for (int64_t b = 0; b < n / 32; b++) synth::q4_0_block(seed, b, out + b * 18);
            return CN_OK;
        case CN_TYPE_Q4_K:
            CN_CHECK(dist == CN_DIST_CFG2_Q4_K && cols % 256 == 0, CN_ERR_INVALID_ARG,
                     "bad Q4_K request");
            for (int64_t b = 0; b < n / 256; b++) synth::q4_k_block(seed, b, out + b * 144);
            return CN_OK;
        case CN_TYPE_Q6_K:
            CN_CHECK(dist == CN_DIST_CFG2_Q6_K && cols % 256 == 0, CN_ERR_INVALID_ARG,
                     "bad Q6_K request");
            for (int64_t b = 0; b < n / 256; b++) synth::q6_k_block(seed, b, out + b * 210);
            return CN_OK;
        case CN_TYPE_F32: {
            CN_CHECK(dist == CN_DIST_NORMAL || dist == CN_DIST_NORM_W, CN_ERR_INVALID_ARG,
                     "bad F32 distribution");
            float* f = reinterpret_cast<float*>(out);
            for (int64_t i = 0; i < n; i++)
                f[i] = dist == CN_DIST_NORM_W ? synth::norm_weight_elem(seed, i)
                                              : synth::normal_elem(seed, i);
            return CN_OK;
        }
        case CN_TYPE_F16: {
            CN_CHECK(dist == CN_DIST_NORMAL, CN_ERR_INVALID_ARG, "bad F16 distribution");
            uint16_t* h = reinterpret_cast<uint16_t*>(out);
            for (int64_t i = 0; i < n; i++) h[i] = synth::f2h(synth::normal_elem(seed, i));
            return CN_OK;
        }
    }
    return set_error(CN_ERR_UNSUPPORTED, "no generator for type %d", type);
}

// ---- op level -----------------------------------------------------------------

static int stage(cn_ctx* ctx, size_t dev_bytes) {
    return ensure(&ctx->dstage, &ctx->dstage_bytes, dev_bytes, false);
}

int cn_dequantize(cn_ctx* ctx, const cn_tensor* W, int64_t row0, int64_t nrows, float* host_out) {
    CN_CHECK(ctx && W && host_out, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(row0 >= 0 && nrows >= 0 && row0 + nrows <= W->rows, CN_ERR_INVALID_ARG,
             "rows [%lld, %lld) outside [0, %lld)", (long long)row0, (long long)(row0 + nrows),
             (long long)W->rows);
    if (nrows == 0) return CN_OK;
    DeviceGuard dg(ctx->device);
    size_t out_bytes = (size_t)nrows * W->cols * sizeof(float);
    int rc = stage(ctx, out_bytes);
    if (rc) return rc;
    const uint8_t* src = static_cast<const uint8_t*>(W->d) + (size_t)row0 * W->row_bytes;
    float* d_out = static_cast<float*>(ctx->dstage);
    if (W->type == CN_TYPE_Q4_0 && W->cols % 32 != 0) {
        // rows are separate Dequantize calls: each ends with a partial block
        for (int64_t r = 0; r < nrows; r++) {
            rc = dequant_launch(W->type, src + r * W->row_bytes, d_out + r * W->cols, W->cols,
                                ctx->stream);
            if (rc) return rc;
        }
    } else if ((W->type == CN_TYPE_Q4_K || W->type == CN_TYPE_Q6_K) && W->cols % 256 != 0) {
        return set_error(CN_ERR_INVALID_ARG, "K-quant rows must hold whole super-blocks");
    } else {
        rc = dequant_launch(W->type, src, d_out, nrows * W->cols, ctx->stream,
                            static_cast<const uint8_t*>(W->d) + W->bytes);
        if (rc) return rc;
    }
    CN_CUDA(cudaMemcpyAsync(host_out, d_out, out_bytes, cudaMemcpyDeviceToHost, ctx->stream));
    CN_CUDA(cudaStreamSynchronize(ctx->stream));
    return check_dev_err(ctx);
}

int cn_matvec(cn_ctx* ctx, const cn_tensor* W, const float* host_x, float* host_y, int batch) {
    CN_CHECK(ctx && W && host_x && host_y, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(batch >= 1 && batch <= 32, CN_ERR_INVALID_ARG, "batch %d outside [1, 32]", batch);
    DeviceGuard dg(ctx->device);
    size_t xb = (size_t)batch * W->cols * sizeof(float);
    size_t yb = (size_t)batch * W->rows * sizeof(float);
    size_t xoff = 0, yoff = (xb + 255) & ~size_t(255);
    int rc = stage(ctx, yoff + yb);
    if (rc) return rc;
    float* dx = reinterpret_cast<float*>(static_cast<uint8_t*>(ctx->dstage) + xoff);
    float* dy = reinterpret_cast<float*>(static_cast<uint8_t*>(ctx->dstage) + yoff);
    CN_CUDA(cudaMemcpyAsync(dx, host_x, xb, cudaMemcpyHostToDevice, ctx->stream));
    rc = gemv_launch(ctx, W->type, W->d, W->rows, W->cols, W->has_map ? &W->map : nullptr, dx, dy,
                     batch);
    if (rc) return rc;
    CN_CUDA(cudaMemcpyAsync(host_y, dy, yb, cudaMemcpyDeviceToHost, ctx->stream));
    CN_CUDA(cudaStreamSynchronize(ctx->stream));
    return check_dev_err(ctx);
}

static int matmul_dev(cn_ctx* ctx, int type, const void* d_w, int64_t rows, int64_t cols,
                      const float* d_x, float* d_y, int n_tokens, const CUtensorMap* wmap_opt = nullptr) {
    CN_CHECK(matmul_type_ok(type), CN_ERR_UNSUPPORTED, "matmul: type %d not supported (Q4_0, Q4_K)", type);
    CN_CHECK(n_tokens >= 1 && rows >= 1 && cols >= 256 && cols % 256 == 0, CN_ERR_INVALID_ARG,
             "matmul: bad shape (%lld x %lld, %d tokens)", (long long)rows, (long long)cols, n_tokens);
    // fp16 rows of x (each scaled by a power of two), then their inverse scales
    const size_t hb = (size_t)n_tokens * cols * sizeof(__half);
    int rc = ensure(&ctx->xhalf, &ctx->xhalf_bytes, hb + (size_t)n_tokens * sizeof(float), false);
    if (rc) return rc;
    __half* xh = static_cast<__half*>(ctx->xhalf);
    float* xs = reinterpret_cast<float*>(static_cast<uint8_t*>(ctx->xhalf) + hb);
    rc = to_half_rows(ctx->stream, d_x, xh, xs, (int)cols, n_tokens);
    if (rc) return rc;
    const int64_t ldy = rows;
    return matmul_quant(ctx->stream, ctx->dev_err, type, 1, &d_w, wmap_opt ? &wmap_opt : nullptr, &rows, cols,
                        xh, xs, n_tokens, &d_y, &ldy, false);
}

int cn_matmul(cn_ctx* ctx, const cn_tensor* W, const float* host_x, float* host_y, int n_tokens) {
    CN_CHECK(ctx && W && host_x && host_y, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(n_tokens >= 1, CN_ERR_INVALID_ARG, "n_tokens %d < 1", n_tokens);
    DeviceGuard dg(ctx->device);
    size_t xb = (size_t)n_tokens * W->cols * sizeof(float);
    size_t yb = (size_t)n_tokens * W->rows * sizeof(float);
    size_t yoff = (xb + 255) & ~size_t(255);
    int rc = stage(ctx, yoff + yb);
    if (rc) return rc;
    float* dx = reinterpret_cast<float*>(ctx->dstage);
    float* dy = reinterpret_cast<float*>(static_cast<uint8_t*>(ctx->dstage) + yoff);
    CN_CUDA(cudaMemcpyAsync(dx, host_x, xb, cudaMemcpyHostToDevice, ctx->stream));
    rc = matmul_dev(ctx, W->type, W->d, W->rows, W->cols, dx, dy, n_tokens, W->has_map ? &W->map : nullptr);
    if (rc) return rc;
    CN_CUDA(cudaMemcpyAsync(host_y, dy, yb, cudaMemcpyDeviceToHost, ctx->stream));
    CN_CUDA(cudaStreamSynchronize(ctx->stream));
    return check_dev_err(ctx);
}

// ---- device level --------------------------------------------------------------

int cn_matmul_dev(cn_ctx* ctx, int type, const void* d_w, int out_dim, int in_dim,
                  const float* d_x, float* d_y, int n_tokens) {
    CN_CHECK(ctx && d_w && d_x && d_y, CN_ERR_INVALID_ARG, "null argument");
    DeviceGuard dg(ctx->device);
    return matmul_dev(ctx, type, d_w, out_dim, in_dim, d_x, d_y, n_tokens);
}

int cn_dequantize_dev(int type, const void* d_blocks, float* d_out, int64_t n_elements,
                      void* stream) {
    return dequant_launch(type, d_blocks, d_out, n_elements, (cudaStream_t)stream);
}

int cn_matvec_dev(cn_ctx* ctx, int type, const void* d_w, int out_dim, int in_dim,
                  const float* d_x, float* d_y, int batch) {
    CN_CHECK(ctx && d_w && d_x && d_y, CN_ERR_INVALID_ARG, "null argument");
    DeviceGuard dg(ctx->device);
    return gemv_launch(ctx, type, d_w, out_dim, in_dim, nullptr, d_x, d_y, batch);
}

int cn_time_matvec(cn_ctx* ctx, const cn_tensor* const* ws, int n_w, const float* d_x, float* d_y, int batch,
                   int launches, int reps, float* us_out, int* kernels_per_launch) {
    CN_CHECK(ctx && ws && d_x && d_y && us_out, CN_ERR_INVALID_ARG, "null argument");
    DeviceGuard dg(ctx->device);
    int rc = gemv_time(ctx, ws, n_w, d_x, d_y, batch, launches, reps, us_out, kernels_per_launch);
    if (rc) return rc;
    return check_dev_err(ctx);
}

}  // extern "C"
