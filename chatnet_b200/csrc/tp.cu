// tp.cu -- tensor-parallel exchange buffers shared between GPUs.
//
// One process per GPU.  Each rank allocates one buffer, exports it with a
// CUDA IPC handle, and maps every other rank's buffer after the host has
// passed the handles around.  The GEMVs whose outputs must be combined
// (O and down: partial sums; lm_head: row slices) store into every rank's
// buffer from their epilogue (gemv_i8.cu) and the next kernel on each rank
// reads its own buffer (gemv.cu).  Every exchange has a sequence number,
// step * uses_per_step + use.  The residual partial sums travel as 8-byte
// {value, seq} pairs that the reader checks one by one (no flag, no fence);
// the lm_head slices are plain floats followed by a flag per rank holding
// the sequence number of the last gather that rank completed.  Neither
// needs a reset.
#include <string.h>

#include <new>

#include "cn_common.cuh"
#include "cn_internal.h"

namespace cn {

__global__ void tp_step_kernel(uint32_t* step) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) *step += 1u;
}

int tp_step_launch(const cn_tp* tp, cudaStream_t s) {
    CN_CUDA(launch_k(true, tp_step_kernel, dim3(1), dim3(32), 0, s, tp->step));
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

XchgOut tp_reduce_out(const cn_tp* tp, uint32_t uses, uint32_t use, int done_index) {
    XchgOut x;
    x.size = tp->size;
    x.rank = tp->rank;
    const int64_t per_rank = (int64_t)tp->max_batch * tp->dim;
    x.ll = 1;
    for (int p = 0; p < tp->size; p++) {
        x.dst[p] = reinterpret_cast<float*>(
            reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(tp->peer[p]) + tp->slots_off) + tp->rank * per_rank);
        x.flag[p] = reinterpret_cast<uint32_t*>(tp->peer[p]) + tp->rank;
    }
    x.parity_stride = tp->size * per_rank;
    x.dst_ld = tp->dim;
    x.dst_row0 = 0;
    x.seq_base = tp->step;
    x.uses = uses;
    x.seq_add = use;
    x.done = tp->done + done_index;
    return x;
}

XchgIn tp_reduce_in(const cn_tp* tp, uint32_t uses, uint32_t use, uint32_t* err) {
    XchgIn x;
    x.size = tp->size;
    x.src = reinterpret_cast<const float*>(tp->buf + tp->slots_off);  // 8-byte {value, seq} elements
    x.ll = 1;
    x.rank_stride = (int64_t)tp->max_batch * tp->dim;
    x.parity_stride = tp->size * x.rank_stride;
    x.flags = reinterpret_cast<const uint32_t*>(tp->buf);
    x.seq_base = tp->step;
    x.uses = uses;
    x.seq_add = use;
    x.err = err;
    return x;
}

XchgIn tp_gather_in(const cn_tp* tp, uint32_t uses, uint32_t use, uint32_t* err) {
    XchgIn x = tp_reduce_in(tp, uses, use, err);
    x.ll = 0;
    return x;
}

XchgOut tp_gather_out(const cn_tp* tp, int64_t local_rows, uint32_t uses, uint32_t use, int done_index) {
    XchgOut x = tp_reduce_out(tp, uses, use, done_index);
    x.ll = 0;
    for (int p = 0; p < tp->size; p++)
        x.dst[p] = reinterpret_cast<float*>(static_cast<uint8_t*>(tp->peer[p]) + tp->logits_off);
    x.parity_stride = 0;
    x.dst_ld = tp->vocab;
    x.dst_row0 = tp->rank * local_rows;
    return x;
}

float* tp_logits(const cn_tp* tp) { return reinterpret_cast<float*>(tp->buf + tp->logits_off); }

}  // namespace cn

using namespace cn;

extern "C" {

int cn_tp_create(cn_ctx* ctx, int rank, int size, int max_batch, int dim, int vocab, cn_tp** out) {
    CN_CHECK(ctx && out, CN_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    CN_CHECK(size >= 1 && size <= kMaxTp && rank >= 0 && rank < size, CN_ERR_INVALID_ARG,
             "rank %d of %d (at most %d ranks)", rank, size, kMaxTp);
    CN_CHECK(max_batch >= 1 && dim > 0 && dim % 4 == 0 && vocab > 0 && vocab % size == 0, CN_ERR_INVALID_ARG,
             "bad tensor-parallel sizes");
    cn_tp* t = new (std::nothrow) cn_tp();
    CN_CHECK(t, CN_ERR_OOM, "host allocation failed");
    t->ctx = ctx;
    t->rank = rank;
    t->size = size;
    t->max_batch = max_batch;
    t->dim = dim;
    t->vocab = vocab;
    t->slots_off = 256;
    t->logits_off = t->slots_off + (size_t)2 * size * max_batch * dim * 8;
    t->bytes = t->logits_off + (size_t)max_batch * vocab * 4;
    CN_CUDA(cudaSetDevice(ctx->device));
    cudaError_t e = cudaMalloc(&t->buf, t->bytes);
    if (e == cudaSuccess) e = cudaMemset(t->buf, 0, t->bytes);
    if (e == cudaSuccess) e = cudaMalloc(&t->step, 256);
    if (e == cudaSuccess) e = cudaMemset(t->step, 0, 256);
    if (e == cudaSuccess) e = cudaMalloc(&t->done, 16 * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(t->done, 0, 16 * sizeof(int));
    if (e != cudaSuccess) {
        cudaFree(t->buf);
        cudaFree(t->step);
        cudaFree(t->done);
        delete t;
        return cuda_error(e, "tensor-parallel buffers");
    }
    t->peer[rank] = t->buf;
    *out = t;
    return CN_OK;
}

int cn_tp_handle(const cn_tp* tp, void* handle_out) {
    CN_CHECK(tp && handle_out, CN_ERR_INVALID_ARG, "null argument");
    static_assert(sizeof(cudaIpcMemHandle_t) == CN_TP_HANDLE_BYTES, "IPC handle size");
    CN_CUDA(cudaSetDevice(tp->ctx->device));
    cudaIpcMemHandle_t h;
    CN_CUDA(cudaIpcGetMemHandle(&h, tp->buf));
    memcpy(handle_out, &h, sizeof(h));
    return CN_OK;
}

int cn_tp_connect(cn_tp* tp, const void* handles) {
    CN_CHECK(tp && handles, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(!tp->connected, CN_ERR_INVALID_ARG, "already connected");
    CN_CUDA(cudaSetDevice(tp->ctx->device));
    const uint8_t* hb = static_cast<const uint8_t*>(handles);
    for (int p = 0; p < tp->size; p++) {
        if (p == tp->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + (size_t)p * CN_TP_HANDLE_BYTES, sizeof(h));
        cudaError_t e = cudaIpcOpenMemHandle(&tp->peer[p], h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < p; q++)
                if (q != tp->rank && tp->peer[q]) {
                    cudaIpcCloseMemHandle(tp->peer[q]);
                    tp->peer[q] = nullptr;
                }
            return cuda_error(e, "cudaIpcOpenMemHandle (peer rank buffer)");
        }
    }
    tp->connected = true;
    return CN_OK;
}

int cn_tp_destroy(cn_tp* tp) {
    if (!tp) return CN_OK;
    cudaSetDevice(tp->ctx->device);
    cudaStreamSynchronize(tp->ctx->stream);
    for (int p = 0; p < tp->size; p++)
        if (p != tp->rank && tp->peer[p]) cudaIpcCloseMemHandle(tp->peer[p]);
    cudaFree(tp->buf);
    cudaFree(tp->step);
    cudaFree(tp->done);
    delete tp;
    return CN_OK;
}

}  // extern "C"
