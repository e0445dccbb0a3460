"""chatnet_b200 -- B200-native engine for ChatNet's quantized-weight hot path.

The compute lives in libchatnet_cuda (CUDA, sm_100a) behind a C ABI
(include/chatnet_cuda.h).  This package is the Python host side of that ABI:
thin RAII wrappers (Context, Tensor) plus mirrors of the reference's
operator interface (tensor_math.TensorMath, llama.CudaLlamaModel) so tests
and tools can drive the library the way ChatNet's C# host does.
"""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np

from . import _native as N
from ._native import (CudaError, NotSupportedError, TYPE_F16, TYPE_F32, TYPE_Q4_0, TYPE_Q4_K,
                      TYPE_Q6_K, TYPE_Q4_1, TYPE_Q5_0, TYPE_Q5_1, TYPE_Q8_0, TYPE_Q2_K, TYPE_Q3_K, TYPE_Q5_K,
                      TYPE_Q8_K, TYPE_IQ4_NL, TYPE_IQ4_XS, TYPE_IQ2_XXS, TYPE_IQ2_XS, TYPE_IQ3_XXS,
                      TYPE_IQ1_S, TYPE_IQ3_S, TYPE_IQ2_S, TYPE_IQ1_M, DIST_CFG0_Q4_0, DIST_CFG2_Q4_K, DIST_CFG2_Q6_K, DIST_NORMAL,
                      DIST_NORM_W, check, byte_size)

__all__ = [
    "Context", "Tensor", "CudaError", "NotSupportedError", "check", "byte_size", "synth_fill",
    "synth_seed", "device_count", "TYPE_F32", "TYPE_F16", "TYPE_Q4_0", "TYPE_Q4_K", "TYPE_Q6_K",
    "TYPE_Q4_1", "TYPE_Q5_0", "TYPE_Q5_1", "TYPE_Q8_0", "TYPE_Q2_K", "TYPE_Q3_K", "TYPE_Q5_K", "TYPE_Q8_K",
    "TYPE_IQ4_NL", "TYPE_IQ4_XS", "TYPE_IQ2_XXS", "TYPE_IQ2_XS", "TYPE_IQ3_XXS", "TYPE_IQ1_S", "TYPE_IQ3_S",
    "TYPE_IQ2_S", "TYPE_IQ1_M",
    "DIST_CFG0_Q4_0", "DIST_CFG2_Q4_K", "DIST_CFG2_Q6_K", "DIST_NORMAL", "DIST_NORM_W",
]

_DEFAULT_DIST = {TYPE_Q4_0: DIST_CFG0_Q4_0, TYPE_Q4_K: DIST_CFG2_Q4_K, TYPE_Q6_K: DIST_CFG2_Q6_K}


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def device_count() -> int:
    n = C.c_int(0)
    rc = N.lib().cn_device_count(C.byref(n))
    return n.value if rc == 0 else 0


def synth_seed(config_id: int, name: str) -> int:
    return int(N.lib().cn_synth_seed(config_id, name.encode()))


def synth_fill(type_: int, rows: int, cols: int, seed: int, dist: int | None = None) -> np.ndarray:
    """Host bytes of a synthetic tensor (identical to what the device generator writes)."""
    if dist is None:
        dist = _DEFAULT_DIST.get(type_, DIST_NORMAL)
    nbytes = byte_size(type_, cols) * rows
    out = np.empty(nbytes, dtype=np.uint8)
    check(N.lib().cn_synth_fill(type_, rows, cols, seed, dist, out.ctypes.data, nbytes),
          "cn_synth_fill")
    if type_ == TYPE_F32:
        return out.view(np.float32).reshape(rows, cols)
    if type_ == TYPE_F16:
        return out.view(np.float16).reshape(rows, cols)
    return out.reshape(rows, -1)


class Tensor:
    """A weight tensor resident in HBM (GGUF block bytes, untouched)."""

    def __init__(self, ctx: "Context", handle: int, type_: int, rows: int, cols: int):
        self.ctx, self.handle, self.type, self.rows, self.cols = ctx, handle, type_, rows, cols

    @property
    def nbytes(self) -> int:
        return int(N.lib().cn_tensor_bytes(self.handle))

    @property
    def device_ptr(self) -> int:
        return int(N.lib().cn_tensor_device_ptr(self.handle))

    def download(self) -> np.ndarray:
        out = np.empty(self.nbytes, dtype=np.uint8)
        check(N.lib().cn_tensor_download(self.handle, out.ctypes.data, out.nbytes), "download")
        return out

    def free(self) -> None:
        if self.handle:
            N.lib().cn_tensor_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Context:
    """One device, one stream, the scratch the kernels need (cn_create)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(N.lib().cn_create(device, C.byref(h)), "cn_create")
        self.handle = h.value
        self.device = device
        self._tensors: "weakref.WeakSet[Tensor]" = weakref.WeakSet()
        # decoders built on this context (closed before it, since they use its stream)
        self._models: weakref.WeakSet = weakref.WeakSet()

    def _own(self, t: "Tensor") -> "Tensor":
        self._tensors.add(t)
        return t

    @property
    def stream(self) -> int:
        return int(N.lib().cn_ctx_stream(self.handle) or 0)

    def synchronize(self) -> None:
        check(N.lib().cn_synchronize(self.handle), "cn_synchronize")

    def upload(self, blocks: np.ndarray, type_: int, rows: int, cols: int) -> Tensor:
        buf = np.ascontiguousarray(blocks).view(np.uint8).reshape(-1)
        h = C.c_void_p()
        check(N.lib().cn_tensor_upload(self.handle, buf.ctypes.data, buf.nbytes, type_, rows, cols,
                                       C.byref(h)), "cn_tensor_upload")
        return self._own(Tensor(self, h.value, type_, rows, cols))

    def upload_slice(self, blocks: np.ndarray, type_: int, rows: int, cols: int, row0: int, nrows: int,
                     col0: int, ncols: int) -> Tensor:
        """Region [row0, row0+nrows) x [col0, col0+ncols) (whole blocks) of the
        host tensor `blocks` ([rows][ByteSize(cols)] bytes): a tensor-parallel shard."""
        buf = np.ascontiguousarray(blocks).view(np.uint8).reshape(-1)
        h = C.c_void_p()
        check(N.lib().cn_tensor_upload_slice(self.handle, buf.ctypes.data, buf.nbytes, type_, rows, cols, row0,
                                             nrows, col0, ncols, C.byref(h)), "cn_tensor_upload_slice")
        return self._own(Tensor(self, h.value, type_, nrows, ncols))

    def synth(self, type_: int, rows: int, cols: int, seed: int, dist: int | None = None) -> Tensor:
        if dist is None:
            dist = _DEFAULT_DIST.get(type_, DIST_NORMAL)
        h = C.c_void_p()
        check(N.lib().cn_tensor_synth(self.handle, type_, rows, cols, seed, dist, C.byref(h)),
              "cn_tensor_synth")
        return self._own(Tensor(self, h.value, type_, rows, cols))

    def synth_slice(self, type_: int, rows: int, cols: int, row0: int, nrows: int, col0: int, ncols: int,
                    seed: int, dist: int | None = None) -> Tensor:
        """Region [row0, row0+nrows) x [col0, col0+ncols) of what synth(type_, rows, cols, seed)
        would generate (a tensor-parallel shard), generated in place."""
        if dist is None:
            dist = _DEFAULT_DIST.get(type_, DIST_NORMAL)
        h = C.c_void_p()
        check(N.lib().cn_tensor_synth_slice(self.handle, type_, rows, cols, row0, nrows, col0, ncols, seed,
                                            dist, C.byref(h)), "cn_tensor_synth_slice")
        return self._own(Tensor(self, h.value, type_, nrows, ncols))

    def dequantize(self, W: Tensor, row0: int = 0, nrows: int | None = None) -> np.ndarray:
        if nrows is None:
            nrows = W.rows - row0
        out = np.empty((nrows, W.cols), dtype=np.float32)
        check(N.lib().cn_dequantize(self.handle, W.handle, row0, nrows, _fptr(out)),
              "cn_dequantize")
        return out

    def matvec(self, W: Tensor, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        squeeze = x.ndim == 1
        x2 = x.reshape(-1, W.cols)
        y = np.empty((x2.shape[0], W.rows), dtype=np.float32)
        check(N.lib().cn_matvec(self.handle, W.handle, _fptr(x2), _fptr(y), x2.shape[0]),
              "cn_matvec")
        return y[0] if squeeze else y

    def matmul(self, W: Tensor, x: np.ndarray) -> np.ndarray:
        """Prefill matmul (cn_matmul): y[t] = W x[t] for every row t of x."""
        x2 = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, W.cols)
        y = np.empty((x2.shape[0], W.rows), dtype=np.float32)
        check(N.lib().cn_matmul(self.handle, W.handle, _fptr(x2), _fptr(y), x2.shape[0]), "cn_matmul")
        return y

    def sample_dev(self, d_logits: int, vocab: int, batch: int, temperature: float, top_k: int = 40,
                   top_p: float = 0.9, r=None) -> np.ndarray:
        """TemperatureSampler.Sample on device logits [batch][vocab] (cn_sample_dev)."""
        rr = np.ascontiguousarray(np.zeros(batch) if r is None else r, dtype=np.float32)
        out = np.empty(batch, dtype=np.int32)
        check(N.lib().cn_sample_dev(self.handle, C.c_void_p(d_logits), vocab, batch, float(temperature),
                                    int(top_k), float(top_p), rr.ctypes.data, out.ctypes.data), "cn_sample_dev")
        return out

    def close(self) -> None:
        if self.handle:
            for m in list(self._models):
                m.close()
            for t in list(self._tensors):
                t.free()
            N.lib().cn_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TensorParallel:
    """This process's rank of a tensor-parallel group (cn_tp_*): one process
    per GPU; the exchange buffers are shared between GPUs with CUDA IPC."""

    def __init__(self, ctx: Context, rank: int, size: int, max_batch: int, dim: int, vocab: int):
        h = C.c_void_p()
        check(N.lib().cn_tp_create(ctx.handle, rank, size, max_batch, dim, vocab, C.byref(h)), "cn_tp_create")
        self.handle, self.rank, self.size = h.value, rank, size

    def ipc_handle(self) -> bytes:
        buf = (C.c_uint8 * N.TP_HANDLE_BYTES)()
        check(N.lib().cn_tp_handle(self.handle, buf), "cn_tp_handle")
        return bytes(buf)

    def connect(self, handles: list[bytes]) -> None:
        """handles: every rank's ipc_handle(), in rank order."""
        assert len(handles) == self.size and all(len(h) == N.TP_HANDLE_BYTES for h in handles)
        blob = b"".join(handles)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        check(N.lib().cn_tp_connect(self.handle, buf), "cn_tp_connect")

    def close(self) -> None:
        if self.handle:
            N.lib().cn_tp_destroy(self.handle)
            self.handle = None
