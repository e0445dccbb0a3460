"""GGUF files (cn_gguf_*): the host side of GgufReader + MemoryMappedWeights.

    GgufReader(path).Load()            (Gguf/GgufReader.cs:34-75)   -> GgufFile(path)
    GgufReader.ExtractModelConfig()    (GgufReader.cs:80-176)       -> GgufFile.llama_config()
    MemoryMappedWeights.GetTensorInfo  (Memory/MemoryMappedWeights.cs:63)
                                                                    -> GgufFile.tensors / .info(name)
    LlamaWeights + LlamaModel ctor     (Models/Llama/LlamaWeights.cs:78-145)
                                                                    -> GgufFile.llama_model(ctx, ...)
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _native as N
from ._native import check
from .llama import CudaLlamaModel, LlamaConfig


@dataclass(frozen=True)
class TensorInfo:
    name: str
    type: int
    dims: tuple      # innermost first, as stored
    bytes: int
    file_offset: int

    @property
    def shape(self) -> tuple[int, int]:
        """[rows, cols] as uploaded: cols = dims[0], rows = the product of the rest."""
        rows = 1
        for d in self.dims[1:]:
            rows *= d
        return rows, self.dims[0]


class GgufFile:
    def __init__(self, path: str):
        h = C.c_void_p()
        check(N.lib().cn_gguf_open(str(path).encode(), C.byref(h)), "cn_gguf_open")
        self.handle = h.value
        n = C.c_int(0)
        check(N.lib().cn_gguf_tensor_count(self.handle, C.byref(n)), "cn_gguf_tensor_count")
        self.tensors = [self._info(i) for i in range(n.value)]

    def _info(self, i: int) -> TensorInfo:
        name, t, nd = C.c_char_p(), C.c_int(0), C.c_int(0)
        dims = (C.c_uint64 * 4)()
        nb, off = C.c_uint64(0), C.c_uint64(0)
        check(N.lib().cn_gguf_tensor_info(self.handle, i, C.byref(name), C.byref(t), C.byref(nd), dims,
                                          C.byref(nb), C.byref(off)), "cn_gguf_tensor_info")
        return TensorInfo(name.value.decode(), t.value, tuple(dims[d] for d in range(nd.value)), nb.value,
                          off.value)

    def info(self, name: str) -> TensorInfo:
        i = C.c_int(0)
        check(N.lib().cn_gguf_find(self.handle, name.encode(), C.byref(i)), "cn_gguf_find")
        return self.tensors[i.value]

    def get_int(self, key: str) -> int:
        v = C.c_int64(0)
        check(N.lib().cn_gguf_get_int(self.handle, key.encode(), C.byref(v)), "cn_gguf_get_int")
        return v.value

    def get_float(self, key: str) -> float:
        v = C.c_double(0)
        check(N.lib().cn_gguf_get_float(self.handle, key.encode(), C.byref(v)), "cn_gguf_get_float")
        return v.value

    def get_string(self, key: str) -> str:
        v = C.c_char_p()
        check(N.lib().cn_gguf_get_string(self.handle, key.encode(), C.byref(v)), "cn_gguf_get_string")
        return v.value.decode()

    def llama_config(self, max_batch: int = 1, kv_f16: bool = False) -> LlamaConfig:
        c = N.LlamaConfigC()
        check(N.lib().cn_gguf_llama_config(self.handle, C.byref(c)), "cn_gguf_llama_config")
        return LlamaConfig(c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.vocab,
                           c.ctx_len, c.rope_base, c.rms_eps, kv_f16, max_batch)

    def upload(self, ctx, name: str):
        from . import Tensor
        h = C.c_void_p()
        check(N.lib().cn_gguf_upload(ctx.handle, self.handle, name.encode(), C.byref(h)), "cn_gguf_upload")
        info = self.info(name)
        rows, cols = info.shape
        return ctx._own(Tensor(ctx, h.value, info.type, rows, cols))

    def llama_model(self, ctx, max_batch: int = 1, kv_f16: bool = False, tp=None) -> CudaLlamaModel:
        """The whole decoder from this file (cn_llama_create_from_gguf), or,
        with a connected TensorParallel group, this rank's shards of it
        (cn_llama_create_from_gguf_tp)."""
        from . import Tensor
        cfg = self.llama_config(max_batch, kv_f16)
        n = 3 + 9 * cfg.n_layers
        arr = (C.c_void_p * n)()
        h = C.c_void_p()
        kv = N.KV_F16 if kv_f16 else N.KV_F32
        if tp is None:
            check(N.lib().cn_llama_create_from_gguf(ctx.handle, self.handle, max_batch, kv, C.byref(h), arr, n),
                  "cn_llama_create_from_gguf")
        else:
            check(N.lib().cn_llama_create_from_gguf_tp(ctx.handle, self.handle, tp.handle, max_batch, kv, C.byref(h),
                                                       arr, n), "cn_llama_create_from_gguf_tp")
        seen, tensors = {}, []
        for v in arr:
            if v not in seen:
                seen[v] = ctx._own(Tensor(ctx, v, 0, 0, 0))
            tensors.append(seen[v])
        model = CudaLlamaModel.__new__(CudaLlamaModel)
        model.ctx, model.cfg, model.tp = ctx, cfg, tp
        model._tensors = tensors
        model.handle = h.value
        return model

    def close(self) -> None:
        if getattr(self, "handle", None):
            N.lib().cn_gguf_close(self.handle)
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
