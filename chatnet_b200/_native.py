"""ctypes binding of libchatnet_cuda (include/chatnet_cuda.h).

The library is the product: there is no Python or CPU fallback.  Loading
fails loudly when the shared object is missing, and every call checks the
returned status and raises the exception the reference would have thrown:

    CN_ERR_UNSUPPORTED -> NotSupportedError   (NotSupportedException)
    CN_ERR_NOT_FOUND   -> KeyError            (KeyNotFoundException)
    CN_ERR_INVALID_ARG -> ValueError          (ArgumentException)
    CN_ERR_TIMEOUT     -> TimeoutError
    others             -> CudaError
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("CHATNET_CUDA_LIB", _PKG / "_build" / "libchatnet_cuda.so"))

CN_OK = 0
CN_ERR_INVALID_ARG = -1
CN_ERR_UNSUPPORTED = -2
CN_ERR_CUDA = -3
CN_ERR_OOM = -4
CN_ERR_TIMEOUT = -5
CN_ERR_NOT_FOUND = -6
CN_ERR_NCCL = -7

TYPE_F32 = 0
TYPE_F16 = 1
TYPE_Q4_0 = 2
TYPE_Q4_1 = 3
TYPE_Q5_0 = 6
TYPE_Q5_1 = 7
TYPE_Q8_0 = 8
TYPE_Q2_K = 10
TYPE_Q3_K = 11
TYPE_Q4_K = 12
TYPE_Q5_K = 13
TYPE_Q6_K = 14
TYPE_Q8_K = 15
TYPE_IQ2_XXS = 16
TYPE_IQ2_XS = 17
TYPE_IQ3_XXS = 18
TYPE_IQ1_S = 19
TYPE_IQ4_NL = 20
TYPE_IQ3_S = 21
TYPE_IQ2_S = 22
TYPE_IQ4_XS = 23
TYPE_IQ1_M = 29

DIST_CFG0_Q4_0 = 1
DIST_CFG2_Q4_K = 2
DIST_CFG2_Q6_K = 3
DIST_NORMAL = 4
DIST_NORM_W = 5


class NotSupportedError(NotImplementedError):
    """The reference's NotSupportedException (LlamaModel.cs:564-565)."""


class CudaError(RuntimeError):
    pass


_vp = C.c_void_p
_i = C.c_int
_i64 = C.c_int64
_u64 = C.c_uint64
_f = C.c_float
_fp = C.POINTER(C.c_float)

# name -> (restype, argtypes); mirrors include/chatnet_cuda.h
SIGNATURES: dict[str, tuple] = {
    "cn_abi_version": (_i, []),
    "cn_last_error": (C.c_char_p, []),
    "cn_byte_size": (_u64, [_i, _u64]),
    "cn_device_count": (_i, [C.POINTER(_i)]),
    "cn_create": (_i, [_i, C.POINTER(_vp)]),
    "cn_destroy": (_i, [_vp]),
    "cn_ctx_stream": (_vp, [_vp]),
    "cn_synchronize": (_i, [_vp]),
    "cn_tensor_upload": (_i, [_vp, _vp, _u64, _i, _i64, _i64, C.POINTER(_vp)]),
    "cn_tensor_synth": (_i, [_vp, _i, _i64, _i64, _u64, _i, C.POINTER(_vp)]),
    "cn_tensor_download": (_i, [_vp, _vp, _u64]),
    "cn_tensor_free": (_i, [_vp]),
    "cn_tensor_device_ptr": (_vp, [_vp]),
    "cn_tensor_bytes": (_u64, [_vp]),
    "cn_synth_fill": (_i, [_i, _i64, _i64, _u64, _i, _vp, _u64]),
    "cn_synth_seed": (_u64, [_i, C.c_char_p]),
    "cn_dequantize": (_i, [_vp, _vp, _i64, _i64, _fp]),
    "cn_matvec": (_i, [_vp, _vp, _fp, _fp, _i]),
    "cn_dequantize_dev": (_i, [_i, _vp, _vp, _i64, _vp]),
    "cn_matvec_dev": (_i, [_vp, _i, _vp, _i, _i, _vp, _vp, _i]),
    "cn_time_matvec": (_i, [_vp, C.POINTER(_vp), _i, _vp, _vp, _i, _i, _i, _fp, C.POINTER(_i)]),
    "cn_matmul": (_i, [_vp, _vp, _fp, _fp, _i]),
    "cn_matmul_dev": (_i, [_vp, _i, _vp, _i, _i, _vp, _vp, _i]),
    "cn_matvec_noalloc_dev": (_i, [_i, _vp, _i, _i, _vp, _vp, _i, _vp]),
    "cn_matvec_noalloc_status": (_i, [_vp]),
    "cn_llama_create": (_i, [_vp, _vp, C.POINTER(_vp), _i, C.POINTER(_vp)]),
    "cn_llama_destroy": (_i, [_vp]),
    "cn_llama_forward": (_i, [_vp, C.POINTER(_i), _i, _i, _fp]),
    "cn_llama_prefill_hidden_dev": (_i, [_vp, _vp, _i, _i, _vp]),
    "cn_gguf_open": (_i, [C.c_char_p, C.POINTER(_vp)]),
    "cn_gguf_close": (_i, [_vp]),
    "cn_gguf_tensor_count": (_i, [_vp, C.POINTER(_i)]),
    "cn_gguf_tensor_info": (_i, [_vp, _i, C.POINTER(C.c_char_p), C.POINTER(_i), C.POINTER(_i),
                                 C.POINTER(_u64), C.POINTER(_u64), C.POINTER(_u64)]),
    "cn_gguf_find": (_i, [_vp, C.c_char_p, C.POINTER(_i)]),
    "cn_gguf_get_int": (_i, [_vp, C.c_char_p, C.POINTER(C.c_int64)]),
    "cn_gguf_get_float": (_i, [_vp, C.c_char_p, C.POINTER(C.c_double)]),
    "cn_gguf_get_string": (_i, [_vp, C.c_char_p, C.POINTER(C.c_char_p)]),
    "cn_gguf_llama_config": (_i, [_vp, _vp]),
    "cn_gguf_upload": (_i, [_vp, _vp, C.c_char_p, C.POINTER(_vp)]),
    "cn_llama_create_from_gguf": (_i, [_vp, _vp, _i, _i, C.POINTER(_vp), C.POINTER(_vp), _i]),
    "cn_llama_create_from_gguf_tp": (_i, [_vp, _vp, _vp, _i, _i, C.POINTER(_vp), C.POINTER(_vp), _i]),
    "cn_tensor_upload_slice": (_i, [_vp, _vp, _u64, _i, _i64, _i64, _i64, _i64, _i64, _i64, C.POINTER(_vp)]),
    "cn_llama_prefill_kernels": (_i, [_vp, C.POINTER(_i)]),
    "cn_llama_decode": (_i, [_vp, C.POINTER(_i), C.POINTER(_i), _i, _fp, C.POINTER(_i)]),
    "cn_llama_kv_write": (_i, [_vp, _i, _i, _i, _i, _vp, _vp]),
    "cn_llama_kv_read": (_i, [_vp, _i, _i, _i, _i, _vp, _vp]),
    "cn_llama_kv_synth": (_i, [_vp, _i, _i, _u64, _u64]),
    "cn_llama_set_inputs": (_i, [_vp, C.POINTER(_i), C.POINTER(_i), _i]),
    "cn_llama_step": (_i, [_vp, _i]),
    "cn_llama_set_prefill": (_i, [_vp, _i]),
    "cn_llama_set_prefill_precision": (_i, [_vp, _i]),
    "cn_llama_sample": (_i, [_vp, _i, C.c_float, _i, C.c_float, _vp, _vp]),
    "cn_sample_dev": (_i, [_vp, _vp, _i, _i, C.c_float, _i, C.c_float, _vp, _vp]),
    "cn_llama_step_kernels": (_i, [_vp, _i, C.POINTER(_i)]),
    "cn_llama_time_gemv": (_i, [_vp, _i, _i, _i, C.POINTER(_f), C.POINTER(C.c_double)]),
    "cn_llama_time_matmul": (_i, [_vp, _i, _i, _i, C.POINTER(_f), C.POINTER(C.c_double)]),
    "cn_llama_profile_step": (_i, [_vp, _i, C.POINTER(_f), _i]),
    "cn_tensor_synth_slice": (_i, [_vp, _i, _i64, _i64, _i64, _i64, _i64, _i64, _u64, _i, C.POINTER(_vp)]),
    "cn_tp_create": (_i, [_vp, _i, _i, _i, _i, _i, C.POINTER(_vp)]),
    "cn_tp_handle": (_i, [_vp, _vp]),
    "cn_tp_connect": (_i, [_vp, _vp]),
    "cn_tp_destroy": (_i, [_vp]),
    "cn_llama_create_tp": (_i, [_vp, _vp, C.POINTER(_vp), _i, _vp, C.POINTER(_vp)]),
    "cn_llama_prepare": (_i, [_vp, _i]),
}

TP_HANDLE_BYTES = 64

KV_F32 = 0
KV_F16 = 1


class LlamaConfigC(C.Structure):
    """cn_llama_config (include/chatnet_cuda.h)."""
    _fields_ = [("dim", _i), ("hidden_dim", _i), ("n_layers", _i), ("n_heads", _i),
                ("n_kv_heads", _i), ("head_dim", _i), ("vocab", _i), ("ctx_len", _i),
                ("rope_base", _f), ("rms_eps", _f), ("kv_dtype", _i), ("max_batch", _i),
                ("rope_neox", _i), ("act_gelu", _i), ("norm_offset", _i)]

_lib = None


def lib() -> C.CDLL:
    """Loads libchatnet_cuda once; raises if it is missing (no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"libchatnet_cuda not built: {LIB_PATH} is missing "
                "(run `python -m chatnet_b200.build`)")
        h = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def last_error() -> str:
    return lib().cn_last_error().decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    if rc == CN_OK:
        return
    msg = f"{what}: {last_error()} (status {rc})" if what else f"{last_error()} (status {rc})"
    if rc == CN_ERR_UNSUPPORTED:
        raise NotSupportedError(msg)
    if rc == CN_ERR_NOT_FOUND:
        raise KeyError(msg)
    if rc == CN_ERR_INVALID_ARG:
        raise ValueError(msg)
    if rc == CN_ERR_TIMEOUT:
        raise TimeoutError(msg)
    if rc == CN_ERR_OOM:
        raise MemoryError(msg)
    raise CudaError(msg)


def byte_size(type_: int, elements: int) -> int:
    return int(lib().cn_byte_size(type_, elements))
