"""Model-level host side: CudaLlamaModel mirrors ChatNet's IModel for Llama.

    IModel.Forward(ReadOnlySpan<int> tokenIds, int position, Span<float> logits)
        (Abstractions/IModel.cs:18, Models/Llama/LlamaModel.cs:93-238)
    -> CudaLlamaModel.forward(token_ids, position, logits)

Weights are uploaded once (byte-identical GGUF blocks) and the KV cache and
scratch live on the device; each call crosses the host/device boundary only
for the token ids in and the logits out.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _native as N
from ._native import check

LAYER_TENSORS = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm",
                 "ffn_gate", "ffn_up", "ffn_down")


@dataclass
class LlamaConfig:
    """Hyper-parameters, as LlamaConfig (Models/Llama/LlamaConfig.cs:23-39)."""
    dim: int
    hidden_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    ctx_len: int
    rope_base: float = 10000.0
    rms_eps: float = 1e-5
    kv_f16: bool = False
    max_batch: int = 1
    # variants of other ChatNet models on the same loop (cn_llama_config)
    rope_neox: bool = False    # TensorMath.ApplyRoPENeox (split-half pairs)
    act_gelu: bool = False     # TensorMath.GeluElementwiseMul
    norm_offset: bool = False  # TensorMath.RmsNormWithOffset (weights stored as w - 1)

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def kv_mul(self) -> int:
        return self.n_heads // self.n_kv_heads

    def to_c(self) -> N.LlamaConfigC:
        return N.LlamaConfigC(self.dim, self.hidden_dim, self.n_layers, self.n_heads,
                              self.n_kv_heads, self.head_dim, self.vocab, self.ctx_len,
                              self.rope_base, self.rms_eps, N.KV_F16 if self.kv_f16 else N.KV_F32,
                              self.max_batch, int(self.rope_neox), int(self.act_gelu), int(self.norm_offset))


def tensor_names(n_layers: int) -> list[str]:
    """GGUF tensor names in cn_llama_create order (LlamaWeights.cs:78-145)."""
    names = ["token_embd.weight", "output.weight", "output_norm.weight"]
    for l in range(n_layers):
        names += [f"blk.{l}.{t}.weight" for t in LAYER_TENSORS]
    return names


def tensor_shape(cfg: LlamaConfig, name: str) -> tuple[int, int]:
    """[rows, cols] of a tensor (rows = output dim)."""
    if name in ("token_embd.weight", "output.weight"):
        return cfg.vocab, cfg.dim
    if name.endswith("norm.weight"):
        return 1, cfg.dim
    kind = name.split(".")[2]
    return {"attn_q": (cfg.dim, cfg.dim), "attn_k": (cfg.kv_dim, cfg.dim),
            "attn_v": (cfg.kv_dim, cfg.dim), "attn_output": (cfg.dim, cfg.dim),
            "ffn_gate": (cfg.hidden_dim, cfg.dim), "ffn_up": (cfg.hidden_dim, cfg.dim),
            "ffn_down": (cfg.dim, cfg.hidden_dim)}[kind]


def shard_region(cfg: LlamaConfig, name: str, rank: int, size: int) -> tuple[int, int, int, int]:
    """(row0, nrows, col0, ncols) of tensor `name` held by tensor-parallel rank
    `rank` of `size`: rows of q/k/v/gate/up/lm_head (heads, FFN rows,
    vocabulary), columns of O/down (their input), everything else whole."""
    rows, cols = tensor_shape(cfg, name)
    if size == 1 or name == "token_embd.weight" or name.endswith("norm.weight"):
        return 0, rows, 0, cols
    kind = "output" if name == "output.weight" else name.split(".")[2]
    if kind in ("attn_output", "ffn_down"):
        n = cols // size
        return 0, rows, rank * n, n
    n = rows // size
    return rank * n, n, 0, cols


class CudaLlamaModel:
    """IModel for Llama on one B200 (cn_llama_*)."""

    def __init__(self, ctx, cfg: LlamaConfig, tensors: list, tp=None):
        """tensors: the whole model's (or, with `tp`, this rank's shards, see shard_shape)."""
        self.ctx, self.cfg, self.tp = ctx, cfg, tp
        self._tensors = list(tensors)  # keep the borrowed weights alive
        arr = (C.c_void_p * len(tensors))(*[t.handle for t in tensors])
        h = C.c_void_p()
        c = cfg.to_c()
        if tp is None:
            check(N.lib().cn_llama_create(ctx.handle, C.byref(c), arr, len(tensors), C.byref(h)),
                  "cn_llama_create")
        else:
            check(N.lib().cn_llama_create_tp(ctx.handle, C.byref(c), arr, len(tensors), tp.handle,
                                             C.byref(h)), "cn_llama_create_tp")
        self.handle = h.value
        models = getattr(ctx, "_models", None)
        if models is not None:
            models.add(self)

    def prepare(self, batch: int) -> None:
        """Build and graph-capture the step without running it."""
        check(N.lib().cn_llama_prepare(self.handle, batch), "cn_llama_prepare")

    # IModel.Forward
    def forward(self, token_ids, position: int, logits: np.ndarray | None = None) -> np.ndarray:
        ids = np.ascontiguousarray(token_ids, dtype=np.int32)
        if logits is None:
            logits = np.empty(self.cfg.vocab, dtype=np.float32)
        assert logits.dtype == np.float32 and logits.size >= self.cfg.vocab
        check(N.lib().cn_llama_forward(self.handle, ids.ctypes.data_as(C.POINTER(C.c_int)), ids.size,
                                       position, logits.ctypes.data_as(C.POINTER(C.c_float))),
              "cn_llama_forward")
        return logits

    def prefill_hidden_dev(self, x_ptr: int, n: int, pos: int, out_ptr: int) -> None:
        """All layers on n hidden states at once (device pointers, enqueued)."""
        check(N.lib().cn_llama_prefill_hidden_dev(self.handle, C.c_void_p(x_ptr), n, pos, C.c_void_p(out_ptr)),
              "cn_llama_prefill_hidden_dev")

    def prefill_kernels(self) -> int:
        n = C.c_int(0)
        check(N.lib().cn_llama_prefill_kernels(self.handle, C.byref(n)), "cn_llama_prefill_kernels")
        return n.value

    def decode(self, tokens, positions, logits: bool = True, argmax: bool = True):
        """One batched decode step: sequence b (KV slot b) at positions[b]."""
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        B = tok.size
        lg = np.empty((B, self.cfg.vocab), dtype=np.float32) if logits else None
        am = np.empty(B, dtype=np.int32) if argmax else None
        check(N.lib().cn_llama_decode(
            self.handle, tok.ctypes.data_as(C.POINTER(C.c_int)), pos.ctypes.data_as(C.POINTER(C.c_int)),
            B, lg.ctypes.data_as(C.POINTER(C.c_float)) if lg is not None else None,
            am.ctypes.data_as(C.POINTER(C.c_int)) if am is not None else None), "cn_llama_decode")
        return lg, am

    def set_inputs(self, tokens, positions) -> None:
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        check(N.lib().cn_llama_set_inputs(self.handle, tok.ctypes.data_as(C.POINTER(C.c_int)),
                                          pos.ctypes.data_as(C.POINTER(C.c_int)), tok.size),
              "cn_llama_set_inputs")

    def set_prefill(self, min_tokens: int) -> None:
        """Prompts of min_tokens (>= 16; 16 by default) or more take the prefill
        pass in forward(); 0 keeps the reference's token-by-token loop."""
        check(N.lib().cn_llama_set_prefill(self.handle, int(min_tokens)), "cn_llama_set_prefill")

    def set_prefill_precision(self, split: int) -> None:
        """0: every prefill operand rounded to fp16 once; 1: the attention path
        (q/k/v and O projections, the attention's operands) on split (hi + lo
        fp16) operands; 2 (default): every projection split as well."""
        check(N.lib().cn_llama_set_prefill_precision(self.handle, int(split)), "cn_llama_set_prefill_precision")

    def step(self, batch: int) -> None:
        """Enqueue one decode step on the device inputs (no host copies, no wait)."""
        check(N.lib().cn_llama_step(self.handle, batch), "cn_llama_step")

    def sample(self, batch: int, temperature: float, top_k: int = 40, top_p: float = 0.9,
               r=None) -> np.ndarray:
        """TemperatureSampler.Sample on the device logits of the last step
        (cn_llama_sample); r[b] = the caller's uniform draw per sequence."""
        rr = np.ascontiguousarray(np.zeros(batch) if r is None else r, dtype=np.float32)
        out = np.empty(batch, dtype=np.int32)
        check(N.lib().cn_llama_sample(self.handle, batch, float(temperature), int(top_k), float(top_p),
                                      rr.ctypes.data, out.ctypes.data), "cn_llama_sample")
        return out

    def step_kernels(self, batch: int) -> int:
        n = C.c_int(0)
        check(N.lib().cn_llama_step_kernels(self.handle, batch, C.byref(n)), "cn_llama_step_kernels")
        return n.value

    def time_gemv(self, proj: int, batch: int, iters: int) -> tuple[float, float]:
        us, nb = C.c_float(0), C.c_double(0)
        check(N.lib().cn_llama_time_gemv(self.handle, proj, batch, iters, C.byref(us), C.byref(nb)),
              "cn_llama_time_gemv")
        return us.value, nb.value

    STAGES = ("start", "tp_step", "embed", "norm", "qkv", "rope", "attn", "o", "gate_up", "silu", "down",
              "head", "xchg_wait", "argmax")

    def profile_step(self, batch: int) -> dict[str, float]:
        """us per stage of one eagerly run decode step (cn_llama_profile_step)."""
        arr = (C.c_float * len(self.STAGES))()
        check(N.lib().cn_llama_profile_step(self.handle, batch, arr, len(self.STAGES)), "cn_llama_profile_step")
        return {k: arr[i] for i, k in enumerate(self.STAGES) if i > 0}

    def time_matmul(self, group: int, n: int, iters: int) -> tuple[float, float]:
        """Mean us and FLOPs of one prefill matmul launch (0 qkv, 1 O, 2 gate/up, 3 down)."""
        us, fl = C.c_float(0), C.c_double(0)
        check(N.lib().cn_llama_time_matmul(self.handle, group, n, iters, C.byref(us), C.byref(fl)),
              "cn_llama_time_matmul")
        return us.value, fl.value

    def kv_synth(self, seq: int, npos: int, seed_k: int, seed_v: int) -> None:
        check(N.lib().cn_llama_kv_synth(self.handle, seq, npos, seed_k, seed_v), "cn_llama_kv_synth")

    def kv_read(self, seq: int, layer: int, pos0: int, npos: int):
        dt = np.float16 if self.cfg.kv_f16 else np.float32
        k = np.empty((npos, self.cfg.kv_dim), dt)
        v = np.empty((npos, self.cfg.kv_dim), dt)
        check(N.lib().cn_llama_kv_read(self.handle, seq, layer, pos0, npos, k.ctypes.data,
                                       v.ctypes.data), "cn_llama_kv_read")
        return k, v

    def kv_write(self, seq: int, layer: int, pos0: int, k: np.ndarray, v: np.ndarray) -> None:
        dt = np.float16 if self.cfg.kv_f16 else np.float32
        k = np.ascontiguousarray(k, dt)
        v = np.ascontiguousarray(v, dt)
        check(N.lib().cn_llama_kv_write(self.handle, seq, layer, pos0, k.shape[0], k.ctypes.data,
                                        v.ctypes.data), "cn_llama_kv_write")

    def close(self) -> None:
        if getattr(self, "handle", None):
            N.lib().cn_llama_destroy(self.handle)
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
