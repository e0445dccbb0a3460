"""ctypes binding of the CPU oracle (oracle/liboracle.so) -- test infrastructure.

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs use this module.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
ORACLE_DIR = ROOT / "oracle"
LIB = ORACLE_DIR / "_build" / "liboracle.so"

_f = C.c_float
_fp = C.POINTER(C.c_float)
_vp = C.c_void_p
_i = C.c_int


class LlamaConfig(C.Structure):
    _fields_ = [("dim", _i), ("hidden_dim", _i), ("n_layers", _i), ("n_heads", _i),
                ("n_kv_heads", _i), ("head_dim", _i), ("vocab", _i), ("ctx_len", _i),
                ("rope_base", _f), ("eps", _f), ("kv_f16", _i), ("rope_neox", _i), ("act_gelu", _i),
                ("norm_offset", _i)]


_SIG = {
    "or_half_to_float": (_f, [C.c_uint16]),
    "or_float_to_half": (C.c_uint16, [_f]),
    "or_byte_size": (C.c_uint64, [_i, C.c_uint64]),
    "or_dequantize": (_i, [_i, _vp, _fp, C.c_int64]),
    "or_dot": (_f, [_i, _vp, _fp, _i]),
    "or_matvec": (_i, [_i, _vp, _fp, _fp, _i, _i, _i]),
    "or_matvec_batch": (_i, [_i, _vp, _fp, _fp, _i, _i, _i, _i]),
    "or_rmsnorm": (None, [_fp, _fp, _fp, _i, _f]),
    "or_softmax": (None, [_fp, _i]),
    "or_silu_mul": (None, [_fp, _fp, _i]),
    "or_rope": (None, [_fp, _fp, _i, _i, _i, _i, _f]),
    "or_rope_neox": (None, [_fp, _fp, _i, _i, _i, _i, _f]),
    "or_gelu_mul": (None, [_fp, _fp, _i]),
    "or_rmsnorm_offset": (None, [_fp, _fp, _fp, _i, _f]),
    "or_add": (None, [_fp, _fp, _i]),
    "or_argmax": (_i, [_fp, _i]),
    "or_sample_temperature": (_i, [_fp, _i, _f, _i, _f, _f, _fp]),
    "or_llama_forward": (_i, [C.POINTER(LlamaConfig), C.POINTER(_vp), C.POINTER(_i), _vp, _vp,
                              C.POINTER(_i), _i, _i, _fp, _i]),
    "or_llama_layers": (_i, [C.POINTER(LlamaConfig), C.POINTER(_vp), C.POINTER(_i), _vp, _vp,
                             _fp, _i, _i, _i, _i]),
    "or_llama_head": (_i, [C.POINTER(LlamaConfig), C.POINTER(_vp), C.POINTER(_i), _fp, _fp, _i]),
    "or_synth_seed": (C.c_uint64, [_i, C.c_char_p]),
    "or_synth_fill": (_i, [_i, C.c_int64, C.c_int64, C.c_uint64, _i, _vp, C.c_uint64]),
    "or_synth_fill_rows": (_i, [_i, C.c_int64, C.c_int64, C.c_int64, C.c_uint64, _i, _vp, C.c_uint64]),
}


def fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


class Oracle:
    def __init__(self, lib: C.CDLL):
        self.lib = lib

    def dequantize(self, type_: int, blocks: np.ndarray, n: int) -> np.ndarray:
        out = np.zeros(n, dtype=np.float32)
        rc = self.lib.or_dequantize(type_, blocks.ctypes.data, fp(out), n)
        assert rc == 0, rc
        return out

    def dot(self, type_: int, row: np.ndarray, x: np.ndarray) -> float:
        x = np.ascontiguousarray(x, dtype=np.float32)
        return float(self.lib.or_dot(type_, row.ctypes.data, fp(x), x.size))

    def sample(self, logits: np.ndarray, temperature: float, top_k: int, top_p: float, r: float):
        """TemperatureSampler.Sample with draw r: (token, decision margin)."""
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        m = np.zeros(1, np.float32)
        tok = self.lib.or_sample_temperature(fp(lg), lg.size, temperature, top_k, top_p, r, fp(m))
        return int(tok), float(m[0])

    # ---- the configs' seeded synthetic inputs, without the product library ----
    def synth_seed(self, config_id: int, name: str) -> int:
        return int(self.lib.or_synth_seed(config_id, name.encode()))

    def synth_fill(self, type_: int, rows: int, cols: int, seed: int, norm_weight: bool = False,
                   row0: int = 0) -> np.ndarray:
        """Same bytes as chatnet_b200.synth_fill (checked by test_oracle_synth);
        with row0, rows [row0, row0 + rows) of a larger tensor."""
        nbytes = int(self.lib.or_byte_size(type_, cols)) * rows
        out = np.empty(nbytes, dtype=np.uint8)
        rc = self.lib.or_synth_fill_rows(type_, row0, rows, cols, seed, 1 if norm_weight else 0, out.ctypes.data,
                                         nbytes)
        assert rc == 0, rc
        if type_ == 0:
            return out.view(np.float32).reshape(rows, cols)
        if type_ == 1:
            return out.view(np.float16).reshape(rows, cols)
        return out.reshape(rows, -1)

    def matvec(self, type_: int, W: np.ndarray, x: np.ndarray, rows: int, nthreads: int = 0):
        x = np.ascontiguousarray(x, dtype=np.float32)
        x2 = x.reshape(-1, x.shape[-1])
        y = np.empty((x2.shape[0], rows), dtype=np.float32)
        rc = self.lib.or_matvec_batch(type_, W.ctypes.data, fp(x2), fp(y), rows, x2.shape[1],
                                      x2.shape[0], nthreads)
        assert rc == 0, rc
        return y[0] if x.ndim == 1 else y


def build() -> Path:
    if not LIB.exists() or LIB.stat().st_mtime < max(
            p.stat().st_mtime for p in (*ORACLE_DIR.glob("*.cpp"), *ORACLE_DIR.glob("*.h"))):
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    return LIB


def load() -> Oracle:
    lib = C.CDLL(str(build()))
    for name, (res, args) in _SIG.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return Oracle(lib)


def llama_config(cfg) -> LlamaConfig:
    """Oracle config struct from chatnet_b200.llama.LlamaConfig."""
    return LlamaConfig(cfg.dim, cfg.hidden_dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads,
                       cfg.head_dim, cfg.vocab, cfg.ctx_len, cfg.rope_base, cfg.rms_eps,
                       1 if cfg.kv_f16 else 0, int(getattr(cfg, "rope_neox", False)),
                       int(getattr(cfg, "act_gelu", False)), int(getattr(cfg, "norm_offset", False)))


class OracleLlama:
    """One sequence of the oracle Llama: weights (host bytes) + its own KV cache."""

    def __init__(self, oracle: Oracle, cfg, host: dict, types: list[int], names: list[str],
                 kcache: np.ndarray, vcache: np.ndarray):
        self.o, self.cfg = oracle, llama_config(cfg)
        self.arrays = [np.ascontiguousarray(host[n]) for n in names]
        self.ptrs = (C.c_void_p * len(names))(*[a.ctypes.data for a in self.arrays])
        self.types = (C.c_int * len(names))(*types)
        self.k = np.ascontiguousarray(kcache)
        self.v = np.ascontiguousarray(vcache)
        self.vocab = cfg.vocab

    def forward(self, tokens, pos: int, nthreads: int = 0) -> np.ndarray:
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.empty(self.vocab, dtype=np.float32)
        rc = self.o.lib.or_llama_forward(C.byref(self.cfg), self.ptrs, self.types,
                                         self.k.ctypes.data, self.v.ctypes.data,
                                         tok.ctypes.data_as(C.POINTER(C.c_int)), tok.size, pos,
                                         fp(logits), nthreads)
        assert rc == 0, rc
        return logits

    def layers(self, x: np.ndarray, pos: int, nthreads: int = 0) -> np.ndarray:
        """All layers on one hidden state x [dim] at position pos (or_llama_layers)."""
        h = np.array(x, dtype=np.float32, copy=True)
        rc = self.o.lib.or_llama_layers(C.byref(self.cfg), self.ptrs, self.types, self.k.ctypes.data,
                                        self.v.ctypes.data, fp(h), pos, 0, self.cfg.n_layers, nthreads)
        assert rc == 0, rc
        return h


# ---- the configs' tensors from the oracle-side generator (bench CPU legs) ----
def host_tensors(orc: Oracle, dc, names=None) -> dict[str, np.ndarray]:
    """chatnet_b200.configs.host_tensors through the oracle's generator."""
    from chatnet_b200 import configs as cf
    from chatnet_b200.llama import tensor_names, tensor_shape
    out = {}
    for name in names or tensor_names(dc.model.n_layers):
        rows, cols = tensor_shape(dc.model, name)
        out[name] = orc.synth_fill(cf.tensor_type(dc, name), rows, cols, orc.synth_seed(dc.config_id, name),
                                   name.endswith("norm.weight"))
    return out


def token(orc: Oracle, dc, seq: int, step: int = 0) -> int:
    return orc.synth_seed(dc.config_id, f"token.{seq}.{step}") % dc.model.vocab


def host_kv(orc: Oracle, dc, seq: int) -> tuple[np.ndarray, np.ndarray]:
    """chatnet_b200.configs.host_kv through the oracle's generator."""
    m = dc.model
    out = []
    for which in ("k", "v"):
        a = orc.synth_fill(1 if m.kv_f16 else 0, m.n_layers * m.ctx_len, m.kv_dim,
                           orc.synth_seed(dc.config_id, f"kv.{which}.{seq}"))
        a = a.reshape(m.n_layers, m.ctx_len, m.kv_dim).copy()
        a[:, dc.kv_filled:, :] = 0
        out.append(a.reshape(m.n_layers * m.ctx_len, m.kv_dim))
    return out[0], out[1]


def layer_kv(orc: Oracle, dc, seq: int, layer: int) -> tuple[np.ndarray, np.ndarray]:
    """Layer `layer`'s [ctx, kv_dim] slice of host_kv(dc, seq), generated alone."""
    m = dc.model
    out = []
    for which in ("k", "v"):
        a = orc.synth_fill(1 if m.kv_f16 else 0, m.ctx_len, m.kv_dim, orc.synth_seed(dc.config_id, f"kv.{which}.{seq}"),
                           row0=layer * m.ctx_len).copy()
        a[dc.kv_filled:, :] = 0
        out.append(a)
    return out[0], out[1]


def prefill_x(orc: Oracle, dc, n: int | None = None) -> np.ndarray:
    n = dc.prefill if n is None else n
    return orc.synth_fill(0, n, dc.model.dim, orc.synth_seed(dc.config_id, f"prefill.x.{n}"))
