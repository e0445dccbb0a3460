"""The benchmark configurations (BASELINE.json "configs") as seeded synthetic models.

Every tensor is generated from the seed cn_synth_seed(config_id, gguf_name), so
the host (oracle) copy and the device copy hold identical bytes, and a model
with fewer layers is a prefix of the full one.

  config 1: TinyLlama-1.1B-shaped decode step, Q4_0 weights (token_embd and
            a separate output included), fp32 KV cache with positions 0..510
            filled with N(0,1) and 511 left zero (the reference's cache starts
            zeroed, LlamaModel.cs:60-61), decoding position 512.
  config 3: prefill of 512 tokens through one Llama-2-7B-shaped layer, Q4_0
            weights, 32/32 heads of 128; the layer input is seeded N(0,1)
            activations [512][4096] (prefill_x), positions 0..511, fp32 KV
            cache starting empty.
  config 4: Llama-2-70B-shaped decode, Q4_K weights, fp16 KV cache with
            positions 0..2046 filled, decoding position 2047 (context 2048).
Norm weights are fp32 1 + N(0, 0.01); N(0,1) is the exact Irwin-Hall(12)
approximation of the generator.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np

from . import (DIST_NORM_W, DIST_NORMAL, TYPE_F16, TYPE_F32, TYPE_Q4_0, TYPE_Q4_K, byte_size, synth_fill,
               synth_seed)
from .llama import LlamaConfig, shard_region, tensor_names, tensor_shape


@dataclass(frozen=True)
class DecodeConfig:
    config_id: int
    model: LlamaConfig
    weight_type: int
    kv_filled: int      # positions 0..kv_filled-1 hold N(0,1)
    decode_pos: int
    name: str
    prefill: int = 0    # prompt tokens of a prefill config (0: decode config)


TINYLLAMA = LlamaConfig(dim=2048, hidden_dim=5632, n_layers=22, n_heads=32, n_kv_heads=4,
                        head_dim=64, vocab=32000, ctx_len=2048, rope_base=10000.0, rms_eps=1e-5,
                        kv_f16=False)
LLAMA2_70B = LlamaConfig(dim=8192, hidden_dim=28672, n_layers=80, n_heads=64, n_kv_heads=8,
                         head_dim=128, vocab=32000, ctx_len=2048, rope_base=10000.0, rms_eps=1e-5,
                         kv_f16=True)

LLAMA2_7B_LAYER = LlamaConfig(dim=4096, hidden_dim=11008, n_layers=1, n_heads=32, n_kv_heads=32,
                              head_dim=128, vocab=32000, ctx_len=512, rope_base=10000.0, rms_eps=1e-5,
                              kv_f16=False)

CONFIGS = {
    1: DecodeConfig(1, TINYLLAMA, TYPE_Q4_0, kv_filled=511, decode_pos=512,
                    name="tinyllama-1.1b-q4_0-decode@512"),
    3: DecodeConfig(3, LLAMA2_7B_LAYER, TYPE_Q4_0, kv_filled=0, decode_pos=0,
                    name="llama2-7b-layer-q4_0-prefill@512", prefill=512),
    4: DecodeConfig(4, LLAMA2_70B, TYPE_Q4_K, kv_filled=2047, decode_pos=2047,
                    name="llama2-70b-q4_k-decode@2047"),
}


def with_layers(dc: DecodeConfig, n_layers: int, max_batch: int = 1) -> DecodeConfig:
    return replace(dc, model=replace(dc.model, n_layers=n_layers, max_batch=max_batch))


def with_batch(dc: DecodeConfig, max_batch: int) -> DecodeConfig:
    return replace(dc, model=replace(dc.model, max_batch=max_batch))


def tensor_type(dc: DecodeConfig, name: str) -> int:
    return TYPE_F32 if name.endswith("norm.weight") else dc.weight_type


def tensor_dist(dc: DecodeConfig, name: str) -> int | None:
    return DIST_NORM_W if name.endswith("norm.weight") else None


def host_tensors(dc: DecodeConfig) -> dict[str, np.ndarray]:
    """Host bytes of every tensor (for the oracle and for uploads)."""
    out = {}
    for name in tensor_names(dc.model.n_layers):
        rows, cols = tensor_shape(dc.model, name)
        out[name] = synth_fill(tensor_type(dc, name), rows, cols, synth_seed(dc.config_id, name),
                               tensor_dist(dc, name))
    return out


def device_tensors(ctx, dc: DecodeConfig, host: dict[str, np.ndarray] | None = None, rank: int = 0,
                   size: int = 1) -> list:
    """The model's tensors in HBM: uploaded from `host`, or generated on the device.
    With size > 1, tensor-parallel rank `rank`'s shards (shard_region)."""
    ts = []
    for name in tensor_names(dc.model.n_layers):
        rows, cols = tensor_shape(dc.model, name)
        t = tensor_type(dc, name)
        r0, nr, c0, nc = shard_region(dc.model, name, rank, size)
        if host is not None:
            ts.append(ctx.upload(host_slice(host[name], t, cols, r0, nr, c0, nc), t, nr, nc))
        elif size == 1:
            ts.append(ctx.synth(t, rows, cols, synth_seed(dc.config_id, name), tensor_dist(dc, name)))
        else:
            ts.append(ctx.synth_slice(t, rows, cols, r0, nr, c0, nc, synth_seed(dc.config_id, name),
                                      tensor_dist(dc, name)))
    return ts


def host_slice(a: np.ndarray, type_: int, cols: int, r0: int, nr: int, c0: int, nc: int) -> np.ndarray:
    """Rows [r0, r0+nr) and columns [c0, c0+nc) (whole blocks) of a host tensor's bytes."""
    raw = np.ascontiguousarray(a).view(np.uint8).reshape(a.shape[0], -1)
    if c0 == 0 and nc == cols:
        return raw[r0:r0 + nr].copy()
    blk = {TYPE_F32: 1, TYPE_F16: 1}.get(type_, 32 if type_ == TYPE_Q4_0 else 256)
    bpb = byte_size(type_, blk)
    return raw[r0:r0 + nr, (c0 // blk) * bpb:((c0 + nc) // blk) * bpb].copy()


def token(dc: DecodeConfig, seq: int, step: int = 0) -> int:
    return synth_seed(dc.config_id, f"token.{seq}.{step}") % dc.model.vocab


def kv_seeds(dc: DecodeConfig, seq: int) -> tuple[int, int]:
    return synth_seed(dc.config_id, f"kv.k.{seq}"), synth_seed(dc.config_id, f"kv.v.{seq}")


def host_kv(dc: DecodeConfig, seq: int) -> tuple[np.ndarray, np.ndarray]:
    """[layers*ctx, kv_dim] caches of sequence `seq` (fp32 or fp16), positions >= kv_filled zero."""
    m = dc.model
    t = TYPE_F16 if m.kv_f16 else TYPE_F32
    sk, sv = kv_seeds(dc, seq)
    out = []
    for s in (sk, sv):
        a = synth_fill(t, m.n_layers * m.ctx_len, m.kv_dim, s, DIST_NORMAL)
        a = a.reshape(m.n_layers, m.ctx_len, m.kv_dim).copy()
        a[:, dc.kv_filled:, :] = 0
        out.append(a.reshape(m.n_layers * m.ctx_len, m.kv_dim))
    return out[0], out[1]


def prefill_x(dc: DecodeConfig, n: int | None = None) -> np.ndarray:
    """Seeded N(0,1) layer input [n][dim] of a prefill config."""
    n = dc.prefill if n is None else n
    return synth_fill(TYPE_F32, n, dc.model.dim, synth_seed(dc.config_id, f"prefill.x.{n}"), DIST_NORMAL)
