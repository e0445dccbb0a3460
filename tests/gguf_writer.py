"""Writes GGUF files for the tests (the layout GgufReader.Load reads,
Gguf/GgufReader.cs:34-75): magic, version, tensor and metadata counts,
metadata key/values, tensor descriptors, then the tensor data, each tensor at
a multiple of the alignment from the start of the aligned data section."""
from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B",
           U64: "<Q", I64: "<q", F64: "<d"}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(t: int, v) -> bytes:
    if t == STR:
        return _str(v)
    if t == ARR:
        et, items = v
        out = struct.pack("<IQ", et, len(items))
        return out + b"".join(_value(et, x) for x in items)
    return struct.pack(_SCALAR[t], v)


def write_gguf(path, metadata, tensors, alignment: int = 32, version: int = 3, magic: int = 0x46554747) -> dict:
    """metadata: [(key, type, value)] (arrays: (ARR, (element_type, items)));
    tensors: [(name, ggml_type, dims innermost first, raw bytes)].  Returns
    {name: absolute file offset of its data}."""
    head = struct.pack("<IIQQ", magic, version, len(tensors), len(metadata))
    head += b"".join(_str(k) + struct.pack("<I", t) + _value(t, v) for k, t, v in metadata)
    offs, off = [], 0
    for _, _, _, raw in tensors:
        offs.append(off)
        off += (len(raw) + alignment - 1) // alignment * alignment
    for (name, t, dims, _), o in zip(tensors, offs):
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", t, o)
    data_off = (len(head) + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(head + b"\0" * (data_off - len(head)))
        for (_, _, _, raw), o in zip(tensors, offs):
            f.seek(data_off + o)
            f.write(bytes(raw))
    return {name: data_off + o for (name, _, _, _), o in zip(tensors, offs)}


def llama_metadata(cfg, arch: str = "llama", vocab_tokens: bool = True) -> list:
    """Metadata of a Llama-shaped model (the keys ExtractModelConfig reads)."""
    md = [("general.architecture", STR, arch), ("general.name", STR, "synthetic"),
          (f"{arch}.embedding_length", U32, cfg.dim), (f"{arch}.block_count", U32, cfg.n_layers),
          (f"{arch}.attention.head_count", U32, cfg.n_heads),
          (f"{arch}.attention.head_count_kv", U32, cfg.n_kv_heads),
          (f"{arch}.feed_forward_length", U32, cfg.hidden_dim), (f"{arch}.context_length", U32, cfg.ctx_len),
          (f"{arch}.rope.freq_base", F32, cfg.rope_base),
          (f"{arch}.attention.layer_norm_rms_epsilon", F32, cfg.rms_eps)]
    if vocab_tokens:
        md.append(("tokenizer.ggml.tokens", ARR, (STR, [f"t{i}" for i in range(cfg.vocab)])))
    else:
        md.append((f"{arch}.vocab_size", U32, cfg.vocab))
    return md


def llama_tensors(host: dict, names: list, types: list, cfg, tie_output: bool = False) -> list:
    """GGUF tensor entries of a model's host tensors (norms 1-D, matrices [cols, rows])."""
    from chatnet_b200.llama import tensor_shape
    out = []
    for n, t in zip(names, types):
        if tie_output and n == "output.weight":
            continue
        rows, cols = tensor_shape(cfg, n)
        dims = (cols,) if rows == 1 else (cols, rows)
        out.append((n, t, dims, np.ascontiguousarray(host[n]).view(np.uint8).tobytes()))
    return out
