"""GGUF reading (cn_gguf_*), against files written by tests/gguf_writer.py:
header and metadata parsing, tensor descriptors and data offsets
(GgufReader.Load, Gguf/GgufReader.cs:34-75; GgufTensorInfo.ByteSize), the
model config (GgufReader.ExtractModelConfig, GgufReader.cs:80-176) with its
defaults and fallbacks, and the reader's errors.  CPU only, except the last
test, which builds a decoder from a file on the GPU."""
from __future__ import annotations

import numpy as np
import pytest

import chatnet_b200 as cn
from chatnet_b200 import configs as cf
from chatnet_b200.gguf import GgufFile
from chatnet_b200.llama import CudaLlamaModel, LlamaConfig, tensor_names
from tests import _oracle
from tests import gguf_writer as gw
from tests.parity import REL_TOL, rel_err


def _raw(t, rows, cols, seed):
    return cn.synth_fill(t, rows, cols, seed).view(np.uint8).tobytes()


def test_descriptors_offsets_and_bytes(tmp_path):
    tensors = [("a.weight", cn.TYPE_Q4_0, (64, 3), _raw(cn.TYPE_Q4_0, 3, 64, 1)),
               ("b.weight", cn.TYPE_Q4_K, (512, 2), _raw(cn.TYPE_Q4_K, 2, 512, 2)),
               ("c.weight", cn.TYPE_Q6_K, (256, 5), _raw(cn.TYPE_Q6_K, 5, 256, 3)),
               ("norm.weight", cn.TYPE_F32, (7,), _raw(cn.TYPE_F32, 1, 7, 4)),
               # the generic codecs: GGUF byte sizes from cn_byte_size (GgufTensorInfo.ByteSize)
               ("q5k.weight", cn.TYPE_Q5_K, (512, 3), bytes(range(256)) * 4 + bytes(32)),
               ("iq4nl.weight", cn.TYPE_IQ4_NL, (64, 2), bytes(72)),
               ("q8k.weight", cn.TYPE_Q8_K, (256, 1), bytes(292)),
               ("iq2s.weight", cn.TYPE_IQ2_S, (256, 2), bytes(164)), ("iq1m.weight", cn.TYPE_IQ1_M, (512, 1), bytes(112))]
    md = [("general.architecture", gw.STR, "llama"), ("x.u8", gw.U8, 7), ("x.i8", gw.I8, -3),
          ("x.u16", gw.U16, 500), ("x.i16", gw.I16, -500), ("x.i32", gw.I32, -70000),
          ("x.u64", gw.U64, 1 << 40), ("x.i64", gw.I64, -(1 << 40)), ("x.f64", gw.F64, 0.125),
          ("x.bool", gw.BOOL, 1), ("x.ints", gw.ARR, (gw.I32, [1, 2, 3])),
          ("x.nested", gw.ARR, (gw.ARR, [(gw.U8, [1]), (gw.U8, [2, 3])]))]
    p = tmp_path / "t.gguf"
    offs = gw.write_gguf(p, md, tensors)
    blob = p.read_bytes()
    with GgufFile(p) as g:
        assert [t.name for t in g.tensors] == [t[0] for t in tensors]
        for (name, t, dims, raw), info in zip(tensors, g.tensors):
            assert info.type == t and info.dims == dims
            assert info.bytes == len(raw) == cn.byte_size(t, int(np.prod(dims)))
            assert info.file_offset == offs[name] and info.file_offset % 32 == 0
            assert blob[info.file_offset:info.file_offset + info.bytes] == raw
        assert g.info("c.weight").shape == (5, 256)
        assert g.get_int("x.u8") == 7 and g.get_int("x.i8") == -3 and g.get_int("x.i16") == -500
        assert g.get_int("x.u64") == 1 << 40 and g.get_int("x.i64") == -(1 << 40)
        assert g.get_int("x.bool") == 1 and g.get_float("x.f64") == 0.125
        assert g.get_string("general.architecture") == "llama"
        with pytest.raises(KeyError):
            g.info("missing.weight")
        with pytest.raises(KeyError):
            g.get_int("no.such.key")
        with pytest.raises(ValueError):
            g.get_int("general.architecture")


def test_custom_alignment(tmp_path):
    tensors = [("a", cn.TYPE_F32, (3,), _raw(cn.TYPE_F32, 1, 3, 5)), ("b", cn.TYPE_F32, (5,), _raw(cn.TYPE_F32, 1, 5, 6))]
    p = tmp_path / "a.gguf"
    offs = gw.write_gguf(p, [("general.alignment", gw.U32, 64)], tensors, alignment=64)
    with GgufFile(p) as g:
        assert [t.file_offset for t in g.tensors] == [offs["a"], offs["b"]]
        assert all(t.file_offset % 64 == 0 for t in g.tensors)


def test_llama_config_keys_defaults_fallbacks(tmp_path):
    cfg = LlamaConfig(dim=256, hidden_dim=512, n_layers=3, n_heads=4, n_kv_heads=2, head_dim=64, vocab=77,
                      ctx_len=128, rope_base=500000.0, rms_eps=1e-6)
    p = tmp_path / "c.gguf"
    gw.write_gguf(p, gw.llama_metadata(cfg), [])
    with GgufFile(p) as g:
        c = g.llama_config()
    assert (c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.vocab, c.ctx_len) == \
        (256, 512, 3, 4, 2, 64, 77, 128)
    assert c.rope_base == 500000.0 and abs(c.rms_eps - 1e-6) < 1e-12
    # defaults (no keys), bare-key fallback, freq_base stored as an integer,
    # vocab_size without a token list, kv heads defaulting to heads, key_length
    md = [("general.architecture", gw.STR, "llama"), ("embedding_length", gw.U32, 1024),
          ("llama.rope.freq_base", gw.U32, 10000), ("llama.vocab_size", gw.U32, 999),
          ("llama.attention.head_count", gw.U32, 8), ("llama.attention.key_length", gw.U32, 128)]
    p2 = tmp_path / "d.gguf"
    gw.write_gguf(p2, md, [])
    with GgufFile(p2) as g:
        c = g.llama_config()
    assert (c.dim, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.hidden_dim, c.ctx_len, c.vocab) == \
        (1024, 22, 8, 8, 128, 5632, 2048, 999)
    assert c.rope_base == 10000.0 and abs(c.rms_eps - 1e-5) < 1e-12
    p3 = tmp_path / "e.gguf"
    gw.write_gguf(p3, [("general.architecture", gw.STR, "qwen2")], [])
    with GgufFile(p3) as g:
        with pytest.raises(NotImplementedError):
            g.llama_config()


def test_llama_config_key_types(tmp_path):
    """GetInt32 counts only 32/64-bit integers and casts to int (a uint32 0xFFFFFFFF under the
    architecture's key is -1, so the bare key is used); GetArchFloat counts float, double,
    uint32 and int32 only (Gguf/GgufMetadata.cs:53-63, Gguf/GgufReader.cs:84-108)."""
    md = [("general.architecture", gw.STR, "llama"),
          ("llama.embedding_length", gw.U8, 64),            # u8: not an int to GetInt32 -> bare/default
          ("llama.block_count", gw.U32, 0xFFFFFFFF),       # reads as -1 -> bare key
          ("block_count", gw.U32, 5),
          ("llama.context_length", gw.U64, (1 << 32) + 300),  # (int) of a ulong: the low 32 bits
          ("llama.feed_forward_length", gw.I16, 999),      # i16: ignored -> default 5632
          ("llama.rope.freq_base", gw.I64, 77),            # long: not a GetArchFloat type -> bare key
          ("rope.freq_base", gw.I32, 5000),
          ("llama.attention.layer_norm_rms_epsilon", gw.U16, 3)]  # ignored -> default
    p = tmp_path / "k.gguf"
    gw.write_gguf(p, md, [])
    with GgufFile(p) as g:
        c = g.llama_config()
    assert c.dim == 2048 and c.n_layers == 5 and c.ctx_len == 300 and c.hidden_dim == 5632
    assert c.rope_base == 5000.0 and abs(c.rms_eps - 1e-5) < 1e-12


def test_reader_rejects_overflowing_shapes(tmp_path):
    # 256 x 2^60 Q4_K elements: the element count and byte size would wrap around
    p = tmp_path / "o.gguf"
    gw.write_gguf(p, [], [("big", cn.TYPE_Q4_K, (256, 1 << 60), b"")])
    with pytest.raises(ValueError, match="too many elements"):
        GgufFile(p)
    p2 = tmp_path / "o2.gguf"
    gw.write_gguf(p2, [], [("wrap", cn.TYPE_F32, (1 << 33, 1 << 33), b"")])
    with pytest.raises(ValueError):
        GgufFile(p2)


def test_reader_errors(tmp_path):
    good = tmp_path / "g.gguf"
    gw.write_gguf(good, [("general.architecture", gw.STR, "llama")],
                  [("a", cn.TYPE_F32, (4,), _raw(cn.TYPE_F32, 1, 4, 7))])
    bad_magic = tmp_path / "m.gguf"
    gw.write_gguf(bad_magic, [], [], magic=0x12345678)
    old = tmp_path / "v.gguf"
    gw.write_gguf(old, [], [], version=1)
    trunc = tmp_path / "tr.gguf"
    trunc.write_bytes(good.read_bytes()[:40])
    short_data = tmp_path / "sd.gguf"
    short_data.write_bytes(good.read_bytes()[:-8])
    for p in (bad_magic, old, trunc, short_data):
        with pytest.raises(ValueError):
            GgufFile(p)
    with pytest.raises(KeyError):
        GgufFile(tmp_path / "does-not-exist.gguf")
    with GgufFile(good) as g:  # still fine
        assert g.info("a").bytes == 16


@pytest.mark.gpu
@pytest.mark.parametrize("tied", [False, True])
def test_model_from_gguf_matches_oracle(ctx, oracle, tmp_path, tied):
    """A small Q4_K Llama written to a GGUF file and built with
    cn_llama_create_from_gguf decodes the oracle's logits; without
    output.weight the lm_head is token_embd.weight (LlamaWeights.cs:89-98)."""
    dc = cf.with_layers(cf.CONFIGS[4], 2, 1)
    m = cf.replace(dc.model, dim=512, hidden_dim=1024, n_heads=8, n_kv_heads=2, head_dim=64, vocab=300,
                   ctx_len=64, kv_f16=False)
    dc = cf.replace(dc, model=m, kv_filled=0, decode_pos=0)
    host = cf.host_tensors(dc)
    if tied:
        host["output.weight"] = host["token_embd.weight"]
    names = tensor_names(m.n_layers)
    types = [cf.tensor_type(dc, n) for n in names]
    p = tmp_path / "model.gguf"
    gw.write_gguf(p, gw.llama_metadata(m), gw.llama_tensors(host, names, types, m, tie_output=tied))
    with GgufFile(p) as g:
        assert g.llama_config().dim == 512
        model = g.llama_model(ctx, max_batch=1)
    k = np.zeros((m.n_layers * m.ctx_len, m.kv_dim), np.float32)
    orc = _oracle.OracleLlama(oracle, m, host, types, names, k, k.copy())
    toks = [cf.token(dc, 0, s) for s in range(4)]
    for pos, t in enumerate(toks):
        got = model.forward([t], pos)
        ref = orc.forward([t], pos)
        assert rel_err(got, ref) <= REL_TOL, pos
    model.close()
