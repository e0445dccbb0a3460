"""Model-level parity: the CUDA decode step (cn_llama_*) against the oracle's
restatement of LlamaModel.Forward on the same seeded weights, KV cache and
tokens.  Logits: max relative error 1e-3 (normalised by max |logit|);
greedy argmax must match."""
from __future__ import annotations

import numpy as np
import pytest

import chatnet_b200 as cn
from chatnet_b200 import configs as cf
from chatnet_b200.llama import CudaLlamaModel, tensor_names, tensor_shape
from tests import _oracle
from tests.parity import REL_TOL, rel_err

pytestmark = pytest.mark.gpu


def small_dc(weight_type=cn.TYPE_Q4_0, kv_f16=False, n_layers=2, max_batch=1, ctx_len=64):
    dc = cf.with_layers(cf.CONFIGS[1], n_layers, max_batch)
    m = cf.replace(dc.model, dim=256, hidden_dim=512, n_heads=4, n_kv_heads=2, head_dim=64,
                   vocab=500, ctx_len=ctx_len, kv_f16=kv_f16)
    return cf.replace(dc, model=m, weight_type=weight_type, kv_filled=10, decode_pos=12)


class Pair:
    """A GPU model and per-sequence oracles built from the same host bytes."""

    def __init__(self, ctx, oracle, dc, host=None, seqs=1, tie_output=False):
        self.dc = dc
        self.host = host if host is not None else cf.host_tensors(dc)
        if tie_output:
            self.host["output.weight"] = self.host["token_embd.weight"]
        self.names = tensor_names(dc.model.n_layers)
        self.types = [cf.tensor_type(dc, n) for n in self.names]
        self.tensors = cf.device_tensors(ctx, dc, self.host)
        if tie_output:
            self.tensors[1] = self.tensors[0]
        self.gpu = CudaLlamaModel(ctx, dc.model, self.tensors)
        self.oracles = []
        for s in range(seqs):
            k, v = cf.host_kv(dc, s)
            self.gpu.kv_synth(s, dc.kv_filled, *cf.kv_seeds(dc, s))
            self.oracles.append(_oracle.OracleLlama(oracle, dc.model, self.host, self.types,
                                                    self.names, k.copy(), v.copy()))

    def close(self):
        self.gpu.close()
        for t in self.tensors:
            t.free()


def test_kv_synth_matches_host(ctx, oracle):
    for f16 in (False, True):
        dc = small_dc(kv_f16=f16)
        p = Pair(ctx, oracle, dc)
        k, v = p.gpu.kv_read(0, 1, 0, dc.model.ctx_len)
        hk, hv = cf.host_kv(dc, 0)
        L, C = dc.model.n_layers, dc.model.ctx_len
        np.testing.assert_array_equal(k, hk.reshape(L, C, -1)[1])
        np.testing.assert_array_equal(v, hv.reshape(L, C, -1)[1])
        p.close()


@pytest.mark.parametrize("wtype", [cn.TYPE_Q4_0, cn.TYPE_Q4_K])
@pytest.mark.parametrize("kv_f16", [False, True])
def test_small_model_decode_parity(ctx, oracle, wtype, kv_f16):
    dc = small_dc(wtype, kv_f16)
    p = Pair(ctx, oracle, dc)
    tok = cf.token(dc, 0)
    got = p.gpu.forward([tok], dc.decode_pos)
    ref = p.oracles[0].forward([tok], dc.decode_pos)
    assert rel_err(got, ref) <= REL_TOL
    assert int(np.argmax(got)) == int(np.argmax(ref))
    # the new K/V rows landed in the cache like the oracle's
    kd = dc.model.kv_dim
    for layer in range(dc.model.n_layers):
        k, v = p.gpu.kv_read(0, layer, dc.decode_pos, 1)
        ok = p.oracles[0].k.reshape(dc.model.n_layers, dc.model.ctx_len, kd)[layer, dc.decode_pos]
        ov = p.oracles[0].v.reshape(dc.model.n_layers, dc.model.ctx_len, kd)[layer, dc.decode_pos]
        assert rel_err(k.astype(np.float32)[0], ok.astype(np.float32)) <= REL_TOL
        assert rel_err(v.astype(np.float32)[0], ov.astype(np.float32)) <= REL_TOL
    p.close()


def test_multi_token_forward_from_zero(ctx, oracle):
    """IModel.Forward with several tokens from position 0 (the engine's prompt path)."""
    dc = cf.replace(small_dc(), kv_filled=0)
    p = Pair(ctx, oracle, dc)
    toks = [cf.token(dc, 0, s) for s in range(6)]
    got = p.gpu.forward(toks, 0)
    ref = p.oracles[0].forward(toks, 0)
    assert rel_err(got, ref) <= REL_TOL
    p.close()


def test_tied_output_and_last_position(ctx, oracle):
    """lm_head tied to token_embd (LlamaWeights.cs:89-98); decode at ctx_len-1."""
    dc = cf.replace(small_dc(), kv_filled=63, decode_pos=63)
    p = Pair(ctx, oracle, dc, tie_output=True)
    tok = cf.token(dc, 0)
    got = p.gpu.forward([tok], 63)
    ref = p.oracles[0].forward([tok], 63)
    assert rel_err(got, ref) <= REL_TOL
    p.close()


def test_batched_decode_matches_sequences(ctx, oracle):
    B = 5
    dc = small_dc(cn.TYPE_Q4_K, True, max_batch=B)
    p = Pair(ctx, oracle, dc, seqs=B)
    toks = [cf.token(dc, s) for s in range(B)]
    pos = [12, 13, 14, 12, 40]
    lg, am = p.gpu.decode(toks, pos)
    for s in range(B):
        ref = p.oracles[s].forward([toks[s]], pos[s])
        assert rel_err(lg[s], ref) <= REL_TOL, s
        assert am[s] == int(np.argmax(lg[s]))
    p.close()


def test_decode_rejects_bad_input(ctx, oracle):
    dc = small_dc()
    p = Pair(ctx, oracle, dc)
    with pytest.raises(ValueError):
        p.gpu.decode([dc.model.vocab], [0])
    with pytest.raises(ValueError):
        p.gpu.decode([0], [dc.model.ctx_len])
    with pytest.raises(ValueError):
        p.gpu.decode([0, 1], [0, 0])  # batch above max_batch
    p.gpu.forward([1], 0)  # still usable afterwards
    p.close()


def test_create_validates_tensors(ctx):
    dc = small_dc()
    host = cf.host_tensors(dc)
    ts = cf.device_tensors(ctx, dc, host)
    with pytest.raises(ValueError):
        CudaLlamaModel(ctx, dc.model, ts[:-1])  # wrong count
    bad = list(ts)
    bad[4], bad[5] = bad[5], bad[4]  # attn_q <-> attn_k: shape mismatch
    with pytest.raises(ValueError):
        CudaLlamaModel(ctx, dc.model, bad)
    for t in ts:
        t.free()


@pytest.fixture(scope="module")
def tiny_full(ctx, oracle):
    """Config 1 at full size: 22 layers, TinyLlama shapes, Q4_0, fp32 KV."""
    dc = cf.CONFIGS[1]
    p = Pair(ctx, oracle, dc)
    yield p
    p.close()


def test_config1_decode_step(tiny_full):
    p, dc = tiny_full, tiny_full.dc
    tok = cf.token(dc, 0)
    got = p.gpu.forward([tok], dc.decode_pos)
    ref = p.oracles[0].forward([tok], dc.decode_pos)
    err = rel_err(got, ref)
    top2 = np.sort(ref)[-2:]
    print(f"config1 logits rel err {err:.2e}, top-1/top-2 margin {top2[1] - top2[0]:.4f}")
    assert err <= REL_TOL
    assert int(np.argmax(got)) == int(np.argmax(ref))


def test_config1_greedy_32_steps(tiny_full):
    """The greedy token matches the oracle for 32 decode steps."""
    p, dc = tiny_full, tiny_full.dc
    o = p.oracles[0]
    tok_g = tok_o = cf.token(dc, 0, 1)
    pos = dc.decode_pos + 1  # after test_config1_decode_step wrote position 512
    for step in range(32):
        lg, am = p.gpu.decode([tok_g], [pos + step])
        ref = o.forward([tok_o], pos + step)
        assert rel_err(lg[0], ref) <= REL_TOL, step
        tok_g, tok_o = int(am[0]), int(np.argmax(ref))
        assert tok_g == tok_o, (step, tok_g, tok_o)


def test_config4_two_layers_batched(ctx, oracle):
    """Config 4 shapes (70B: d 8192, FFN 28672, 64/8 heads, Q4_K, fp16 KV at
    2047) with 2 of its 80 layers, 2 sequences decoded together."""
    dc = cf.with_layers(cf.CONFIGS[4], 2, max_batch=2)
    p = Pair(ctx, oracle, dc, seqs=2)
    toks = [cf.token(dc, s) for s in range(2)]
    lg, am = p.gpu.decode(toks, [dc.decode_pos] * 2)
    for s in range(2):
        ref = p.oracles[s].forward([toks[s]], dc.decode_pos)
        assert rel_err(lg[s], ref) <= REL_TOL
        assert am[s] == int(np.argmax(ref))
    p.close()


def _oracle_full_depth(orc, dc, toks: list[int]) -> np.ndarray:
    """LlamaModel.Forward of every sequence's token at dc.decode_pos through all
    of dc's layers, generating one layer's weights (and that layer's slice of
    each sequence's KV cache) at a time from the seeded generator, so host
    memory holds one layer (481 MB at config 4) instead of the model."""
    from chatnet_b200.llama import LAYER_TENSORS
    m = dc.model
    one = cf.with_layers(dc, 1)
    head = _oracle.host_tensors(orc, dc, names=["token_embd.weight", "output.weight", "output_norm.weight"])
    names1 = tensor_names(1)
    types1 = [cf.tensor_type(dc, n) for n in names1]
    xs = [orc.dequantize(types1[0], head["token_embd.weight"][t], m.dim) for t in toks]
    ol = None
    for layer in range(m.n_layers):
        lay = _oracle.host_tensors(orc, dc, names=[f"blk.{layer}.{k}.weight" for k in LAYER_TENSORS])
        host = dict(head)
        host.update({f"blk.0.{k}.weight": lay[f"blk.{layer}.{k}.weight"] for k in LAYER_TENSORS})
        for b in range(len(toks)):
            k, v = _oracle.layer_kv(orc, dc, b, layer)
            ol = _oracle.OracleLlama(orc, one.model, host, types1, names1, k, v)
            xs[b] = ol.layers(xs[b], dc.decode_pos)
    out = np.empty((len(toks), m.vocab), np.float32)
    for b in range(len(toks)):
        rc = orc.lib.or_llama_head(_oracle.C.byref(ol.cfg), ol.ptrs, ol.types, _oracle.fp(xs[b]), _oracle.fp(out[b]), 0)
        assert rc == 0
    return out


def test_config4_full_depth_b16_and_b1(ctx, oracle):
    """Config 4 at its full depth and both of its batch sizes: all 80
    Llama-2-70B-shaped Q4_K layers with the fp16 cache filled to position
    2046, one decode step of 16 sequences (the fp16 hi + lo GEMV family) and
    one of sequence 0 alone (the integer GEMV), against the oracle's Forward of
    each sequence: logits within 1e-3 and the same greedy token."""
    B = 16
    dc = cf.with_batch(cf.CONFIGS[4], B)
    m = dc.model
    ts = cf.device_tensors(ctx, dc)  # 38.5 GB generated on the device
    g = CudaLlamaModel(ctx, m, ts)
    for b in range(B):
        g.kv_synth(b, dc.kv_filled, *cf.kv_seeds(dc, b))
    toks = [cf.token(dc, b) for b in range(B)]
    lg16, am16 = g.decode(toks, [dc.decode_pos] * B)
    lg1, am1 = g.decode(toks[:1], [dc.decode_pos])
    g.close()
    for t in ts:
        t.free()
    ref = _oracle_full_depth(oracle, dc, toks)
    errs = [rel_err(lg16[b], ref[b]) for b in range(B)]
    print(f"config4 80 layers: B=16 worst logits rel err {max(errs):.2e}, B=1 {rel_err(lg1[0], ref[0]):.2e}")
    for b in range(B):
        assert errs[b] <= REL_TOL, (b, errs[b])
        assert int(am16[b]) == int(np.argmax(ref[b])), b
    assert rel_err(lg1[0], ref[0]) <= REL_TOL
    assert int(am1[0]) == int(np.argmax(ref[0]))


@pytest.mark.parametrize("kinds", [
    # every projection Q8_0: the tiled fp16 GEMV, q/k/v and gate/up as one launch each
    {"attn_q": "q8_0", "attn_k": "q8_0", "attn_v": "q8_0", "attn_output": "q8_0", "ffn_gate": "q8_0",
     "ffn_up": "q8_0", "ffn_down": "q8_0", "token_embd": "q8_0", "output": "q8_0"},
    # the reference's simplified importance-quant decodes, one per tensor kind
    {"attn_q": "iq3_s", "attn_k": "iq3_xxs", "attn_v": "iq2_xs", "attn_output": "iq2_xxs", "ffn_gate": "iq2_s",
     "ffn_up": "iq1_s", "ffn_down": "iq1_m", "token_embd": "iq3_s", "output": "iq2_s"},
], ids=["q8_0", "iq"])
@pytest.mark.parametrize("batch", [1, 3])
def test_codec_family_models(ctx, oracle, kinds, batch):
    """Whole decoders on Q8_0 (tiled GEMV, grouped launches) and on the IQ
    codecs (generic kernel) match the oracle's Forward at batch 1 and 3."""
    from tests.test_gpu_quant import _rand_b32, _rand_sb
    dc = cf.replace(small_dc(max_batch=3), kv_filled=0, decode_pos=0)
    m = dc.model
    host = cf.host_tensors(dc)
    names = tensor_names(m.n_layers)
    types = []
    for i, n in enumerate(names):
        rows, cols = tensor_shape(m, n)
        kind = n.split(".")[2] if n.startswith("blk.") else n.split(".")[0]
        codec = kinds.get(kind)
        if codec is None:  # norms stay fp32
            types.append(cf.tensor_type(dc, n))
            continue
        t, blocks = (_rand_b32 if codec == "q8_0" else _rand_sb)(codec, rows, cols, 300 + i)
        host[n] = blocks
        types.append(t)
    tensors = [ctx.upload(host[n], t, *tensor_shape(m, n)) for n, t in zip(names, types)]
    g = CudaLlamaModel(ctx, m, tensors)
    orcs = []
    for _ in range(batch):
        k = np.zeros((m.n_layers * m.ctx_len, m.kv_dim), np.float32)
        orcs.append(_oracle.OracleLlama(oracle, m, host, types, names, k, k.copy()))
    for step in range(2):
        toks = [cf.token(dc, b, step) for b in range(batch)]
        lg, am = g.decode(toks, [step] * batch)
        for b in range(batch):
            ref = orcs[b].forward([toks[b]], step)
            assert rel_err(lg[b], ref) <= REL_TOL, (step, b)
            assert am[b] == int(np.argmax(lg[b]))
    g.close()
    for t in tensors:
        t.free()


def test_mixed_codec_model(ctx, oracle):
    """A decoder whose projections, embedding and lm_head use the generic
    codecs (every K-quant and IQ4 type the reference decodes besides Q4_K /
    Q6_K, one per tensor kind) matches the oracle's Forward."""
    from tests.test_gpu_quant import _rand_b32, _rand_sb
    dc = cf.replace(small_dc(), kv_filled=0, decode_pos=0)
    m = dc.model
    kinds = {"attn_q": "q5_k", "attn_k": "q3_k", "attn_v": "q2_k", "attn_output": "iq4_xs",
             "ffn_gate": "q8_k", "ffn_up": "iq4_nl", "ffn_down": "q5_k"}
    host = cf.host_tensors(dc)
    names = tensor_names(m.n_layers)
    types = []
    for i, n in enumerate(names):
        rows, cols = tensor_shape(m, n)
        kind = n.split(".")[2] if n.startswith("blk.") else n.split(".")[0]
        codec = {"token_embd": "q2_k", "output": "iq4_xs"}.get(kind, kinds.get(kind))
        if codec is None:  # norms stay fp32
            types.append(cf.tensor_type(dc, n))
            continue
        t, blocks = (_rand_b32 if codec == "iq4_nl" else _rand_sb)(codec, rows, cols, 100 + i)
        host[n] = blocks
        types.append(t)
    tensors = [ctx.upload(host[n], t, *tensor_shape(m, n)) for n, t in zip(names, types)]
    g = CudaLlamaModel(ctx, m, tensors)
    k = np.zeros((m.n_layers * m.ctx_len, m.kv_dim), np.float32)
    orc = _oracle.OracleLlama(oracle, m, host, types, names, k, k.copy())
    for pos in range(3):
        t = cf.token(dc, 0, pos)
        got, ref = g.forward([t], pos), orc.forward([t], pos)
        assert rel_err(got, ref) <= REL_TOL, pos
        assert int(np.argmax(got)) == int(np.argmax(ref))
    g.close()
    for t in tensors:
        t.free()
