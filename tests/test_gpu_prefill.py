"""Prefill parity: n tokens through the decoder at once (tcgen05 matmul,
flash attention) against the oracle running the same tokens one at a time
(or_llama_layers / or_llama_forward, the reference's sequential prompt loop).
Hidden states and logits: max relative error 1e-3 per token, normalised by
the token's largest reference magnitude."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import chatnet_b200 as cn
from chatnet_b200 import configs as cf
from chatnet_b200.llama import CudaLlamaModel, LlamaConfig, tensor_names
from tests import _oracle
from tests.parity import REL_TOL, rel_err

pytestmark = pytest.mark.gpu


def small(n_layers=2, kv_f16=False, ctx=256, head_dim=64, n_heads=4, n_kv=2, wtype=cn.TYPE_Q4_0):
    m = LlamaConfig(dim=n_heads * head_dim, hidden_dim=512, n_layers=n_layers, n_heads=n_heads,
                    n_kv_heads=n_kv, head_dim=head_dim, vocab=500, ctx_len=ctx, kv_f16=kv_f16)
    return cf.DecodeConfig(3, m, wtype, kv_filled=0, decode_pos=0, name="small-prefill")


class Rig:
    """GPU model + oracle on the same host bytes; KV caches start empty."""

    def __init__(self, ctx, oracle, dc):
        self.dc, self.ctx = dc, ctx
        self.host = cf.host_tensors(dc)
        names = tensor_names(dc.model.n_layers)
        types = [cf.tensor_type(dc, n) for n in names]
        self.tensors = cf.device_tensors(ctx, dc, self.host)
        self.gpu = CudaLlamaModel(ctx, dc.model, self.tensors)
        m = dc.model
        dt = np.float16 if m.kv_f16 else np.float32
        k = np.zeros((m.n_layers * m.ctx_len, m.kv_dim), dt)
        self.oracle = _oracle.OracleLlama(oracle, m, self.host, types, names, k, k.copy())

    def prefill(self, x: np.ndarray, pos: int) -> np.ndarray:
        xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
        out = torch.empty_like(xd)
        torch.cuda.synchronize()
        self.gpu.prefill_hidden_dev(xd.data_ptr(), x.shape[0], pos, out.data_ptr())
        self.ctx.synchronize()
        return out.cpu().numpy()

    def close(self):
        self.gpu.close()
        for t in self.tensors:
            t.free()


def _check_tokens(got, ref_fn, x, pos):
    worst = 0.0
    for t in range(x.shape[0]):
        err = rel_err(got[t], ref_fn(x[t], pos + t))
        assert err <= REL_TOL, (t, err)
        worst = max(worst, err)
    return worst


@pytest.mark.parametrize("n,head_dim,kv_f16", [(100, 64, False), (64, 128, False), (130, 64, True),
                                               (17, 64, False)])
def test_prefill_hidden_matches_sequential(ctx, oracle, n, head_dim, kv_f16):
    dc = small(kv_f16=kv_f16, head_dim=head_dim, n_heads=4 if head_dim == 64 else 2,
               n_kv=2 if head_dim == 64 else 1)
    r = Rig(ctx, oracle, dc)
    x = cf.prefill_x(dc, n)
    got = r.prefill(x, 0)
    _check_tokens(got, r.oracle.layers, x, 0)
    # the cache rows the prefill wrote match the oracle's
    m = dc.model
    for layer in range(m.n_layers):
        k, v = r.gpu.kv_read(0, layer, 0, n)
        ok = r.oracle.k.reshape(m.n_layers, m.ctx_len, m.kv_dim)[layer, :n]
        ov = r.oracle.v.reshape(m.n_layers, m.ctx_len, m.kv_dim)[layer, :n]
        assert rel_err(k.astype(np.float32), ok.astype(np.float32)) <= REL_TOL
        assert rel_err(v.astype(np.float32), ov.astype(np.float32)) <= REL_TOL
    r.close()


def test_prefill_q4_k_model(ctx, oracle):
    """A Q4_K model (config 4's weight type) takes the same prefill path."""
    dc = small(wtype=cn.TYPE_Q4_K, kv_f16=True)
    r = Rig(ctx, oracle, dc)
    assert r.gpu.prefill_kernels() == 10 * dc.model.n_layers
    x = cf.prefill_x(dc, 90)
    _check_tokens(r.prefill(x, 0), r.oracle.layers, x, 0)
    toks = [cf.token(dc, 1, s) for s in range(24)]
    got = r.gpu.forward(toks, 90)
    ref = r.oracle.forward(toks, 90)
    assert rel_err(got, ref) <= REL_TOL and int(np.argmax(got)) == int(np.argmax(ref))
    r.close()


def test_prefill_q4_k_m_style_model(ctx, oracle):
    """Q4_K projections with Q6_K attn_v and ffn_down, as Q4_K_M files mix
    them: every projection runs on the prefill matmul (Q6_K rows of dim 2048
    / hidden 4096 are 16-byte multiples; q/k and v take two launches), and
    the K/V rows the pass stores -- the Q4_K and Q6_K projections' outputs
    after RoPE -- match the oracle's.  The hidden states are not compared
    here: with these weights the fp16 rounding of the normalised input,
    shared by every row of the q and k projections, moves the scores of a
    peaked softmax enough to put some tokens' outputs ~1e-2 from the
    sequential reference; cn_llama_forward keeps the sequential steps unless
    cn_llama_set_prefill turns the pass on."""
    from chatnet_b200.llama import tensor_shape
    m = LlamaConfig(dim=2048, hidden_dim=4096, n_layers=1, n_heads=16, n_kv_heads=4, head_dim=128, vocab=300,
                    ctx_len=128, kv_f16=True)
    dc = cf.DecodeConfig(3, m, cn.TYPE_Q4_K, kv_filled=0, decode_pos=0, name="q4_k_m-prefill")
    names = tensor_names(m.n_layers)
    types = [cn.TYPE_F32 if n.endswith("norm.weight") else
             cn.TYPE_Q6_K if (".attn_v." in n or ".ffn_down." in n) else cn.TYPE_Q4_K for n in names]
    host = {n: cn.synth_fill(t, *tensor_shape(m, n), cn.synth_seed(3, "qkm." + n),
                             cn.DIST_NORM_W if t == cn.TYPE_F32 else None) for n, t in zip(names, types)}
    tensors = [ctx.upload(host[n], t, *tensor_shape(m, n)) for n, t in zip(names, types)]
    g = CudaLlamaModel(ctx, m, tensors)
    assert g.prefill_kernels() == 11 * m.n_layers
    k = np.zeros((m.n_layers * m.ctx_len, m.kv_dim), np.float16)
    orc = _oracle.OracleLlama(oracle, m, host, types, names, k, k.copy())
    n = 40
    x = cf.prefill_x(dc, n)
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    out = torch.empty_like(xd)
    torch.cuda.synchronize()
    g.prefill_hidden_dev(xd.data_ptr(), n, 0, out.data_ptr())
    ctx.synchronize()
    assert np.isfinite(out.cpu().numpy()).all()
    for t in range(n):
        orc.layers(x[t], t)
    kg, vg = g.kv_read(0, 0, 0, n)
    assert rel_err(kg.astype(np.float32), orc.k[:n].astype(np.float32)) <= REL_TOL
    assert rel_err(vg.astype(np.float32), orc.v[:n].astype(np.float32)) <= REL_TOL
    g.close()
    for t in tensors:
        t.free()


def test_prefill_after_cached_positions(ctx, oracle):
    """A second prompt chunk attends to the first chunk's cache rows."""
    dc = small()
    r = Rig(ctx, oracle, dc)
    x1, x2 = cf.prefill_x(dc, 40), cf.prefill_x(dc, 70)
    _check_tokens(r.prefill(x1, 0), r.oracle.layers, x1, 0)
    _check_tokens(r.prefill(x2, 40), r.oracle.layers, x2, 40)
    r.close()


def test_forward_prompt_takes_prefill(ctx, oracle):
    """IModel.Forward with a 48-token prompt (prefill path, turned on) matches
    the oracle's token-by-token Forward, then decoding continues from the
    cache."""
    dc = small()
    r = Rig(ctx, oracle, dc)
    with pytest.raises(ValueError):
        r.gpu.set_prefill(8)  # below the smallest threshold
    r.gpu.set_prefill(16)
    toks = [cf.token(dc, 0, s) for s in range(48)]
    got = r.gpu.forward(toks, 0)
    ref = r.oracle.forward(toks, 0)
    assert rel_err(got, ref) <= REL_TOL
    assert int(np.argmax(got)) == int(np.argmax(ref))
    nxt = int(np.argmax(ref))
    assert rel_err(r.gpu.forward([nxt], 48), r.oracle.forward([nxt], 48)) <= REL_TOL
    r.close()


def test_prefill_config3_layer(ctx, oracle):
    """Config 3 at full size: 512 tokens through one Llama-2-7B-shaped Q4_0 layer."""
    dc = cf.CONFIGS[3]
    r = Rig(ctx, oracle, dc)
    x = cf.prefill_x(dc)
    got = r.prefill(x, 0)
    assert np.isfinite(got).all()
    worst = _check_tokens(got, r.oracle.layers, x, 0)
    print(f"config3 prefill worst per-token rel err {worst:.2e}")
    r.close()


def test_prefill_rejects_unsupported(ctx):
    dc = cf.replace(small(), weight_type=cn.TYPE_Q6_K)
    ts = cf.device_tensors(ctx, dc)
    g = CudaLlamaModel(ctx, dc.model, ts)
    x = torch.zeros(20, 256, device="cuda")
    with pytest.raises(NotImplementedError):
        g.prefill_hidden_dev(x.data_ptr(), 20, 0, x.data_ptr())
    with pytest.raises(ValueError):
        g.prefill_hidden_dev(x.data_ptr(), 20, dc.model.ctx_len - 5, x.data_ptr())
    g.close()
    for t in ts:
        t.free()
