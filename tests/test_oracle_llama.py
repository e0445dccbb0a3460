"""The oracle's Llama forward on a small seeded model (CPU only): runs, is
deterministic, and fills the KV cache at the decoded position."""
from __future__ import annotations

import numpy as np

from chatnet_b200 import configs as cf
from chatnet_b200.llama import tensor_names
from tests import _oracle


def small_dc():
    dc = cf.with_layers(cf.CONFIGS[1], 2)
    m = cf.replace(dc.model, dim=256, hidden_dim=512, n_heads=4, n_kv_heads=2, head_dim=64,
                   vocab=500, ctx_len=64)
    return cf.replace(dc, model=m, kv_filled=10, decode_pos=12)


def make_oracle(oracle, dc):
    host = cf.host_tensors(dc)
    names = tensor_names(dc.model.n_layers)
    types = [cf.tensor_type(dc, n) for n in names]
    k, v = cf.host_kv(dc, 0)
    return _oracle.OracleLlama(oracle, dc.model, host, types, names, k, v)


def test_oracle_forward_runs(oracle):
    dc = small_dc()
    o1 = make_oracle(oracle, dc)
    o2 = make_oracle(oracle, dc)
    tok = cf.token(dc, 0)
    l1 = o1.forward([tok], dc.decode_pos)
    l2 = o2.forward([tok], dc.decode_pos, nthreads=1)
    assert np.isfinite(l1).all()
    np.testing.assert_array_equal(l1, l2)  # thread count does not change results
    kv = dc.model.kv_dim
    row = o1.k.reshape(dc.model.n_layers, dc.model.ctx_len, kv)[:, dc.decode_pos]
    assert np.abs(row).sum() > 0   # K written at the decoded position
    assert o1.k.reshape(dc.model.n_layers, dc.model.ctx_len, kv)[:, dc.decode_pos + 1:].sum() == 0


def test_oracle_multi_token_equals_sequential(oracle):
    dc = small_dc()
    toks = [cf.token(dc, 0, s) for s in range(3)]
    a = make_oracle(oracle, dc)
    la = a.forward(toks, 12)
    b = make_oracle(oracle, dc)
    for i, t in enumerate(toks):
        lb = b.forward([t], 12 + i)
    np.testing.assert_array_equal(la, lb)
