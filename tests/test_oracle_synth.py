"""The oracle-side generator (oracle/synth.cpp) writes the same bytes as the
product's host generator (cn_synth_seed / cn_synth_fill), so the CPU legs of
bench.py can build the configs' tensors without loading libchatnet_cuda.
Runs on the CPU: both generators are host code."""
from __future__ import annotations

import numpy as np
import pytest

import chatnet_b200 as cn
from chatnet_b200 import configs as cf
from tests import _oracle


@pytest.mark.parametrize("name", ["token_embd.weight", "blk.3.attn_q.weight", "kv.k.0", "", "x" * 200])
@pytest.mark.parametrize("config_id", [0, 1, 3, 4, -7])
def test_seed_matches(oracle, config_id, name):
    assert oracle.synth_seed(config_id, name) == cn.synth_seed(config_id, name)


@pytest.mark.parametrize("type_,rows,cols,norm_w", [
    (cn.TYPE_Q4_0, 37, 2048, False), (cn.TYPE_Q4_0, 1, 32, False),
    (cn.TYPE_Q4_K, 19, 4096, False), (cn.TYPE_Q4_K, 300, 256, False),
    (cn.TYPE_Q6_K, 23, 4096, False), (cn.TYPE_F32, 7, 4100, False), (cn.TYPE_F32, 1, 8192, True),
    (cn.TYPE_F16, 33, 1024, False)])
def test_fill_matches(oracle, type_, rows, cols, norm_w):
    seed = cn.synth_seed(4, f"t{type_}.{rows}x{cols}")
    want = cn.synth_fill(type_, rows, cols, seed, cn.DIST_NORM_W if norm_w else None)
    got = oracle.synth_fill(type_, rows, cols, seed, norm_w)
    assert got.dtype == want.dtype and got.shape == want.shape
    assert np.array_equal(got.view(np.uint8), want.view(np.uint8))


def test_config_helpers_match(oracle):
    dc = cf.with_layers(cf.CONFIGS[1], 1)
    want = cf.host_tensors(dc)
    got = _oracle.host_tensors(oracle, dc)
    assert want.keys() == got.keys()
    for k in want:
        assert np.array_equal(got[k].view(np.uint8), want[k].view(np.uint8)), k
    for seq in (0, 3):
        assert _oracle.token(oracle, dc, seq, 2) == cf.token(dc, seq, 2)
        for a, b in zip(_oracle.host_kv(oracle, dc, seq), cf.host_kv(dc, seq)):
            assert np.array_equal(a.view(np.uint8), b.view(np.uint8))
    d3 = cf.CONFIGS[3]
    assert np.array_equal(_oracle.prefill_x(oracle, d3, 9), cf.prefill_x(d3, 9))


@pytest.mark.parametrize("type_,cols", [(cn.TYPE_Q4_0, 2048), (cn.TYPE_Q4_K, 512), (cn.TYPE_Q6_K, 256),
                                        (cn.TYPE_F32, 100), (cn.TYPE_F16, 64)])
def test_row_slices(oracle, type_, cols):
    seed = oracle.synth_seed(4, "rows")
    full = oracle.synth_fill(type_, 23, cols, seed).view(np.uint8).reshape(23, -1)
    part = oracle.synth_fill(type_, 9, cols, seed, row0=7).view(np.uint8).reshape(9, -1)
    assert np.array_equal(full[7:16], part)


def test_layer_kv_slices(oracle):
    dc = cf.with_layers(cf.CONFIGS[4], 3)
    dc = cf.replace(dc, model=cf.replace(dc.model, ctx_len=16, n_kv_heads=1, head_dim=8), kv_filled=11)
    k, v = _oracle.host_kv(oracle, dc, 2)
    for layer in range(3):
        lk, lv = _oracle.layer_kv(oracle, dc, 2, layer)
        assert np.array_equal(lk, k[layer * 16:(layer + 1) * 16]) and np.array_equal(lv, v[layer * 16:(layer + 1) * 16])


def test_bad_requests(oracle):
    buf = np.empty(18, np.uint8)
    assert oracle.lib.or_synth_fill(cn.TYPE_Q4_0, 1, 32, 1, 0, buf.ctypes.data, 17) == -1
    assert oracle.lib.or_synth_fill(cn.TYPE_Q4_0, 1, 16, 1, 0, buf.ctypes.data, 9) == -1
    assert oracle.lib.or_synth_fill(cn.TYPE_Q8_0, 1, 32, 1, 0, buf.ctypes.data, 34) == -2
