"""Tensor parallelism across GPUs (one process per GPU, cn_tp_* + CUDA IPC):
a small Q4_K Llama sharded over 2 ranks decodes the same logits as the
oracle's single-CPU restatement (max relative error 1e-3, equal argmax), and
every rank ends with bitwise the same all-gathered logits.  Needs two GPUs;
skipped otherwise."""
from __future__ import annotations

import multiprocessing as mp
import queue

import numpy as np
import pytest
import torch

import chatnet_b200 as cn
from chatnet_b200 import configs as cf
from chatnet_b200.llama import tensor_names
from tests import _oracle
from tests.parity import REL_TOL, rel_err
from tests.tp_worker import run_rank, run_rank_stalled

pytestmark = pytest.mark.gpu


def tp_dc(max_batch=1, n_layers=2):
    dc = cf.with_layers(cf.CONFIGS[4], n_layers, max_batch)
    m = cf.replace(dc.model, dim=512, hidden_dim=1024, n_heads=8, n_kv_heads=2, head_dim=64,
                   vocab=512, ctx_len=64, kv_f16=True)
    return cf.replace(dc, model=m, kv_filled=20, decode_pos=20)


def tp8_dc(n_layers=2):
    """Shapes that shard over 2, 4 and 8 ranks: 32 heads of 64 over 8 kv heads (one
    per rank at 8), O and down input split into whole 256-column super-blocks."""
    dc = cf.with_layers(cf.CONFIGS[4], n_layers, 1)
    m = cf.replace(dc.model, dim=2048, hidden_dim=2048, n_heads=32, n_kv_heads=8, head_dim=64,
                   vocab=512, ctx_len=64, kv_f16=True)
    return cf.replace(dc, model=m, kv_filled=20, decode_pos=20)


def run_group(dc, size, steps, gguf_path=None):
    ctx = mp.get_context("spawn")
    to_parent = ctx.Queue()
    to_child = [ctx.Queue() for _ in range(size)]
    procs = [ctx.Process(target=run_rank, args=(r, size, dc, steps, to_parent, to_child[r], gguf_path), daemon=True)
             for r in range(size)]
    for p in procs:
        p.start()
    try:
        def collect(kind):
            got = {}
            while len(got) < size:
                k, r, v = to_parent.get(timeout=300)
                if k == "error":
                    raise AssertionError(f"rank {r}: {v}")
                assert k == kind, (k, kind)
                got[r] = v
            return [got[r] for r in range(size)]
        handles = collect("handle")
        for q in to_child:
            q.put(handles)
        collect("ready")
        for q in to_child:
            q.put("go")
        return collect("done")
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("batch", [1, 3])
def test_tp2_decode_matches_oracle(oracle, batch):
    dc = tp_dc(max_batch=batch)
    steps = 3
    res = run_group(dc, 2, steps)
    # every rank holds the same all-gathered logits
    for s in range(steps):
        np.testing.assert_array_equal(res[0][s][0], res[1][s][0])
        np.testing.assert_array_equal(res[0][s][1], res[1][s][1])
    host = cf.host_tensors(dc)
    names = tensor_names(dc.model.n_layers)
    types = [cf.tensor_type(dc, n) for n in names]
    for b in range(batch):
        k, v = cf.host_kv(dc, b)
        orc = _oracle.OracleLlama(oracle, dc.model, host, types, names, k.copy(), v.copy())
        for s in range(steps):
            ref = orc.forward([cf.token(dc, b, s)], dc.decode_pos + s)
            got = res[0][s][0][b]
            assert rel_err(got, ref) <= REL_TOL, (b, s, rel_err(got, ref))
            assert int(res[0][s][1][b]) == int(np.argmax(ref))


def _check_against_oracle(oracle, dc, res, steps, batch):
    size = len(res)
    for s in range(steps):
        for r in range(1, size):
            np.testing.assert_array_equal(res[0][s][0], res[r][s][0])
            np.testing.assert_array_equal(res[0][s][1], res[r][s][1])
    host = cf.host_tensors(dc)
    names = tensor_names(dc.model.n_layers)
    types = [cf.tensor_type(dc, n) for n in names]
    for b in range(batch):
        k, v = cf.host_kv(dc, b)
        orc = _oracle.OracleLlama(oracle, dc.model, host, types, names, k.copy(), v.copy())
        for s in range(steps):
            ref = orc.forward([cf.token(dc, b, s)], dc.decode_pos + s)
            got = res[0][s][0][b]
            assert rel_err(got, ref) <= REL_TOL, (b, s, rel_err(got, ref))
            assert int(res[0][s][1][b]) == int(np.argmax(ref))


@pytest.mark.parametrize("size", [2, 4, 8])
def test_tp_n_decode_matches_oracle(oracle, size):
    """The same model on 2, 4 and 8 ranks (where that many GPUs exist)."""
    if torch.cuda.device_count() < size:
        pytest.skip(f"needs {size} GPUs")
    dc = tp8_dc()
    steps = 3
    _check_against_oracle(oracle, dc, run_group(dc, size, steps), steps, 1)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("tied", [False, True])
def test_tp2_from_gguf_file(oracle, tmp_path, tied):
    """Each rank builds its shards straight from a GGUF file
    (cn_llama_create_from_gguf_tp, cn_tensor_upload_slice), with lm_head
    tied to token_embd or not; the logits match the oracle's."""
    from tests import gguf_writer as gw
    dc = tp8_dc()
    m = dc.model
    host = cf.host_tensors(dc)
    if tied:
        host["output.weight"] = host["token_embd.weight"]
    names = tensor_names(m.n_layers)
    types = [cf.tensor_type(dc, n) for n in names]
    path = tmp_path / "tp.gguf"
    gw.write_gguf(path, gw.llama_metadata(m), gw.llama_tensors(host, names, types, m, tie_output=tied))
    steps = 2
    res = run_group(dc, 2, steps, gguf_path=str(path))
    for s in range(steps):
        np.testing.assert_array_equal(res[0][s][0], res[1][s][0])
    k, v = cf.host_kv(dc, 0)
    orc = _oracle.OracleLlama(oracle, m, host, types, names, k.copy(), v.copy())
    for s in range(steps):
        ref = orc.forward([cf.token(dc, 0, s)], dc.decode_pos + s)
        assert rel_err(res[0][s][0][0], ref) <= REL_TOL, (s, rel_err(res[0][s][0][0], ref))
        assert int(res[0][s][1][0]) == int(np.argmax(ref))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_missing_rank_times_out():
    """Failure detection without a GPU fault: rank 1 joins the group (its
    exchange buffer mapped, its process alive) but never runs the step, so
    rank 0's first exchange wait runs out.  Rank 0's decode returns
    CN_ERR_TIMEOUT (TimeoutError) after about the 2 s wait limit -- the later
    waits of the step give up at once -- and its context still runs work."""
    dc = tp8_dc()
    ctx = mp.get_context("spawn")
    to_parent = ctx.Queue()
    to_child = [ctx.Queue() for _ in range(2)]
    procs = [ctx.Process(target=run_rank_stalled, args=(r, 2, dc, to_parent, to_child[r]), daemon=True)
             for r in range(2)]
    for p in procs:
        p.start()
    try:
        def collect(kind):
            got = {}
            while len(got) < 2:
                k, r, v = to_parent.get(timeout=300)
                if k == "error":
                    raise AssertionError(f"rank {r}: {v}")
                assert k == kind, (k, kind)
                got[r] = v
            return [got[r] for r in range(2)]
        handles = collect("handle")
        for q in to_child:
            q.put(handles)
        collect("ready")
        for q in to_child:
            q.put("go")
        done = collect("done")
        for q in to_child:  # the host barrier: both ranks are idle, now they may tear down
            q.put("teardown")
        collect("closed")
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    kind, elapsed, usable = done[0]
    assert kind == "timeout", kind
    assert 1.5 < elapsed < 30.0, elapsed
    assert usable
