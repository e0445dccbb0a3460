"""The tensor-parallel sharding scheme on CPU (world size 2, gloo): each rank
takes its shard of every projection (shard_region / host_slice, the same
regions cn_tensor_synth_slice generates), runs the oracle's matvec on it,
and the ranks combine like the GPU path does: partial sums added in rank
order for O/down (input split), slices gathered for q/k/v/gate/up/lm_head
(row split).  The combination must equal the unsharded matvec."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as tmp

import chatnet_b200 as cn
from chatnet_b200 import configs as cf
from chatnet_b200.llama import shard_region, tensor_shape

NAMES = ["blk.0.attn_q.weight", "blk.0.attn_k.weight", "blk.0.attn_output.weight", "blk.0.ffn_up.weight",
         "blk.0.ffn_down.weight", "output.weight"]


def _dc():
    dc = cf.with_layers(cf.CONFIGS[4], 1, 1)
    m = cf.replace(dc.model, dim=512, hidden_dim=1024, n_heads=8, n_kv_heads=2, head_dim=64, vocab=512,
                   ctx_len=64, kv_f16=True)
    return cf.replace(dc, model=m)


def _worker(rank, size, port, results):
    from tests import _oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=size)
    try:
        orc = _oracle.load()
        dc = _dc()
        out = {}
        for name in NAMES:
            rows, cols = tensor_shape(dc.model, name)
            t = cf.tensor_type(dc, name)
            full = cn.synth_fill(t, rows, cols, cn.synth_seed(dc.config_id, name))
            x = cn.synth_fill(cn.TYPE_F32, 1, cols, cn.synth_seed(9, "x." + name))[0]
            r0, nr, c0, nc = shard_region(dc.model, name, rank, size)
            shard = cf.host_slice(full, t, cols, r0, nr, c0, nc)
            y = orc.matvec(t, shard.reshape(-1), x[c0:c0 + nc].copy(), nr)
            y = torch.from_numpy(np.ascontiguousarray(y, dtype=np.float32).reshape(-1))
            if nc != cols:  # input split: gather the partials, add them in rank order
                parts = [torch.empty_like(y) for _ in range(size)]
                dist.all_gather(parts, y)
                comb = parts[0].clone()
                for p in parts[1:]:
                    comb += p
            else:           # row split: concatenate the slices
                parts = [torch.empty_like(y) for _ in range(size)]
                dist.all_gather(parts, y)
                comb = torch.cat(parts)
            if rank == 0:
                ref = orc.matvec(t, full.reshape(-1), x, rows).reshape(-1)
                out[name] = float(np.max(np.abs(comb.numpy() - ref)) / max(1e-30, np.max(np.abs(ref))))
        if rank == 0:
            results.put(out)
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shards_combine_to_full_matvec():
    ctx = tmp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    out = results.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert set(out) == set(NAMES)
    for name, err in out.items():
        assert err <= 1e-5, (name, err)


def test_shard_regions_cover_the_tensor():
    dc = _dc()
    for size in (1, 2):  # 4 would cut O's 512 inputs into 128-column (partial super-block) shards
        for name in NAMES:
            rows, cols = tensor_shape(dc.model, name)
            regs = [shard_region(dc.model, name, r, size) for r in range(size)]
            if all(c0 == 0 and nc == cols for _, _, c0, nc in regs):
                assert [r0 for r0, _, _, _ in regs] == [r * (rows // size) for r in range(size)]
                assert sum(nr for _, nr, _, _ in regs) == rows
            else:
                assert sum(nc for _, _, _, nc in regs) == cols
                assert all(nc % 256 == 0 for _, _, _, nc in regs)  # whole Q4_K super-blocks
