"""One tensor-parallel rank for the multi-GPU parity test (run in a spawned
process, one per GPU).  Builds this rank's shards of a small Q4_K model,
joins the group through IPC handles passed by the parent, decodes, and
returns the logits."""
from __future__ import annotations

import numpy as np


def run_rank(rank: int, size: int, dc, steps: int, to_parent, from_parent) -> None:
    import chatnet_b200 as cn
    from chatnet_b200 import configs as cf
    from chatnet_b200.llama import CudaLlamaModel
    try:
        ctx = cn.Context(rank)
        m = dc.model
        tp = cn.TensorParallel(ctx, rank, size, m.max_batch, m.dim, m.vocab)
        to_parent.put(("handle", rank, tp.ipc_handle()))
        handles = from_parent.get(timeout=120)
        tp.connect(handles)
        ts = cf.device_tensors(ctx, dc, rank=rank, size=size)
        model = CudaLlamaModel(ctx, m, ts, tp=tp)
        for b in range(m.max_batch):
            model.kv_synth(b, dc.kv_filled, *cf.kv_seeds(dc, b))
        model.prepare(m.max_batch)
        to_parent.put(("ready", rank, None))
        assert from_parent.get(timeout=120) == "go"
        B = m.max_batch
        outs = []
        for s in range(steps):
            toks = [cf.token(dc, b, s) for b in range(B)]
            lg, am = model.decode(toks, [dc.decode_pos + s] * B)
            outs.append((lg.copy(), am.copy()))
        model.close()
        for t in ts:
            t.free()
        tp.close()
        ctx.close()
        to_parent.put(("done", rank, outs))
    except Exception as e:  # reported to the parent, which fails the test
        to_parent.put(("error", rank, repr(e)))
