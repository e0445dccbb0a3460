"""One tensor-parallel rank for the multi-GPU parity test (run in a spawned
process, one per GPU).  Builds this rank's shards of a small Q4_K model,
joins the group through IPC handles passed by the parent, decodes, and
returns the logits."""
from __future__ import annotations

import numpy as np


def run_rank(rank: int, size: int, dc, steps: int, to_parent, from_parent, gguf_path: str | None = None) -> None:
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
        if gguf_path:  # this rank's shards straight from the file (cn_llama_create_from_gguf_tp)
            from chatnet_b200.gguf import GgufFile
            with GgufFile(gguf_path) as g:
                model = g.llama_model(ctx, m.max_batch, kv_f16=m.kv_f16, tp=tp)
            ts = []
        else:
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


def run_rank_stalled(rank: int, size: int, dc, to_parent, from_parent) -> None:
    """Failure-detection worker: every rank joins the group; rank 0 then
    decodes a step while rank 1 never does.  Rank 0 reports how its decode
    ended, and whether its context still runs work afterwards; every rank
    tears down only when the parent says so (after all ranks are done), so
    no rank unmaps an exchange buffer a peer's kernels may still write."""
    import time

    import numpy as np

    import chatnet_b200 as cn
    from chatnet_b200 import configs as cf
    from chatnet_b200.llama import CudaLlamaModel
    try:
        ctx = cn.Context(rank)
        m = dc.model
        tp = cn.TensorParallel(ctx, rank, size, m.max_batch, m.dim, m.vocab)
        to_parent.put(("handle", rank, tp.ipc_handle()))
        tp.connect(from_parent.get(timeout=120))
        ts = cf.device_tensors(ctx, dc, rank=rank, size=size)
        model = CudaLlamaModel(ctx, m, ts, tp=tp)
        model.kv_synth(0, dc.kv_filled, *cf.kv_seeds(dc, 0))
        model.prepare(1)
        to_parent.put(("ready", rank, None))
        assert from_parent.get(timeout=120) == "go"
        result = None
        if rank == 0:
            t0 = time.time()
            kind = "no error"
            try:
                model.decode([cf.token(dc, 0, 0)], [dc.decode_pos])
            except TimeoutError:
                kind = "timeout"
            elapsed = time.time() - t0
            # the context still runs work: a small GEMV on the same stream
            W = ctx.synth(cn.TYPE_Q4_K, 256, 512, 7)
            y = ctx.matvec(W, np.ones(512, np.float32))
            result = (kind, elapsed, bool(np.isfinite(y).all()))
            W.free()
        to_parent.put(("done", rank, result))
        assert from_parent.get(timeout=120) == "teardown"
        model.close()
        for t in ts:
            t.free()
        tp.close()
        ctx.close()
        to_parent.put(("closed", rank, None))
    except Exception as e:  # reported to the parent, which fails the test
        to_parent.put(("error", rank, repr(e)))
