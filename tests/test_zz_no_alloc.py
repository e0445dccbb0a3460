"""cn_matvec_noalloc_dev: the fused dequant-GEMV for hosts that cannot allocate
device memory (they own every buffer, or forbid cudaMalloc/cudaFree while
running).  Its scratch is a fixed array inside the library, so the check here
is that it computes what cn_matvec_dev computes, call after call on the same
reused array, and that it turns away work that does not fit that array.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test."""
from __future__ import annotations

import numpy as np
import pytest

import chatnet_b200 as cn
from chatnet_b200 import _native as N
from tests.parity import REL_TOL, rel_err

pytestmark = pytest.mark.gpu


def _matvec_dev(ctx, t, W, rows, cols, x, batch):
    import torch
    y = torch.empty(batch, rows, device="cuda")
    ctx.synchronize()
    torch.cuda.synchronize()
    N.check(N.lib().cn_matvec_dev(ctx.handle, t, W.device_ptr, rows, cols, x.data_ptr(),
                                  y.data_ptr(), batch), "cn_matvec_dev")
    ctx.synchronize()
    return y.cpu().numpy()


def _noalloc(t, W, rows, cols, x, batch):
    import torch
    y = torch.full((batch, rows), float("nan"), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    N.check(N.lib().cn_matvec_noalloc_dev(t, W.device_ptr, rows, cols, x.data_ptr(), y.data_ptr(),
                                          batch, stream), "cn_matvec_noalloc_dev")
    # no kernel of the call gave up waiting (the status call reads and clears the error word)
    N.check(N.lib().cn_matvec_noalloc_status(stream), "cn_matvec_noalloc_status")
    torch.cuda.synchronize()
    return y.cpu().numpy()


# Q4_0 300x2080 and Q8_0 130x1056 take the untiled (warp-per-row) path (an
# inner dimension that is not a multiple of 256); Q8_0 257x1024 and Q5_K
# 129x768 the tiled fp16 GEMV
CASES = [(cn.TYPE_Q4_K, 11008, 4096, 1), (cn.TYPE_Q4_0, 5632, 2048, 3),
         (cn.TYPE_Q6_K, 4096, 4096, 4), (cn.TYPE_Q4_K, 37, 512, 2),
         (cn.TYPE_Q4_0, 300, 2080, 2), (cn.TYPE_Q8_0, 257, 1024, 1), (cn.TYPE_Q8_0, 130, 1056, 2),
         (cn.TYPE_Q5_K, 129, 768, 3)]


def test_noalloc_matches_matvec_dev(ctx):
    import torch
    for i, (t, rows, cols, batch) in enumerate(CASES):
        if t in (cn.TYPE_Q4_0, cn.TYPE_Q4_K, cn.TYPE_Q6_K):
            W = ctx.synth(t, rows, cols, cn.synth_seed(7, f"noalloc.w.{i}"))
        else:  # no seeded generator for this codec: random block bytes with a small fp16 scale
            W = ctx.upload(_random_blocks(t, rows, cols, i), t, rows, cols)
        x = torch.from_numpy(
            cn.synth_fill(cn.TYPE_F32, batch, cols, cn.synth_seed(7, f"noalloc.x.{i}"))).cuda()
        ref = _matvec_dev(ctx, t, W, rows, cols, x, batch)
        # two calls in a row on the shared array (the second sees the first's leftovers)
        y1 = _noalloc(t, W, rows, cols, x, batch)
        y2 = _noalloc(t, W, rows, cols, x, batch)
        assert np.isfinite(y1).all() and np.isfinite(y2).all()
        assert rel_err(y1, ref) <= REL_TOL, (i, rel_err(y1, ref))
        assert rel_err(y2, ref) <= REL_TOL, (i, rel_err(y2, ref))
        W.free()


def _random_blocks(t, rows, cols, seed):
    """Random bytes of `rows` rows of type t whose fp16 scale fields hold 0.01 (so values stay finite)."""
    rng = np.random.default_rng(1000 + seed)
    rb = cn.byte_size(t, cols)
    raw = rng.integers(0, 256, size=(rows, rb), dtype=np.uint8)
    blk, bpb = {cn.TYPE_Q8_0: (32, 34), cn.TYPE_Q5_K: (256, 176)}[t]
    v = raw.reshape(rows, cols // blk, bpb)
    half = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    v[:, :, 0:2] = half  # Q8_0: d; Q5_K: d
    if t == cn.TYPE_Q5_K:
        v[:, :, 2:4] = half  # dmin
    return raw


def test_noalloc_allocates_nothing(ctx):
    import torch
    t, rows, cols, batch = cn.TYPE_Q4_K, 4096, 8192, 1
    W = ctx.synth(t, rows, cols, cn.synth_seed(7, "noalloc.mem.w"))
    x = torch.from_numpy(cn.synth_fill(cn.TYPE_F32, batch, cols, cn.synth_seed(7, "noalloc.mem.x"))).cuda()
    y = torch.empty(batch, rows, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        N.check(N.lib().cn_matvec_noalloc_dev(t, W.device_ptr, rows, cols, x.data_ptr(),
                                              y.data_ptr(), batch, stream))
        torch.cuda.synchronize()
    call()  # the first call on the device loads the array's address
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        call()
    assert torch.cuda.mem_get_info()[0] == free0
    W.free()


def test_noalloc_rejects_oversized_work(ctx):
    import torch
    t, rows, cols, batch = cn.TYPE_Q4_K, 1024, 28672, 32
    W = ctx.synth(t, rows, cols, cn.synth_seed(7, "noalloc.big.w"))
    x = torch.zeros(batch, cols, device="cuda")
    y = torch.zeros(batch, rows, device="cuda")
    with pytest.raises(ValueError, match="scratch"):
        N.check(N.lib().cn_matvec_noalloc_dev(t, W.device_ptr, rows, cols, x.data_ptr(),
                                              y.data_ptr(), batch, None))
    W.free()
