"""GPU parity of the prefill dequant-matmul (cn_matmul, tcgen05) against the
CPU oracle's matvec (TensorMath.MatVecMulQ4_0 run once per token, the way
ChatNet prefills).  Tolerance: max relative error 1e-3 normalised by the
largest reference magnitude of each token's output (
the kernel rounds activations and expanded weights to fp16 and accumulates
in fp32)."""
from __future__ import annotations

import numpy as np
import pytest

import chatnet_b200 as cn
from tests.parity import REL_TOL, rel_err

pytestmark = pytest.mark.gpu


def _w(rows, cols, key):
    return cn.synth_fill(cn.TYPE_Q4_0, rows, cols, seed=cn.synth_seed(3, key))


def _x(tokens, cols, key):
    return cn.synth_fill(cn.TYPE_F32, tokens, cols, cn.synth_seed(3, key))


MATMUL_CASES = [
    # (rows, cols, tokens): config 3's projections at M = 512, then edges
    (4096, 4096, 512),    # q / k / v / o
    (11008, 4096, 512),   # gate / up
    (4096, 11008, 512),   # down (43 runs of 8 blocks per row)
    (4096, 4096, 64),     # the smallest prefill the engine routes here
    (200, 256, 1),        # one token, ragged row tile, one 256-position run
    (128, 2304, 300),     # ragged token tile (300 = 256 + 44)
    (5632, 2048, 37),     # TinyLlama FFN shape, few tokens
]


@pytest.mark.parametrize("rows,cols,tokens", MATMUL_CASES,
                         ids=[f"{r}x{c}-m{m}" for r, c, m in MATMUL_CASES])
def test_matmul_parity(ctx, oracle, rows, cols, tokens):
    blocks = _w(rows, cols, f"mm.{rows}x{cols}")
    W = ctx.upload(blocks, cn.TYPE_Q4_0, rows, cols)
    x = _x(tokens, cols, f"mm.x.{rows}.{cols}.{tokens}")
    y = ctx.matmul(W, x)
    assert y.shape == (tokens, rows) and np.isfinite(y).all()
    # the oracle on a sample of rows (all of them for small shapes)
    rng = np.random.default_rng(rows * 7 + cols)
    sample = np.arange(rows) if rows <= 512 else np.sort(rng.choice(rows, 384, replace=False))
    Ws = blocks.reshape(rows, -1)[sample].copy()
    ref = oracle.matvec(cn.TYPE_Q4_0, Ws, x, len(sample))
    err = rel_err(y[:, sample], ref)
    assert err <= REL_TOL, err


def test_matmul_matches_matvec_rows(ctx):
    """Token t of the matmul is the matvec of x[t] (same weights, 1e-3)."""
    rows, cols = 1024, 4096
    W = ctx.upload(_w(rows, cols, "mm.mv"), cn.TYPE_Q4_0, rows, cols)
    x = _x(96, cols, "mm.mv.x")
    y = ctx.matmul(W, x)
    for t in (0, 1, 63, 95):
        assert rel_err(y[t], ctx.matvec(W, x[t])) <= REL_TOL


def test_matmul_rejects_bad_input(ctx):
    W = ctx.upload(_w(16, 96, "mm.bad"), cn.TYPE_Q4_0, 16, 96)  # cols not a multiple of 256
    with pytest.raises(ValueError):
        ctx.matmul(W, np.zeros((4, 96), np.float32))
    Wk = ctx.upload(cn.synth_fill(cn.TYPE_Q4_K, 16, 256, 5), cn.TYPE_Q4_K, 16, 256)
    with pytest.raises((ValueError, NotImplementedError)):
        ctx.matmul(Wk, np.zeros((4, 256), np.float32))
