"""GPU parity of the prefill dequant-matmul (cn_matmul, tcgen05) against the
CPU oracle's matvec (TensorMath.MatVecMulQ4_0 / MatVecMulGeneric for Q4_K,
run once per token, the way ChatNet prefills).  Tolerance: max relative
error 1e-3 normalised by the largest reference magnitude of each token's
output (the kernel rounds activations and expanded
weights to fp16 and accumulates in fp32)."""
from __future__ import annotations

import numpy as np
import pytest

import chatnet_b200 as cn
from tests.parity import REL_TOL, rel_err

pytestmark = pytest.mark.gpu


def _w(rows, cols, key, t=cn.TYPE_Q4_0):
    return cn.synth_fill(t, rows, cols, seed=cn.synth_seed(3, key))


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


@pytest.mark.parametrize("wtype", [cn.TYPE_Q4_0, cn.TYPE_Q4_K, cn.TYPE_Q6_K], ids=["q4_0", "q4_k", "q6_k"])
@pytest.mark.parametrize("rows,cols,tokens", MATMUL_CASES,
                         ids=[f"{r}x{c}-m{m}" for r, c, m in MATMUL_CASES])
def test_matmul_parity(ctx, oracle, rows, cols, tokens, wtype):
    if wtype == cn.TYPE_Q6_K and cn.byte_size(wtype, cols) % 16:
        pytest.skip("Q6_K rows of this width are not 16-byte multiples (no TMA tiling)")
    blocks = _w(rows, cols, f"mm.{rows}x{cols}", wtype)
    W = ctx.upload(blocks, wtype, rows, cols)
    x = _x(tokens, cols, f"mm.x.{rows}.{cols}.{tokens}")
    y = ctx.matmul(W, x)
    assert y.shape == (tokens, rows) and np.isfinite(y).all()
    # the oracle on a sample of rows (all of them for small shapes)
    rng = np.random.default_rng(rows * 7 + cols)
    sample = np.arange(rows) if rows <= 512 else np.sort(rng.choice(rows, 384, replace=False))
    Ws = blocks.reshape(rows, -1)[sample].copy()
    ref = oracle.matvec(wtype, Ws, x, len(sample))
    err = rel_err(y[:, sample], ref)
    assert err <= REL_TOL, err


@pytest.mark.parametrize("wtype", [cn.TYPE_Q4_0, cn.TYPE_Q4_K], ids=["q4_0", "q4_k"])
def test_matmul_matches_matvec_rows(ctx, wtype):
    """Token t of the matmul is the matvec of x[t] (same weights, 1e-3)."""
    rows, cols = 1024, 4096
    W = ctx.upload(_w(rows, cols, "mm.mv", wtype), wtype, rows, cols)
    x = _x(96, cols, "mm.mv.x")
    y = ctx.matmul(W, x)
    for t in (0, 1, 63, 95):
        assert rel_err(y[t], ctx.matvec(W, x[t])) <= REL_TOL


def test_matmul_rejects_bad_input(ctx):
    W = ctx.upload(_w(16, 96, "mm.bad"), cn.TYPE_Q4_0, 16, 96)  # cols not a multiple of 256
    with pytest.raises(ValueError):
        ctx.matmul(W, np.zeros((4, 96), np.float32))
    W6 = ctx.upload(cn.synth_fill(cn.TYPE_Q6_K, 16, 256, 5), cn.TYPE_Q6_K, 16, 256)  # 210-byte rows
    with pytest.raises((ValueError, NotImplementedError)):
        ctx.matmul(W6, np.zeros((4, 256), np.float32))
    W2 = ctx.upload(np.zeros(16 * 84, np.uint8), cn.TYPE_Q2_K, 16, 256)  # no matmul decoder
    with pytest.raises((ValueError, NotImplementedError)):
        ctx.matmul(W2, np.zeros((4, 256), np.float32))


def test_matmul_q4_k_scale_extremes(ctx, oracle):
    """Q4_K super-blocks whose 6-bit scales and minima take every value 0..63
    (both halves of the packed scale bytes, DequantQ4K.cs:218-241)."""
    rows, cols = 256, 1024
    blocks = _w(rows, cols, "mm.q4k.sc", cn.TYPE_Q4_K).reshape(rows * cols // 256, 144)
    rng = np.random.default_rng(5)
    blocks[:, 4:16] = rng.integers(0, 256, size=(blocks.shape[0], 12), dtype=np.uint8)
    blocks = blocks.ravel()
    W = ctx.upload(blocks, cn.TYPE_Q4_K, rows, cols)
    x = _x(80, cols, "mm.q4k.sc.x")
    assert rel_err(ctx.matmul(W, x), oracle.matvec(cn.TYPE_Q4_K, blocks, x, rows)) <= REL_TOL


@pytest.mark.parametrize("wtype", [cn.TYPE_Q4_0, cn.TYPE_Q4_K], ids=["q4_0", "q4_k"])
@pytest.mark.parametrize("magnitude", [1e-6, 1.0, 3e5])
def test_matmul_activation_range(ctx, oracle, wtype, magnitude):
    """Tokens far outside fp16 range (either way), with very different scales
    in one call, keep fp32-level accuracy: each token's row is scaled by an
    exact power of two before the fp16 operand is formed."""
    rows, cols = 256, 2048
    blocks = _w(rows, cols, f"mm.range.{wtype}", wtype)
    W = ctx.upload(blocks, wtype, rows, cols)
    x = _x(70, cols, f"mm.range.x.{wtype}") * np.float32(magnitude)
    x[1::3] *= np.float32(1e-3)
    x[5] = 0.0  # an all-zero token
    y = ctx.matmul(W, x)
    ref = oracle.matvec(wtype, blocks, x, rows)
    assert np.isfinite(y).all() and not y[5].any()
    assert rel_err(y, ref) <= REL_TOL
