"""GPU parity of the block dequantizers (bit-exact) and the fused dequant-GEMVs
(max relative error 1e-3) against the CPU oracle, through the C ABI."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import chatnet_b200 as cn
from tests.parity import REL_TOL, bits_equal, rel_err

pytestmark = pytest.mark.gpu

KAT = json.loads((Path(__file__).parent / "golden" / "kat_quant.json").read_text())
Q = {"q4_0": cn.TYPE_Q4_0, "q4_k": cn.TYPE_Q4_K, "q6_k": cn.TYPE_Q6_K}


@pytest.mark.parametrize("case", KAT["cases"], ids=lambda c: c["name"])
def test_kat_on_gpu(ctx, oracle, case):
    blocks = np.array(case["blocks"], dtype=np.uint8)
    n = case["n"]
    W = ctx.upload(blocks, case["type"], 1, n)
    got = ctx.dequantize(W).ravel()
    assert bits_equal(got, oracle.dequantize(case["type"], blocks, n))
    np.testing.assert_allclose(got, case["dequant"], rtol=0, atol=case["tol"])
    if "x" in case:
        y = ctx.matvec(W, np.array(case["x"], np.float32))
        assert abs(float(y[0]) - case["dot"]) <= case["tol"]


@pytest.mark.parametrize("name,rows,cols", [
    ("q4_0", 5632, 2048), ("q4_0", 7, 96), ("q4_k", 4096, 4096), ("q4_k", 3, 512),
    ("q6_k", 512, 4096), ("q6_k", 5, 768)])
def test_dequantize_bit_exact(ctx, oracle, name, rows, cols):
    t = Q[name]
    blocks = cn.synth_fill(t, rows, cols, seed=cn.synth_seed(2, f"deq.{name}.{rows}x{cols}"))
    W = ctx.upload(blocks, t, rows, cols)
    got = ctx.dequantize(W)
    ref = oracle.dequantize(t, blocks, rows * cols).reshape(rows, cols)
    assert bits_equal(got, ref)
    # a row window
    part = ctx.dequantize(W, 1, rows - 2) if rows > 2 else got
    assert bits_equal(part, ref[1:rows - 1] if rows > 2 else ref)


def test_dequantize_q4_0_partial_block(ctx, oracle):
    """Dequantize handles a partial last block (DequantQ4_0.cs:39-53)."""
    rows, cols = 3, 45  # 2 blocks per row, the second holds 13 values
    blocks = np.random.default_rng(0).integers(0, 256, size=rows * 36, dtype=np.uint8)
    blocks.reshape(rows, 2, 18)[:, :, 1] = 0x1C  # finite fp16 scales
    W = ctx.upload(blocks, cn.TYPE_Q4_0, rows, cols)
    got = ctx.dequantize(W)
    for r in range(rows):
        ref = oracle.dequantize(cn.TYPE_Q4_0, blocks[r * 36:(r + 1) * 36], cols)
        assert bits_equal(got[r], ref)


def test_device_synth_matches_host(ctx):
    for t, rows, cols in [(cn.TYPE_Q4_0, 33, 2048), (cn.TYPE_Q4_K, 17, 4096),
                          (cn.TYPE_Q6_K, 9, 4096), (cn.TYPE_F32, 3, 999), (cn.TYPE_F16, 5, 128)]:
        seed = cn.synth_seed(9, f"synth.{t}")
        host = cn.synth_fill(t, rows, cols, seed).view(np.uint8).ravel()
        dev = ctx.synth(t, rows, cols, seed).download()
        assert np.array_equal(host, dev), t
    w = ctx.synth(cn.TYPE_F32, 1, 4096, 11, dist=cn.DIST_NORM_W).download()
    assert np.array_equal(w, cn.synth_fill(cn.TYPE_F32, 1, 4096, 11, cn.DIST_NORM_W).view(np.uint8).ravel())


def _x(batch, cols, key):
    return cn.synth_fill(cn.TYPE_F32, batch, cols, cn.synth_seed(2, key))


MATVEC_CASES = [
    # (type, rows, cols, batches) -- configs 0 and 2 of the benchmark, every batch size
    ("q4_0", 5632, 2048, (1, 4, 16, 32)),
    ("q4_k", 4096, 4096, (1, 4, 16, 32)),
    ("q4_k", 11008, 4096, (1, 4, 16, 32)),
    ("q4_k", 4096, 11008, (1, 4, 16, 32)),
    ("q6_k", 32000, 4096, (1, 4, 16, 32)),
]


@pytest.mark.parametrize("name,rows,cols,batches", MATVEC_CASES,
                         ids=[f"{c[0]}-{c[1]}x{c[2]}" for c in MATVEC_CASES])
def test_matvec_parity(ctx, oracle, name, rows, cols, batches):
    t = Q[name]
    blocks = cn.synth_fill(t, rows, cols, seed=cn.synth_seed(2, f"mv.{name}.{rows}x{cols}"))
    W = ctx.upload(blocks, t, rows, cols)
    for b in batches:  # every output row against the oracle
        x = _x(b, cols, f"mv.x.{name}.{rows}.{b}")
        y = ctx.matvec(W, x)
        ref = oracle.matvec(t, blocks, x, rows)
        err = rel_err(y, ref)
        assert err <= REL_TOL, (b, err)
        assert np.isfinite(y).all()


@pytest.mark.parametrize("name,rows,cols", [
    ("q4_0", 37, 96),      # rows not 16-aligned; row bytes not 16-aligned -> generic path
    ("q4_0", 16, 256),
    ("q4_0", 100, 2304),   # row bytes 1296 = 81*16 -> tiled path, ragged tile
    ("q4_k", 21, 256),
    ("q6_k", 19, 768),     # 630-byte rows -> generic path
    ("q6_k", 40, 2048)])
@pytest.mark.parametrize("batch", [1, 3, 5, 13])
def test_matvec_edge_shapes(ctx, oracle, name, rows, cols, batch):
    t = Q[name]
    blocks = cn.synth_fill(t, rows, cols, seed=cn.synth_seed(2, f"edge.{name}.{rows}x{cols}"))
    W = ctx.upload(blocks, t, rows, cols)
    x = _x(batch, cols, f"edge.x.{rows}.{cols}.{batch}")
    y = ctx.matvec(W, x)
    ref = oracle.matvec(t, blocks, x, rows)
    assert rel_err(y, ref) <= REL_TOL


TC_CASES = [
    # Q4_K decode at batch 1..8: integer mma.sync path (128-row tiles, stream-K)
    (300, 768),     # ragged last tile
    (1, 256),       # one row, one unit
    (7, 4096),      # one tile shared by 7 CTAs
    (1024, 8192),   # Llama-2-70B k/v projection: 7 CTAs per tile (clusters of 7 at batch 1-2)
    (2048, 5632),   # inner dimension not a power of two
    (8000, 8192),   # 63 tiles, ragged last: two CTAs per tile, clusters of 2 at batch 1-2
]


@pytest.mark.parametrize("rows,cols", TC_CASES, ids=[f"{r}x{c}" for r, c in TC_CASES])
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 8])
def test_matvec_q4_k_decode(ctx, oracle, rows, cols, batch):
    t = cn.TYPE_Q4_K
    blocks = cn.synth_fill(t, rows, cols, seed=cn.synth_seed(2, f"tc.{rows}x{cols}"))
    W = ctx.upload(blocks, t, rows, cols)
    x = _x(batch, cols, f"tc.x.{rows}.{cols}.{batch}")
    y = ctx.matvec(W, x)
    ref = oracle.matvec(t, blocks, x, rows)
    assert np.isfinite(y).all()
    assert rel_err(y, ref) <= REL_TOL


@pytest.mark.parametrize("rows,cols,batch", [(4096, 11008, 4), (8192, 8192, 1), (1024, 8192, 2)])
def test_matvec_repeatable(ctx, rows, cols, batch):
    """Stream-K partials (and cluster splits of 2 and 7 CTAs per tile) are
    combined in a fixed order: results are bitwise stable."""
    blocks = cn.synth_fill(cn.TYPE_Q4_K, rows, cols, seed=5)
    W = ctx.upload(blocks, cn.TYPE_Q4_K, rows, cols)
    x = _x(batch, cols, "rep")
    y0 = ctx.matvec(W, x)
    for _ in range(3):
        assert bits_equal(ctx.matvec(W, x), y0)


def test_matvec_errors(ctx):
    blocks = cn.synth_fill(cn.TYPE_Q4_0, 16, 64, seed=1)
    W = ctx.upload(blocks, cn.TYPE_Q4_0, 16, 64)
    with pytest.raises(ValueError):
        ctx.matvec(W, np.zeros((33, 64), np.float32))
    with pytest.raises(cn.NotSupportedError):
        ctx.upload(np.zeros(36, np.uint8), 9, 1, 32)  # Q8_1: no decoder (and none in the reference)
    with pytest.raises(ValueError):
        ctx.upload(np.zeros(17, np.uint8), cn.TYPE_Q4_0, 1, 32)  # wrong byte count


@pytest.mark.parametrize("name", ["q4_0", "q4_k", "q6_k"])
@pytest.mark.parametrize("magnitude", [1e-6, 1.0, 3e5])
def test_matvec_activation_range(ctx, oracle, name, magnitude):
    """Activations far outside fp16 range (either way) keep fp32-level accuracy:
    the prep rescales each sequence by an exact power of two."""
    t = Q[name]
    rows, cols = 256, 2048
    blocks = cn.synth_fill(t, rows, cols, seed=cn.synth_seed(2, f"range.{name}"))
    W = ctx.upload(blocks, t, rows, cols)
    x = _x(3, cols, f"range.x.{name}") * np.float32(magnitude)
    x[1] *= np.float32(1e-3)   # sequences with very different scales in one batch
    y = ctx.matvec(W, x)
    ref = oracle.matvec(t, blocks, x, rows)
    assert np.isfinite(y).all()
    assert rel_err(y, ref) <= REL_TOL


# The 32-weight codecs decoded through the generic paths: Q4_1, Q5_0, Q5_1, Q8_0
# (block bytes, offsets of the fp16 fields d and m)
B32 = {"q4_1": (cn.TYPE_Q4_1, 20, (0, 2)), "q5_0": (cn.TYPE_Q5_0, 22, (0,)),
       "q5_1": (cn.TYPE_Q5_1, 24, (0, 2)), "q8_0": (cn.TYPE_Q8_0, 34, (0,)),
       "iq4_nl": (cn.TYPE_IQ4_NL, 18, (0,))}


def _rand_b32(name, rows, cols, seed):
    t, bpb, halves = B32[name]
    rng = np.random.default_rng(seed)
    nb = rows * ((cols + 31) // 32)
    blocks = rng.integers(0, 256, size=(nb, bpb), dtype=np.uint8)
    for k, off in enumerate(halves):  # finite scales (d) and minima (m)
        v = (np.abs(rng.standard_normal(nb)) * 0.01 if k == 0 else rng.standard_normal(nb) * 0.01).astype(np.float16)
        blocks[:, off:off + 2] = v.view(np.uint8).reshape(nb, 2)
    return t, blocks.ravel()


@pytest.mark.parametrize("name", list(B32))
def test_block32_dequantize_bit_exact(ctx, oracle, name):
    t, blocks = _rand_b32(name, 37, 96, 11)
    W = ctx.upload(blocks, t, 37, 96)
    assert bits_equal(ctx.dequantize(W), oracle.dequantize(t, blocks, 37 * 96).reshape(37, 96))
    # a partial last block (45 = 32 + 13 values in one row)
    t, blocks = _rand_b32(name, 1, 45, 12)
    W = ctx.upload(blocks, t, 1, 45)
    assert bits_equal(ctx.dequantize(W).ravel(), oracle.dequantize(t, blocks, 45))


@pytest.mark.parametrize("name", list(B32))
@pytest.mark.parametrize("batch", [1, 3])
def test_block32_matvec_parity(ctx, oracle, name, batch):
    rows, cols = 300, 2048
    t, blocks = _rand_b32(name, rows, cols, 13)
    W = ctx.upload(blocks, t, rows, cols)
    x = _x(batch, cols, f"b32.x.{name}.{batch}")
    assert rel_err(ctx.matvec(W, x), oracle.matvec(t, blocks, x, rows)) <= REL_TOL


@pytest.mark.parametrize("name", ["q4_1", "q5_0", "q5_1"])
@pytest.mark.parametrize("rows,cols,batch", [(4096, 4096, 1), (300, 2048, 3), (1000, 4096, 8), (129, 768, 16),
                                            (257, 1024, 32), (96, 1056, 2)])
def test_b32_tiled_matvec_parity(ctx, oracle, name, rows, cols, batch):
    """Q4_1 / Q5_0 / Q5_1 on the tiled fp16 GEMV (whole 256-column units:
    every n-tile count, partial row tiles, the cluster split at batch 1-8)
    and, at 1056 columns, on the generic kernel."""
    t, blocks = _rand_b32(name, rows, cols, 51 + batch)
    W = ctx.upload(blocks, t, rows, cols)
    x = _x(batch, cols, f"b32t.x.{name}.{rows}.{cols}.{batch}")
    assert rel_err(ctx.matvec(W, x), oracle.matvec(t, blocks, x, rows)) <= REL_TOL


@pytest.mark.parametrize("rows,cols,batch", [(4096, 4096, 1), (300, 2048, 5), (1000, 4096, 16), (129, 768, 32),
                                            (96, 1056, 2)])
def test_q8_0_matvec_parity(ctx, oracle, rows, cols, batch):
    """Q8_0 on the tiled fp16 GEMV (whole 256-column units: every n-tile
    count, a partial row tile) and, at 1056 columns, on the generic kernel."""
    t, blocks = _rand_b32("q8_0", rows, cols, 31 + batch)
    W = ctx.upload(blocks, t, rows, cols)
    x = _x(batch, cols, f"q8.x.{rows}.{cols}.{batch}")
    assert rel_err(ctx.matvec(W, x), oracle.matvec(t, blocks, x, rows)) <= REL_TOL


# The 256-weight super-block codecs on the generic paths: Q2_K, Q3_K, Q5_K,
# Q8_K, IQ4_XS and the reference's simplified IQ2/IQ3/IQ1 decodes (block
# bytes, offsets of the fp16 scale fields; Q8_K's scale is an fp32 at 0).
# IQ3_S reads sign and scale bytes past its 110-byte block (the next block's
# bytes; 0 past the tensor): the row slice below starts inside the tensor, so
# its last block reads the following row's bytes, as the whole tensor does.
SB = {"q2_k": (cn.TYPE_Q2_K, 84, (80, 82)), "q3_k": (cn.TYPE_Q3_K, 110, (108,)),
      "q5_k": (cn.TYPE_Q5_K, 176, (0, 2)), "q8_k": (cn.TYPE_Q8_K, 292, ()),
      "iq4_xs": (cn.TYPE_IQ4_XS, 136, (0,)), "iq3_s": (cn.TYPE_IQ3_S, 110, (0,)),
      "iq3_xxs": (cn.TYPE_IQ3_XXS, 98, (0,)), "iq2_xs": (cn.TYPE_IQ2_XS, 74, (0,)),
      "iq2_xxs": (cn.TYPE_IQ2_XXS, 66, (0,)), "iq2_s": (cn.TYPE_IQ2_S, 82, (0,)),
      "iq1_s": (cn.TYPE_IQ1_S, 50, (0,)), "iq1_m": (cn.TYPE_IQ1_M, 56, (0,))}


def _rand_sb(name, rows, cols, seed):
    t, bpb, halves = SB[name]
    rng = np.random.default_rng(seed)
    nb = rows * (cols // 256)
    blocks = rng.integers(0, 256, size=(nb, bpb), dtype=np.uint8)
    for off in halves:  # finite scales
        v = (np.abs(rng.standard_normal(nb)) * 0.01).astype(np.float16)
        blocks[:, off:off + 2] = v.view(np.uint8).reshape(nb, 2)
    if t == cn.TYPE_Q8_K:
        v = (np.abs(rng.standard_normal(nb)) * 0.01).astype("<f4")
        blocks[:, 0:4] = v.view(np.uint8).reshape(nb, 4)
    return t, blocks.ravel()


@pytest.mark.parametrize("rows,cols,batch", [(4096, 4096, 1), (300, 2048, 5), (1000, 4096, 16), (129, 768, 32)])
def test_q5_k_matvec_parity(ctx, oracle, rows, cols, batch):
    """Q5_K on the tiled fp16 GEMV (high bits into the fp16 subnormals):
    every n-tile count and a partial row tile."""
    t, blocks = _rand_sb("q5_k", rows, cols, 41 + batch)
    W = ctx.upload(blocks, t, rows, cols)
    x = _x(batch, cols, f"q5k.x.{rows}.{cols}.{batch}")
    assert rel_err(ctx.matvec(W, x), oracle.matvec(t, blocks, x, rows)) <= REL_TOL


@pytest.mark.parametrize("name", list(SB))
def test_superblock_dequantize_bit_exact(ctx, oracle, name):
    t, blocks = _rand_sb(name, 37, 768, 21)
    W = ctx.upload(blocks, t, 37, 768)
    assert bits_equal(ctx.dequantize(W), oracle.dequantize(t, blocks, 37 * 768).reshape(37, 768))
    assert bits_equal(ctx.dequantize(W, 5, 7), oracle.dequantize(t, blocks, 37 * 768).reshape(37, 768)[5:12])


@pytest.mark.parametrize("name", list(SB))
@pytest.mark.parametrize("batch", [1, 3])
def test_superblock_matvec_parity(ctx, oracle, name, batch):
    rows, cols = 300, 2048
    t, blocks = _rand_sb(name, rows, cols, 23)
    W = ctx.upload(blocks, t, rows, cols)
    x = _x(batch, cols, f"sb.x.{name}.{batch}")
    assert rel_err(ctx.matvec(W, x), oracle.matvec(t, blocks, x, rows)) <= REL_TOL
