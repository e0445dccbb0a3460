"""The oracle's restatements of the reference's simplified importance-quant
decodes (DequantIQ.cs: IQ3_S, IQ3_XXS, IQ2_XS, IQ2_XXS, IQ2_S, IQ1_S, IQ1_M)
checked against a second, independent restatement written here in NumPy
straight from the reference's Dequantize loops: bit-exact dequantization,
and the fused dot products (DotProductScalar) within the parity tolerance.
The reference's tests pin only these types' byte sizes
(QuantizationTests.cs:642-698, tests/golden/kat_quant.json); this is the
pin for the values.  CPU only."""
from __future__ import annotations

import numpy as np
import pytest

import chatnet_b200 as cn
from tests.parity import REL_TOL, bits_equal, rel_err

BPB = {cn.TYPE_IQ3_S: 110, cn.TYPE_IQ3_XXS: 98, cn.TYPE_IQ2_XS: 74, cn.TYPE_IQ2_XXS: 66,
       cn.TYPE_IQ2_S: 82, cn.TYPE_IQ1_S: 50, cn.TYPE_IQ1_M: 56}
F32 = np.float32


def _blocks(t: int, nb: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(nb, BPB[t]), dtype=np.uint8)
    d = (np.abs(rng.standard_normal(nb)) * 0.01 + 1e-3).astype(np.float16)
    b[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    return b


def _np_dequant(t: int, blocks: np.ndarray) -> np.ndarray:
    """Element values in the reference's operation order, float32 throughout."""
    nb = blocks.shape[0]
    flat = blocks.ravel()
    d = blocks[:, 0:2].copy().view(np.float16).astype(F32).ravel()
    e = np.arange(256)
    out = np.zeros((nb, 256), F32)
    for b in range(nb):
        p = blocks[b]
        if t == cn.TYPE_IQ3_S:
            base = b * 110

            def byte(k):  # reads past the block into the next one, 0 past the buffer
                i = base + k
                return np.where(i < flat.size, flat[np.minimum(i, flat.size - 1)], 0).astype(np.int64)
            sub, j = e // 8, e % 8
            sc = ((byte(130 + sub // 4) >> ((sub % 4) * 2)) & 3) + 1
            q3 = ((p[2 + e // 4].astype(np.int64) >> ((e % 4) * 2)) & 3) | \
                 (((p[66 + e // 8].astype(np.int64) >> (e % 8)) & 1) << 2)
            v = (d[b] * sc.astype(F32)).astype(F32) * q3.astype(F32)
            neg = ((byte(98 + sub) >> j) & 1) == 1
            out[b] = np.where(neg, -v, v)
        elif t == cn.TYPE_IQ3_XXS:
            sub, j = e // 8, e % 8
            g = p[2:98].astype(np.int64).reshape(32, 3)
            packed = g[:, 0] | (g[:, 1] << 8) | (g[:, 2] << 16)
            q3 = (packed[sub] >> (3 * j)) & 7
            out[b] = d[b] * (q3 - 4).astype(F32)
        elif t in (cn.TYPE_IQ2_XS, cn.TYPE_IQ2_XXS, cn.TYPE_IQ2_S):
            sub, r = e // 16, e % 16
            q = (p[2 + 4 * sub + r // 4].astype(np.int64) >> (2 * (r % 4))) & 3
            if t == cn.TYPE_IQ2_XXS:
                out[b] = d[b] * (q - 1).astype(F32)
            elif t == cn.TYPE_IQ2_XS:
                raw = p[66 + sub // 2].astype(np.int64)
                sc = np.where(sub % 2 == 0, raw & 15, (raw >> 4) & 15) - 8
                out[b] = (d[b] * sc.astype(F32)).astype(F32) * (q - 1).astype(F32)
            else:
                qh = p[66 + sub].astype(np.int64)
                v = (d[b] * ((qh & 15) + 1).astype(F32)).astype(F32) * q.astype(F32)
                neg = (r < 4) & (((qh >> (4 + r)) & 1) == 1)
                out[b] = np.where(neg, -v, v)
        else:  # IQ1_S, IQ1_M
            sub, j = e // 8, e % 8
            bit = (p[2 + sub].astype(np.int64) >> j) & 1
            hbit = (p[34 + sub // 2].astype(np.int64) >> ((sub % 2) * 4 + j // 2)) & 1
            w = np.full(256, d[b], F32)
            if t == cn.TYPE_IQ1_M:
                sc = np.where(((p[50 + sub // 8].astype(np.int64) >> (sub % 8)) & 1) == 1, F32(1.0), F32(0.5))
                w = (d[b] * sc).astype(F32)
            out[b] = np.where(bit == 1, w, np.where(hbit == 1, -w, F32(0.0)))
    return out.ravel()


@pytest.mark.parametrize("t", list(BPB))
def test_dequantize_matches_independent_restatement(oracle, t):
    blocks = _blocks(t, 9, 100 + t)
    got = oracle.dequantize(t, blocks.ravel(), 9 * 256)
    assert bits_equal(got, _np_dequant(t, blocks))


@pytest.mark.parametrize("t", list(BPB))
def test_matvec_matches_dequantized_dot(oracle, t):
    """The oracle's fused dot (DotProductScalar's order) against the float64
    dot of the independently dequantized rows.  IQ3_S rows read the next
    row's bytes, as the reference's pointer-based dot does."""
    rows, cols = 7, 1024
    blocks = _blocks(t, rows * cols // 256, 200 + t)
    x = np.random.default_rng(t).standard_normal(cols).astype(F32)
    y = oracle.matvec(t, blocks.ravel(), x, rows)
    w = _np_dequant(t, blocks).reshape(rows, cols).astype(np.float64)
    assert rel_err(y, w @ x.astype(np.float64)) <= REL_TOL


def test_iq3_s_reads_past_its_block(oracle):
    """Signs and scales of IQ3_S sit at bytes 98-137 of a 110-byte block: the
    last block of a buffer reads them as 0 (scale 1, no sign), earlier blocks
    from the next block's bytes 0-27."""
    t = cn.TYPE_IQ3_S
    blocks = _blocks(t, 2, 7)
    both = oracle.dequantize(t, blocks.ravel(), 512).reshape(2, 256)
    alone = oracle.dequantize(t, blocks[1].copy(), 256)
    assert bits_equal(both[1], alone)
    # the first block's values depend on the second block's bytes
    b2 = blocks.copy()
    b2[1, 0:28] ^= 0xFF
    changed = oracle.dequantize(t, b2.ravel(), 512).reshape(2, 256)[0]
    assert not bits_equal(changed, both[0])
