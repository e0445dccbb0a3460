"""The oracle's restatements of the architecture variants other ChatNet
models run on the Llama loop, pinned to the reference's own tests
(tests/ChatNet.Tests/ArchitectureTests.cs: GELU :237-338, RmsNormWithOffset
:344-422) and, for split-half RoPE (TensorMath.ApplyRoPENeox, which the
reference does not test), to its relation with the interleaved form."""
from __future__ import annotations

import numpy as np
import pytest

from tests._oracle import fp


def _gelu(oracle, gate, up):
    g = np.array(gate, np.float32)
    u = np.array(up, np.float32)
    oracle.lib.or_gelu_mul(fp(g), fp(u), g.size)
    return g


def test_gelu_known_answers(oracle):
    # ArchitectureTests.cs:237-318
    assert np.allclose(_gelu(oracle, np.zeros(32), np.ones(32)), 0.0, atol=1e-3)
    g = _gelu(oracle, np.full(32, 2.0), np.ones(32))
    assert np.all((g > 1.9) & (g < 2.1))
    g = _gelu(oracle, np.full(32, -3.0), np.ones(32))
    assert np.all((g > -0.1) & (g < 0.1))
    g = _gelu(oracle, np.ones(32), np.full(32, 2.0))  # GELU(1) * 2 ~= 1.68
    assert np.all((g > 1.5) & (g < 1.9))
    for n in (1, 2, 3, 5, 7, 15, 17, 33):  # ArchitectureTests.cs:320-338
        assert np.isfinite(_gelu(oracle, np.ones(n), np.ones(n))).all()


def test_rmsnorm_offset_known_answers(oracle):
    # ArchitectureTests.cs:344-422
    y = np.zeros(64, np.float32)
    oracle.lib.or_rmsnorm_offset(fp(np.ones(64, np.float32)), fp(np.zeros(64, np.float32)), fp(y), 64, 1e-5)
    assert np.allclose(y, 1.0, atol=0.01)
    x = ((np.arange(256) - 128) / 256).astype(np.float32)
    w = (0.01 * np.arange(256)).astype(np.float32)
    y = np.zeros(256, np.float32)
    oracle.lib.or_rmsnorm_offset(fp(x), fp(w), fp(y), 256, 1e-5)
    assert np.isfinite(y).all()
    w5 = np.full(64, 0.5, np.float32)
    a, b = np.zeros(64, np.float32), np.zeros(64, np.float32)
    oracle.lib.or_rmsnorm(fp(np.ones(64, np.float32)), fp(w5), fp(a), 64, 1e-5)
    oracle.lib.or_rmsnorm_offset(fp(np.ones(64, np.float32)), fp(w5), fp(b), 64, 1e-5)
    assert np.max(np.abs(a - b)) > 0.01
    # exactly RmsNorm with the weights + 1 formed in fp32
    c = np.zeros(256, np.float32)
    oracle.lib.or_rmsnorm(fp(x), fp((w + np.float32(1)).astype(np.float32)), fp(c), 256, 1e-5)
    oracle.lib.or_rmsnorm_offset(fp(x), fp(w), fp(y), 256, 1e-5)
    assert np.array_equal(c, y)


@pytest.mark.parametrize("hd", [64, 128])
def test_rope_neox_is_interleaved_on_paired_layout(oracle, hd):
    """Split-half RoPE rotates (i, i + hd/2) by the angle interleaved RoPE gives
    the pair (2i, 2i + 1): moving element i + hd/2 next to element i turns one
    into the other, bit for bit (same table values, same rounding order)."""
    rng = np.random.default_rng(hd)
    nh, nkv, pos = 4, 2, 37
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal(nkv * hd).astype(np.float32)
    perm = np.empty(hd, np.int64)
    perm[0::2] = np.arange(hd // 2)
    perm[1::2] = np.arange(hd // 2) + hd // 2

    def to_pairs(v, n):
        return np.ascontiguousarray(v.reshape(n, hd)[:, perm].reshape(-1))

    qn, kn = q.copy(), k.copy()
    oracle.lib.or_rope_neox(fp(qn), fp(kn), pos, hd, nh, nkv, 10000.0)
    qi, ki = to_pairs(q, nh), to_pairs(k, nkv)
    oracle.lib.or_rope(fp(qi), fp(ki), pos, hd, nh, nkv, 10000.0)
    assert np.array_equal(to_pairs(qn, nh), qi) and np.array_equal(to_pairs(kn, nkv), ki)
