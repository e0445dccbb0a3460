"""Pins the CPU oracle to the reference's own known-answer tests
(tests/ChatNet.Tests/QuantizationTests.cs, fixtures in tests/golden/kat_quant.json)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

KAT = json.loads((Path(__file__).parent / "golden" / "kat_quant.json").read_text())


@pytest.mark.parametrize("case", KAT["cases"], ids=lambda c: c["name"])
def test_kat_dequantize(oracle, case):
    blocks = np.array(case["blocks"], dtype=np.uint8)
    out = oracle.dequantize(case["type"], blocks, case["n"])
    assert np.all(np.isfinite(out))
    np.testing.assert_allclose(out, np.array(case["dequant"], np.float32), rtol=0,
                               atol=case["tol"])


@pytest.mark.parametrize("case", [c for c in KAT["cases"] if "dot" in c], ids=lambda c: c["name"])
def test_kat_dot_matches_dequantize(oracle, case):
    blocks = np.array(case["blocks"], dtype=np.uint8)
    x = np.array(case["x"], dtype=np.float32)
    got = oracle.dot(case["type"], blocks, x)
    deq = oracle.dequantize(case["type"], blocks, case["n"])
    expected_from_dequant = float(np.sum(deq.astype(np.float64) * x))
    assert abs(got - case["dot"]) <= case["tol"]
    assert abs(got - expected_from_dequant) <= case["tol"]


@pytest.mark.parametrize("row", KAT["byte_size"], ids=lambda r: f"type{r['type']}")
def test_kat_byte_size(oracle, row):
    elements = 1024 if row["block"] == 1 else row["block"] * 4
    blocks = (elements + row["block"] - 1) // row["block"]
    assert oracle.lib.or_byte_size(row["type"], elements) == blocks * row["bytes_per_block"]


def test_kat_fixture_is_current():
    """tests/golden/make_kat.py reproduces the committed fixture."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_kat",
                                                  Path(__file__).parent / "golden" / "make_kat.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    assert m.cases() == KAT["cases"]


def test_half_roundtrip_exhaustive(oracle):
    """fp16 -> fp32 is exact and fp32 -> fp16 is round-to-nearest-even (numpy agrees)."""
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    f = np.array([oracle.lib.or_half_to_float(int(v)) for v in h[::97]], dtype=np.float32)
    ref = h[::97].view(np.float16).astype(np.float32)
    same = (f == ref) | (np.isnan(f) & np.isnan(ref))
    assert same.all()
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.standard_normal(4000).astype(np.float32) * s
                         for s in (1e-6, 1e-3, 1, 100, 6e4)])
    got = np.array([oracle.lib.or_float_to_half(float(v)) for v in xs], dtype=np.uint16)
    np.testing.assert_array_equal(got, xs.astype(np.float16).view(np.uint16))


# Every codec the oracle restates: (type, elements per block, bytes per block,
# offsets of fp16 scale fields)
_CODECS = [(2, 32, 18, (0,)), (3, 32, 20, (0, 2)), (6, 32, 22, (0,)), (7, 32, 24, (0, 2)),
           (8, 32, 34, (0,)), (10, 256, 84, (80, 82)), (11, 256, 110, (108,)), (12, 256, 144, (0, 2)),
           (13, 256, 176, (0, 2)), (14, 256, 210, (208,)), (15, 256, 292, ()), (20, 32, 18, (0,)),
           (23, 256, 136, (0,))]


@pytest.mark.parametrize("t,blk,bpb,halves", _CODECS, ids=lambda v: str(v))
def test_dot_matches_dequantize_random(oracle, t, blk, bpb, halves):
    """Each codec's fused DotProduct agrees with its Dequantize on random
    blocks (the two restated code paths of one format check each other)."""
    rng = np.random.default_rng(t)
    nb = 2048 // blk
    b = rng.integers(0, 256, size=(nb, bpb), dtype=np.uint8)
    for off in halves:
        b[:, off:off + 2] = (np.abs(rng.standard_normal(nb)) * 0.01).astype(np.float16).view(np.uint8).reshape(nb, 2)
    if t == 15:  # Q8_K: fp32 scale
        b[:, 0:4] = (np.abs(rng.standard_normal(nb)) * 0.01).astype("<f4").view(np.uint8).reshape(nb, 4)
    blocks = b.ravel()
    x = rng.standard_normal(2048).astype(np.float32)
    deq = oracle.dequantize(t, blocks, 2048).astype(np.float64)
    assert np.all(np.isfinite(deq))
    want = float(np.dot(deq, x))
    got = oracle.dot(t, blocks, x)
    scale = float(np.sum(np.abs(deq * x))) + 1e-30
    assert abs(got - want) <= 1e-5 * scale, (got, want)
