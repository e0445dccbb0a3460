"""Parity helpers shared by the GPU tests."""
from __future__ import annotations

import numpy as np

# North-star tolerance for matvec / matmul outputs and logits: max relative
# error 1e-3, normalised by the largest reference magnitude of the vector.
REL_TOL = 1e-3


def rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    denom = np.max(np.abs(ref), axis=-1, keepdims=True)
    denom = np.where(denom == 0, 1.0, denom)
    return float(np.max(np.abs(got - ref) / denom))


def bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and bool(np.array_equal(a.view(np.uint32), b.view(np.uint32)))
