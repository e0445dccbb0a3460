"""The C-ABI library loads and exports every entry point include/chatnet_cuda.h
declares; host-only logic (sizes, synthetic generator, argument checks) works
without a GPU."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

import chatnet_b200 as cn
from chatnet_b200 import _native as N

HEADER = Path(__file__).resolve().parent.parent / "include" / "chatnet_cuda.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(cn_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_something():
    assert len(declared_functions()) >= 15


@pytest.mark.parametrize("name", declared_functions())
def test_symbol_exported(name):
    lib = N.lib()
    assert hasattr(lib, name), f"{name} declared in chatnet_cuda.h but not exported"


def test_binding_covers_header():
    assert set(declared_functions()) <= set(N.SIGNATURES)


def test_abi_version():
    assert N.lib().cn_abi_version() == 2


@pytest.mark.parametrize("t,elems,expected", [
    (cn.TYPE_Q4_0, 2048, 1152), (cn.TYPE_Q4_0, 33, 36), (cn.TYPE_Q4_K, 4096, 2304),
    (cn.TYPE_Q4_K, 257, 288), (cn.TYPE_Q6_K, 4096, 3360), (cn.TYPE_F32, 10, 40),
    (cn.TYPE_F16, 10, 20), (cn.TYPE_Q4_1, 32, 20), (cn.TYPE_Q5_0, 64, 44), (cn.TYPE_Q5_1, 33, 48),
    (cn.TYPE_Q8_0, 32, 34), (cn.TYPE_Q2_K, 256, 84), (cn.TYPE_Q3_K, 512, 220), (cn.TYPE_Q5_K, 257, 352),
    (cn.TYPE_Q8_K, 256, 292), (cn.TYPE_IQ4_NL, 33, 36), (cn.TYPE_IQ4_XS, 256, 136),
    (cn.TYPE_IQ2_XXS, 256, 66), (cn.TYPE_IQ2_XS, 512, 148), (cn.TYPE_IQ3_XXS, 256, 98), (cn.TYPE_IQ1_S, 257, 100),
    (cn.TYPE_IQ3_S, 256, 110), (cn.TYPE_IQ2_S, 256, 82), (cn.TYPE_IQ1_M, 256, 56), (9, 32, 0)])
def test_byte_size(t, elems, expected, oracle):
    assert cn.byte_size(t, elems) == expected
    assert oracle.lib.or_byte_size(t, elems) == expected


def test_synth_deterministic_and_distinct():
    a = cn.synth_fill(cn.TYPE_Q4_0, 8, 64, seed=1)
    b = cn.synth_fill(cn.TYPE_Q4_0, 8, 64, seed=1)
    c = cn.synth_fill(cn.TYPE_Q4_0, 8, 64, seed=2)
    assert a.shape == (8, 36) and (a == b).all() and not (a == c).all()
    assert cn.synth_seed(1, "blk.0.attn_q.weight") != cn.synth_seed(1, "blk.1.attn_q.weight")
    assert cn.synth_seed(1, "x") != cn.synth_seed(2, "x")


def test_synth_normal_moments():
    x = cn.synth_fill(cn.TYPE_F32, 1, 200000, seed=7).ravel()
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1) < 0.01
    assert np.abs(x).max() <= 6.0
    # exact multiples of 2^-16
    assert np.all((x * 65536) == np.round(x * 65536))


def test_synth_block_statistics(oracle):
    W = cn.synth_fill(cn.TYPE_Q4_0, 64, 2048, seed=3)
    d = W.reshape(-1, 18)[:, :2].copy().view(np.float16).astype(np.float32).ravel()
    assert (d >= 0).all() and 0.0015 < d.mean() < 0.0025   # E|N| * 0.0025 ~ 0.002
    w = oracle.dequantize(cn.TYPE_Q4_0, W, 64 * 2048)
    assert np.isfinite(w).all()
    K = cn.synth_fill(cn.TYPE_Q4_K, 4, 256, seed=3).reshape(-1, 144)
    sc = oracle.dequantize(cn.TYPE_Q4_K, K, 4 * 256)
    assert np.isfinite(sc).all()
    Q6 = cn.synth_fill(cn.TYPE_Q6_K, 4, 256, seed=3).reshape(-1, 210)
    assert (Q6[:, 192:208] <= 63).all()


def test_synth_norm_weight():
    w = cn.synth_fill(cn.TYPE_F32, 1, 50000, seed=5, dist=cn.DIST_NORM_W).ravel()
    assert abs(w.mean() - 1) < 1e-3 and abs(w.std() - 0.01) < 1e-3


def test_synth_rejects_bad_requests():
    with pytest.raises(ValueError):
        cn.synth_fill(cn.TYPE_Q4_0, 2, 33, seed=1)
    with pytest.raises(cn.NotSupportedError):
        cn.synth_fill(3, 2, 32, seed=1)


def test_last_error_is_string():
    assert isinstance(N.last_error(), str)


def test_create_without_gpu_fails_cleanly():
    if cn.device_count() > 0:
        pytest.skip("a GPU is visible")
    h = C.c_void_p()
    rc = N.lib().cn_create(0, C.byref(h))
    assert rc != 0 and h.value is None
    assert N.last_error()
