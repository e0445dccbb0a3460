"""CPU restatement of the tiled fp16 GEMV's element decode for the 32-weight
codecs (gemv.cu: unit_q4_0, block_b32), checked against the oracle's
dequantization.

For every lane quad t the kernel reads the block's quant bytes 4t..4t+3 as
one 32-bit word and builds four half2 A-fragment registers:
  * low nibbles of bytes (0, 2) and (1, 3) under the fp16 exponent of 1024:
    1024 + q for elements 4t + {0, 2} and 4t + {1, 3};
  * high nibbles left at mantissa bits 4-7: 1024 + 16 q for elements
    16 + 4t + {0, 2} and 16 + 4t + {1, 3};
  * Q5: the element's fifth bit (bit j of qh) ORed in at mantissa bit 4 (low
    nibbles) or 8 (high nibbles);
then one half2 subtraction (low) or FMA with 1/16 (high) gives the exact
integer q (Q4_1, Q5_1), q - 8 (Q4_0) or q - 16 (Q5_0).  This test restates
that arithmetic in numpy fp16 and checks, for random blocks, that q * d (+ m)
in fp32 equals the oracle's dequantized element bit for bit, which pins the
element order and the fifth-bit positions the kernel relies on.  (The GPU
parity tests check the kernel itself.)
"""
from __future__ import annotations

import numpy as np
import pytest

import chatnet_b200 as cn

# type: (block bytes, quant offset, qh offset or None, has minimum, low constant, high addend)
FMT = {
    "q4_0": (cn.TYPE_Q4_0, 18, 2, None, False, 1032.0, -72.0),
    "q4_1": (cn.TYPE_Q4_1, 20, 4, None, True, 1024.0, -64.0),
    "q5_0": (cn.TYPE_Q5_0, 22, 6, 2, False, 1040.0, -80.0),
    "q5_1": (cn.TYPE_Q5_1, 24, 8, 4, True, 1024.0, -64.0),
}
MAGIC = 0x6400  # fp16 1024


def _half(bits: int) -> np.float16:
    return np.array([bits & 0xFFFF], np.uint16).view(np.float16)[0]


def _decode_block(blk: np.ndarray, name: str) -> list[float]:
    """The kernel's per-element integers for one block, element order 0..31."""
    _, _, qs, qh_off, _, lo_c, hi_c = FMT[name]
    qh = int.from_bytes(bytes(blk[qh_off:qh_off + 4]), "little") if qh_off is not None else 0
    out = [0.0] * 32
    for t in range(4):
        w = int.from_bytes(bytes(blk[qs + 4 * t:qs + 4 * t + 4]), "little")
        for k in range(4):  # byte k of the word: element 4t + k and 16 + 4t + k
            lo = ((w >> (8 * k)) & 0x0F) | MAGIC
            hi = ((w >> (8 * k)) & 0xF0) | MAGIC
            if qh_off is not None:
                lo |= ((qh >> (4 * t + k)) & 1) << 4
                hi |= ((qh >> (16 + 4 * t + k)) & 1) << 8
            q_lo = np.float16(_half(lo) - np.float16(lo_c))
            q_hi = np.float16(_half(hi) * np.float16(1.0 / 16.0) + np.float16(hi_c))
            out[4 * t + k] = float(q_lo)
            out[16 + 4 * t + k] = float(q_hi)
    return out


@pytest.mark.parametrize("name", list(FMT))
def test_fp16_decode_matches_oracle(oracle, name):
    t, bpb, _, _, has_min, _, _ = FMT[name]
    rng = np.random.default_rng(7)
    nb = 64
    blocks = rng.integers(0, 256, size=(nb, bpb), dtype=np.uint8)
    d = (np.abs(rng.standard_normal(nb)) * 0.01).astype(np.float16)
    blocks[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    if has_min:
        m = (rng.standard_normal(nb) * 0.01).astype(np.float16)
        blocks[:, 2:4] = m.view(np.uint8).reshape(nb, 2)
    ref = oracle.dequantize(t, blocks.ravel(), nb * 32).reshape(nb, 32)
    for b in range(nb):
        q = np.array(_decode_block(blocks[b], name), np.float32)
        assert np.all(q == np.round(q)) and np.all(np.abs(q) <= 31)
        scale = np.float32(np.frombuffer(blocks[b, 0:2].tobytes(), np.float16)[0])
        got = q * scale
        if has_min:
            got = got + np.float32(np.frombuffer(blocks[b, 2:4].tobytes(), np.float16)[0])
        assert np.array_equal(got.view(np.uint32), ref[b].view(np.uint32)), (name, b)
