"""Writes kat_quant.json: the reference's own known-answer tests for the hot path.

The cases restate the fixtures of ChatNet's tests/ChatNet.Tests/
QuantizationTests.cs (block bytes built exactly as each test builds them,
WriteHalf = IEEE round-to-nearest fp16) together with the values the test
asserts and its tolerance.  Where the test compares DotProduct against the
sum of Dequantize, the expected sum is derived here from the block formula
(exact in fp32 for these fixtures), so the check does not depend on the
oracle it pins.

Run: python tests/golden/make_kat.py   (rewrites tests/golden/kat_quant.json)
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
T = "tests/ChatNet.Tests/QuantizationTests.cs"


def half_bytes(v: float) -> list[int]:
    h = np.array([v], dtype=np.float16).view(np.uint16)[0]
    return [int(h & 0xFF), int(h >> 8)]


def f16(v: float) -> float:
    return float(np.float16(v))


def cases() -> list[dict]:
    out = []

    # Q4_0_Dequantize_ProducesCorrectValues (:23-41): d=1, qs=0 -> all -8
    blk = half_bytes(1.0) + [0] * 16
    out.append(dict(name="Q4_0_Dequantize_ProducesCorrectValues", ref=f"{T}:23-41", type=2, n=32,
                    blocks=blk, dequant=[-8.0] * 32, tol=0.01))

    # Q4_0_Dequantize_MidpointValues (:43-60): d=0.5, 0x88 -> 0
    blk = half_bytes(0.5) + [0x88] * 16
    out.append(dict(name="Q4_0_Dequantize_MidpointValues", ref=f"{T}:43-60", type=2, n=32,
                    blocks=blk, dequant=[0.0] * 32, tol=0.01))

    # Q4_0_DotProduct_MatchesScalar (:62-87): d=2, 0x37 (lo 7, hi 3), x=1
    blk = half_bytes(2.0) + [0x37] * 16
    deq = [(7 - 8) * 2.0] * 16 + [(3 - 8) * 2.0] * 16
    out.append(dict(name="Q4_0_DotProduct_MatchesScalar", ref=f"{T}:62-87", type=2, n=32,
                    blocks=blk, dequant=deq, x=[1.0] * 32, dot=float(sum(deq)), tol=0.01))

    # Q6K_Dequantize_ProducesFiniteValues (:302-319): d=1 at byte 208, scales=1
    blk = [0] * 210
    blk[192:208] = [1] * 16
    blk[208:210] = half_bytes(1.0)
    out.append(dict(name="Q6K_Dequantize_ProducesFiniteValues", ref=f"{T}:302-319", type=14,
                    n=256, blocks=blk, dequant=[-32.0] * 256, finite=True, tol=0.01))

    # Q6K_DotProduct_MatchesDequantize (:321-345): d=0.1, scales=2, ql=0x22, x=1
    blk = [0x22] * 128 + [0] * 64 + [2] * 16 + half_bytes(0.1)
    v = np.float32(np.float32(f16(0.1)) * np.float32(2)) * np.float32(-30)
    out.append(dict(name="Q6K_DotProduct_MatchesDequantize", ref=f"{T}:321-345", type=14, n=256,
                    blocks=blk, dequant=[float(v)] * 256, x=[1.0] * 256,
                    dot=float(np.float32(v) * 256), tol=0.1))

    # Q4K_Dequantize_ProducesFiniteValues (:445-462): d=1, dmin=0.5, scales 0x11
    blk = half_bytes(1.0) + half_bytes(0.5) + [0x11] * 12 + [0] * 128
    # sc = m = 17 for sub-blocks 0..3, 1 for 4..7 (DecodeScales); q = 0
    deq = [(-8.5 if (i // 32) < 4 else -0.5) for i in range(256)]
    out.append(dict(name="Q4K_Dequantize_ProducesFiniteValues", ref=f"{T}:445-462", type=12,
                    n=256, blocks=blk, dequant=deq, finite=True, tol=0.01))

    # Q4K_DotProduct_MatchesDequantize (:464-489): d=.5, dmin=.25, 0x11, qs 0x33, x=1
    blk = half_bytes(0.5) + half_bytes(0.25) + [0x11] * 12 + [0x33] * 128
    deq = [(0.5 * 17 * 3 - 0.25 * 17) if (i // 32) < 4 else (0.5 * 1 * 3 - 0.25 * 1)
           for i in range(256)]
    out.append(dict(name="Q4K_DotProduct_MatchesDequantize", ref=f"{T}:464-489", type=12, n=256,
                    blocks=blk, dequant=deq, x=[1.0] * 256, dot=float(sum(deq)), tol=0.1))

    # Q4_0_MultiBlock_Dequantize (:704-726): two blocks d=1 and d=2, 0x88 -> 0
    blk = half_bytes(1.0) + [0x88] * 16 + half_bytes(2.0) + [0x88] * 16
    out.append(dict(name="Q4_0_MultiBlock_Dequantize", ref=f"{T}:704-726", type=2, n=64,
                    blocks=blk, dequant=[0.0] * 64, tol=0.01))

    # Q4K_MultiBlock_DotProduct (:728-759): 2 super-blocks, qs 0x55, x=0.5
    one = half_bytes(0.5) + half_bytes(0.25) + [0x11] * 12 + [0x55] * 128
    blk = one + one
    deq1 = [(0.5 * 17 * 5 - 0.25 * 17) if (i // 32) < 4 else (0.5 * 1 * 5 - 0.25 * 1)
            for i in range(256)]
    deq = deq1 + deq1
    out.append(dict(name="Q4K_MultiBlock_DotProduct", ref=f"{T}:728-759", type=12, n=512,
                    blocks=blk, dequant=deq, x=[0.5] * 512,
                    dot=float(sum(d * 0.5 for d in deq)), tol=0.1))
    # Q4_1_Dequantize_ProducesCorrectValues (:93-110): d=2, m=1, qs=0 -> 0*2+1
    blk = half_bytes(2.0) + half_bytes(1.0) + [0] * 16
    out.append(dict(name="Q4_1_Dequantize_ProducesCorrectValues", ref=f"{T}:93-110", type=3, n=32,
                    blocks=blk, dequant=[1.0] * 32, tol=0.01))

    # Q4_1_DotProduct_MatchesScalar (:111-136): d=1, m=0.5, nibbles 5, x=1
    blk = half_bytes(1.0) + half_bytes(0.5) + [0x55] * 16
    out.append(dict(name="Q4_1_DotProduct_MatchesScalar", ref=f"{T}:111-136", type=3, n=32,
                    blocks=blk, dequant=[5.5] * 32, x=[1.0] * 32, dot=5.5 * 32, tol=0.01))

    # Q5_0_Dequantize_ZeroQuants (:141-157): d=1, qh=qs=0 -> (0-16)*1
    blk = half_bytes(1.0) + [0] * 20
    out.append(dict(name="Q5_0_Dequantize_ZeroQuants", ref=f"{T}:141-157", type=6, n=32,
                    blocks=blk, dequant=[-16.0] * 32, tol=0.01))

    # Q5_0_DotProduct_MatchesDequantize (:158-186): d=0.5, qh bits 0-15 set,
    # nibbles 0xA, x=0.5: positions 0-15 (26-16)*0.5, 16-31 (10-16)*0.5
    blk = half_bytes(0.5) + [0xFF, 0xFF, 0x00, 0x00] + [0xAA] * 16
    deq = [5.0] * 16 + [-3.0] * 16
    out.append(dict(name="Q5_0_DotProduct_MatchesDequantize", ref=f"{T}:158-186", type=6, n=32,
                    blocks=blk, dequant=deq, x=[0.5] * 32, dot=float(sum(d * 0.5 for d in deq)), tol=0.01))

    # Q5_1_Dequantize_WithMinOffset (:189-206): d=1, m=2, zero quants -> 2
    blk = half_bytes(1.0) + half_bytes(2.0) + [0] * 20
    out.append(dict(name="Q5_1_Dequantize_WithMinOffset", ref=f"{T}:189-206", type=7, n=32,
                    blocks=blk, dequant=[2.0] * 32, tol=0.01))

    # Q5_1_DotProduct_MatchesDequantize (:207-231): d=0.25, m=0.5, nibbles 3, x=1
    blk = half_bytes(0.25) + half_bytes(0.5) + [0] * 4 + [0x33] * 16
    out.append(dict(name="Q5_1_DotProduct_MatchesDequantize", ref=f"{T}:207-231", type=7, n=32,
                    blocks=blk, dequant=[1.25] * 32, x=[1.0] * 32, dot=1.25 * 32, tol=0.01))

    # Q8_0_Dequantize_ProducesCorrectValues (:237-254): d=0.5, q=10 -> 5
    blk = half_bytes(0.5) + [10] * 32
    out.append(dict(name="Q8_0_Dequantize_ProducesCorrectValues", ref=f"{T}:237-254", type=8, n=32,
                    blocks=blk, dequant=[5.0] * 32, tol=0.01))

    # Q8_0_Dequantize_NegativeValues (:255-272): d=1, q=0xF6 (-10)
    blk = half_bytes(1.0) + [0xF6] * 32
    out.append(dict(name="Q8_0_Dequantize_NegativeValues", ref=f"{T}:255-272", type=8, n=32,
                    blocks=blk, dequant=[-10.0] * 32, tol=0.01))

    # Q8_0_DotProduct_MatchesDequantize (:273-299): d=0.25, q=0..31, x=1
    blk = half_bytes(0.25) + list(range(32))
    deq = [0.25 * i for i in range(32)]
    out.append(dict(name="Q8_0_DotProduct_MatchesDequantize", ref=f"{T}:273-299", type=8, n=32,
                    blocks=blk, dequant=deq, x=[1.0] * 32, dot=float(sum(deq)), tol=0.01))

    # Q2K_Dequantize_ProducesFiniteValues (:351-367): d=1 @80, dmin=0.5 @82,
    # scale bytes 0x21 (sc 1, m 2), quants 0 -> 1*1*0 - 0.5*2
    blk = [0x21] * 16 + [0] * 64 + half_bytes(1.0) + half_bytes(0.5)
    out.append(dict(name="Q2K_Dequantize_ProducesFiniteValues", ref=f"{T}:351-367", type=10, n=256,
                    blocks=blk, dequant=[-1.0] * 256, finite=True, tol=0.01))

    # Q2K_DotProduct_MatchesDequantize (:369-394): d=.5, dmin=.25, scales 0x11,
    # quant bytes 0x55 (every 2-bit field 1), x=1 -> 0.5*1*1 - 0.25*1 each
    blk = [0x11] * 16 + [0x55] * 64 + half_bytes(0.5) + half_bytes(0.25)
    out.append(dict(name="Q2K_DotProduct_MatchesDequantize", ref=f"{T}:369-394", type=10, n=256,
                    blocks=blk, dequant=[0.25] * 256, x=[1.0] * 256, dot=64.0, tol=0.1))

    # Q3K_Dequantize_ProducesFiniteValues (:400-414): d=1 @108, all else 0:
    # scales 0 - 32, q3 0 -> 1 * -32 * (0 - 4)
    blk = [0] * 108 + half_bytes(1.0)
    out.append(dict(name="Q3K_Dequantize_ProducesFiniteValues", ref=f"{T}:400-414", type=11, n=256,
                    blocks=blk, dequant=[128.0] * 256, finite=True, tol=0.01))

    # Q3K_DotProduct_MatchesDequantize (:416-439): d=0.1, qs bytes 0x55 (q2 1),
    # hmask 0, scales -32 -> d * -32 * (1 - 4), x=1
    blk = [0] * 32 + [0x55] * 64 + [0] * 12 + half_bytes(0.1)
    v = np.float32(np.float32(f16(0.1)) * np.float32(-32)) * np.float32(-3)
    out.append(dict(name="Q3K_DotProduct_MatchesDequantize", ref=f"{T}:416-439", type=11, n=256,
                    blocks=blk, dequant=[float(v)] * 256, x=[1.0] * 256, dot=float(v) * 256, tol=0.1))

    # Q5K_Dequantize_ProducesFiniteValues (:495-511): d=1, dmin=0.5, scale
    # bytes 0x11 (sc = m = 17 for sub-blocks 0..3, 1 for 4..7), quants 0
    blk = half_bytes(1.0) + half_bytes(0.5) + [0x11] * 12 + [0] * 160
    deq = [(-8.5 if (i // 32) < 4 else -0.5) for i in range(256)]
    out.append(dict(name="Q5K_Dequantize_ProducesFiniteValues", ref=f"{T}:495-511", type=13, n=256,
                    blocks=blk, dequant=deq, finite=True, tol=0.01))

    # Q5K_DotProduct_MatchesDequantize (:513-538): d=.5, dmin=.25, scales 0x11,
    # qs 0x55, qh 0 (q5 = 5), x=1
    blk = half_bytes(0.5) + half_bytes(0.25) + [0x11] * 12 + [0] * 32 + [0x55] * 128
    deq = [(0.5 * 17 * 5 - 0.25 * 17) if (i // 32) < 4 else (0.5 * 1 * 5 - 0.25 * 1) for i in range(256)]
    out.append(dict(name="Q5K_DotProduct_MatchesDequantize", ref=f"{T}:513-538", type=13, n=256,
                    blocks=blk, dequant=deq, x=[1.0] * 256, dot=float(sum(deq)), tol=0.1))

    # Q8K_Dequantize_ProducesCorrectValues (:544-562): fp32 d=0.5, q=10 -> 5
    f32 = lambda v: list(np.array([v], dtype="<f4").view(np.uint8))
    blk = [int(b) for b in f32(0.5)] + [10] * 256 + [0] * 32
    out.append(dict(name="Q8K_Dequantize_ProducesCorrectValues", ref=f"{T}:544-562", type=15, n=256,
                    blocks=blk, dequant=[5.0] * 256, tol=0.01))

    # Q8K_DotProduct_MatchesDequantize (:564-588): d=0.25, byte i = i % 20, x=1
    blk = [int(b) for b in f32(0.25)] + [i % 20 for i in range(4, 260)] + [0] * 32
    deq = [0.25 * (i % 20) for i in range(4, 260)]
    out.append(dict(name="Q8K_DotProduct_MatchesDequantize", ref=f"{T}:564-588", type=15, n=256,
                    blocks=blk, dequant=deq, x=[1.0] * 256, dot=float(sum(deq)), tol=0.01))

    # IQ4NL_Dequantize_UsesLookupTable (:594-611): scale 1, byte 2 = 0x80:
    # element 0 -> table[0] = -127, element 16 -> table[8] = 1, the rest table[0]
    blk = half_bytes(1.0) + [0x80] + [0] * 15
    deq = [-127.0] * 16 + [1.0] + [-127.0] * 15
    out.append(dict(name="IQ4NL_Dequantize_UsesLookupTable", ref=f"{T}:594-611", type=20, n=32,
                    blocks=blk, dequant=deq, tol=0.01))

    # IQ4NL_DotProduct_MatchesDequantize (:613-636): scale 0.01, all index 8 (1), x=1
    blk = half_bytes(0.01) + [0x88] * 16
    v = float(np.float32(f16(0.01)))
    out.append(dict(name="IQ4NL_DotProduct_MatchesDequantize", ref=f"{T}:613-636", type=20, n=32,
                    blocks=blk, dequant=[v] * 32, x=[1.0] * 32, dot=v * 32, tol=0.1))
    return out


# GgufTensorInfo_ByteSize_AllTypes (:642-698), the rows for the types this
# library decodes: (type, block size, bytes per block)
BYTESIZE = [(0, 1, 4), (1, 1, 2), (2, 32, 18), (3, 32, 20), (6, 32, 22), (7, 32, 24), (8, 32, 34),
            (10, 256, 84), (11, 256, 110), (12, 256, 144), (13, 256, 176), (14, 256, 210), (15, 256, 292),
            (20, 32, 18), (23, 256, 136), (21, 256, 110), (18, 256, 98), (17, 256, 74), (16, 256, 66),
            (22, 256, 82), (19, 256, 50), (29, 256, 56)]


def main() -> None:
    doc = {
        "source": T,
        "note": "fixtures restated from the reference's MSTest known-answer tests",
        "cases": cases(),
        "byte_size": [dict(type=t, block=b, bytes_per_block=p, ref=f"{T}:642-698")
                      for (t, b, p) in BYTESIZE],
    }
    (HERE / "kat_quant.json").write_text(json.dumps(doc, indent=1) + "\n")


if __name__ == "__main__":
    main()
