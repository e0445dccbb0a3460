"""TemperatureSampler.Sample (Samplers/TemperatureSampler.cs:33-113): the
oracle's restatement on hand-checked cases (CPU), and the device sampler
(cn_sample_dev / cn_llama_sample) against it on the same logits and draws
(GPU).  The device softmax sums as a tree, so probabilities agree to fp32
rounding; a draw is compared when the oracle's token stays the same with
top_p and r each moved by +-1e-5 (a decision that rounding cannot flip)."""
from __future__ import annotations

import math

import numpy as np
import pytest

LOGITS3 = np.log(np.array([1.0, 2.0, 3.0], np.float32))  # softmax 1/6, 2/6, 3/6


def test_oracle_sampler_hand_cases(oracle):
    # sorted probabilities 1/2 (index 2), 1/3 (index 1), 1/6 (index 0)
    for r, want in [(0.0, 2), (0.4, 2), (0.6, 1), (0.82, 1), (0.9, 0), (0.9999, 0)]:
        assert oracle.sample(LOGITS3, 1.0, 3, 1.0, r)[0] == want, r
    # nucleus: the first entry already reaches top_p -> always the most probable
    for r in (0.0, 0.5, 0.99):
        assert oracle.sample(LOGITS3, 1.0, 3, 0.5, r)[0] == 2
    # top_k = 2 keeps indices 2 and 1, renormalised to 3/5 and 2/5
    assert oracle.sample(LOGITS3, 1.0, 2, 1.0, 0.59)[0] == 2
    assert oracle.sample(LOGITS3, 1.0, 2, 1.0, 0.61)[0] == 1
    # temperature 0: the argmax, first maximum on ties
    assert oracle.sample(np.array([1, 5, 5, 2], np.float32), 0.0, 40, 0.9, 0.5)[0] == 1
    # low temperature sharpens to the argmax
    rng = np.random.default_rng(0)
    lg = rng.standard_normal(1000).astype(np.float32)
    assert oracle.sample(lg, 1e-3, 40, 0.9, 0.99)[0] == int(np.argmax(lg))


def _robust(oracle, lg, temp, k, p, r, d=1e-5):
    """The oracle's token if no rounding-sized move of top_p or r changes it."""
    toks = {oracle.sample(lg, temp, k, pp, rr)[0] for pp in (p - d, p, p + d) for rr in (r - d, r, r + d)}
    return toks.pop() if len(toks) == 1 else None


def _cases():
    rng = np.random.default_rng(7)
    out = []
    for vocab, temp, k, p in [(32000, 0.7, 40, 0.9), (32000, 1.0, 40, 0.9), (32000, 1.5, 100, 0.95),
                              (32000, 1.0, 32000, 0.9), (1000, 2.0, 1000, 1.0), (77, 0.8, 5, 0.5),
                              (32000, 1.0, 1, 0.9), (2000, 50.0, 2000, 0.9)]:
        lg = (rng.standard_normal(vocab) * 3).astype(np.float32)
        out.append((lg, temp, k, p))
    return out


@pytest.mark.gpu
def test_device_sampler_matches_oracle(ctx, oracle):
    import torch
    rng = np.random.default_rng(11)
    compared = 0
    for lg, temp, k, p in _cases():
        d = torch.from_numpy(lg).cuda()
        torch.cuda.synchronize()
        for _ in range(25):
            r = float(np.float32(rng.random()))
            want = _robust(oracle, lg, temp, k, p, r)
            got = int(ctx.sample_dev(d.data_ptr(), lg.size, 1, temp, k, p, [r])[0])
            if want is None:
                continue
            assert got == want, (lg.size, temp, k, p, r)
            compared += 1
    assert compared >= 180


@pytest.mark.gpu
def test_device_sampler_batch_and_greedy(ctx, oracle):
    import torch
    rng = np.random.default_rng(3)
    lg = (rng.standard_normal((4, 5000)) * 2).astype(np.float32)
    lg[2, 17] = lg[2, 4000] = lg[2].max() + 1  # a tie: the first index wins
    d = torch.from_numpy(lg).cuda()
    torch.cuda.synchronize()
    got = ctx.sample_dev(d.data_ptr(), 5000, 4, 0.0)
    assert list(got) == [int(np.argmax(row)) for row in lg] and got[2] == 17
    rs = [0.1, 0.5, 0.9, 0.3]
    got = ctx.sample_dev(d.data_ptr(), 5000, 4, 0.9, 40, 0.9, rs)
    for b in range(4):
        want = _robust(oracle, lg[b], 0.9, 40, 0.9, rs[b])
        if want is not None:
            assert got[b] == want, b
    with pytest.raises(ValueError):
        ctx.sample_dev(d.data_ptr(), 5000, 1, 1.0, 0, 0.9, [0.5])  # top_k < 1


@pytest.mark.gpu
def test_model_sample_after_forward(ctx, oracle):
    """cn_llama_sample reads the logits the last Forward left on the device."""
    from chatnet_b200 import configs as cf
    from chatnet_b200.llama import CudaLlamaModel
    from tests.test_gpu_llama import small_dc
    dc = cf.replace(small_dc(), kv_filled=0, decode_pos=0)
    ts = cf.device_tensors(ctx, dc)
    g = CudaLlamaModel(ctx, dc.model, ts)
    rng = np.random.default_rng(5)
    for pos in range(3):
        logits = g.forward([cf.token(dc, 0, pos)], pos)
        for temp in (0.0, 0.8, 1.3):
            r = float(np.float32(rng.random()))
            want = _robust(oracle, logits, temp, 40, 0.9, r)
            got = int(g.sample(1, temp, 40, 0.9, [r])[0])
            if want is not None:
                assert got == want, (pos, temp, r)
    g.close()
    for t in ts:
        t.free()
