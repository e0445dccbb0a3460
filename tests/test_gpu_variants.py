"""The architecture variants other ChatNet models run on the Llama loop,
selected in cn_llama_config: split-half RoPE (TensorMath.ApplyRoPENeox,
Tensors/TensorMath.cs:475; Qwen, Phi), GELU * up (GeluElementwiseMul, :294;
Gemma) and RMSNorm weights stored as w - 1 (RmsNormWithOffset, :335; Gemma).
Decode steps (fp32 cache: RoPE kernel + split attention; fp16 cache: RoPE
fused into the tensor-core attention) and the prefill pass against the
oracle's Forward with the same variants: logits within 1e-3, same argmax."""
from __future__ import annotations

import numpy as np
import pytest

from chatnet_b200 import configs as cf
from tests.parity import REL_TOL, rel_err
from tests.test_gpu_llama import Pair, small_dc

pytestmark = pytest.mark.gpu

VARIANTS = [(1, 0, 0), (0, 1, 0), (0, 0, 1), (1, 1, 1)]


def variant_dc(neox, gelu, offset, kv_f16, **kw):
    dc = small_dc(kv_f16=kv_f16, **kw)
    m = cf.replace(dc.model, rope_neox=bool(neox), act_gelu=bool(gelu), norm_offset=bool(offset))
    return cf.replace(dc, model=m)


@pytest.mark.parametrize("kv_f16", [False, True])
@pytest.mark.parametrize("neox,gelu,offset", VARIANTS)
def test_variant_decode(ctx, oracle, neox, gelu, offset, kv_f16):
    dc = variant_dc(neox, gelu, offset, kv_f16)
    p = Pair(ctx, oracle, dc)
    for step in range(3):
        tok = cf.token(dc, 0, step)
        got = p.gpu.forward([tok], dc.decode_pos + step)
        ref = p.oracles[0].forward([tok], dc.decode_pos + step)
        assert rel_err(got, ref) <= REL_TOL, (step, rel_err(got, ref))
        assert int(np.argmax(got)) == int(np.argmax(ref))
    p.close()


@pytest.mark.parametrize("kv_f16", [False, True])
def test_variant_prefill(ctx, oracle, kv_f16):
    """A 24-token prompt through cn_llama_forward (the prefill pass) with all
    three variants, then a decode step from the cache it wrote."""
    dc = cf.replace(variant_dc(1, 1, 1, kv_f16), kv_filled=0, decode_pos=0)
    p = Pair(ctx, oracle, dc)
    toks = [cf.token(dc, 0, s) for s in range(24)]
    got = p.gpu.forward(toks, 0)
    ref = p.oracles[0].forward(toks, 0)
    assert rel_err(got, ref) <= REL_TOL, rel_err(got, ref)
    assert int(np.argmax(got)) == int(np.argmax(ref))
    nxt = int(np.argmax(ref))
    assert rel_err(p.gpu.forward([nxt], 24), p.oracles[0].forward([nxt], 24)) <= REL_TOL
    p.close()


def test_variant_flags_validated(ctx):
    from chatnet_b200.llama import CudaLlamaModel
    dc = small_dc()
    bad = cf.replace(dc.model, head_dim=64)
    c = bad.to_c()
    c.rope_neox = 2
    import ctypes as C
    from chatnet_b200 import _native as N
    ts = cf.device_tensors(ctx, dc)
    arr = (C.c_void_p * len(ts))(*[t.handle for t in ts])
    h = C.c_void_p()
    assert N.lib().cn_llama_create(ctx.handle, C.byref(c), arr, len(ts), C.byref(h)) == N.CN_ERR_INVALID_ARG
    for t in ts:
        t.free()
    del CudaLlamaModel
