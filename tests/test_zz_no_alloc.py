"""spl_sage_quantize_noalloc: the quantiser without any device allocation
(fixed library scratch instead of a workspace).  Its outputs must equal, byte
for byte, what spl_sage_prepare writes for the same inputs, on consecutive
calls with different shapes and data.  This file is collected last so that it
also runs after every other GPU test in the same process."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from sagetest import Case, engine, make_inputs, run_ours, sage, to_device
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _v_to_reference(v8: np.ndarray, b: int, g: int, d: int, tk_pad: int) -> np.ndarray:
    """[b][g][D][tk_pad] (keys in order) -> the reference's
    [b][g][tk_pad/64][D][64] with keys permuted inside each 16 by vpos."""
    v = v8.reshape(b, g, d, tk_pad // 64, 64)
    perm = np.array([(kl & ~15) + O.vpos(kl & 15) for kl in range(64)])
    out = np.empty((b, g, tk_pad // 64, d, 64), np.uint8)
    out[..., perm] = v.transpose(0, 1, 3, 2, 4)
    return out


def _noalloc(c: Case, x):
    tq_pad = (c.tokens + 127) // 128 * 128
    tk_pad = (c.tokens + 63) // 64 * 64
    b, hq, g, d = c.batch, c.heads, c.kv_heads, c.d
    keep, (tq, tk, tv) = to_device(c, x)
    q8 = torch.full((b * hq * tq_pad * d,), 7, dtype=torch.int8, device="cuda")
    qs = torch.full((b * hq * tq_pad // 16,), 7.0, dtype=torch.float32, device="cuda")
    k8 = torch.full((b * g * tk_pad * d,), 7, dtype=torch.int8, device="cuda")
    ks = torch.full((b * g * tk_pad // 64,), 7.0, dtype=torch.float32, device="cuda")
    v8 = torch.full((b * g * d * tk_pad,), 7, dtype=torch.uint8, device="cuda")
    st = torch.full((b * g * 4 * d,), 7.0, dtype=torch.float32, device="cuda")
    opts = sage.Options(smooth_k=c.smooth, smooth_v=c.smooth)
    if c.ln:
        opts.qk_norm = sage.QkNorm(torch.from_numpy(x.ln).cuda(), 1e-5)
    sage.quantize_noalloc(d, sage.Shape(b, hq, c.tokens, g), tq, tk, tv, q8, qs, k8, ks, v8, st, opts,
                          sage.PvAccum.F16 if c.pv16 else sage.PvAccum.F32, torch.cuda.current_stream())
    torch.cuda.synchronize()
    return {
        "q8": q8.cpu().numpy().reshape(b, hq, tq_pad, d),
        "q_scale": qs.cpu().numpy().reshape(b, hq, tq_pad // 16),
        "k8": k8.cpu().numpy().reshape(b, g, tk_pad, d),
        "k_scale": ks.cpu().numpy().reshape(b, g, tk_pad // 64),
        "v8": _v_to_reference(v8.cpu().numpy(), b, g, d, tk_pad),
        "stats": st.cpu().numpy().reshape(b, g, 4, d),
    }


CASES = [
    Case(batch=2, heads=4, kv_heads=2, tokens=1000, d=128, ln=True, seed=5),
    Case(batch=1, heads=8, kv_heads=8, tokens=3001, d=64, pv16=True, seed=9, packed=False),
]


def test_noalloc_matches_workspace_prepare_on_consecutive_calls():
    got = []
    for c in CASES:  # two calls in a row, different shapes and data
        got.append(_noalloc(c, make_inputs(c)))
    for c, mine in zip(CASES, got):
        want = run_ours(c, make_inputs(c)).quant
        for name, arr in mine.items():
            ref = getattr(want, name)
            assert arr.shape == ref.shape, name
            np.testing.assert_array_equal(arr.view(np.uint8), np.ascontiguousarray(ref).view(np.uint8),
                                          err_msg=f"{name} of {c}")


def test_noalloc_rejects_sizes_beyond_its_scratch():
    b, h, t, d = 8, 64, 4096, 128  # 8*64*32*4*128 = 8,388,608 floats of statistics: too big
    x = torch.zeros(16, dtype=torch.bfloat16, device="cuda")  # the size check comes first
    st = sage.Strides.bthd(t, h, d)
    tv = sage.Tensor(x, st)
    small = torch.zeros(16, dtype=torch.float32, device="cuda")
    with pytest.raises(sage.SageError) as e:
        sage.quantize_noalloc(d, sage.Shape(b, h, t, h), tv, tv, tv, small, small, small, small, small, small)
    assert "scratch" in str(e.value)
