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


def _outputs(c: Case):
    tq_pad = (c.tokens + 127) // 128 * 128
    tk_pad = (c.tokens + 63) // 64 * 64
    b, hq, g, d = c.batch, c.heads, c.kv_heads, c.d
    return dict(
        q8=torch.full((b * hq * tq_pad * d,), 7, dtype=torch.int8, device="cuda"),
        q_scale=torch.full((b * hq * tq_pad // 16,), 7.0, dtype=torch.float32, device="cuda"),
        k8=torch.full((b * g * tk_pad * d,), 7, dtype=torch.int8, device="cuda"),
        k_scale=torch.full((b * g * tk_pad // 64,), 7.0, dtype=torch.float32, device="cuda"),
        v8=torch.full((b * g * d * tk_pad,), 7, dtype=torch.uint8, device="cuda"),
        stats=torch.full((b * g * 4 * d,), 7.0, dtype=torch.float32, device="cuda"))


def _call(c: Case, x, tensors, outs):
    """One spl_sage_quantize_noalloc call on caller-owned inputs and outputs."""
    tq, tk, tv = tensors
    opts = sage.Options(smooth_k=c.smooth, smooth_v=c.smooth)
    if c.ln:
        opts.qk_norm = sage.QkNorm(x.ln_dev, 1e-5)
    sage.quantize_noalloc(c.d, sage.Shape(c.batch, c.heads, c.tokens, c.kv_heads), tq, tk, tv, outs["q8"],
                          outs["q_scale"], outs["k8"], outs["k_scale"], outs["v8"], outs["stats"], opts,
                          sage.PvAccum.F16 if c.pv16 else sage.PvAccum.F32, torch.cuda.current_stream())


def _host(c: Case, outs):
    tq_pad = (c.tokens + 127) // 128 * 128
    tk_pad = (c.tokens + 63) // 64 * 64
    b, hq, g, d = c.batch, c.heads, c.kv_heads, c.d
    return {
        "q8": outs["q8"].cpu().numpy().reshape(b, hq, tq_pad, d),
        "q_scale": outs["q_scale"].cpu().numpy().reshape(b, hq, tq_pad // 16),
        "k8": outs["k8"].cpu().numpy().reshape(b, g, tk_pad, d),
        "k_scale": outs["k_scale"].cpu().numpy().reshape(b, g, tk_pad // 64),
        "v8": _v_to_reference(outs["v8"].cpu().numpy(), b, g, d, tk_pad),
        "stats": outs["stats"].cpu().numpy().reshape(b, g, 4, d),
    }


CASES = [
    Case(batch=2, heads=4, kv_heads=2, tokens=1000, d=128, ln=True, seed=5),
    Case(batch=1, heads=8, kv_heads=8, tokens=3001, d=64, pv16=True, seed=9, packed=False),
]


def test_noalloc_matches_workspace_prepare_on_consecutive_calls():
    # Inputs and outputs are the caller's, made before the calls; the calls
    # themselves must not take any device memory (torch's allocator and the
    # device's free bytes stay where they were).
    prepared = []
    for c in CASES:
        x = make_inputs(c)
        x.ln_dev = torch.from_numpy(x.ln).cuda() if c.ln else None
        keep, tensors = to_device(c, x)
        prepared.append((c, x, keep, tensors, _outputs(c)))
    # One call first: with CUDA's lazy module loading the library's module
    # (and its fixed scratch array) may only be placed on the device at its
    # first use, which is not an allocation by the call.
    c0, x0, _, tensors0, outs0 = prepared[0]
    _call(c0, x0, tensors0, outs0)
    torch.cuda.synchronize()
    allocated, free = torch.cuda.memory_allocated(), torch.cuda.mem_get_info()[0]
    for c, x, keep, tensors, outs in prepared:  # two calls in a row, different shapes and data
        _call(c, x, tensors, outs)
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == allocated
    assert torch.cuda.mem_get_info()[0] == free
    got = [_host(c, outs) for c, x, keep, tensors, outs in prepared]
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


@pytest.mark.parametrize("name", ["C4", "C2"])
def test_noalloc_matches_workspace_prepare_at_benchmark_shapes(name):
    """At the benchmark shapes (bench.py's generator): with a workspace the
    slice statistics are reduced by the CTA that finishes a slice's last
    statistics tile, without one by sp_finalize in a launch of its own; the
    bytes are the same (many tiles per slice, every slice's count reset for
    the next call: the workspace path runs twice)."""
    import bench
    w = bench.WORKLOADS[name]
    q, k, v = bench.make_inputs(w, w["batch"], 4, "cuda")
    c = Case(batch=w["batch"], heads=w["heads"], kv_heads=w["kv_heads"], tokens=w["tokens"], d=w["d"],
             packed=False)
    st_q, st_kv = sage.Strides.bthd(c.tokens, c.heads, c.d), sage.Strides.bthd(c.tokens, c.kv_heads, c.d)
    tensors = (sage.Tensor(q.reshape(-1), st_q), sage.Tensor(k.reshape(-1), st_kv), sage.Tensor(v.reshape(-1), st_kv))
    outs = _outputs(c)
    _call(c, None, tensors, outs)
    torch.cuda.synchronize()
    got = _host(c, outs)
    del outs
    eng = engine(c)
    ws = eng.workspace(sage.Shape(c.batch, c.heads, c.tokens, c.kv_heads))
    opts = sage.Options(smooth_k=c.smooth, smooth_v=c.smooth)
    for _ in range(2):
        eng.prepare(ws, *tensors, opts)
    assert eng.status(ws) == 0
    from sagetest import export_quant
    want = export_quant(eng, ws, c)
    for name_, arr in got.items():
        ref = getattr(want, name_)
        assert arr.shape == ref.shape, name_
        np.testing.assert_array_equal(arr.view(np.uint8), np.ascontiguousarray(ref).view(np.uint8),
                                      err_msg=f"{name}: {name_}")
