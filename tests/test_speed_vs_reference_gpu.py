"""Speed on the same B200 against the reference's own kernels.

The reference's SageAttention2 kernels (platform/spl-nn/cuda/sage_quant.cu,
sage_attn.cu: mma.sync INT8/FP8, built for sm_100a from their sources into
oracle/_ref) are the GPU implementation this library replaces.  For the
benchmark configurations they support (non-causal, equal head counts: C1,
C2's attention, C3) both are timed here on the same inputs (bench.py's
generator), with CUDA events on one stream after warm-up: the whole forward
(quantiser + attention, sg_prep/sg_finalize/sg_quant_kv/sg_attn launched
with the grids of src/sage/mod.rs:789-870) and the attention alone.  The
gate: ours is faster in both.  Each case prints one JSON line with the
times, the TOPS (4*B*H*N^2*D / t) and the speed-up."""
from __future__ import annotations

import ctypes
import json
import statistics

import numpy as np
import pytest
import torch

import bench
import sagetest as st
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _time(fn, iters=10, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


class _Reference:
    """The reference kernels on device tensors q/k/v [B][T][H][D] (bthd)."""

    def __init__(self, c: st.Case, q, k, v):
        self.L = O.ref_lib(c.d)
        self.g = g = st.geom(c)
        b, h, d = c.batch, c.heads, c.d
        so = st.sage.Strides.bthd(c.tokens, h, d)
        sq = st.sage.Strides.bthd(c.tokens, h, d)
        self.strides = np.array([sq.batch, sq.token, sq.head] * 3 + [so.batch, so.token, so.head], np.int64)
        self.dims = O.ref_dims(g)
        z = lambda n, dt: torch.zeros(n, dtype=dt, device="cuda")
        self.q8, self.qs = z(b * h * g.tq_pad * d, torch.int8), z(b * h * g.tq_pad // 16, torch.float32)
        self.k8, self.ks = z(b * h * g.tk_pad * d, torch.int8), z(b * h * g.tk_pad // 64, torch.float32)
        self.v8, self.stats = z(b * h * g.tk_pad * d, torch.uint8), z(b * h * 4 * d, torch.float32)
        self.kb, self.part = z(g.tk_pad, torch.float32), z(b * h * g.q_tiles * 4 * d, torch.float32)
        self.out = z(b * c.tokens * h * d, torch.bfloat16)
        self.q, self.k, self.v = q, k, v

    def _p(self, t):
        return None if t is None else ctypes.c_void_p(t.data_ptr())

    def forward(self):
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = self.L.ref_sage_run(self._p(self.q), self._p(self.k), self._p(self.v), None,
                                 self.strides.ctypes.data_as(ctypes.c_void_p), self.dims.ctypes.data_as(ctypes.c_void_p),
                                 self.g.q_mul, self.g.ln_eps, self.g.v_range, self._p(self.q8), self._p(self.qs),
                                 self._p(self.k8), self._p(self.ks), self._p(self.v8), self._p(self.stats),
                                 self._p(self.kb), self._p(self.part), self._p(self.out), s)
        assert rc == 0, rc

    def attend(self):
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = self.L.ref_sage_attend(self.strides.ctypes.data_as(ctypes.c_void_p),
                                    self.dims.ctypes.data_as(ctypes.c_void_p), self.g.q_mul, self.g.v_range,
                                    self._p(self.q8), self._p(self.qs), self._p(self.k8), self._p(self.ks),
                                    self._p(self.v8), self._p(self.stats), self._p(self.kb), self._p(self.out), s)
        assert rc == 0, rc


@pytest.mark.parametrize("name", ["C1", "C2", "C3"])
def test_faster_than_reference_kernels_on_this_gpu(name):
    w = bench.WORKLOADS[name]
    if not O.ref_available(w["d"]):
        pytest.skip("oracle/_ref not built")
    B, H, T, D = w["batch"], w["heads"], w["tokens"], w["d"]
    q, k, v = bench.make_inputs(w, B, 1, "cuda")
    c = st.Case(batch=B, heads=H, kv_heads=H, tokens=T, d=D, packed=False)
    eng = st.engine(c)
    ws = eng.workspace(st.sage.Shape(B, H, T, H, False))
    st_ = st.sage.Strides.bthd(T, H, D)
    tq, tk, tv = (st.sage.Tensor(x.reshape(-1), st_) for x in (q, k, v))
    out = torch.empty(B * T * H * D, dtype=torch.bfloat16, device="cuda")
    to = st.sage.Tensor(out, st_)
    ours_fwd = _time(lambda: eng.forward(ws, tq, tk, tv, to))
    ours_att = _time(lambda: eng.attend(ws, to))
    assert eng.status(ws) == 0
    ref = _Reference(c, q, k, v)
    ref_fwd = _time(ref.forward)
    ref_att = _time(ref.attend)
    # the two outputs agree (the same gate as the parity tests)
    e = O.errors(O.bf16_to_f32(out.view(torch.int16).cpu().numpy().view(np.uint16)),
                 O.bf16_to_f32(ref.out.view(torch.int16).cpu().numpy().view(np.uint16)))
    assert st.attention_gate(e), e
    fl = 4.0 * B * H * T * T * D
    line = dict(config=name, ours_forward_ms=round(ours_fwd, 4), ref_forward_ms=round(ref_fwd, 4),
                ours_attend_ms=round(ours_att, 4), ref_attend_ms=round(ref_att, 4),
                ours_forward_tops=round(fl / ours_fwd / 1e9, 1), ref_forward_tops=round(fl / ref_fwd / 1e9, 1),
                speedup_forward=round(ref_fwd / ours_fwd, 2), speedup_attend=round(ref_att / ours_att, 2),
                cos=round(e["cos"], 6), rel_l1=round(e["rel_l1"], 5))
    print("SPEED " + json.dumps(line))
    assert ours_fwd < ref_fwd and ours_att < ref_att, line
