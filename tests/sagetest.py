"""Helpers shared by the GPU parity tests: run the product through its C ABI,
run the CPU oracle and the reference's own kernels (oracle/_ref) on the same
seeded inputs, and compare."""
from __future__ import annotations

import ctypes
import importlib
from dataclasses import dataclass

import numpy as np
import torch

from oracle import oracle as O

sage = importlib.import_module("sota-papers-lab_b200")


def small_layout():
    # tests.rs:596-605
    return O.Layout(frames=3, special=5, grid_h=7, grid_w=10, dense_frames=1)


def ln_params(d: int, seed: int) -> np.ndarray:
    # tests.rs:422-435
    r = O.Rng(seed)
    out = []
    for part in range(4):
        for _ in range(d):
            out.append(1.0 + 0.5 * r.normal() if part % 2 == 0 else 0.8 * r.normal())
    return np.array(out, np.float32)


@dataclass
class Case:
    batch: int
    heads: int
    kv_heads: int
    tokens: int
    d: int
    merge: int = 1
    layout: O.Layout | None = None
    ln: bool = False
    smooth: bool = True
    causal: bool = False
    pv16: bool = False
    seed: int = 11
    packed: bool = True  # packed [b][t][3][h][d] when heads == kv_heads

    def flags(self):
        f = 0
        if self.ln:
            f |= O.LN_Q | O.LN_K
        if self.smooth:
            f |= O.SMOOTH_K | O.SMOOTH_V
        return f


@dataclass
class Inputs:
    q: np.ndarray  # bf16 bits [b][t][hq][d]
    k: np.ndarray  # [b][t][hkv][d]
    v: np.ndarray
    ln: np.ndarray | None


def make_inputs(c: Case) -> Inputs:
    if c.heads == c.kv_heads:
        q, k, v = O.synthetic(c.batch, c.heads, c.tokens, c.d, c.seed)
    else:
        q, _, _ = O.synthetic(c.batch, c.heads, c.tokens, c.d, c.seed)
        _, k, v = O.synthetic(c.batch, c.kv_heads, c.tokens, c.d, c.seed + 1)
    ln = ln_params(c.d, 3) if c.ln else None
    return Inputs(q, k, v, ln)


def geom(c: Case) -> O.Geom:
    sq = O.bthd_strides(c.tokens, c.heads, c.d)
    skv = O.bthd_strides(c.tokens, c.kv_heads, c.d)
    return O.make_geom(c.batch, c.heads, c.kv_heads, c.tokens, c.d, sq, skv, skv, flags=c.flags(), merge=c.merge,
                       layout=c.layout, v_range=O.PV16_V_RANGE if c.pv16 else O.FP8_MAX)


def _dev_bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.bfloat16)


def to_device(c: Case, x: Inputs):
    """Device tensors and their sage.Tensor views (packed QKV when possible,
    like the reference's run_gpu, tests.rs:372-420)."""
    d, h, t, b = c.d, c.heads, c.tokens, c.batch
    if c.packed and c.heads == c.kv_heads:
        packed = np.stack([x.q, x.k, x.v], axis=2)  # [b][t][3][h][d]
        buf = _dev_bf16(packed).reshape(-1)
        st = sage.Strides.packed_qkv(t, h, d)
        hd = h * d
        return (buf,), (sage.Tensor(buf[0:], st), sage.Tensor(buf[hd:], st), sage.Tensor(buf[2 * hd:], st))
    qd, kd, vd = _dev_bf16(x.q).reshape(-1), _dev_bf16(x.k).reshape(-1), _dev_bf16(x.v).reshape(-1)
    sq = sage.Strides.bthd(t, c.heads, d)
    skv = sage.Strides.bthd(t, c.kv_heads, d)
    return (qd, kd, vd), (sage.Tensor(qd, sq), sage.Tensor(kd, skv), sage.Tensor(vd, skv))


def engine(c: Case):
    cfg = sage.Config(sage.Tile.for_head_dim(c.d), sage.PvAccum.F16 if c.pv16 else sage.PvAccum.F32)
    return sage.SageAttention(torch.cuda.current_stream(), c.d, cfg)


def merge_of(c: Case):
    if c.merge == 1:
        return sage.KvMerge.dense()
    L = c.layout
    return sage.KvMerge.pool(c.merge, sage.FrameLayout(L.frames, L.special, L.grid_h, L.grid_w, L.dense_frames))


@dataclass
class Run:
    out: np.ndarray  # f32 [b][t][hq][d]
    quant: O.Quant | None
    ws: object
    eng: object


def run_ours(c: Case, x: Inputs, *, export=True) -> Run:
    eng = engine(c)
    ws = eng.workspace(sage.Shape(c.batch, c.heads, c.tokens, c.kv_heads, c.causal), merge_of(c))
    keep, (tq, tk, tv) = to_device(c, x)
    out = torch.zeros(c.batch * c.tokens * c.heads * c.d, dtype=torch.bfloat16, device="cuda")
    opts = sage.Options(smooth_k=c.smooth, smooth_v=c.smooth)
    ln_dev = None
    if c.ln:
        ln_dev = torch.from_numpy(x.ln).cuda()
        opts.qk_norm = sage.QkNorm(ln_dev, 1e-5)
    eng.forward(ws, tq, tk, tv, sage.Tensor(out, sage.Strides.bthd(c.tokens, c.heads, c.d)), opts)
    quant = export_quant(eng, ws, c) if export else None
    word = eng.status(ws)
    assert word == 0
    o = out.view(torch.int16).cpu().numpy().view(np.uint16)
    return Run(O.bf16_to_f32(o).reshape(c.batch, c.tokens, c.heads, c.d), quant, ws, eng)


def export_quant(eng, ws, c: Case) -> O.Quant:
    """The workspace's quantised tensors in the reference's byte layouts."""
    p = ws.plan
    b, hq, hkv, d = c.batch, c.heads, c.kv_heads, c.d
    q8 = torch.zeros(b * hq * p.tq_pad * d, dtype=torch.int8, device="cuda")
    qs = torch.zeros(b * hq * p.tq_pad // 16, dtype=torch.float32, device="cuda")
    k8 = torch.zeros(b * hkv * p.tk_pad * d, dtype=torch.int8, device="cuda")
    ks = torch.zeros(b * hkv * p.tk_pad // 64, dtype=torch.float32, device="cuda")
    v8 = torch.zeros(b * hkv * p.tk_pad * d, dtype=torch.uint8, device="cuda")
    st = torch.zeros(b * hkv * 4 * d, dtype=torch.float32, device="cuda")
    kb = torch.zeros(p.tk_pad, dtype=torch.float32, device="cuda")
    eng.export_reference_layout(ws, q8, qs, k8, ks, v8, st, kb)
    torch.cuda.synchronize()
    return O.Quant(q8=q8.cpu().numpy().reshape(b, hq, p.tq_pad, d),
                   q_scale=qs.cpu().numpy().reshape(b, hq, p.tq_pad // 16),
                   k8=k8.cpu().numpy().reshape(b, hkv, p.tk_pad, d),
                   k_scale=ks.cpu().numpy().reshape(b, hkv, p.tk_pad // 64),
                   v8=v8.cpu().numpy().reshape(b, hkv, p.tk_pad // 64, d, 64),
                   stats=st.cpu().numpy().reshape(b, hkv, 4, d), kbias=kb.cpu().numpy(), part=None)


def run_reference_gpu(c: Case, x: Inputs, *, attend=True):
    """The reference's own kernels (oracle/_ref) on the same inputs: returns
    (out f32 [b][t][h][d] or None, Quant).  Needs heads == kv_heads."""
    assert c.heads == c.kv_heads and not c.causal
    L = O.ref_lib(c.d, c.pv16)
    g = geom(c)
    b, h, d = c.batch, c.heads, c.d
    keep, (tq, tk, tv) = to_device(c, x)
    st_q, st_k = tq.strides, tk.strides
    so = sage.Strides.bthd(c.tokens, h, d)
    strides = np.array([st_q.batch, st_q.token, st_q.head, st_k.batch, st_k.token, st_k.head,
                        tv.strides.batch, tv.strides.token, tv.strides.head, so.batch, so.token, so.head], np.int64)
    dims = O.ref_dims(g)
    q8 = torch.zeros(b * h * g.tq_pad * d, dtype=torch.int8, device="cuda")
    qs = torch.zeros(b * h * g.tq_pad // 16, dtype=torch.float32, device="cuda")
    k8 = torch.zeros(b * h * g.tk_pad * d, dtype=torch.int8, device="cuda")
    ks = torch.zeros(b * h * g.tk_pad // 64, dtype=torch.float32, device="cuda")
    v8 = torch.zeros(b * h * g.tk_pad * d, dtype=torch.uint8, device="cuda")
    stt = torch.zeros(b * h * 4 * d, dtype=torch.float32, device="cuda")
    kb = torch.zeros(g.tk_pad, dtype=torch.float32, device="cuda")
    part = torch.zeros(b * h * g.q_tiles * 4 * d, dtype=torch.float32, device="cuda")
    out = torch.zeros(b * c.tokens * h * d, dtype=torch.bfloat16, device="cuda") if attend else None
    ln_dev = torch.from_numpy(x.ln).cuda() if c.ln else None
    vp = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
    rc = L.ref_sage_run(vp(tq.data), vp(tk.data), vp(tv.data), vp(ln_dev), strides.ctypes.data_as(ctypes.c_void_p),
                        dims.ctypes.data_as(ctypes.c_void_p), g.q_mul, g.ln_eps, g.v_range, vp(q8), vp(qs), vp(k8),
                        vp(ks), vp(v8), vp(stt), vp(kb), vp(part), vp(out),
                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, rc
    torch.cuda.synchronize()
    quant = O.Quant(q8=q8.cpu().numpy().reshape(b, h, g.tq_pad, d), q_scale=qs.cpu().numpy().reshape(b, h, -1),
                    k8=k8.cpu().numpy().reshape(b, h, g.tk_pad, d), k_scale=ks.cpu().numpy().reshape(b, h, -1),
                    v8=v8.cpu().numpy().reshape(b, h, g.tk_pad // 64, d, 64), stats=stt.cpu().numpy().reshape(b, h, 4, d),
                    kbias=kb.cpu().numpy(), part=part.cpu().numpy())
    o = None
    if attend:
        o = O.bf16_to_f32(out.view(torch.int16).cpu().numpy().view(np.uint16)).reshape(b, c.tokens, h, d)
    return o, quant


def assert_quant_equal(a: O.Quant, b: O.Quant, *, kbias=True, what=""):
    for name in ("q8", "q_scale", "k8", "k_scale", "v8", "stats"):
        x, y = getattr(a, name), getattr(b, name)
        assert x.shape == y.shape, (what, name, x.shape, y.shape)
        if x.dtype == np.float32:
            same = x.view(np.uint32) == y.view(np.uint32)
        else:
            same = x == y
        if not same.all():
            idx = np.argwhere(~same)[:5]
            raise AssertionError(f"{what}: {name} differs at {len(np.argwhere(~same))} places, first "
                                 f"{idx.tolist()}: {x[tuple(idx[0])]} vs {y[tuple(idx[0])]}")
    if kbias:
        np.testing.assert_allclose(a.kbias, b.kbias, rtol=0, atol=1e-6)


def attention_gate(e: dict) -> bool:
    """The north-star gate against the reference implementation."""
    return e["cos"] >= 0.9995 and e["rel_l1"] <= 1e-2


def reference_gate(e: dict) -> bool:
    """The reference's own gate against f64 attention (tests.rs:699)."""
    return e["cos"] > 0.999 and e["rel_l2"] < 0.04
