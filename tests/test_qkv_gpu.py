"""The fused QKV GEMM (spl_sage_qkv_gemm: tcgen05 bf16 GEMM + bias + RoPE
epilogue; one SM per tile, and SM pairs with cta_group::2) against the f64 oracle of the reference's GEMM + QKV prologue
(host::linear + qkv::reference), with the reference's own tolerance for its
GEMM (src/tests.rs:652-684: rel-RMS 4e-3 against f64, here on bf16 outputs
5e-3), and parity at the quantiser boundary: the quantised workspace equals
the oracle quantiser applied to the bf16 Q/K/V the GEMM wrote, bit for bit."""

import importlib

import numpy as np
import pytest
import torch

import sagetest as st
from oracle import oracle as O

pytestmark = pytest.mark.gpu
sage = importlib.import_module("sota-papers-lab_b200")


def _bf16(a):
    return O.f32_to_bf16(np.ascontiguousarray(a, np.float32))


def _dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda().view(torch.bfloat16)


def _host(t):
    return O.bf16_to_f32(t.view(torch.int16).cpu().numpy().view(np.uint16))


CASES = {
    # name: batch, tokens, hidden, heads, kv, d, rope kind
    "vit_d64_norope": (2, 137, 1024, 16, 16, 64, None),
    "llama_d128_rope1d": (2, 200, 512, 4, 2, 128, "llama"),
    "vggt_d64_rope2d": (1, 3 * 75, 256, 4, 4, 64, "vggt"),
}


@pytest.mark.parametrize("pairs", [False, True], ids=["1sm", "2sm"])
@pytest.mark.parametrize("name", list(CASES))
def test_qkv_gemm_matches_f64_oracle(name, pairs):
    b, t, hidden, hq, hkv, d, rk = CASES[name]
    rng = np.random.default_rng(5)
    m, n = b * t, (hq + 2 * hkv) * d
    # LayerNormed activations and N(0, 0.02^2) weights (BASELINE configs C2/C4)
    x = rng.normal(size=(m, hidden)).astype(np.float32)
    x = (x - x.mean(1, keepdims=True)) / x.std(1, keepdims=True)
    xb, wb = _bf16(x), _bf16(rng.normal(0, 0.02, size=(n, hidden)))
    bias = _bf16(rng.normal(0, 0.1, size=n))
    rope, half, frame = None, 0, 1
    if rk == "llama":
        rope, half, frame = sage.rope_table_1d(500000.0, d, t), d // 2, t
    elif rk == "vggt":
        tab = sage.RopeTable.vggt(7, 10, 5)
        rope, half, frame = tab.cos_sin, tab.half, tab.frame_len
    eng = st.engine(st.Case(batch=b, heads=hq, kv_heads=hkv, tokens=t, d=d))
    eng.gemm_pairs(pairs)
    q = torch.empty(b, t, hq, d, dtype=torch.bfloat16, device="cuda")
    k = torch.empty(b, t, hkv, d, dtype=torch.bfloat16, device="cuda")
    v = torch.empty(b, t, hkv, d, dtype=torch.bfloat16, device="cuda")
    rd = None if rope is None else torch.from_numpy(rope).cuda()
    eng.qkv_gemm(_dev(xb), _dev(wb), _dev(bias), rd, q, k, v, batch=b, tokens=t, heads=hq, kv_heads=hkv,
                 rope_half=half, frame_len=frame)
    assert eng.engine_status() == 0
    want = O.qkv_reference(xb, wb, bias, rope, tokens=t, hq=hq, hkv=hkv, d=d, rope_half=half, frame_len=frame)
    for got, ref, what in zip((q, k, v), want, "qkv"):
        g = _host(got).reshape(ref.shape)
        e = O.errors(g, ref)
        rel_rms = e["rel_l2"]
        print(name, what, e)
        assert rel_rms < 5e-3 and e["max_abs"] < 0.05 * max(1.0, e["ref_max"]), (what, e)


def test_qkv_gemm_quant_is_the_quantiser_on_its_own_output():
    b, t, hidden, hq, hkv, d = 1, 300, 512, 4, 2, 128
    rng = np.random.default_rng(9)
    m, n = b * t, (hq + 2 * hkv) * d
    xb, wb = _bf16(rng.normal(size=(m, hidden))), _bf16(rng.normal(0, 0.02, size=(n, hidden)))
    rope = sage.rope_table_1d(500000.0, d, t)
    c = st.Case(batch=b, heads=hq, kv_heads=hkv, tokens=t, d=d, causal=True, packed=False)
    eng = st.engine(c)
    ws = eng.workspace(sage.Shape(b, hq, t, hkv, True))
    q = torch.empty(b, t, hq, d, dtype=torch.bfloat16, device="cuda")
    k = torch.empty(b, t, hkv, d, dtype=torch.bfloat16, device="cuda")
    v = torch.empty(b, t, hkv, d, dtype=torch.bfloat16, device="cuda")
    eng.qkv_gemm_quant(ws, _dev(xb), _dev(wb), None, torch.from_numpy(rope).cuda(), q, k, v, rope_half=64,
                       frame_len=t)
    p = ws.plan
    got = O.Quant(q8=None, q_scale=None, k8=None, k_scale=None, v8=None, stats=None, kbias=None, part=None)
    bufs = dict(q8=torch.zeros(b * hq * p.tq_pad * d, dtype=torch.int8, device="cuda"),
                q_scale=torch.zeros(b * hq * p.tq_pad // 16, device="cuda"),
                k8=torch.zeros(b * hkv * p.tk_pad * d, dtype=torch.int8, device="cuda"),
                k_scale=torch.zeros(b * hkv * p.tk_pad // 64, device="cuda"),
                v8=torch.zeros(b * hkv * p.tk_pad * d, dtype=torch.uint8, device="cuda"),
                stats=torch.zeros(b * hkv * 4 * d, device="cuda"), kbias=torch.zeros(p.tk_pad, device="cuda"))
    eng.export_reference_layout(ws, **bufs)
    torch.cuda.synchronize()
    qb = q.view(torch.int16).cpu().numpy().view(np.uint16)
    kb = k.view(torch.int16).cpu().numpy().view(np.uint16)
    vb = v.view(torch.int16).cpu().numpy().view(np.uint16)
    want = O.prepare(qb, kb, vb, st.geom(c))
    got.q8 = bufs["q8"].cpu().numpy().reshape(want.q8.shape)
    got.q_scale = bufs["q_scale"].cpu().numpy().reshape(want.q_scale.shape)
    got.k8 = bufs["k8"].cpu().numpy().reshape(want.k8.shape)
    got.k_scale = bufs["k_scale"].cpu().numpy().reshape(want.k_scale.shape)
    got.v8 = bufs["v8"].cpu().numpy().reshape(want.v8.shape)
    got.stats = bufs["stats"].cpu().numpy().reshape(want.stats.shape)
    got.kbias = bufs["kbias"].cpu().numpy()
    st.assert_quant_equal(got, want, kbias=False, what="qkv_gemm_quant")
