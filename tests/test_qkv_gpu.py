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
    # one kv head (C4 sharded over 8 GPUs): a 256-channel tile holds a K and
    # a V head; at D = 64 one tile holds Q, K and V heads
    "llama_d128_kv1": (2, 200, 512, 4, 1, 128, "llama"),
    "d64_q2_kv1": (1, 160, 256, 2, 1, 64, None),
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


QUANT_CASES = {
    # name: batch, tokens, hidden, heads, kv, d, rope kind, pairs (SM-pair GEMM)
    "fused_d128_rope1d": (2, 304, 512, 4, 2, 128, "llama", True),      # Q quantised in the epilogue
    "fused_d64_norope": (2, 256, 256, 4, 4, 64, None, True),
    "fused_d64_vggt": (1, 3 * 80, 256, 4, 4, 64, "vggt", True),
    "fused_d128_kv1": (2, 304, 512, 4, 1, 128, "llama", True),        # the per-rank shape of C4 on 8 GPUs
    "unfused_ragged": (1, 300, 512, 4, 2, 128, "llama", True),         # tokens % 16 != 0: whole quantiser
    "unfused_1sm": (1, 304, 512, 4, 2, 128, "llama", False),
}


@pytest.mark.parametrize("name", list(QUANT_CASES))
def test_qkv_gemm_quant_is_the_quantiser_on_its_own_output(name):
    """spl_sage_qkv_gemm_quant's workspace equals, byte for byte, the oracle
    quantiser run on the bf16 Q/K/V the same call wrote (A.7: the GEMM output
    rounded to bf16 after the GEMM and after RoPE, then quantised), whether Q
    is quantised in the GEMM's epilogue (fused) or by the quantiser."""
    b, t, hidden, hq, hkv, d, rk, pairs = QUANT_CASES[name]
    rng = np.random.default_rng(9)
    m, n = b * t, (hq + 2 * hkv) * d
    xb, wb = _bf16(rng.normal(size=(m, hidden))), _bf16(rng.normal(0, 0.02, size=(n, hidden)))
    bias = _bf16(rng.normal(0, 0.1, size=n))
    rope, half, frame = None, 0, 1
    if rk == "llama":
        rope, half, frame = sage.rope_table_1d(500000.0, d, t), d // 2, t
    elif rk == "vggt":
        tab = sage.RopeTable.vggt(5, 15, 5)
        rope, half, frame = tab.cos_sin, tab.half, tab.frame_len
    c = st.Case(batch=b, heads=hq, kv_heads=hkv, tokens=t, d=d, causal=True, packed=False)
    eng = st.engine(c)
    eng.gemm_pairs(pairs)
    ws = eng.workspace(sage.Shape(b, hq, t, hkv, True))
    q = torch.empty(b, t, hq, d, dtype=torch.bfloat16, device="cuda")
    k = torch.empty(b, t, hkv, d, dtype=torch.bfloat16, device="cuda")
    v = torch.empty(b, t, hkv, d, dtype=torch.bfloat16, device="cuda")
    rd = None if rope is None else torch.from_numpy(rope).cuda()
    eng.qkv_gemm_quant(ws, _dev(xb), _dev(wb), _dev(bias), rd, q, k, v, rope_half=half, frame_len=frame)
    assert eng.status(ws) == 0
    got = st.export_quant(eng, ws, c)
    qb = q.view(torch.int16).cpu().numpy().view(np.uint16)
    kb = k.view(torch.int16).cpu().numpy().view(np.uint16)
    vb = v.view(torch.int16).cpu().numpy().view(np.uint16)
    want = O.prepare(qb, kb, vb, st.geom(c))
    st.assert_quant_equal(got, want, kbias=False, what=f"qkv_gemm_quant {name}")
    # the bf16 outputs are the GEMM's own (unchanged by the fusion)
    ref = O.qkv_reference(xb, wb, bias, rope, tokens=t, hq=hq, hkv=hkv, d=d, rope_half=half, frame_len=frame)
    for got_t, r, what in zip((q, k, v), ref, "qkv"):
        e = O.errors(_host(got_t).reshape(r.shape), r)
        assert e["rel_l2"] < 5e-3, (what, e)
    if name.startswith("fused"):
        # with q NULL the fused path writes no bf16 Q and the same bytes
        ws2 = eng.workspace(sage.Shape(b, hq, t, hkv, True))
        eng.qkv_gemm_quant(ws2, _dev(xb), _dev(wb), _dev(bias), rd, None, k, v, rope_half=half, frame_len=frame)
        got2 = st.export_quant(eng, ws2, c)
        st.assert_quant_equal(got2, got, kbias=False, what=f"qkv_gemm_quant {name} without bf16 Q")
