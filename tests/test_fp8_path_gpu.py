"""The FP8 QKV side of the reference's FP8 transformer block
(apps/image-to-3d/src/vggt/trunk/block.rs:326-395): LN1 -> per-token E4M3
(spl_sage_layer_norm_fp8, norm.cu:37-137) and the FP8 QKV GEMM with the
prologue's token / channel scales, bias and RoPE fused
(spl_sage_qkv_gemm_fp8).

* LayerNorm: byte-identical to the reference's own kernels (built from its
  sources into oracle/_ref) on the reference's widths, f32 and bf16 inputs,
  ragged row counts and an all-zero row; against the CPU restatement (whose
  1/sqrtf may differ from rsqrtf in the last place) within one E4M3 step.
* GEMM: the f64 oracle of Gemm::linear_fp8 + qkv::reference with tok/chan on
  the same E4M3 operands, with the bf16 GEMM's gate (rel-RMS 5e-3).
* The chain LN -> FP8 GEMM -> quantiser: the quantised workspace is the
  oracle quantiser applied to the bf16 Q/K/V the GEMM wrote, bit for bit."""
import importlib

import numpy as np
import pytest
import torch

import sagetest as st
from oracle import oracle as O

pytestmark = pytest.mark.gpu
sage = importlib.import_module("sota-papers-lab_b200")


def _engine(d=128):
    return sage.SageAttention(torch.cuda.current_stream(), d)


def _ln_inputs(rows, c, seed, xf32=True):
    rng = np.random.default_rng(seed)
    # a residual stream: per-channel offsets, a few large channels, one zero
    # row (which normalises to beta)
    x = rng.normal(size=(rows, c)).astype(np.float32) * 2.0 + rng.normal(size=c).astype(np.float32)
    x[:, ::97] *= 20.0
    x[min(3, rows - 1)] = 0.0
    gamma = (1.0 + 0.2 * rng.normal(size=c)).astype(np.float32)
    beta = (0.1 * rng.normal(size=c)).astype(np.float32)
    if xf32:
        return x, torch.from_numpy(x).cuda(), gamma, beta
    xb = O.f32_to_bf16(x)
    return xb, torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16), gamma, beta


def _run_ln(eng_or_ref, xd, gamma, beta, eps, with_out):
    rows, c = xd.shape
    q8 = torch.zeros(rows, c, dtype=torch.uint8, device="cuda")
    sc = torch.zeros(rows, dtype=torch.float32, device="cuda")
    out = torch.zeros(rows, c, dtype=torch.bfloat16, device="cuda") if with_out else None
    g, b = torch.from_numpy(gamma).cuda(), torch.from_numpy(beta).cuda()
    if eng_or_ref == "ref":
        assert O.ref_layer_norm_fp8(xd, g, b, eps, out, q8, sc, torch.cuda.current_stream().cuda_stream) == 0
    else:
        eng_or_ref.layer_norm_fp8(xd, g, b, eps, q8, sc, out)
    torch.cuda.synchronize()
    return q8.cpu().numpy(), sc.cpu().numpy(), None if out is None else out.view(torch.int16).cpu().numpy()


@pytest.mark.parametrize("c", [256, 768, 1024, 2048])
@pytest.mark.parametrize("xf32", [True, False], ids=["f32", "bf16"])
def test_layer_norm_fp8_bytes_equal_the_reference_kernel(c, xf32):
    if not O.norm_ref_available():
        pytest.skip("the reference's LayerNorm kernels were not built (oracle/_ref)")
    rows = 157  # not a multiple of the 4 rows per block
    _, xd, gamma, beta = _ln_inputs(rows, c, seed=c + xf32, xf32=xf32)
    eng = _engine()
    ours = _run_ln(eng, xd, gamma, beta, 1e-6, True)
    ref = _run_ln("ref", xd, gamma, beta, 1e-6, True)
    assert np.array_equal(ours[1].view(np.uint32), ref[1].view(np.uint32)), "scales"
    assert np.array_equal(ours[0], ref[0]), "q8"
    assert np.array_equal(ours[2], ref[2]), "bf16 out"
    # the zero row normalises to beta
    assert ours[1][3] == np.float32(np.abs(beta).max()) / np.float32(448.0)


@pytest.mark.parametrize("c,xf32", [(512, True), (3072, False), (4096, True), (4096, False)])
def test_layer_norm_fp8_against_the_cpu_restatement(c, xf32):
    # 63 rows: the wide rows' kernel (two warps per row, two rows per block)
    # then has a block whose second row is past the end
    rows = 63
    x, xd, gamma, beta = _ln_inputs(rows, c, seed=7, xf32=xf32)
    eng = _engine()
    q8, sc, _ = _run_ln(eng, xd, gamma, beta, 1e-5, False)
    # the restatement reduces in one-warp order; rows wider than 2048 add two
    # warp sums instead, which moves mean and variance in the last bits
    rq8, rsc, _ = O.layer_norm_fp8(x, gamma, beta, 1e-5)
    np.testing.assert_allclose(sc, rsc, rtol=1e-6)
    # rsqrtf against 1/sqrtf: at most one E4M3 step apart, and rarely
    diff = np.abs(q8.astype(np.int32) - rq8.astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() < 0.01, ((diff > 0).mean(), diff.max())


def test_layer_norm_fp8_arguments_are_checked():
    eng = _engine()
    x = torch.zeros(4, 640, device="cuda")
    g = torch.ones(640, device="cuda")
    with pytest.raises(sage.SageError):
        eng.layer_norm_fp8(x, g, g, 1e-5, torch.zeros(4, 640, dtype=torch.uint8, device="cuda"),
                           torch.zeros(4, device="cuda"))


def _quant_weights(w):
    """Per-output-channel E4M3 weights (amax / 448), as the reference's FP8
    weight preparation stores them: returns (w8 bytes, scales)."""
    amax = np.abs(w).max(axis=1)
    scale = np.where(amax > 0, amax / 448.0, 1.0).astype(np.float32)
    w8 = np.stack([O.f32_to_e4m3_array(w[i] / scale[i]) for i in range(w.shape[0])])
    return w8, scale


FP8_CASES = {
    # name: batch, tokens, hidden, heads, kv, d, rope
    "vit_d64": (2, 137, 1024, 16, 16, 64, None),
    "llama_d128_rope": (1, 300, 512, 4, 2, 128, "llama"),
}


@pytest.mark.parametrize("pairs", [False, True], ids=["1sm", "2sm"])
@pytest.mark.parametrize("name", list(FP8_CASES))
def test_fp8_qkv_gemm_matches_f64_oracle(name, pairs):
    b, t, hidden, hq, hkv, d, rk = FP8_CASES[name]
    m, n = b * t, (hq + 2 * hkv) * d
    rng = np.random.default_rng(11)
    x, xd, gamma, beta = _ln_inputs(m, hidden, seed=3)
    eng = _engine(d)
    eng.gemm_pairs(pairs)
    q8d = torch.zeros(m, hidden, dtype=torch.uint8, device="cuda")
    xsd = torch.zeros(m, device="cuda")
    eng.layer_norm_fp8(xd, torch.from_numpy(gamma).cuda(), torch.from_numpy(beta).cuda(), 1e-6, q8d, xsd)
    w8, ws = _quant_weights(rng.normal(0, 0.02, size=(n, hidden)).astype(np.float32))
    bias = O.f32_to_bf16(rng.normal(0, 0.1, size=n))
    rope, half, frame = None, 0, 1
    if rk == "llama":
        rope, half, frame = sage.rope_table_1d(500000.0, d, t), d // 2, t
    q = torch.empty(b, t, hq, d, dtype=torch.bfloat16, device="cuda")
    k = torch.empty(b, t, hkv, d, dtype=torch.bfloat16, device="cuda")
    v = torch.empty(b, t, hkv, d, dtype=torch.bfloat16, device="cuda")
    eng.qkv_gemm_fp8(q8d, xsd, torch.from_numpy(w8).cuda(), torch.from_numpy(ws).cuda(),
                     torch.from_numpy(bias.view(np.int16)).cuda().view(torch.bfloat16),
                     None if rope is None else torch.from_numpy(rope).cuda(), q, k, v, batch=b, tokens=t, heads=hq,
                     kv_heads=hkv, rope_half=half, frame_len=frame)
    torch.cuda.synchronize()
    assert eng.engine_status() == 0
    want = O.qkv_reference_fp8(q8d.cpu().numpy(), xsd.cpu().numpy(), w8, ws, bias, rope, tokens=t, hq=hq, hkv=hkv,
                               d=d, rope_half=half, frame_len=frame)
    for got, ref, what in zip((q, k, v), want, "qkv"):
        g = O.bf16_to_f32(got.view(torch.int16).cpu().numpy().view(np.uint16)).reshape(ref.shape)
        e = O.errors(g, ref)
        print(name, what, e)
        assert e["rel_l2"] < 5e-3 and e["max_abs"] < 0.05 * max(1.0, e["ref_max"]), (what, e)


def test_fp8_chain_feeds_the_quantiser_bit_exactly():
    """LN -> FP8 GEMM -> prepare: the quantised workspace equals the oracle
    quantiser applied to the bf16 Q/K/V the FP8 GEMM wrote."""
    b, t, hidden, hq, hkv, d = 1, 256, 768, 4, 2, 128
    m, n = b * t, (hq + 2 * hkv) * d
    rng = np.random.default_rng(21)
    _, xd, gamma, beta = _ln_inputs(m, hidden, seed=5, xf32=False)
    eng = _engine(d)
    q8d = torch.zeros(m, hidden, dtype=torch.uint8, device="cuda")
    xsd = torch.zeros(m, device="cuda")
    eng.layer_norm_fp8(xd, torch.from_numpy(gamma).cuda(), torch.from_numpy(beta).cuda(), 1e-6, q8d, xsd)
    w8, ws = _quant_weights(rng.normal(0, 0.02, size=(n, hidden)).astype(np.float32))
    q = torch.empty(b, t, hq, d, dtype=torch.bfloat16, device="cuda")
    k = torch.empty(b, t, hkv, d, dtype=torch.bfloat16, device="cuda")
    v = torch.empty(b, t, hkv, d, dtype=torch.bfloat16, device="cuda")
    rope = sage.rope_table_1d(500000.0, d, t)
    eng.qkv_gemm_fp8(q8d, xsd, torch.from_numpy(w8).cuda(), torch.from_numpy(ws).cuda(), None,
                     torch.from_numpy(rope).cuda(), q, k, v, batch=b, tokens=t, heads=hq, kv_heads=hkv, rope_half=64,
                     frame_len=t)
    c = st.Case(batch=b, heads=hq, kv_heads=hkv, tokens=t, d=d, causal=True, packed=False)
    ws_ = eng.workspace(sage.Shape(b, hq, t, hkv, True))
    sq, skv = sage.Strides.bthd(t, hq, d), sage.Strides.bthd(t, hkv, d)
    eng.prepare(ws_, sage.Tensor(q, sq), sage.Tensor(k, skv), sage.Tensor(v, skv))
    got = st.export_quant(eng, ws_, c)
    torch.cuda.synchronize()
    qb, kb, vb = (a.view(torch.int16).cpu().numpy().view(np.uint16) for a in (q, k, v))
    want = O.prepare(qb, kb, vb, st.geom(c))
    st.assert_quant_equal(got, want, kbias=False, what="fp8 chain")
    ws_.close()


# ---------------------------------------------------------------- the output side: attention -> FP8 -> proj

def _bf16_dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda().view(torch.bfloat16)


@pytest.mark.parametrize("c,ld", [(1024, 1024), (2048, 2056), (4096, 4096)])
def test_rows_fp8_bytes_equal_the_reference_kernel(c, ld):
    if not O.norm_ref_available():
        pytest.skip("the reference's LayerNorm kernels were not built (oracle/_ref)")
    rows = 77
    rng = np.random.default_rng(c)
    y = O.f32_to_bf16(rng.normal(size=(rows, ld)) * 3)
    y[5] = 0
    tok = rng.uniform(0.5, 2, size=rows).astype(np.float32)
    yd, td = _bf16_dev(y), torch.from_numpy(tok).cuda()
    eng = _engine()
    for t in (None, td):
        ours = (torch.zeros(rows, c, dtype=torch.uint8, device="cuda"), torch.zeros(rows, device="cuda"))
        ref = (torch.zeros(rows, c, dtype=torch.uint8, device="cuda"), torch.zeros(rows, device="cuda"))
        eng.rows_fp8(yd, ours[0], ours[1], c=c, tok=t)
        assert O.ref_rows_fp8(yd, c, t, None, None, ref[0], ref[1], torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(ours[0], ref[0]) and torch.equal(ours[1], ref[1])
        # and the CPU restatement, exactly (no approximate functions on this path)
        q8, sc = O.rows_fp8(y, c, tok=None if t is None else tok)
        assert np.array_equal(ours[0].cpu().numpy(), q8) and np.array_equal(ours[1].cpu().numpy(), sc)
        assert sc[5] == 1.0


@pytest.mark.parametrize("pairs", [False, True], ids=["1sm", "2sm"])
def test_linear_fp8_matches_f64_oracle_and_defers_scales(pairs):
    m, n, k = 300, 1024, 1024
    rng = np.random.default_rng(4)
    x8 = O.f32_to_e4m3_array(rng.normal(size=(m, k)) * 40)
    w8, ws = _quant_weights(rng.normal(0, 0.02, size=(n, k)).astype(np.float32))
    xs = rng.uniform(0.005, 0.02, size=m).astype(np.float32)
    bias = O.f32_to_bf16(rng.normal(0, 0.1, size=n))
    eng = _engine()
    eng.gemm_pairs(pairs)
    x8d, w8d = torch.from_numpy(x8).cuda(), torch.from_numpy(w8).cuda()
    y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    eng.linear_fp8(x8d, torch.from_numpy(xs).cuda(), w8d, torch.from_numpy(ws).cuda(), _bf16_dev(bias), y)
    yd = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    eng.linear_fp8(x8d, None, w8d, None, None, yd)
    torch.cuda.synchronize()
    assert eng.engine_status() == 0
    want, _, _ = O.qkv_reference_fp8(x8, xs, w8, ws, bias, None, tokens=m, hq=n // 128, hkv=0, d=128)
    e = O.errors(O.bf16_to_f32(y.view(torch.int16).cpu().numpy().view(np.uint16)), want.reshape(m, n))
    assert e["rel_l2"] < 5e-3, e
    ones_m, ones_n = np.ones(m, np.float32), np.ones(n, np.float32)
    raw, _, _ = O.qkv_reference_fp8(x8, ones_m, w8, ones_n, None, None, tokens=m, hq=n // 128, hkv=0, d=128)
    e = O.errors(O.bf16_to_f32(yd.view(torch.int16).cpu().numpy().view(np.uint16)), raw.reshape(m, n))
    assert e["rel_l2"] < 5e-3, e
    with pytest.raises(sage.SageError):  # one scale without the other
        eng.linear_fp8(x8d, torch.from_numpy(xs).cuda(), w8d, None, None, yd)


def test_attention_output_to_fp8_proj():
    """The reference's FP8 block after attention: the bf16 attention output
    [T][H*D] -> per-token E4M3 -> FP8 proj GEMM (deferred weight scales), then
    y * tok * chan, against the f64 oracle on the quantised operands."""
    c = st.Case(batch=1, heads=8, kv_heads=8, tokens=384, d=128, causal=False, packed=False, seed=3)
    x = st.make_inputs(c)
    run = st.run_ours(c, x, export=False)
    dim = c.heads * c.d
    o_bits = O.f32_to_bf16(run.out.reshape(c.tokens, dim))
    eng = _engine()
    o8 = torch.zeros(c.tokens, dim, dtype=torch.uint8, device="cuda")
    osc = torch.zeros(c.tokens, device="cuda")
    eng.rows_fp8(_bf16_dev(o_bits), o8, osc)
    rng = np.random.default_rng(8)
    w8, ws = _quant_weights(rng.normal(0, 0.02, size=(dim, dim)).astype(np.float32))
    y = torch.empty(c.tokens, dim, dtype=torch.bfloat16, device="cuda")
    eng.linear_fp8(o8, osc, torch.from_numpy(w8).cuda(), torch.from_numpy(ws).cuda(), None, y)
    torch.cuda.synchronize()
    q8, sc = O.rows_fp8(o_bits)
    assert np.array_equal(o8.cpu().numpy(), q8) and np.array_equal(osc.cpu().numpy(), sc)
    want, _, _ = O.qkv_reference_fp8(q8, sc, w8, ws, None, None, tokens=c.tokens, hq=dim // 128, hkv=0, d=128)
    e = O.errors(O.bf16_to_f32(y.view(torch.int16).cpu().numpy().view(np.uint16)), want.reshape(c.tokens, dim))
    assert e["rel_l2"] < 5e-3, e
    # and the FP8 path against the bf16 projection of the unquantised output
    exact = O.bf16_to_f32(o_bits).astype(np.float64) @ (O.e4m3_to_f32(w8) * ws[:, None]).T.astype(np.float64)
    e = O.errors(O.bf16_to_f32(y.view(torch.int16).cpu().numpy().view(np.uint16)), exact)
    assert e["cos"] > 0.999, e
