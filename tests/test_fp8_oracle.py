"""CPU checks of the oracle's FP8-path restatements (no GPU): LN -> per-token
E4M3 (norm.cu:37-137) against float64 numpy LayerNorm, and the FP8 QKV
reference (Gemm::linear_fp8 + qkv::reference with token / channel scales)
against a numpy matmul of the decoded E4M3 operands."""
import numpy as np
import pytest

from oracle import oracle as O


@pytest.mark.parametrize("c", [256, 1024, 4096])
@pytest.mark.parametrize("xf32", [True, False], ids=["f32", "bf16"])
def test_layer_norm_fp8_oracle_against_numpy(c, xf32):
    rng = np.random.default_rng(c)
    rows = 9
    x = (rng.normal(size=(rows, c)) * 3 + rng.normal(size=c)).astype(np.float32)
    x[4] = 0.0
    gamma = (1 + 0.3 * rng.normal(size=c)).astype(np.float32)
    beta = (0.2 * rng.normal(size=c)).astype(np.float32)
    xin = x if xf32 else O.f32_to_bf16(x)
    xv = x.astype(np.float64) if xf32 else O.bf16_to_f32(xin).astype(np.float64)
    q8, sc, out = O.layer_norm_fp8(xin, gamma, beta, 1e-5, with_out=True)
    mean = xv.mean(1, keepdims=True)
    y = (xv - mean) / np.sqrt(((xv - mean) ** 2).mean(1, keepdims=True) + 1e-5) * gamma + beta
    amax = np.abs(y).max(1)
    np.testing.assert_allclose(sc, np.where(amax > 0, amax / 448, 1.0), rtol=1e-5)
    assert sc[4] == np.float32(np.abs(beta).max() / 448) or np.abs(beta).max() == 0
    deq = O.e4m3_to_f32(q8).astype(np.float64) * sc[:, None]
    # E4M3: 3 mantissa bits, half a step of relative error (subnormals: 2^-10 of the scale)
    tol = np.maximum(np.abs(y) * 2.0 ** -4, sc[:, None] * 2.0 ** -9) * 1.01
    assert np.all(np.abs(deq - y) <= tol)
    np.testing.assert_allclose(O.bf16_to_f32(out), y, rtol=2 ** -8, atol=1e-6)


def test_fp8_qkv_oracle_against_numpy():
    rng = np.random.default_rng(3)
    m, k, hq, hkv, d = 5, 64, 2, 1, 64
    n = (hq + 2 * hkv) * d
    x8 = rng.integers(0, 256, size=(m, k), dtype=np.uint8)
    x8[(x8 & 0x7f) == 0x7f] = 0x10  # no NaN codes
    w8 = rng.integers(0, 256, size=(n, k), dtype=np.uint8)
    w8[(w8 & 0x7f) == 0x7f] = 0x20
    xs = rng.uniform(0.01, 0.1, size=m).astype(np.float32)
    wsc = rng.uniform(0.001, 0.01, size=n).astype(np.float32)
    bias = O.f32_to_bf16(rng.normal(size=n))
    q, kk, v = O.qkv_reference_fp8(x8, xs, w8, wsc, bias, None, tokens=m, hq=hq, hkv=hkv, d=d)
    y = (O.e4m3_to_f32(x8).astype(np.float64) @ O.e4m3_to_f32(w8).astype(np.float64).T) * xs[:, None] * wsc[None, :]
    y += O.bf16_to_f32(bias)[None, :]
    np.testing.assert_allclose(q.reshape(m, -1), y[:, :hq * d], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(kk.reshape(m, -1), y[:, hq * d:(hq + hkv) * d], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(v.reshape(m, -1), y[:, (hq + hkv) * d:], rtol=1e-6, atol=1e-6)


def test_rows_fp8_oracle_against_numpy():
    rng = np.random.default_rng(5)
    y = O.f32_to_bf16(rng.normal(size=(6, 2056)) * 5)
    y[2] = 0
    tok = rng.uniform(0.5, 2, size=6).astype(np.float32)
    q8, sc = O.rows_fp8(y, 2048, tok=tok)
    v = O.bf16_to_f32(y)[:, :2048].astype(np.float64) * tok[:, None]
    amax = np.abs(v).max(1)
    np.testing.assert_allclose(sc, np.where(amax > 0, amax / 448, 1.0), rtol=1e-6)
    deq = O.e4m3_to_f32(q8) * sc[:, None]
    assert np.all(np.abs(deq - v) <= np.maximum(np.abs(v) * 2.0 ** -4, sc[:, None] * 2.0 ** -9) * 1.01)
    assert sc[2] == 1.0 and not q8[2].any()
