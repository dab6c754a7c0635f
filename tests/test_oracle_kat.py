"""Known-answer tests of the CPU oracle: the reference's own CPU tests for
this path (platform/spl-nn/src/sage/tests.rs:25-232), restated against the
C restatement in oracle/, plus independent cross-checks (torch's E4M3 and
bf16 casts)."""
import math

import numpy as np
import pytest
import torch


def test_e4m3_codes_round_trip(oracle):
    # tests.rs:25-37
    for b in range(256):
        x = oracle.lib().or_e4m3_to_f32(b)
        if b & 0x7F == 0x7F:
            assert math.isnan(x)
            continue
        assert oracle.f32_to_e4m3(x) == b, f"code {b:#04x} = {x}"
    assert oracle.lib().or_e4m3_to_f32(0x7E) == 448.0
    assert oracle.lib().or_e4m3_to_f32(0x01) == 2.0 ** -9
    assert oracle.lib().or_e4m3_to_f32(0x38) == 1.0


def test_e4m3_rounds_to_nearest_even_and_saturates(oracle):
    # tests.rs:40-55
    dec = oracle.lib().or_e4m3_to_f32
    enc = oracle.f32_to_e4m3
    assert dec(enc(1.0625)) == 1.0
    assert dec(enc(1.1875)) == 1.25
    assert dec(enc(-3.3)) == -3.25
    assert enc(1000.0) == 0x7E
    assert enc(-1000.0) == 0xFE
    assert enc(2.0 ** -10) == 0
    assert dec(enc(3.0 * 2.0 ** -10)) == 2.0 ** -8
    assert dec(enc(15.9)) == 16.0
    assert enc(float("nan")) == 0x7F


def test_e4m3_matches_torch_in_range(oracle):
    # Independent check: torch's float8_e4m3fn cast is RNE inside the finite range.
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.normal(0, 30, 20000), rng.normal(0, 0.01, 5000), rng.uniform(-447, 447, 5000)])
    x = x.astype(np.float32)
    ours = np.array([oracle.f32_to_e4m3(float(v)) for v in x], np.uint8)
    theirs = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert (ours == theirs).all()


def test_bf16_rounds_to_nearest_even(oracle):
    # tests.rs:58-66
    enc = oracle.lib().or_f32_to_bf16
    dec = oracle.lib().or_bf16_to_f32
    assert enc(1.0) == 0x3F80
    assert dec(enc(1.0 + 1.0 / 256.0)) == 1.0
    assert dec(enc(1.0 + 3.0 / 256.0)) == 1.0 + 4.0 / 256.0
    assert dec(enc(-2.5)) == -2.5
    x = np.random.default_rng(1).normal(0, 10, 100000).astype(np.float32)
    assert (oracle.f32_to_bf16(x) == torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)).all()


def test_v_permutation_matches_the_p_fragment(oracle):
    # tests.rs:69-83
    seen = [False] * 16
    for t in range(4):
        for e, key in enumerate([2 * t, 2 * t + 1, 8 + 2 * t, 9 + 2 * t]):
            assert oracle.vpos(key) == 4 * t + e
            seen[oracle.vpos(key)] = True
    assert all(seen)


def _vggt_layout(oracle, frames, dense_frames=0):
    return oracle.Layout(frames=frames, special=17, grid_h=21, grid_w=32, dense_frames=dense_frames)


def _geom(oracle, tokens, merge=1, layout=None, d=64, heads=1):
    s = oracle.bthd_strides(tokens, heads, d)
    return oracle.make_geom(1, heads, heads, tokens, d, s, s, s, merge=merge, layout=layout)


def test_dense_first_frame_keeps_its_keys(oracle):
    # tests.rs:96-133
    lay = _vggt_layout(oracle, 3, dense_frames=1)
    g = _geom(oracle, 3 * 689, merge=4, layout=lay)
    assert g.tk == 689 + 2 * 65
    for j in range(689):
        assert oracle.members(g, j) == [j]
    for j in range(689, 689 + 17):
        assert oracle.members(g, j) == [j]
    assert oracle.members(g, 689 + 17) == [706, 707, 708, 709, 738, 739, 740, 741, 770, 771, 772, 773, 802, 803,
                                          804, 805]
    seen = [False] * (3 * 689)
    for j in range(g.tk):
        for t in oracle.members(g, j):
            assert not seen[t], f"token {t} pooled twice"
            seen[t] = True
    assert all(seen)


def test_vggt_merge_geometry(oracle):
    # tests.rs:136-172
    lay = _vggt_layout(oracle, 200)
    assert lay.tokens_per_frame() == 689
    dense = _geom(oracle, 200 * 689)
    assert (dense.tq_pad, dense.tk, dense.tk_pad) == (137856, 137800, 137856)
    m2 = _geom(oracle, 200 * 689, merge=2, layout=lay)
    assert m2.tk == 200 * (17 + 11 * 16)
    m4 = _geom(oracle, 200 * 689, merge=4, layout=lay)
    assert m4.tk == 200 * (17 + 6 * 8)
    for g, s in [(m2, 2), (m4, 4)]:
        per = lay.merged_per_frame(s)
        hit = [0] * 689
        for j in range(per, 2 * per):
            for t in oracle.members(g, j):
                hit[t - 689] += 1
        assert all(h == 1 for h in hit)
        assert oracle.members(g, per + 3) == [689 + 3]
    assert len(oracle.members(m4, 17)) == 16
    assert len(oracle.members(m4, 17 + 5 * 8)) == 4
    assert len(oracle.members(m2, 17 + 10 * 16)) == 2


def test_merged_attention_equals_dense_on_uniform_cells(oracle):
    # tests.rs:193-232, on the f64 oracle attention
    lay = oracle.Layout(frames=2, special=3, grid_h=5, grid_w=7)
    tokens = 2 * lay.tokens_per_frame()
    d = 16
    for stride in (2, 4):
        g = _geom(oracle, tokens, merge=stride, layout=lay, d=d)
        rng = oracle.Rng(7)
        cell_k = rng.normals(g.tk * d).reshape(g.tk, d)
        cell_v = rng.normals(g.tk * d).reshape(g.tk, d)
        k = np.zeros((tokens, d), np.float32)
        v = np.zeros((tokens, d), np.float32)
        for j in range(g.tk):
            for t in oracle.members(g, j):
                k[t] = cell_k[j]
                v[t] = cell_v[j]
        q = (2.0 * rng.normals(tokens * d)).reshape(tokens, d).astype(np.float32)
        dense = np.zeros((tokens, d), np.float32)
        oracle.lib().or_attention_f64(oracle._p(q), oracle._p(k), oracle._p(v), None, tokens, tokens, d, 0.25, 0, 0,
                                      oracle._p(dense))
        km = np.ascontiguousarray(cell_k, np.float32)
        vm = np.ascontiguousarray(cell_v, np.float32)
        bias = np.array([math.log2(len(oracle.members(g, j))) for j in range(g.tk)], np.float32)
        merged = np.zeros((tokens, d), np.float32)
        oracle.lib().or_attention_f64(oracle._p(q), oracle._p(km), oracle._p(vm), oracle._p(bias), tokens, g.tk, d,
                                      0.25, 0, 0, oracle._p(merged))
        e = oracle.errors(merged, dense)
        assert e["max_abs"] < 1e-5, (stride, e)


def test_f64_attention_matches_torch_sdpa(oracle):
    # Independent check of the f64 oracle (and its causal / GQA extensions)
    # against torch's fp32 SDPA on the CPU.
    b, hq, hkv, t, d = 1, 4, 2, 70, 32
    rng = np.random.default_rng(3)
    q = oracle.f32_to_bf16(rng.normal(size=(b, t, hq, d)).astype(np.float32))
    k = oracle.f32_to_bf16(rng.normal(size=(b, t, hkv, d)).astype(np.float32))
    v = oracle.f32_to_bf16(rng.normal(size=(b, t, hkv, d)).astype(np.float32))
    g = oracle.make_geom(b, hq, hkv, t, d, oracle.bthd_strides(t, hq, d), oracle.bthd_strides(t, hkv, d),
                         oracle.bthd_strides(t, hkv, d))
    for causal in (False, True):
        ours = oracle.attention_bthd(q, k, v, g, causal=causal, nthreads=2)
        tq = torch.from_numpy(oracle.bf16_to_f32(q)).permute(0, 2, 1, 3)
        tk = torch.from_numpy(oracle.bf16_to_f32(k)).permute(0, 2, 1, 3).repeat_interleave(hq // hkv, dim=1)
        tv = torch.from_numpy(oracle.bf16_to_f32(v)).permute(0, 2, 1, 3).repeat_interleave(hq // hkv, dim=1)
        ref = torch.nn.functional.scaled_dot_product_attention(tq, tk, tv, is_causal=causal).permute(0, 2, 1, 3)
        e = oracle.errors(ours, ref.numpy())
        assert e["max_abs"] < 1e-5, (causal, e)


def test_rng_is_splitmix64(oracle):
    # reference.rs:235-241: the first outputs of seed 0 (published SplitMix64 vectors).
    r = oracle.Rng(0)
    assert [r.next_u64() for _ in range(3)] == [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F]
