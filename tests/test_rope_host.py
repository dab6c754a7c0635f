"""CPU tests of the RoPE tables the QKV epilogue reads, after the
reference's own known-answer tests (platform/spl-nn/src/qkv.rs:376-452):
the channel-to-pair layout, the VGGT and DINOv3 table formulas, the 1-D
(Llama) table the library builds, and a rotation by the f64 prologue
restatement that keeps pair norms and leaves V and special tokens alone."""
import math

import numpy as np
import pytest


def test_pair_layout(sage):
    # qkv.rs:378-392
    L = sage.RopeLayout
    v, d = L.VGGT, L.DINOV3
    assert (L.pair(v, 0), L.pair(v, 16), L.pair(v, 15)) == (0, 0, 15)
    assert (L.pair(v, 32), L.pair(v, 48), L.pair(v, 63)) == (16, 16, 31)
    assert (L.pair(d, 0), L.pair(d, 32), L.pair(d, 31), L.pair(d, 63)) == (0, 0, 31, 31)
    for half, dim in ((v, 64), (d, 64), (L.one_d(128), 128), (L.one_d(64), 64)):
        for c in range(dim):
            assert L.pair(half, c) == L.pair(half, c ^ half), (half, c)
            assert L.pair(half, c) < dim // 2


def test_vggt_table_matches_its_formula(sage):
    # qkv.rs:395-412: 2 special tokens, a 3 x 4 grid
    t = sage.RopeTable.vggt(3, 4, 2, 100.0)
    assert t.frame_len == 14 and t.cos_sin.shape == (14, 32, 2) and t.half == 16
    assert tuple(t.cos_sin[1, 5]) == (1.0, 0.0)  # special tokens do not rotate
    row = t.cos_sin[9]  # token 2 + 1*4 + 3: patch (y=1, x=3), positions (2, 4)
    a = 2.0 * 100.0 ** (-3.0 / 16.0)
    assert abs(row[3][0] - math.cos(a)) < 1e-7 and abs(row[3][1] - math.sin(a)) < 1e-7
    a = 4.0 * 100.0 ** (-5.0 / 16.0)
    assert abs(row[16 + 5][1] - math.sin(a)) < 1e-7


def test_dinov3_table_matches_its_formula(sage):
    # qkv.rs:414-424
    t = sage.RopeTable.dinov3(2, 2, 1, 100.0)
    assert t.half == 32
    row = t.cos_sin[2]  # patch (0, 1): coordinates (-0.5, 0.5)
    a = 2.0 * math.pi * -0.5
    assert abs(row[0][1] - math.sin(a)) < 1e-7
    a = 2.0 * math.pi * 0.5 / 100.0 ** (2.0 / 16.0)
    assert abs(row[18][0] - math.cos(a)) < 1e-7


@pytest.mark.parametrize("d", [64, 128])
def test_one_d_table_matches_its_formula(sage, d):
    t = sage.RopeTable.one_d(500000.0, d, 300)
    assert t.cos_sin.shape == (300, d // 2, 2) and t.half == d // 2
    pos = np.arange(300, dtype=np.float64)[:, None]
    ang = pos * 500000.0 ** (-np.arange(d // 2, dtype=np.float64) / (d // 2))
    assert np.array_equal(t.cos_sin[..., 0], np.cos(ang).astype(np.float32))
    assert np.array_equal(t.cos_sin[..., 1], np.sin(ang).astype(np.float32))
    assert np.all(t.cos_sin[0] == np.array([1.0, 0.0], np.float32))
    with pytest.raises(sage.SageError):
        sage.rope_table_1d(500000.0, 96, 4)
    with pytest.raises(sage.SageError):
        sage.rope_table_1d(1.0, 64, 4)


def test_rotation_keeps_pair_norms(sage, oracle):
    # qkv.rs:426-452, through the f64 GEMM + prologue restatement with an
    # identity weight, so the prologue sees the bf16 inputs themselves
    tokens, heads, d = 3, 2, 64
    ld = 3 * heads * d
    y = np.array([((i * 37 % 101) - 50.0) / 25.0 for i in range(tokens * ld)], np.float32).reshape(tokens, ld)
    x = oracle.f32_to_bf16(y)
    w = oracle.f32_to_bf16(np.eye(ld, dtype=np.float32))
    rope = sage.RopeTable.vggt(1, 2, 1, 100.0)
    kw = dict(tokens=tokens, hq=heads, hkv=heads, d=d, nthreads=1)
    q0, _, v0 = oracle.qkv_reference(x, w, None, None, **kw)
    q1, _, v1 = oracle.qkv_reference(x, w, None, rope.cos_sin, rope_half=rope.half, frame_len=rope.frame_len, **kw)
    assert np.array_equal(v0, v1)  # V is never rotated
    assert np.array_equal(q0[0], q1[0])  # token 0 is special: unrotated
    assert not np.array_equal(q0[1:], q1[1:])
    for c in range(d):
        if c & rope.half:
            continue
        n0 = q0[..., c].astype(np.float64) ** 2 + q0[..., c ^ rope.half].astype(np.float64) ** 2
        n1 = q1[..., c].astype(np.float64) ** 2 + q1[..., c ^ rope.half].astype(np.float64) ** 2
        # the rotated pair is rounded to bf16 (8 significant bits) once more
        assert np.all(np.abs(n0 - n1) <= 2 * 2.0 ** -8 * np.maximum(n0, 1.0)), c

