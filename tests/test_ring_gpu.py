"""Context-parallel (ring) attention on one GPU: all ranks of a P-rank ring
emulated in one process (statistics combined and K/V handed over by copies,
in the multi-GPU order), and the real RingAttention at P = 1.  The result
must equal single-GPU causal attention within the attention gate, and the
f64 oracle within the reference's gate."""
from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

import sagetest as st
from oracle import oracle as O

sage = st.sage
ring = importlib.import_module("sota-papers-lab_b200.ring")

pytestmark = pytest.mark.gpu


def _inputs(c: st.Case):
    x = st.make_inputs(c)
    keep, (tq, tk, tv) = st.to_device(c, x)
    b, t = c.batch, c.tokens
    q = tq.data.view(b, t, c.heads, c.d)
    k = tk.data.view(b, t, c.kv_heads, c.d)
    v = tv.data.view(b, t, c.kv_heads, c.d)
    return x, q, k, v


def _f64_rows(c, x, rows):
    return O.attention_bthd(x.q, x.k, x.v, st.geom(c), causal=True, rows=rows)[:, rows[0]:rows[1]]


@pytest.mark.parametrize("world,d,heads,kv_heads,tokens", [(2, 128, 4, 2, 2048), (4, 64, 4, 4, 2048),
                                                           (4, 128, 8, 2, 4096), (8, 128, 4, 1, 4096)])
def test_emulated_ring_matches_single_gpu_causal(world, d, heads, kv_heads, tokens):
    c = st.Case(batch=1, heads=heads, kv_heads=kv_heads, tokens=tokens, d=d, causal=True, packed=False, seed=17)
    x, q, k, v = _inputs(c)
    single = st.run_ours(c, x, export=False).out
    eng = st.engine(c)
    T = tokens // world
    rings = [ring.RingAttention(eng, 1, heads, kv_heads, T, r, world, d) for r in range(world)]
    sq, skv = sage.Strides.bthd(T, heads, d), sage.Strides.bthd(T, kv_heads, d)
    shards = [(ring.shard_zigzag(q, r, world), ring.shard_zigzag(k, r, world), ring.shard_zigzag(v, r, world))
              for r in range(world)]
    outs = [torch.zeros(1, T, heads, d, dtype=torch.bfloat16, device="cuda") for _ in range(world)]
    ring.emulate_ring(rings, [sage.Tensor(a, sq) for a, _, _ in shards], [sage.Tensor(b, skv) for _, b, _ in shards],
                      [sage.Tensor(cc, skv) for _, _, cc in shards], [sage.Tensor(o, sq) for o in outs])
    torch.cuda.synchronize()
    for rg in rings:
        assert eng.status(rg.ws) == 0
    full = ring.unshard_zigzag(outs, world, dim=1)
    ours = O.bf16_to_f32(full.view(torch.int16).cpu().numpy().view(np.uint16)).reshape(single.shape)
    e = O.errors(ours, single)
    assert st.attention_gate(e), e
    # the exact reference on rows of the first, a middle and the last chunk
    for r0 in (0, tokens // 2 - 64, tokens - 128):
        rows = (r0, r0 + 128)
        ef = O.errors(ours[:, rows[0]:rows[1]], _f64_rows(c, x, rows))
        assert st.reference_gate(ef), (rows, ef)
    for rg in rings:
        rg.close()


def test_ring_attention_single_rank_path():
    """RingAttention.forward itself (the code the multi-GPU run executes) at
    P = 1: one GPU, the sequence as two zig-zag chunks."""
    c = st.Case(batch=2, heads=8, kv_heads=2, tokens=1024, d=128, causal=True, packed=False, seed=23)
    x, q, k, v = _inputs(c)
    single = st.run_ours(c, x, export=False).out
    eng = st.engine(c)
    rg = ring.RingAttention(eng, 2, 8, 2, 1024, 0, 1, 128)
    out = torch.zeros(2, 1024, 8, 128, dtype=torch.bfloat16, device="cuda")
    sq, skv = sage.Strides.bthd(1024, 8, 128), sage.Strides.bthd(1024, 2, 128)
    rg.forward(sage.Tensor(q.contiguous(), sq), sage.Tensor(k.contiguous(), skv), sage.Tensor(v.contiguous(), skv),
               sage.Tensor(out, sq))
    torch.cuda.synchronize()
    assert eng.status(rg.ws) == 0
    ours = O.bf16_to_f32(out.view(torch.int16).cpu().numpy().view(np.uint16)).reshape(single.shape)
    e = O.errors(ours, single)
    assert st.attention_gate(e), e
    rg.close()


def test_pairwise_segments_equal_one_launch_per_step():
    """The ring's one launch per step (contiguous chunk pairs together, the
    first step writing the accumulator) against one launch per chunk pair
    merged into a zeroed accumulator: the same attention within the gate."""
    world, d, heads, kv_heads, tokens = 4, 128, 4, 2, 4096
    c = st.Case(batch=1, heads=heads, kv_heads=kv_heads, tokens=tokens, d=d, causal=True, packed=False, seed=31)
    x, q, k, v = _inputs(c)
    eng = st.engine(c)
    T = tokens // world
    rings = [ring.RingAttention(eng, 1, heads, kv_heads, T, r, world, d) for r in range(world)]
    sq, skv = sage.Strides.bthd(T, heads, d), sage.Strides.bthd(T, kv_heads, d)
    shards = [(ring.shard_zigzag(q, r, world), ring.shard_zigzag(k, r, world), ring.shard_zigzag(v, r, world))
              for r in range(world)]
    outs = [torch.zeros(1, T, heads, d, dtype=torch.bfloat16, device="cuda") for _ in range(world)]
    ring.emulate_ring(rings, [sage.Tensor(a, sq) for a, _, _ in shards], [sage.Tensor(b, skv) for _, b, _ in shards],
                      [sage.Tensor(cc, skv) for _, _, cc in shards], [sage.Tensor(o, sq) for o in outs])
    torch.cuda.synchronize()
    for i, rg in enumerate(rings):
        acc1, lse1 = rg.acc.clone(), rg.lse.clone()
        rg.acc.zero_()
        rg.lse.fill_(float("-inf"))
        for src, pairs in ring.ring_schedule(i, world):
            for pr in pairs:
                eng.cp_attend(rg.ws, rings[src].kv[0], pr.q_local * rg.C, rg.C, pr.k_local * rg.C, rg.C, pr.causal,
                              rg.acc, rg.lse)
        torch.cuda.synchronize()
        assert eng.status(rg.ws) == 0
        # P is rounded to E4M3 against the running row maximum, which a
        # longer key segment reaches at other blocks: attention tolerance for
        # the output; the denominators are fp32 sums of the unrounded P
        e = O.errors(rg.acc.cpu().numpy().astype(np.float64), acc1.cpu().numpy().astype(np.float64))
        assert st.attention_gate(e), e
        assert torch.allclose(rg.lse, lse1, rtol=1e-5, atol=1e-3), (rg.lse - lse1).abs().max()
    for rg in rings:
        rg.close()


def test_reserved_sms_give_the_same_result():
    """Attention on all but n SMs (fewer persistent CTAs, more tiles each)
    is bit-identical to attention on all SMs."""
    c = st.Case(batch=2, heads=8, kv_heads=2, tokens=2048, d=128, causal=True, packed=False, seed=5)
    x, q, k, v = _inputs(c)
    eng = st.engine(c)
    ws = eng.workspace(sage.Shape(2, 8, 2048, 2, True))
    sq, skv = sage.Strides.bthd(2048, 8, 128), sage.Strides.bthd(2048, 2, 128)
    tq, tk, tv = sage.Tensor(q.contiguous(), sq), sage.Tensor(k.contiguous(), skv), sage.Tensor(v.contiguous(), skv)
    outs = []
    for n in (0, 8, 100):
        eng.reserve_sms(n)
        o = torch.zeros(2, 2048, 8, 128, dtype=torch.bfloat16, device="cuda")
        eng.forward(ws, tq, tk, tv, sage.Tensor(o, sq))
        outs.append(o)
    eng.reserve_sms(0)
    torch.cuda.synchronize()
    assert eng.status(ws) == 0
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    with pytest.raises(sage.SageError):
        eng.reserve_sms(-1)
    ws.close()


def test_segment_arguments_are_checked():
    c = st.Case(batch=1, heads=2, kv_heads=2, tokens=512, d=128, causal=True, packed=False)
    eng = st.engine(c)
    rg = ring.RingAttention(eng, 1, 2, 2, 512, 0, 1, 128)
    acc = torch.zeros(1, 512, 2, 128, device="cuda")
    lse = torch.zeros(1, 2, 512, device="cuda")
    with pytest.raises(sage.SageError):  # not prepared
        eng.cp_attend(rg.ws, rg.kv[0], 0, 256, 0, 256, True, acc, lse)
    rg.close()


@pytest.mark.parametrize("world,d,heads,kv_heads,tokens", [(2, 128, 4, 2, 2048), (4, 64, 4, 4, 2048),
                                                           (8, 128, 4, 1, 4096)])
def test_emulated_gather_matches_single_gpu_causal(world, d, heads, kv_heads, tokens):
    """The gather schedule (all ranks' quantised K/V gathered into the whole
    sequence, one causal launch per rank over it): single-GPU causal
    attention within the gate, f64 within the reference's gate, and equal to
    the ring schedule within the gate."""
    c = st.Case(batch=2, heads=heads, kv_heads=kv_heads, tokens=tokens, d=d, causal=True, packed=False, seed=19)
    x, q, k, v = _inputs(c)
    single = st.run_ours(c, x, export=False).out
    eng = st.engine(c)
    T = tokens // world
    sq, skv = sage.Strides.bthd(T, heads, d), sage.Strides.bthd(T, kv_heads, d)
    shards = [(ring.shard_zigzag(q, r, world), ring.shard_zigzag(k, r, world), ring.shard_zigzag(v, r, world))
              for r in range(world)]
    views = ([sage.Tensor(a, sq) for a, _, _ in shards], [sage.Tensor(b, skv) for _, b, _ in shards],
             [sage.Tensor(cc, skv) for _, _, cc in shards])
    results = {}
    for schedule, emulate in (("gather", ring.emulate_gather), ("ring", ring.emulate_ring)):
        rings = [ring.RingAttention(eng, 2, heads, kv_heads, T, r, world, d, schedule=schedule) for r in range(world)]
        outs = [torch.zeros(2, T, heads, d, dtype=torch.bfloat16, device="cuda") for _ in range(world)]
        emulate(rings, *views, [sage.Tensor(o, sq) for o in outs])
        torch.cuda.synchronize()
        for rg in rings:
            assert eng.status(rg.ws) == 0
            rg.close()
        full = ring.unshard_zigzag(outs, world, dim=1)
        results[schedule] = O.bf16_to_f32(full.view(torch.int16).cpu().numpy().view(np.uint16)).reshape(single.shape)
    ours = results["gather"]
    e = O.errors(ours, single)
    print(f"gather P={world} vs single GPU: {e}")
    assert st.attention_gate(e), e
    e = O.errors(ours, results["ring"])
    assert st.attention_gate(e), e
    for r0 in (0, tokens // 2 - 64, tokens - 128):
        rows = (r0, r0 + 128)
        ef = O.errors(ours[:, rows[0]:rows[1]], _f64_rows(c, x, rows))
        assert st.reference_gate(ef), (rows, ef)


def test_gather_single_rank_path():
    """RingAttention.forward with the gather schedule at P = 1 (the code the
    multi-GPU run executes, without the collective)."""
    c = st.Case(batch=2, heads=8, kv_heads=2, tokens=1024, d=128, causal=True, packed=False, seed=29)
    x, q, k, v = _inputs(c)
    single = st.run_ours(c, x, export=False).out
    eng = st.engine(c)
    rg = ring.RingAttention(eng, 2, 8, 2, 1024, 0, 1, 128, schedule="gather")
    out = torch.zeros(2, 1024, 8, 128, dtype=torch.bfloat16, device="cuda")
    sq, skv = sage.Strides.bthd(1024, 8, 128), sage.Strides.bthd(1024, 2, 128)
    rg.forward(sage.Tensor(q.contiguous(), sq), sage.Tensor(k.contiguous(), skv), sage.Tensor(v.contiguous(), skv),
               sage.Tensor(out, sq))
    torch.cuda.synchronize()
    assert eng.status(rg.ws) == 0
    ours = O.bf16_to_f32(out.view(torch.int16).cpu().numpy().view(np.uint16)).reshape(single.shape)
    e = O.errors(ours, single)
    assert st.attention_gate(e), e
    with pytest.raises(sage.SageError):  # query chunks past the gathered keys
        eng.cp_attend_gathered(rg.ws, rg.kv_all, 0, 1024, sage.Tensor(out, sq))
    rg.close()
