"""Parity of the tcgen05 attention kernel (spl_sage_attend): against the
reference's own kernels run on the same GPU (the gate: cos >= 0.9995,
rel-L1 <= 1e-2), against f64 exact attention (the reference's own gate,
tests.rs:699: cos > 0.999, rel-L2 < 0.04) and against an emulation of the
quantised arithmetic on the same quantised tensors (tighter)."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _small(st, d, **kw):
    lay = st.small_layout()
    args = dict(batch=2, heads=3, kv_heads=3, tokens=lay.frames * lay.tokens_per_frame(), d=d, layout=lay, seed=5)
    args.update(kw)
    return st.Case(**args)


def _exact(c, x):
    return O.attention_bthd(x.q, x.k, x.v, __import__("sagetest").geom(c), causal=c.causal)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("kw", [dict(), dict(smooth=False), dict(ln=True), dict(merge=2), dict(merge=4, ln=True),
                                dict(pv16=True), dict(pv16=True, merge=4)],
                         ids=["dense", "nosmooth", "ln", "merge2", "merge4_ln", "pv16", "pv16_merge4"])
def test_attention_matches_reference_kernels(d, kw):
    """pv16: PvAccum::F16 against the reference's SG_PV16 kernel (FP16 PV
    accumulation per block); ours keeps FP32 accumulation with the same
    quantiser (V scaled to +-2.25)."""
    import sagetest as st
    if not O.ref_available(d, kw.get("pv16", False)):
        pytest.skip("oracle/_ref not built")
    c = _small(st, d, **kw)
    x = st.make_inputs(c)
    ours = st.run_ours(c, x, export=False).out
    ref, _ = st.run_reference_gpu(c, x)
    e = O.errors(ours, ref)
    print(f"d{d} {kw} vs reference kernels: {e}")
    assert st.attention_gate(e), e


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("kw", [dict(), dict(smooth=False), dict(merge=2), dict(merge=4)],
                         ids=["dense", "nosmooth", "merge2", "merge4"])
def test_attention_matches_f64_and_emulation(d, kw):
    import sagetest as st
    c = _small(st, d, **kw)
    x = st.make_inputs(c)
    run = st.run_ours(c, x)
    g = st.geom(c)
    # f64 exact attention over the (merged) bf16 inputs
    exact = O.attention_bthd(x.q, x.k, x.v, g)
    e = O.errors(run.out, exact)
    print(f"d{d} {kw} vs f64: {e}")
    assert st.reference_gate(e), e
    # the quantised arithmetic evaluated exactly on our own quantised tensors
    emu = O.sage_emulate(run.quant, g)
    e2 = O.errors(run.out, emu)
    print(f"d{d} {kw} vs emulation: {e2}")
    assert e2["cos"] > 0.9999 and e2["rel_l1"] < 5e-3, e2


@pytest.mark.parametrize("d", [64, 128])
def test_causal_gqa_attention(d):
    import sagetest as st
    c = st.Case(batch=2, heads=8, kv_heads=2, tokens=700, d=d, causal=True, packed=False, seed=9)
    x = st.make_inputs(c)
    run = st.run_ours(c, x)
    g = st.geom(c)
    exact = O.attention_bthd(x.q, x.k, x.v, g, causal=True)
    e = O.errors(run.out, exact)
    print(f"causal gqa d{d} vs f64: {e}")
    assert st.reference_gate(e), e
    emu = O.sage_emulate(run.quant, g, causal=True)
    e2 = O.errors(run.out, emu)
    print(f"causal gqa d{d} vs emulation: {e2}")
    assert e2["cos"] > 0.9999 and e2["rel_l1"] < 5e-3, e2


def test_long_sequence_single_head():
    import sagetest as st
    # tests.rs:704-729: T = 3001, ragged tails, many key blocks.
    c = st.Case(batch=1, heads=2, kv_heads=2, tokens=3001, d=64, seed=21)
    x = st.make_inputs(c)
    run = st.run_ours(c, x, export=False)
    exact = O.attention_bthd(x.q, x.k, x.v, st.geom(c))
    e = O.errors(run.out, exact)
    print(f"T3001 vs f64: {e}")
    assert st.reference_gate(e), e
    if O.ref_available(64):
        ref, _ = st.run_reference_gpu(c, x)
        e2 = O.errors(run.out, ref)
        print(f"T3001 vs reference kernels: {e2}")
        assert st.attention_gate(e2), e2


def test_attention_kernel_does_not_spill():
    import sagetest as st
    for d in (64, 128):
        eng = st.engine(st.Case(batch=1, heads=1, kv_heads=1, tokens=1, d=d))
        regs, spill = eng.attn_resources()
        print(f"d{d}: {regs} registers, {spill} spill bytes")
        assert spill == 0
