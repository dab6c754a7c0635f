"""The CPU oracle against golden outputs of the reference's own kernels
(tests/golden/ref_*.npz, written by tests/golden/gen_ref_fixtures.py on a B200
from oracle/_ref).  Bit-exact for the quantiser; the oracle's f64 attention
and its emulation of the quantised arithmetic against the reference kernel's
attention output within the reference's own tolerances."""
import glob
import os

import numpy as np
import pytest

import sagetest as st
from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
FILES = sorted(glob.glob(os.path.join(HERE, "golden", "ref_*.npz")))
CASES = {"dense": dict(), "nosmooth": dict(smooth=False), "merge2": dict(merge=2), "merge4": dict(merge=4),
         "pv16": dict(pv16=True)}


def _case(path):
    f = np.load(path)
    b, h, t, d, merge, smooth, pv16, seed = (int(v) for v in f["meta"])
    name = os.path.basename(path)[len("ref_d") + len(str(d)) + 1:-4]
    lay = st.small_layout()
    c = st.Case(batch=b, heads=h, kv_heads=h, tokens=t, d=d, layout=lay, seed=seed, **CASES[name])
    return f, c


def test_fixtures_present():
    assert len(FILES) == 10, FILES


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(p) for p in FILES])
def test_oracle_quantiser_matches_reference_kernels(path):
    f, c = _case(path)
    x = st.make_inputs(c)
    import hashlib
    h = hashlib.sha256()
    for a in (x.q, x.k, x.v):
        h.update(np.ascontiguousarray(a).tobytes())
    assert h.hexdigest() == str(f["input_sha256"]), "input generator drifted"
    ours = O.prepare(x.q, x.k, x.v, st.geom(c), None)
    ref = O.Quant(q8=f["q8"], q_scale=f["q_scale"], k8=f["k8"], k_scale=f["k_scale"], v8=f["v8"], stats=f["stats"],
                  kbias=f["kbias"], part=None)
    st.assert_quant_equal(ours, ref, kbias=c.merge > 1, what=os.path.basename(path))


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(p) for p in FILES])
def test_oracle_attention_matches_reference_kernels(path):
    f, c = _case(path)
    x = st.make_inputs(c)
    g = st.geom(c)
    ref_out = f["out"]
    exact = O.attention_bthd(x.q, x.k, x.v, g, nthreads=4)
    e = O.errors(ref_out, exact)
    # the reference's own gate for its kernel against f64 (tests.rs:699)
    assert e["cos"] > 0.999 and e["rel_l2"] < 0.04, e
    emu = O.sage_emulate(O.prepare(x.q, x.k, x.v, g, None), g, nthreads=4)
    e2 = O.errors(ref_out, emu)
    assert e2["cos"] > 0.9999 and e2["rel_l1"] < 5e-3, e2


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(p) for p in FILES])
def test_online_emulation_matches_reference_kernels(path):
    """or_sage_online with the reference kernel's 64-key blocks restates that
    kernel's online arithmetic; against its bf16 output only rounding noise
    is left (exp2f vs ex2.approx, the PV summation order), which the bf16
    output almost always absorbs: most fixtures match bit for bit."""
    f, c = _case(path)
    x = st.make_inputs(c)
    g = st.geom(c)
    quant = O.prepare(x.q, x.k, x.v, g, None)
    on64 = O.bf16_to_f32(O.f32_to_bf16(O.sage_online(quant, g, block=O.REF_BLOCK, nthreads=4)))
    e = O.errors(f["out"], on64)
    print(os.path.basename(path), e)
    assert e["cos"] > 0.9999999 and e["rel_l1"] < 1e-5, e
