"""Failure detection without a GPU fault.  A bounded wait inside a kernel
runs into its limit on purpose (spl_sage_wait_selftest: an mbarrier that
nothing arrives on, the same wait code every kernel uses).  The device error
word carries the timeout and its site back to the host through
spl_sage_engine_status, a second warp leaves as soon as it sees the word
set, and the engine and its CUDA context stay usable afterwards."""
import ctypes
import importlib

import numpy as np
import pytest
import torch

import sagetest as st
from oracle import oracle as O

pytestmark = pytest.mark.gpu
sage = importlib.import_module("sota-papers-lab_b200")

ERR_KERNEL = 5      # SPL_SAGE_ERR_KERNEL
TIMEOUT_BIT = 0x1   # SPL_SAGE_DEVERR_TIMEOUT
SITE = 99           # SPL_SAGE_SELFTEST_SITE


def test_bounded_wait_times_out_and_the_engine_stays_usable():
    c = st.Case(batch=1, heads=4, kv_heads=2, tokens=300, d=128, causal=True)
    eng = st.engine(c)
    assert eng.engine_status() == 0
    ok0, ns0, ok1, ns1 = eng.wait_selftest()
    assert not ok0 and not ok1
    assert 0.2e9 <= ns0 < 1.0e9, ns0   # its own 0.2 s limit
    assert ns1 < 1.2e9, ns1            # left on the error word, before its 1.5 s limit
    with pytest.raises(sage.SageError, match=f"timeout site {SITE}") as ei:
        eng.engine_status()
    assert ei.value.code == ERR_KERNEL
    assert eng.engine_status() == 0    # read and cleared: the word is 0 again
    # a second run, refused again while its word is pending, the word read
    # through the C ABI
    assert not eng.wait_selftest()[0]
    with pytest.raises(sage.SageError, match="already set"):
        eng.wait_selftest()
    word = ctypes.c_uint32()
    rc = sage.lib().spl_sage_engine_status(eng._h, ctypes.byref(word))
    assert rc == ERR_KERNEL and word.value == (TIMEOUT_BIT | (SITE << 8)), hex(word.value)
    # the context and the engine still work: causal GQA attention within the
    # reference's gate against f64 attention (tests.rs:699)
    x = st.make_inputs(c)
    ws = eng.workspace(sage.Shape(c.batch, c.heads, c.tokens, c.kv_heads, c.causal))
    keep, (tq, tk, tv) = st.to_device(c, x)
    out = torch.zeros(c.batch * c.tokens * c.heads * c.d, dtype=torch.bfloat16, device="cuda")
    eng.forward(ws, tq, tk, tv, sage.Tensor(out, sage.Strides.bthd(c.tokens, c.heads, c.d)))
    assert eng.status(ws) == 0 and eng.engine_status() == 0
    got = O.bf16_to_f32(out.view(torch.int16).cpu().numpy().view(np.uint16)).reshape(c.batch, c.tokens, c.heads,
                                                                                         c.d)
    e = O.errors(got, O.attention_bthd(x.q, x.k, x.v, st.geom(c), causal=True))
    assert st.reference_gate(e), e
    # and byte for byte what a fresh engine computes from the same inputs
    assert np.array_equal(got, st.run_ours(c, x, export=False).out)
