"""CPU tests of the boundary: libsplsage.so loads and exports every symbol
include/splsage.h declares, the ctypes structs match the C layout, host-side
validation mirrors the reference's (mod.rs checks), and without a GPU the
library fails loudly instead of falling back."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "splsage.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(spl_sage_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol(sage):
    names = declared_functions()
    assert len(names) >= 17
    out = subprocess.run(["nm", "-D", "--defined-only", sage.library_path()], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (\w+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    assert set(sage.EXPORTS) == set(names)


def test_struct_layouts_match_the_header(sage, tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "splsage.h"\n'
        'int main(void){printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu %zu\\n",'
        'sizeof(spl_sage_config), sizeof(spl_sage_shape), sizeof(spl_sage_merge), sizeof(spl_sage_tensor),'
        'sizeof(spl_sage_options), sizeof(spl_sage_plan), offsetof(spl_sage_options, qk_norm_params),'
        'offsetof(spl_sage_merge, frames), offsetof(spl_sage_shape, causal), offsetof(spl_sage_options, qk_norm_eps));'
        'return 0;}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    m = sage
    want = [ctypes.sizeof(m._Config), ctypes.sizeof(m._Shape), ctypes.sizeof(m._Merge), ctypes.sizeof(m._Tensor),
            ctypes.sizeof(m._Options), ctypes.sizeof(m._Plan), m._Options.qk_norm_params.offset,
            m._Merge.frames.offset, m._Shape.causal.offset, m._Options.qk_norm_eps.offset]
    assert got == want


def test_defaults_mirror_the_reference(sage):
    # Config::for_head_dim (mod.rs:195-200), Tile::DEFAULT / D128, Options::default.
    c = sage._Config()
    sage.lib().spl_sage_default_config(64, ctypes.byref(c))
    assert (c.warps, c.m_tiles, c.stages, c.pv_accum) == (4, 2, 3, 0)
    sage.lib().spl_sage_default_config(128, ctypes.byref(c))
    assert (c.warps, c.m_tiles, c.stages, c.pv_accum) == (4, 1, 3, 0)
    o = sage._Options()
    sage.lib().spl_sage_default_options(ctypes.byref(o))
    assert (o.smooth_k, o.smooth_v, o.has_softmax_scale, o.qk_norm_params) == (1, 1, 0, None)


def test_strides_cover_the_tensor(sage):
    # tests.rs:246-261
    shape = sage.Shape(batch=2, heads=3, tokens=5)
    d = 64
    assert sage.Strides.bthd(5, 3, d).extent(shape, d) == 2 * 5 * 3 * d
    assert sage.Strides.bhtd(5, 3, d).extent(shape, d) == 2 * 3 * 5 * d
    assert sage.Strides.packed_qkv(5, 3, d).extent(shape, d) + 2 * 3 * d == 2 * 5 * 3 * 3 * d


def test_create_validates_before_touching_the_gpu(sage):
    h = ctypes.c_void_p()
    rc = sage.lib().spl_sage_create(None, 96, None, ctypes.byref(h))
    assert rc == 1 and b"head dim 64 or 128" in sage.lib().spl_sage_last_error()
    bad = sage._Config(3, 1, 3, 0)
    rc = sage.lib().spl_sage_create(None, 64, ctypes.byref(bad), ctypes.byref(h))
    assert rc == 1 and b"unsupported sage tile" in sage.lib().spl_sage_last_error()


def test_no_gpu_fails_loudly(sage):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(sage.SageError) as e:
        sage.SageAttention(None, 64)
    assert e.value.code in (2, 3)


def test_flops_definition(sage):
    plan = sage.Plan(sage.Shape(1, 16, 137800), sage.KvMerge.dense(), 137856, 137800, 137856)
    assert sage.flops(plan, 64) == 4.0 * 16 * 137800 * 137800 * 64


def test_plan_rejects_bad_layouts(sage):
    # tests.rs:174-190 (Plan::new, mod.rs:405-440), on the host: no engine, no GPU
    lay = lambda frames: sage.FrameLayout(frames, 17, 21, 32, 0)  # noqa: E731  (tests.rs:85-93)
    with pytest.raises(sage.SageError, match="covers 1378 tokens, the sequence has 1000"):
        sage.Plan.new(sage.Shape(1, 2, 1000), sage.KvMerge.pool(2, lay(2)))
    with pytest.raises(sage.SageError, match="stride must be 2 or 4, got 3"):
        sage.Plan.new(sage.Shape(1, 2, 2 * 689), sage.KvMerge.pool(3, lay(2)))
    p = sage.Plan.new(sage.Shape(1, 2, 2 * 689), sage.KvMerge.pool(4, lay(2)))
    assert (p.tq_pad, p.tk, p.tk_pad) == (1408, 2 * (17 + 6 * 8), 192)
    with pytest.raises(sage.SageError, match="empty attention shape"):
        sage.Plan.new(sage.Shape(1, 2, 0))
    with pytest.raises(sage.SageError, match="patch grid"):
        sage.Plan.new(sage.Shape(1, 2, 34), sage.KvMerge.pool(2, sage.FrameLayout(2, 17, 0, 32)))
    with pytest.raises(sage.SageError, match="multiple of kv_heads"):
        sage.Plan.new(sage.Shape(1, 6, 128, kv_heads=4))
    with pytest.raises(sage.SageError, match="causal attention over merged keys"):
        sage.Plan.new(sage.Shape(1, 2, 2 * 689, causal=True), sage.KvMerge.pool(2, lay(2)))


def test_plan_sizes(sage):
    # the padding of mod.rs:429-434 at the BASELINE shapes (N = 1370 -> 1408 / 1408)
    for tokens, tq_pad, tk_pad in ((1024, 1024, 1024), (1370, 1408, 1408), (8192, 8192, 8192), (1, 128, 64),
                                   (130, 256, 192)):
        p = sage.Plan.new(sage.Shape(8, 16, tokens))
        assert (p.tq_pad, p.tk, p.tk_pad, p.key_ratio()) == (tq_pad, tokens, tk_pad, 1.0)
    # a merged layout keeps its dense frames whole (tests.rs:96-133)
    lay = sage.FrameLayout(3, 5, 7, 10, 1)
    p = sage.Plan.new(sage.Shape(2, 3, 3 * 75), sage.KvMerge.pool(2, lay))
    assert p.tk == lay.merged_keys(2) == 75 + 2 * (5 + 4 * 5)
    assert p.tk_pad == 128 and 0 < p.key_ratio() < 1
    # every index the kernels form must fit in i32 (mod.rs:435-439)
    with pytest.raises(sage.SageError, match="does not fit in i32"):
        sage.Plan.new(sage.Shape(1, 1, 2**31))
    with pytest.raises(sage.SageError, match="does not fit in i32"):
        sage.Plan.new(sage.Shape(2**16, 2**16, 128))


def test_noalloc_rejects_misaligned_outputs_before_any_launch(sage):
    # The alignment checks of spl_sage_quantize_noalloc come before any CUDA
    # call, so fake (never dereferenced) addresses show them on the CPU.
    L = sage.lib()
    sh = sage._Shape(1, 2, 2, 128, 0, 0)
    t = sage._Tensor(0x100000, 1 << 20, 0, 0, 0)
    base, f4 = 0x200000, 0x300000
    ok = dict(q8=base, q_scale=f4, k8=base + 0x10000, k_scale=f4 + 0x1000, v8=base + 0x20000, stats=f4 + 0x2000)
    for name, bad in (("q8", 8), ("k8", 4), ("v8", 1), ("q_scale", 2), ("k_scale", 1), ("stats", 3)):
        args = dict(ok)
        args[name] += bad
        rc = L.spl_sage_quantize_noalloc(None, 64, 0, ctypes.byref(sh), t, t, t, None,
                                         *[ctypes.c_void_p(args[k]) for k in
                                           ("q8", "q_scale", "k8", "k_scale", "v8", "stats")])
        assert rc == 1, (name, rc)
        assert b"must start on" in L.spl_sage_last_error(), name


class _FakeCuda:
    """Stands in for a CUDA tensor in the wrapper's host-side size checks."""
    is_cuda = True

    def __init__(self, nbytes):
        self.n = nbytes

    def numel(self):
        return self.n

    def element_size(self):
        return 1

    def data_ptr(self):
        raise AssertionError("the wrapper must reject before it reads an address")


def test_noalloc_wrapper_checks_output_sizes_on_the_host(sage):
    import torch
    b, h, g, t, d = 1, 4, 2, 200, 64  # tq_pad 256, tk_pad 256
    need = dict(q8=b * h * 256 * d, q_scale=4 * b * h * 16, k8=b * g * 256 * d, k_scale=4 * b * g * 4,
                v8=b * g * d * 256, stats=4 * b * g * 4 * d)
    x = torch.zeros(8, dtype=torch.bfloat16)
    tq = sage.Tensor(x, sage.Strides.bthd(t, h, d))
    order = ("q8", "q_scale", "k8", "k_scale", "v8", "stats")
    for short in order:
        outs = [_FakeCuda(need[k] - (1 if k == short else 0)) for k in order]
        with pytest.raises(sage.SageError, match=short):
            sage.quantize_noalloc(d, sage.Shape(b, h, t, g), tq, tq, tq, *outs)
    with pytest.raises(sage.SageError, match="CUDA tensor"):
        sage.quantize_noalloc(d, sage.Shape(b, h, t, g), tq, tq, tq, torch.zeros(need["q8"], dtype=torch.int8),
                              *[_FakeCuda(need[k]) for k in order[1:]])
