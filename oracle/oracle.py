"""ctypes/numpy front end of the CPU oracle (liboracle.so) and of the
reference's own kernels built as a GPU oracle (oracle/_ref).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference arm may use this module, as the checker; the
product (libsplsage.so and its Python mirror) never imports it.

What each function restates is documented in sage_oracle.h with the
reference file:line it follows (platform/spl-nn/src/sage/reference.rs,
platform/spl-nn/cuda/sage_quant.cu).
"""
from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
QGROUP, QTILE, KBLOCK = 16, 128, 64
LN_Q, LN_K, SMOOTH_K, SMOOTH_V = 1, 2, 4, 8
FP8_MAX = 448.0
PV16_V_RANGE = 2.25
LOG2_E = np.float32(1.4426950408889634)


class Geom(ctypes.Structure):
    """or_geom of sage_oracle.h."""

    _fields_ = [(n, ctypes.c_int64) for n in
                ("q_sb", "q_st", "q_sh", "k_sb", "k_st", "k_sh", "v_sb", "v_st", "v_sh")] + [
        (n, ctypes.c_int32) for n in
        ("batch", "heads", "kv_heads", "tokens", "tq_pad", "tk", "tk_pad", "d", "merge", "frames",
         "frame_tokens", "special", "grid_h", "grid_w", "merged_frame", "merged_w", "dense_frames",
         "q_tiles", "flags", "pad0")] + [(n, ctypes.c_float) for n in ("q_mul", "ln_eps", "v_range", "pad1")]


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} missing: run `make -C oracle`")
        L = ctypes.CDLL(path)
        P = ctypes.c_void_p
        L.or_bf16_to_f32.restype = ctypes.c_float
        L.or_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.or_f32_to_bf16.restype = ctypes.c_uint16
        L.or_f32_to_bf16.argtypes = [ctypes.c_float]
        L.or_e4m3_to_f32.restype = ctypes.c_float
        L.or_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.or_f32_to_e4m3.restype = ctypes.c_uint8
        L.or_f32_to_e4m3.argtypes = [ctypes.c_float]
        L.or_f32_to_e4m3_n.argtypes = [P, P, ctypes.c_int64]
        L.or_vpos.restype = ctypes.c_int
        L.or_vpos.argtypes = [ctypes.c_int]
        L.or_rng_next.restype = ctypes.c_uint64
        L.or_rng_next.argtypes = [ctypes.POINTER(ctypes.c_uint64)]
        L.or_rng_normal.restype = ctypes.c_float
        L.or_rng_normal.argtypes = [ctypes.POINTER(ctypes.c_uint64)]
        L.or_rng_normals.argtypes = [ctypes.POINTER(ctypes.c_uint64), P, ctypes.c_int64, ctypes.c_float,
                                     ctypes.c_float]
        L.or_synthetic.argtypes = [ctypes.c_int] * 4 + [ctypes.c_uint64, P, P, P]
        L.or_members.restype = ctypes.c_int
        L.or_members.argtypes = [ctypes.POINTER(Geom), ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                 ctypes.POINTER(ctypes.c_int)]
        L.or_prepare.argtypes = [P] * 12 + [ctypes.POINTER(Geom)]
        L.or_prep.argtypes = [P] * 7 + [ctypes.POINTER(Geom)]
        L.or_finalize.argtypes = [P, P, ctypes.POINTER(Geom)]
        L.or_quant_kv.argtypes = [P] * 8 + [ctypes.POINTER(Geom)]
        L.or_attention_f64.argtypes = [P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                       ctypes.c_int, ctypes.c_int, P]
        L.or_attention_bthd.restype = ctypes.c_int
        L.or_attention_bthd.argtypes = [P, P, P, ctypes.POINTER(Geom), ctypes.c_float, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
        L.or_sage_emulate.argtypes = [P] * 7 + [ctypes.POINTER(Geom)] + [ctypes.c_int] * 4 + [P]
        L.or_sage_online.argtypes = [P] * 7 + [ctypes.POINTER(Geom)] + [ctypes.c_int] * 5 + [P]
        L.or_layer_norm.argtypes = [P, P, P, ctypes.c_int, ctypes.c_float]
        L.or_qkv_reference.argtypes = [P, P, P, P] + [ctypes.c_int] * 10 + [P, P, P]
        L.or_qkv_reference_fp8.argtypes = [P] * 6 + [ctypes.c_int] * 10 + [P, P, P]
        L.or_layer_norm_fp8.argtypes = [P, ctypes.c_int, ctypes.c_int64, ctypes.c_int, P, P, ctypes.c_float, P, P, P]
        L.or_rows_fp8.argtypes = [P, ctypes.c_int64, ctypes.c_int, ctypes.c_int64, P, P, P, P, P]
        L.or_errors.argtypes = [P, P, ctypes.c_int64, P]
        L.or_flops.restype = ctypes.c_double
        L.or_flops.argtypes = [ctypes.c_int] * 5
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------- codecs

def bf16_to_f32(b):
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x):
    """reference.rs:13-20, vectorised."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32)
    rnd = np.uint32(0x7FFF) + ((bits >> 16) & 1)
    out = ((bits + rnd) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = ((bits[nan] >> 16) | 0x40).astype(np.uint16)
    return out


_E4M3_TABLE = None


def e4m3_table() -> np.ndarray:
    global _E4M3_TABLE
    if _E4M3_TABLE is None:
        _E4M3_TABLE = np.array([lib().or_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)
    return _E4M3_TABLE


def e4m3_to_f32(b):
    return e4m3_table()[np.asarray(b, dtype=np.uint8)]


def f32_to_e4m3(x: float) -> int:
    return int(lib().or_f32_to_e4m3(float(x)))


def f32_to_e4m3_array(x) -> np.ndarray:
    """or_f32_to_e4m3 over an array (same shape, uint8)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(x.shape, np.uint8)
    lib().or_f32_to_e4m3_n(_p(x), _p(out), x.size)
    return out


def vpos(k: int) -> int:
    return int(lib().or_vpos(k))


# ---------------------------------------------------------------- RNG / data

class Rng:
    """SplitMix64 + Box-Muller (reference.rs:228-254)."""

    def __init__(self, seed: int):
        self.s = ctypes.c_uint64(seed)

    def next_u64(self) -> int:
        return int(lib().or_rng_next(ctypes.byref(self.s)))

    def normal(self) -> float:
        return float(lib().or_rng_normal(ctypes.byref(self.s)))

    def normals(self, n: int, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        lib().or_rng_normals(ctypes.byref(self.s), _p(out), n, std, mean)
        return out


def synthetic(batch: int, heads: int, tokens: int, d: int, seed: int):
    """Data::synthetic (tests.rs:300-329): bf16 bits [b][t][h][d] each."""
    shape = (batch, tokens, heads, d)
    q = np.empty(shape, np.uint16)
    k = np.empty(shape, np.uint16)
    v = np.empty(shape, np.uint16)
    lib().or_synthetic(batch, heads, tokens, d, seed, _p(q), _p(k), _p(v))
    return q, k, v


# ---------------------------------------------------------------- geometry

@dataclass
class Layout:
    """FrameLayout (mod.rs:273-300)."""
    frames: int
    special: int
    grid_h: int
    grid_w: int
    dense_frames: int = 0

    def tokens_per_frame(self) -> int:
        return self.special + self.grid_h * self.grid_w

    def merged_per_frame(self, s: int) -> int:
        return self.special + -(-self.grid_h // s) * -(-self.grid_w // s)

    def merged_keys(self, s: int) -> int:
        d = min(self.dense_frames, self.frames)
        return d * self.tokens_per_frame() + (self.frames - d) * self.merged_per_frame(s)


def make_geom(batch, heads, kv_heads, tokens, d, strides_q, strides_k, strides_v, *, flags=SMOOTH_K | SMOOTH_V,
              softmax_scale=None, merge: int = 1, layout: Layout | None = None, ln_eps=1e-5,
              v_range=FP8_MAX) -> Geom:
    g = Geom()
    g.q_sb, g.q_st, g.q_sh = strides_q
    g.k_sb, g.k_st, g.k_sh = strides_k
    g.v_sb, g.v_st, g.v_sh = strides_v
    g.batch, g.heads, g.kv_heads, g.tokens, g.d = batch, heads, kv_heads, tokens, d
    g.tq_pad = -(-tokens // QTILE) * QTILE
    if merge > 1:
        lay = layout
        g.tk = lay.merged_keys(merge)
        g.frames, g.special, g.grid_h, g.grid_w = lay.frames, lay.special, lay.grid_h, lay.grid_w
        g.dense_frames = min(lay.dense_frames, lay.frames)
        g.frame_tokens = lay.tokens_per_frame()
        g.merged_frame = lay.merged_per_frame(merge)
        g.merged_w = -(-lay.grid_w // merge)
    else:
        g.tk = tokens
        g.frames = 1
    g.merge = merge
    g.tk_pad = -(-g.tk // KBLOCK) * KBLOCK
    g.q_tiles = g.tq_pad // QTILE
    g.flags = flags
    scale = np.float32(1.0) / np.sqrt(np.float32(d)) if softmax_scale is None else np.float32(softmax_scale)
    g.q_mul = float(np.float32(scale) * LOG2_E)
    g.ln_eps = ln_eps
    g.v_range = v_range
    return g


def bthd_strides(tokens, heads, d):
    return (tokens * heads * d, heads * d, d)


def members(g: Geom, j: int):
    base, nx = ctypes.c_int(), ctypes.c_int()
    n = lib().or_members(ctypes.byref(g), j, ctypes.byref(base), ctypes.byref(nx))
    return [base.value + (m // nx.value) * g.grid_w + m % nx.value for m in range(n)]


# ---------------------------------------------------------------- quantiser

@dataclass
class Quant:
    q8: np.ndarray
    q_scale: np.ndarray
    k8: np.ndarray
    k_scale: np.ndarray
    v8: np.ndarray  # reference layout [b][hkv][tk_pad/64][d][64], keys permuted
    stats: np.ndarray
    kbias: np.ndarray
    part: np.ndarray


def prepare(q, k, v, g: Geom, ln: np.ndarray | None = None) -> Quant:
    """SageAttention::prepare on the CPU, bit-exact with sage_quant.cu."""
    b, hq, hkv, d = g.batch, g.heads, g.kv_heads, g.d
    out = Quant(
        q8=np.zeros((b, hq, g.tq_pad, d), np.int8),
        q_scale=np.zeros((b, hq, g.tq_pad // QGROUP), np.float32),
        k8=np.zeros((b, hkv, g.tk_pad, d), np.int8),
        k_scale=np.zeros((b, hkv, g.tk_pad // KBLOCK), np.float32),
        v8=np.zeros((b, hkv, g.tk_pad // KBLOCK, d, KBLOCK), np.uint8),
        stats=np.zeros((b, hkv, 4, d), np.float32),
        kbias=np.zeros(g.tk_pad, np.float32),
        part=np.zeros((b, hkv, g.q_tiles, 4, d), np.float32),
    )
    lnp = None if ln is None else np.ascontiguousarray(ln, np.float32)
    lib().or_prepare(_p(np.ascontiguousarray(q)), _p(np.ascontiguousarray(k)), _p(np.ascontiguousarray(v)),
                     _p(lnp), _p(out.q8), _p(out.q_scale), _p(out.k8), _p(out.k_scale), _p(out.v8), _p(out.stats),
                     _p(out.kbias), _p(out.part), ctypes.byref(g))
    return out


def attention_bthd(q, k, v, g: Geom, *, causal=False, rows=None, nthreads=None, scale=None) -> np.ndarray:
    """f64 exact attention over bf16 [b][t][h][d] inputs (reference.rs:148-184,
    with the causal mask and GQA head mapping as extensions).  Returns f32
    [b][t][hq][d]; only `rows` (a (start, stop) range) are computed."""
    out = np.zeros((g.batch, g.tokens, g.heads, g.d), np.float32)
    r0, r1 = rows if rows is not None else (0, g.tokens)
    sc = np.float32(1.0) / np.sqrt(np.float32(g.d)) if scale is None else np.float32(scale)
    lib().or_attention_bthd(_p(np.ascontiguousarray(q)), _p(np.ascontiguousarray(k)), _p(np.ascontiguousarray(v)),
                            ctypes.byref(g), float(sc), int(causal), r0, r1, nthreads or os.cpu_count() or 1,
                            _p(out))
    return out


def sage_emulate(qt: Quant, g: Geom, *, causal=False, rows=None, nthreads=None) -> np.ndarray:
    """The quantised arithmetic evaluated exactly (or_sage_emulate); only
    `rows` (a (start, stop) range of every (b, h)) are computed."""
    out = np.zeros((g.batch, g.tokens, g.heads, g.d), np.float32)
    r0, r1 = rows if rows is not None else (0, g.tokens)
    lib().or_sage_emulate(_p(qt.q8), _p(qt.q_scale), _p(qt.k8), _p(qt.k_scale), _p(qt.v8), _p(qt.stats),
                          _p(qt.kbias), ctypes.byref(g), int(causal), r0, r1, nthreads or os.cpu_count() or 1,
                          _p(out))
    return out


REF_BLOCK = 64   # keys per online-softmax block in the reference kernel (sage_attn.cu:227)
OUR_BLOCK = 128  # ... in this library's kernel


def sage_online(qt: Quant, g: Geom, *, block=REF_BLOCK, causal=False, rows=None, nthreads=None) -> np.ndarray:
    """The kernels' online softmax, block by block (or_sage_online): block
    64 restates the reference kernel's arithmetic (extended with the causal
    mask and GQA), 128 this library's.  Only `rows` of every (b, h)."""
    out = np.zeros((g.batch, g.tokens, g.heads, g.d), np.float32)
    r0, r1 = rows if rows is not None else (0, g.tokens)
    lib().or_sage_online(_p(qt.q8), _p(qt.q_scale), _p(qt.k8), _p(qt.k_scale), _p(qt.v8), _p(qt.stats),
                         _p(qt.kbias), ctypes.byref(g), int(causal), int(block), r0, r1,
                         nthreads or os.cpu_count() or 1, _p(out))
    return out


def qkv_reference(x, w, bias, rope, *, tokens, hq, hkv, d, rope_half=0, frame_len=1, nthreads=None):
    """f64 QKV GEMM + prologue (host::linear + qkv::reference): x bf16 bits
    [m][k], w [n][k], bias [n] or None, rope f32 [frame_len][d/2][2] or None.
    Returns f32 q [m][hq][d], k [m][hkv][d], v [m][hkv][d]."""
    m, k = x.shape
    n = w.shape[0]
    q = np.zeros((m, hq, d), np.float32)
    kk = np.zeros((m, hkv, d), np.float32)
    v = np.zeros((m, hkv, d), np.float32)
    lib().or_qkv_reference(_p(np.ascontiguousarray(x)), _p(np.ascontiguousarray(w)),
                           _p(None if bias is None else np.ascontiguousarray(bias)),
                           _p(None if rope is None else np.ascontiguousarray(rope, np.float32)), rope_half, frame_len,
                           m, n, k, tokens, hq, hkv, d, nthreads or os.cpu_count() or 1, _p(q), _p(kk), _p(v))
    return q, kk, v


def qkv_reference_fp8(x8, x_scale, w8, w_scale, bias, rope, *, tokens, hq, hkv, d, rope_half=0, frame_len=1,
                      nthreads=None):
    """f64 FP8 QKV GEMM + prologue: x8 E4M3 bytes [m][k] with x_scale f32
    [m], w8 [n][k] with w_scale f32 [n], bias bf16 bits [n] or None.  Returns
    f32 q [m][hq][d], k [m][hkv][d], v [m][hkv][d]."""
    m, k = x8.shape
    n = w8.shape[0]
    q = np.zeros((m, hq, d), np.float32)
    kk = np.zeros((m, hkv, d), np.float32)
    v = np.zeros((m, hkv, d), np.float32)
    c = np.ascontiguousarray
    lib().or_qkv_reference_fp8(_p(c(x8, np.uint8)), _p(c(x_scale, np.float32)), _p(c(w8, np.uint8)),
                               _p(c(w_scale, np.float32)), _p(None if bias is None else c(bias)),
                               _p(None if rope is None else c(rope, np.float32)), rope_half, frame_len, m, n, k, tokens,
                               hq, hkv, d, nthreads or os.cpu_count() or 1, _p(q), _p(kk), _p(v))
    return q, kk, v


def layer_norm_fp8(x, gamma, beta, eps, with_out=False):
    """norm.cu:37-137 on the CPU: x f32 or bf16 bits (uint16) [rows][c].
    Returns (q8 uint8 [rows][c], scales f32 [rows], out bf16 bits or None)."""
    x = np.ascontiguousarray(x)
    rows, c = x.shape
    q8 = np.zeros((rows, c), np.uint8)
    sc = np.zeros(rows, np.float32)
    out = np.zeros((rows, c), np.uint16) if with_out else None
    lib().or_layer_norm_fp8(_p(x), int(x.dtype == np.float32), rows, c, _p(np.ascontiguousarray(gamma, np.float32)),
                            _p(np.ascontiguousarray(beta, np.float32)), float(eps), _p(out), _p(q8), _p(sc))
    return q8, sc, out


def rows_fp8(y, c=None, tok=None, chan=None, bias=None):
    """norm.cu:170-229 on the CPU: y bf16 bits [rows][ld].  Returns (q8, scales)."""
    y = np.ascontiguousarray(y, np.uint16)
    rows, ld = y.shape
    c = c or ld
    q8 = np.zeros((rows, c), np.uint8)
    sc = np.zeros(rows, np.float32)
    a = lambda t, dt: None if t is None else np.ascontiguousarray(t, dt)
    lib().or_rows_fp8(_p(y), rows, c, ld, _p(a(tok, np.float32)), _p(a(chan, np.float32)), _p(a(bias, np.uint16)),
                      _p(q8), _p(sc))
    return q8, sc


def errors(ours, ref) -> dict:
    a = np.ascontiguousarray(ours, np.float32).ravel()
    r = np.ascontiguousarray(ref, np.float32).ravel()
    o = np.zeros(5, np.float64)
    lib().or_errors(_p(a), _p(r), a.size, _p(o))
    return dict(cos=o[0], rel_l1=o[1], rel_l2=o[2], max_abs=o[3], ref_max=o[4])


def flops(batch, heads, tq, tk, d) -> float:
    return 4.0 * batch * heads * tq * tk * d


def causal_flops(batch, heads, n, d) -> float:
    return 4.0 * batch * heads * d * n * (n + 1) / 2


# ---------------------------------------------------------------- reference GPU oracle

_ref_libs: dict[tuple, ctypes.CDLL] = {}


def _ref_name(d: int, pv16: bool) -> str:
    return os.path.join(HERE, "_ref", f"libsage_ref_d{d}{'_pv16' if pv16 else ''}.so")


def ref_available(d: int, pv16: bool = False) -> bool:
    return os.path.exists(_ref_name(d, pv16))


def ref_lib(d: int, pv16: bool = False) -> ctypes.CDLL:
    """The reference's kernels for head dim d (SG_PV16 = pv16)."""
    key = (d, pv16)
    if key not in _ref_libs:
        L = ctypes.CDLL(_ref_name(d, pv16))
        P = ctypes.c_void_p
        L.ref_sage_run.restype = ctypes.c_int
        L.ref_sage_run.argtypes = [P, P, P, P, P, P, ctypes.c_float, ctypes.c_float, ctypes.c_float] + [P] * 10
        L.ref_sage_attend.restype = ctypes.c_int
        L.ref_sage_attend.argtypes = [P, P, ctypes.c_float, ctypes.c_float] + [P] * 9
        _ref_libs[key] = L
    return _ref_libs[key]


def ref_dims(g: Geom) -> np.ndarray:
    return np.array([g.batch, g.heads, g.tokens, g.merge, g.frames, g.special, g.grid_h, g.grid_w,
                     g.dense_frames, g.flags], np.int32)


_norm_ref = None


def norm_ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libnorm_ref.so"))


def _load_norm_ref():
    global _norm_ref
    L = ctypes.CDLL(os.path.join(HERE, "_ref", "libnorm_ref.so"))
    P = ctypes.c_void_p
    L.ref_layer_norm_fp8.restype = ctypes.c_int
    L.ref_layer_norm_fp8.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, ctypes.c_float, P, P, P, P]
    L.ref_rows_fp8.restype = ctypes.c_int
    L.ref_rows_fp8.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P, P, P, P]
    _norm_ref = L


def ref_layer_norm_fp8(x, gamma, beta, eps, out, q8, scales, stream=0) -> int:
    """The reference's own ln_{f32,bf16}_c<n> kernels (norm.cu:37-144), on
    device tensors (x f32 or bf16 [rows][c]); returns a cudaError_t."""
    global _norm_ref
    if _norm_ref is None:
        _load_norm_ref()
    import torch
    p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
    return _norm_ref.ref_layer_norm_fp8(p(x), int(x.dtype == torch.float32), x.shape[0], x.shape[-1], p(gamma),
                                        p(beta), float(eps), p(out), p(q8), p(scales), ctypes.c_void_p(stream))


def ref_rows_fp8(y, c, tok, chan, bias, q8, scales, stream=0) -> int:
    """The reference's own row_c<n> kernels (norm.cu:170-235) on device
    tensors: y bf16 [rows][ld]; returns a cudaError_t."""
    global _norm_ref
    if _norm_ref is None:
        _load_norm_ref()
    p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
    return _norm_ref.ref_rows_fp8(p(y), y.shape[0], c, y.shape[-1], p(tok), p(chan), p(bias), p(q8), p(scales),
                                  ctypes.c_void_p(stream))
