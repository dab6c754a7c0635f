"""Python mirror of the reference's `spl_nn::sage` API over libsplsage.so.

The reference (platform/spl-nn/src/sage/mod.rs) is a Rust API; this module
binds the same types and calls to the C ABI in include/splsage.h so the
tests and the benchmark read like the reference's own tests:

    sage = SageAttention(stream, head_dim=128)            # SageAttention::new
    ws = sage.workspace(Shape(batch, heads, tokens), KvMerge.dense())
    sage.prepare(ws, Tensor(q, strides), Tensor(k, strides), Tensor(v, strides), Options())
    sage.attend(ws, TensorMut(out, Strides.bthd(tokens, heads, d)))

Tensors are torch CUDA tensors (bf16 storage, channels contiguous) viewed
through element strides, exactly as the Rust `Tensor { data, strides }`.
There is no CPU fallback: every call goes to the sm_100a kernels, and the
module refuses to load without the built library.
"""
from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass, field

__all__ = [
    "QGROUP", "QTILE", "KBLOCK", "FP8_MAX", "PV16_V_RANGE", "SageError", "Tile", "PvAccum", "Config", "Strides",
    "Shape", "FrameLayout", "KvMerge", "Options", "QkNorm", "Plan", "Tensor", "TensorMut", "Workspace",
    "SageAttention", "flops", "library_path",
]

QGROUP = 16      # mod.rs:71
QTILE = 128      # mod.rs:73
KBLOCK = 64      # mod.rs:75
FP8_MAX = 448.0  # mod.rs:77
PV16_V_RANGE = 2.25  # mod.rs:185

_HERE = os.path.dirname(os.path.abspath(__file__))


def library_path() -> str:
    return os.path.join(_HERE, "libsplsage.so")


ERR_INVALID = 1  # SPL_SAGE_ERR_INVALID
NOALLOC_SCRATCH_FLOATS = 1 << 20  # the fixed scratch of spl_sage_quantize_noalloc (sage_quant.cu)


class SageError(RuntimeError):
    """A non-zero status from libsplsage, with its message."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


# ---------------------------------------------------------------- C structs

class _Config(ctypes.Structure):
    _fields_ = [("warps", ctypes.c_uint32), ("m_tiles", ctypes.c_uint32), ("stages", ctypes.c_uint32),
                ("pv_accum", ctypes.c_int32)]


class _Shape(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("heads", ctypes.c_int64), ("kv_heads", ctypes.c_int64),
                ("tokens", ctypes.c_int64), ("causal", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class _Merge(ctypes.Structure):
    _fields_ = [("stride", ctypes.c_int32), ("reserved", ctypes.c_int32), ("frames", ctypes.c_int64),
                ("special", ctypes.c_int64), ("grid_h", ctypes.c_int64), ("grid_w", ctypes.c_int64),
                ("dense_frames", ctypes.c_int64)]


class _Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("len", ctypes.c_int64), ("batch", ctypes.c_int64),
                ("token", ctypes.c_int64), ("head", ctypes.c_int64)]


class _Options(ctypes.Structure):
    _fields_ = [("softmax_scale", ctypes.c_float), ("has_softmax_scale", ctypes.c_int32),
                ("smooth_k", ctypes.c_int32), ("smooth_v", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("qk_norm_params", ctypes.c_void_p), ("qk_norm_len", ctypes.c_int64),
                ("qk_norm_eps", ctypes.c_float), ("reserved2", ctypes.c_int32)]


class _QkvShape(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("tokens", ctypes.c_int64), ("hidden", ctypes.c_int64),
                ("heads", ctypes.c_int64), ("kv_heads", ctypes.c_int64), ("rope_half", ctypes.c_int32),
                ("frame_len", ctypes.c_int32)]


class _Plan(ctypes.Structure):
    _fields_ = [("tq_pad", ctypes.c_int64), ("tk", ctypes.c_int64), ("tk_pad", ctypes.c_int64)]


EXPORTS = [
    "spl_sage_default_config", "spl_sage_default_options", "spl_sage_create", "spl_sage_destroy",
    "spl_sage_workspace_create", "spl_sage_ws_destroy", "spl_sage_ws_bytes", "spl_sage_ws_plan", "spl_sage_prepare",
    "spl_sage_attend", "spl_sage_forward", "spl_sage_ws_export_reference_layout", "spl_sage_status",
    "spl_sage_attn_resources", "spl_sage_flops", "spl_sage_last_error", "spl_sage_version", "spl_sage_tensor_peak",
    "spl_sage_qkv_gemm", "spl_sage_qkv_gemm_quant", "spl_sage_rope_table_1d", "spl_sage_engine_status",
    "spl_sage_quantize_noalloc", "spl_sage_kv_bytes", "spl_sage_kv_create", "spl_sage_kv_destroy",
    "spl_sage_cp_prepare", "spl_sage_cp_quantize_kv", "spl_sage_cp_attend", "spl_sage_cp_finish",
    "spl_sage_reserve_sms", "spl_sage_qkv_gemm_fp8", "spl_sage_layer_norm_fp8", "spl_sage_rows_fp8",
    "spl_sage_linear_fp8", "spl_sage_gemm_pairs", "spl_sage_ring_create", "spl_sage_ring_destroy",
    "spl_sage_ring_forward", "spl_sage_plan_new", "spl_sage_wait_selftest", "spl_sage_ring_segment",
    "spl_sage_kv_create_gathered", "spl_sage_cp_attend_gathered", "spl_sage_ring_schedule",
]

# spl_sage_cp_attend flags
CP_CAUSAL = 1
CP_FIRST = 2
# spl_sage_ring_schedule
CP_SCHEDULES = {"ring": 0, "gather": 1}

_lib = None


def lib() -> ctypes.CDLL:
    """Loads libsplsage.so (fails loudly if it was not built)."""
    global _lib
    if _lib is None:
        path = library_path()
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with `make -C sota-papers-lab_b200/csrc` "
                               "(or __graft_entry__.build()); there is no fallback implementation")
        L = ctypes.CDLL(path)
        P, I = ctypes.c_void_p, ctypes.c_int
        L.spl_sage_default_config.argtypes = [I, ctypes.POINTER(_Config)]
        L.spl_sage_default_options.argtypes = [ctypes.POINTER(_Options)]
        L.spl_sage_create.argtypes = [P, I, ctypes.POINTER(_Config), ctypes.POINTER(P)]
        L.spl_sage_destroy.argtypes = [P]
        L.spl_sage_reserve_sms.argtypes = [P, I]
        L.spl_sage_gemm_pairs.argtypes = [P, I]
        L.spl_sage_ring_create.argtypes = [P, ctypes.POINTER(_Shape), I, I, I, ctypes.POINTER(P)]
        L.spl_sage_ring_destroy.argtypes = [P]
        L.spl_sage_ring_forward.argtypes = [P, P, _Tensor, _Tensor, _Tensor, _Tensor, ctypes.POINTER(_Options), P]
        L.spl_sage_ring_schedule.argtypes = [P, I]
        L.spl_sage_kv_create_gathered.argtypes = [P, P, ctypes.c_int64, P, P, P, ctypes.POINTER(P)]
        L.spl_sage_cp_attend_gathered.argtypes = [P, P, P, ctypes.c_int64, ctypes.c_int64, _Tensor]
        L.spl_sage_ring_segment.argtypes = [I, I, I, ctypes.c_int64] + [ctypes.POINTER(ctypes.c_int64)] * 4 + [
            ctypes.POINTER(I)]
        L.spl_sage_workspace_create.argtypes = [P, ctypes.POINTER(_Shape), ctypes.POINTER(_Merge), ctypes.POINTER(P)]
        L.spl_sage_ws_destroy.argtypes = [P]
        L.spl_sage_ws_bytes.restype = ctypes.c_int64
        L.spl_sage_ws_bytes.argtypes = [P]
        L.spl_sage_ws_plan.argtypes = [P, ctypes.POINTER(_Plan)]
        L.spl_sage_plan_new.argtypes = [ctypes.POINTER(_Shape), ctypes.POINTER(_Merge), ctypes.POINTER(_Plan)]
        L.spl_sage_prepare.argtypes = [P, P, _Tensor, _Tensor, _Tensor, ctypes.POINTER(_Options)]
        L.spl_sage_attend.argtypes = [P, P, _Tensor]
        L.spl_sage_forward.argtypes = [P, P, _Tensor, _Tensor, _Tensor, _Tensor, ctypes.POINTER(_Options)]
        L.spl_sage_ws_export_reference_layout.argtypes = [P] * 9
        L.spl_sage_status.argtypes = [P, P, ctypes.POINTER(ctypes.c_uint32)]
        L.spl_sage_attn_resources.argtypes = [P, ctypes.POINTER(I), ctypes.POINTER(I)]
        L.spl_sage_tensor_peak.argtypes = [P, I, I, I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
        L.spl_sage_qkv_gemm.argtypes = [P, ctypes.POINTER(_QkvShape)] + [P] * 7
        L.spl_sage_qkv_gemm_fp8.argtypes = [P, ctypes.POINTER(_QkvShape)] + [P] * 9
        L.spl_sage_layer_norm_fp8.argtypes = [P, P, I, ctypes.c_int64, ctypes.c_int64, P, P, ctypes.c_float, P, P, P]
        L.spl_sage_rows_fp8.argtypes = [P, P] + [ctypes.c_int64] * 3 + [P] * 5
        L.spl_sage_linear_fp8.argtypes = [P] * 6 + [ctypes.c_int64] * 3 + [P]
        L.spl_sage_qkv_gemm_quant.argtypes = [P, P, ctypes.POINTER(_QkvShape)] + [P] * 7 + [ctypes.POINTER(_Options)]
        L.spl_sage_rope_table_1d.argtypes = [ctypes.c_double, I, ctypes.c_int64, P]
        L.spl_sage_engine_status.argtypes = [P, ctypes.POINTER(ctypes.c_uint32)]
        L.spl_sage_wait_selftest.argtypes = [P, ctypes.POINTER(ctypes.c_uint64)]
        L.spl_sage_quantize_noalloc.argtypes = ([P, I, I, ctypes.POINTER(_Shape), _Tensor, _Tensor, _Tensor,
                                                 ctypes.POINTER(_Options)] + [P] * 6)
        I64P = ctypes.POINTER(ctypes.c_int64)
        L.spl_sage_kv_bytes.argtypes = [P, I64P, I64P, I64P]
        L.spl_sage_kv_create.argtypes = [P, P, P, P, P, ctypes.POINTER(P)]
        L.spl_sage_kv_destroy.argtypes = [P]
        L.spl_sage_cp_prepare.argtypes = [P, P, _Tensor, _Tensor, _Tensor, ctypes.POINTER(_Options), P]
        L.spl_sage_cp_quantize_kv.argtypes = [P, P, _Tensor, _Tensor, ctypes.POINTER(_Options), P, ctypes.c_int64, P]
        L.spl_sage_cp_attend.argtypes = [P, P, P] + [ctypes.c_int64] * 4 + [I, P, P]
        L.spl_sage_cp_finish.argtypes = [P, P, P, _Tensor]
        L.spl_sage_flops.restype = ctypes.c_double
        L.spl_sage_flops.argtypes = [P]
        L.spl_sage_last_error.restype = ctypes.c_char_p
        L.spl_sage_version.restype = ctypes.c_char_p
        _lib = L
    return _lib


def _check(rc: int):
    if rc != 0:
        raise SageError(rc, lib().spl_sage_last_error().decode())


# ---------------------------------------------------------------- types (mod.rs)

@dataclass(frozen=True)
class Tile:
    """CTA shape of the reference kernel (mod.rs:119-168); validated, and kept
    for drop-in compatibility (the sm_100a kernel's CTA is fixed)."""
    warps: int = 4
    m_tiles: int = 2
    stages: int = 3

    @staticmethod
    def for_head_dim(head_dim: int) -> "Tile":
        return Tile(4, 1, 3) if head_dim > 64 else Tile(4, 2, 3)

    def rows(self) -> int:
        return 16 * self.m_tiles * self.warps


class PvAccum:
    """mod.rs:172-181."""
    F32 = 0
    F16 = 1


@dataclass(frozen=True)
class Config:
    tile: Tile
    pv_accum: int = PvAccum.F32

    @staticmethod
    def for_head_dim(head_dim: int) -> "Config":
        return Config(Tile.for_head_dim(head_dim), PvAccum.F32)


@dataclass(frozen=True)
class Strides:
    """Element strides of a [batch][token][head][dim] bf16 view (mod.rs:203-260)."""
    batch: int
    token: int
    head: int

    @staticmethod
    def bthd(tokens: int, heads: int, head_dim: int) -> "Strides":
        return Strides(tokens * heads * head_dim, heads * head_dim, head_dim)

    @staticmethod
    def bhtd(tokens: int, heads: int, head_dim: int) -> "Strides":
        return Strides(heads * tokens * head_dim, head_dim, tokens * head_dim)

    @staticmethod
    def packed_qkv(tokens: int, heads: int, head_dim: int) -> "Strides":
        return Strides(tokens * 3 * heads * head_dim, 3 * heads * head_dim, head_dim)

    def extent(self, shape: "Shape", head_dim: int, heads: int | None = None) -> int:
        h = shape.heads if heads is None else heads
        return (shape.batch - 1) * self.batch + (shape.tokens - 1) * self.token + (h - 1) * self.head + head_dim


@dataclass(frozen=True)
class Shape:
    """mod.rs:262-268, plus kv_heads (GQA) and causal (extensions)."""
    batch: int
    heads: int
    tokens: int
    kv_heads: int = 0
    causal: bool = False

    @property
    def kv(self) -> int:
        return self.kv_heads or self.heads


@dataclass(frozen=True)
class FrameLayout:
    """mod.rs:273-300."""
    frames: int
    special: int
    grid_h: int
    grid_w: int
    dense_frames: int = 0

    def tokens_per_frame(self) -> int:
        return self.special + self.grid_h * self.grid_w

    def merged_per_frame(self, stride: int) -> int:
        return self.special + -(-self.grid_h // stride) * -(-self.grid_w // stride)

    def merged_keys(self, stride: int) -> int:
        d = min(self.dense_frames, self.frames)
        return d * self.tokens_per_frame() + (self.frames - d) * self.merged_per_frame(stride)


@dataclass(frozen=True)
class KvMerge:
    """KvMerge::Dense or KvMerge::Pool { stride, layout } (mod.rs:302-311)."""
    stride: int = 1
    layout: FrameLayout | None = None

    @staticmethod
    def dense() -> "KvMerge":
        return KvMerge(1, None)

    @staticmethod
    def pool(stride: int, layout: FrameLayout) -> "KvMerge":
        return KvMerge(stride, layout)


@dataclass
class QkNorm:
    """QK LayerNorm parameters: a CUDA f32 tensor [4][head_dim] (q w, q b, k w, k b)."""
    params: object
    eps: float = 1e-5


@dataclass
class Options:
    """mod.rs:313-335 (smoothing on by default)."""
    softmax_scale: float | None = None
    smooth_k: bool = True
    smooth_v: bool = True
    qk_norm: QkNorm | None = None

    def _c(self) -> _Options:
        o = _Options()
        lib().spl_sage_default_options(ctypes.byref(o))
        if self.softmax_scale is not None:
            o.softmax_scale = float(self.softmax_scale)
            o.has_softmax_scale = 1
        o.smooth_k = int(bool(self.smooth_k))
        o.smooth_v = int(bool(self.smooth_v))
        if self.qk_norm is not None:
            p = self.qk_norm.params
            o.qk_norm_params = p.data_ptr()
            o.qk_norm_len = p.numel()
            o.qk_norm_eps = float(self.qk_norm.eps)
        return o


def _merge_c(merge: "KvMerge") -> _Merge:
    if merge.stride > 1:
        lay = merge.layout
        return _Merge(merge.stride, 0, lay.frames, lay.special, lay.grid_h, lay.grid_w, lay.dense_frames)
    return _Merge()


@dataclass(frozen=True)
class Plan:
    """mod.rs:391-454."""
    shape: Shape
    merge: KvMerge
    tq_pad: int
    tk: int
    tk_pad: int

    @classmethod
    def new(cls, shape: Shape, merge: KvMerge | None = None) -> "Plan":
        """Plan::new (mod.rs:405-440): the sizes that follow from a shape and
        a key merge, with the same checks (spl_sage_plan_new; host only)."""
        merge = merge or KvMerge.dense()
        cs = _Shape(shape.batch, shape.heads, shape.kv_heads, shape.tokens, int(shape.causal), 0)
        cm = _merge_c(merge)
        p = _Plan()
        _check(lib().spl_sage_plan_new(ctypes.byref(cs), ctypes.byref(cm), ctypes.byref(p)))
        return cls(shape, merge, p.tq_pad, p.tk, p.tk_pad)

    def key_ratio(self) -> float:
        """Keys after merging per key before (mod.rs:443-445)."""
        return self.tk / self.shape.tokens


@dataclass
class Tensor:
    """A bf16 tensor view: torch CUDA tensor (any dtype of 2 bytes) + element strides.
    The view starts at data's first element."""
    data: object
    strides: Strides

    def _c(self) -> _Tensor:
        t = self.data
        if t.element_size() != 2:
            raise SageError(1, "sage tensors hold bf16 (2-byte) elements")
        return _Tensor(t.data_ptr(), t.numel(), self.strides.batch, self.strides.token, self.strides.head)


TensorMut = Tensor


def _stream_ptr(stream) -> int:
    if stream is None:
        return 0
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


class Workspace:
    """Device buffers of one Plan (mod.rs:456-495); owned by the library."""

    def __init__(self, handle: int, plan: Plan, head_dim: int):
        self._h = ctypes.c_void_p(handle)
        self.plan = plan
        self.head_dim = head_dim

    def bytes(self) -> int:
        return int(lib().spl_sage_ws_bytes(self._h))

    def close(self):
        if self._h:
            lib().spl_sage_ws_destroy(self._h)
            self._h = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class SageAttention:
    """SageAttention (mod.rs:509-901) on one CUDA stream."""

    def __init__(self, stream=None, head_dim: int = 64, config: Config | None = None):
        cfg = config or Config.for_head_dim(head_dim)
        c = _Config(cfg.tile.warps, cfg.tile.m_tiles, cfg.tile.stages, cfg.pv_accum)
        h = ctypes.c_void_p()
        _check(lib().spl_sage_create(ctypes.c_void_p(_stream_ptr(stream)), head_dim, ctypes.byref(c),
                                     ctypes.byref(h)))
        self._h = h
        self.head_dim = head_dim
        self.config = cfg
        self.stream = stream
        self.reserved_sms = 0

    @staticmethod
    def new(stream, head_dim: int) -> "SageAttention":
        return SageAttention(stream, head_dim)

    @staticmethod
    def with_config(stream, head_dim: int, config: Config) -> "SageAttention":
        return SageAttention(stream, head_dim, config)

    def reserve_sms(self, n: int):
        """Persistent kernels of this engine leave n SMs free (for kernels on
        other streams, e.g. NCCL's during a ring step); 0 restores all."""
        _check(lib().spl_sage_reserve_sms(self._h, n))
        self.reserved_sms = n

    def gemm_pairs(self, on: bool):
        """Run this engine's GEMMs on SM pairs (tcgen05 cta_group::2)."""
        _check(lib().spl_sage_gemm_pairs(self._h, int(on)))

    def close(self):
        if self._h:
            lib().spl_sage_destroy(self._h)
            self._h = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def attn_resources(self) -> tuple[int, int]:
        r, s = ctypes.c_int(), ctypes.c_int()
        _check(lib().spl_sage_attn_resources(self._h, ctypes.byref(r), ctypes.byref(s)))
        return r.value, s.value

    def tensor_peak(self, kind: int, n: int = 128, iters: int = 20000) -> tuple[float, float]:
        """Measured tcgen05 rate: kind 0 INT8, 1 FP8 E4M3, 2 BF16; returns
        (tera-ops/s over all SMs, cycles per M128 x N x 32-byte instruction)."""
        t, c = ctypes.c_double(), ctypes.c_double()
        _check(lib().spl_sage_tensor_peak(self._h, kind, n, iters, ctypes.byref(t), ctypes.byref(c)))
        return t.value, c.value

    def qkv_gemm(self, x, w, bias, rope, q, k, v, *, batch: int, tokens: int, heads: int, kv_heads: int = 0,
                 rope_half: int = 0, frame_len: int = 0):
        """Gemm::linear_bf16 + QkvPrologue::run fused (spl_sage_qkv_gemm): x
        [batch*tokens][hidden], w [(heads+2*kv)*D][hidden], bias or None,
        rope (f32 [frame_len][D/2][2]) or None; writes q/k/v bf16 [B][T][H][D]."""
        p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
        sh = _QkvShape(batch, tokens, x.shape[-1], heads, kv_heads, rope_half, frame_len)
        _check(lib().spl_sage_qkv_gemm(self._h, ctypes.byref(sh), p(x), p(w), p(bias), p(rope), p(q), p(k), p(v)))

    def qkv_gemm_fp8(self, x8, x_scale, w8, w_scale, bias, rope, q, k, v, *, batch: int, tokens: int, heads: int,
                     kv_heads: int = 0, rope_half: int = 0, frame_len: int = 0):
        """The FP8 QKV side (spl_sage_qkv_gemm_fp8): x8 E4M3 (uint8)
        [batch*tokens][hidden] with x_scale f32 [batch*tokens], w8 E4M3
        [(heads+2*kv)*D][hidden] with w_scale f32 per output channel; the
        rest as qkv_gemm."""
        p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
        sh = _QkvShape(batch, tokens, x8.shape[-1], heads, kv_heads, rope_half, frame_len)
        _check(lib().spl_sage_qkv_gemm_fp8(self._h, ctypes.byref(sh), p(x8), p(x_scale), p(w8), p(w_scale), p(bias),
                                           p(rope), p(q), p(k), p(v)))

    def layer_norm_fp8(self, x, gamma, beta, eps: float, q8, scales, out=None):
        """Norm::layer_norm with per-token FP8 output (spl_sage_layer_norm_fp8):
        x f32 or bf16 [rows][c]; writes q8 (uint8 E4M3) [rows][c], scales f32
        [rows] and, when given, out bf16 [rows][c]."""
        import torch
        p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
        rows, c = x.shape[0], x.shape[-1]
        _check(lib().spl_sage_layer_norm_fp8(self._h, p(x), int(x.dtype == torch.float32), rows, c, p(gamma), p(beta),
                                             float(eps), p(out), p(q8), p(scales)))

    def rows_fp8(self, y, q8, scales, *, c: int | None = None, tok=None, chan=None, bias=None):
        """Norm::row_epilogue with per-token FP8 (spl_sage_rows_fp8): y bf16
        [rows][ld] (its first c channels) -> q8 uint8 [rows][c], scales f32."""
        p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
        rows, ld = y.shape[0], y.shape[-1]
        _check(lib().spl_sage_rows_fp8(self._h, p(y), rows, c or ld, ld, p(tok), p(chan), p(bias), p(q8),
                                       p(scales)))

    def linear_fp8(self, x8, x_scale, w8, w_scale, bias, y):
        """Gemm::linear_fp8 (spl_sage_linear_fp8): y bf16 [m][n] from E4M3 x8
        [m][k] and w8 [n][k]; scales None for deferred scales."""
        p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
        m, k = x8.shape
        n = w8.shape[0]
        _check(lib().spl_sage_linear_fp8(self._h, p(x8), p(x_scale), p(w8), p(w_scale), p(bias), m, n, k, p(y)))

    def qkv_gemm_quant(self, ws: Workspace, x, w, bias, rope, q, k, v, opts: Options | None = None, *,
                       rope_half: int = 0, frame_len: int = 0):
        p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
        s = ws.plan.shape
        sh = _QkvShape(s.batch, s.tokens, x.shape[-1], s.heads, s.kv_heads, rope_half, frame_len)
        o = (opts or Options())._c()
        _check(lib().spl_sage_qkv_gemm_quant(self._h, ws._h, ctypes.byref(sh), p(x), p(w), p(bias), p(rope), p(q),
                                             p(k), p(v), ctypes.byref(o)))

    def engine_status(self) -> int:
        """Reads (and clears) the engine's device error word; raises on a
        kernel error."""
        w = ctypes.c_uint32()
        _check(lib().spl_sage_engine_status(self._h, ctypes.byref(w)))
        return w.value

    def wait_selftest(self) -> tuple[bool, int, bool, int]:
        """Runs a bounded wait into its timeout on purpose
        (spl_sage_wait_selftest): (warp 0 succeeded, its wait in ns, warp 1
        succeeded, its wait in ns).  The engine's error word is left set."""
        r = (ctypes.c_uint64 * 4)()
        _check(lib().spl_sage_wait_selftest(self._h, r))
        return bool(r[0]), int(r[1]), bool(r[2]), int(r[3])

    def workspace(self, shape: Shape, merge: KvMerge | None = None) -> Workspace:
        merge = merge or KvMerge.dense()
        cs = _Shape(shape.batch, shape.heads, shape.kv_heads, shape.tokens, int(shape.causal), 0)
        cm = _merge_c(merge)
        h = ctypes.c_void_p()
        _check(lib().spl_sage_workspace_create(self._h, ctypes.byref(cs), ctypes.byref(cm), ctypes.byref(h)))
        p = _Plan()
        _check(lib().spl_sage_ws_plan(h, ctypes.byref(p)))
        return Workspace(h.value, Plan(shape, merge, p.tq_pad, p.tk, p.tk_pad), self.head_dim)

    def prepare(self, ws: Workspace, q: Tensor, k: Tensor, v: Tensor, opts: Options | None = None):
        o = (opts or Options())._c()
        _check(lib().spl_sage_prepare(self._h, ws._h, q._c(), k._c(), v._c(), ctypes.byref(o)))

    def attend(self, ws: Workspace, out: Tensor):
        _check(lib().spl_sage_attend(self._h, ws._h, out._c()))

    def forward(self, ws: Workspace, q: Tensor, k: Tensor, v: Tensor, out: Tensor, opts: Options | None = None):
        o = (opts or Options())._c()
        _check(lib().spl_sage_forward(self._h, ws._h, q._c(), k._c(), v._c(), out._c(), ctypes.byref(o)))

    def export_reference_layout(self, ws: Workspace, q8=None, q_scale=None, k8=None, k_scale=None, v8=None,
                                stats=None, kbias=None):
        """Copies the quantised tensors, in the reference's byte layout, into
        the given CUDA tensors (any may be None)."""
        ptr = (lambda t: None if t is None else ctypes.c_void_p(t.data_ptr()))
        _check(lib().spl_sage_ws_export_reference_layout(self._h, ws._h, ptr(q8), ptr(q_scale), ptr(k8),
                                                         ptr(k_scale), ptr(v8), ptr(stats), ptr(kbias)))

    # ------------------------------------------------------------ context parallelism
    # (no counterpart in the reference; see ring.py for the schedule)

    def cp_prepare(self, ws: Workspace, q: Tensor, k: Tensor, v: Tensor, raw, opts: Options | None = None):
        """Quantise this rank's Q into ws; raw (f32 CUDA, b*g*4*D) receives
        its K/V channel statistics {sum K, sum V, -min V, max V}."""
        o = (opts or Options())._c()
        _check(lib().spl_sage_cp_prepare(self._h, ws._h, q._c(), k._c(), v._c(), ctypes.byref(o),
                                         ctypes.c_void_p(raw.data_ptr())))

    def cp_quantize_kv(self, ws: Workspace, k: Tensor, v: Tensor, raw_global, total_tokens: int, kv: "KvBuffer",
                       opts: Options | None = None):
        """This rank's K/V quantised with the statistics combined over all
        ranks (raw entries 0-1 summed, 2-3 maxed) into kv."""
        o = (opts or Options())._c()
        _check(lib().spl_sage_cp_quantize_kv(self._h, ws._h, k._c(), v._c(), ctypes.byref(o),
                                             ctypes.c_void_p(raw_global.data_ptr()), total_tokens, kv._h))

    def cp_attend(self, ws: Workspace, kv: "KvBuffer", q_begin: int, q_len: int, k_begin: int, k_len: int,
                  causal: bool, acc, lse, first: bool = False):
        """Segment attention merged into acc (f32 [b][t][h][D]) and lse (f32
        [b][h][t]) by log-sum-exp; first: the segment is the first of its
        query rows and overwrites acc and lse instead."""
        flags = (CP_CAUSAL if causal else 0) | (CP_FIRST if first else 0)
        _check(lib().spl_sage_cp_attend(self._h, ws._h, kv._h, q_begin, q_len, k_begin, k_len, flags,
                                        ctypes.c_void_p(acc.data_ptr()), ctypes.c_void_p(lse.data_ptr())))

    def cp_attend_gathered(self, ws: Workspace, kv_all: "KvBuffer", q_off0: int, q_off1: int, out: Tensor):
        """This rank's two query chunks (local rows [0, C) at global rows
        q_off0.., [C, 2C) at q_off1..) against the gathered keys of the whole
        sequence in one causal launch, bf16 into out."""
        _check(lib().spl_sage_cp_attend_gathered(self._h, ws._h, kv_all._h, q_off0, q_off1, out._c()))

    def cp_finish(self, ws: Workspace, acc, out: Tensor):
        _check(lib().spl_sage_cp_finish(self._h, ws._h, ctypes.c_void_p(acc.data_ptr()), out._c()))

    def status(self, ws: Workspace) -> int:
        """Reads (and clears) the device error word; raises on a kernel error."""
        w = ctypes.c_uint32()
        _check(lib().spl_sage_status(self._h, ws._h, ctypes.byref(w)))
        return w.value


def ring_segment(rank: int, world: int, step: int, chunk: int) -> tuple[int, int, int, int, int]:
    """The segment the native ring attends at a step (spl_sage_ring_segment;
    host only): (q_begin, q_len, k_begin, k_len, cp_attend flags)."""
    v = [ctypes.c_int64() for _ in range(4)]
    f = ctypes.c_int()
    _check(lib().spl_sage_ring_segment(rank, world, step, chunk, *[ctypes.byref(x) for x in v], ctypes.byref(f)))
    return v[0].value, v[1].value, v[2].value, v[3].value, f.value


class NativeRing:
    """One rank of the context-parallel ring driven inside the library
    (spl_sage_ring_create / _forward): the schedule of
    ring.RingAttention, over a caller's NCCL communicator (an ncclComm_t as
    an integer; 0 when world = 1)."""

    def __init__(self, eng: "SageAttention", batch: int, heads: int, kv_heads: int, local_tokens: int, rank: int,
                 world: int, reserved_sms: int = 1, schedule: str = "ring"):
        cs = _Shape(batch, heads, kv_heads, local_tokens, 0, 0)
        h = ctypes.c_void_p()
        _check(lib().spl_sage_ring_create(eng._h, ctypes.byref(cs), rank, world, reserved_sms, ctypes.byref(h)))
        self._h, self.eng = h, eng
        if schedule not in CP_SCHEDULES:
            self.close()
            raise SageError(ERR_INVALID, f"unknown context-parallel schedule {schedule!r}")
        _check(lib().spl_sage_ring_schedule(self._h, CP_SCHEDULES[schedule]))

    def forward(self, q: Tensor, k: Tensor, v: Tensor, out: Tensor, opts: Options | None = None, comm: int = 0):
        o = (opts or Options())._c()
        _check(lib().spl_sage_ring_forward(self.eng._h, self._h, q._c(), k._c(), v._c(), out._c(), ctypes.byref(o),
                                           ctypes.c_void_p(comm)))

    def close(self):
        if self._h:
            lib().spl_sage_ring_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class KvBuffer:
    """One rank's quantised K/V (k8, k_scale, v8 as torch CUDA tensors that
    NCCL can send and receive) with the TMA descriptors the attention kernel
    reads them through (spl_sage_kv_create)."""

    def __init__(self, eng: "SageAttention", ws: Workspace, tokens: int | None = None):
        """tokens None: ws's own keys (spl_sage_kv_create); otherwise a
        buffer of `tokens` gathered keys, the whole sequence of a
        context-parallel job (spl_sage_kv_create_gathered)."""
        import torch
        if tokens is None:
            n = [ctypes.c_int64() for _ in range(3)]
            _check(lib().spl_sage_kv_bytes(ws._h, *[ctypes.byref(x) for x in n]))
            sizes = [x.value for x in n]
        else:
            s = ws.plan.shape
            kb = s.batch * s.kv * tokens * ws.head_dim
            sizes = [kb, 4 * s.batch * s.kv * (tokens // KBLOCK), kb]
        self.tokens = tokens
        self.k8 = torch.empty(sizes[0], dtype=torch.uint8, device="cuda")
        self.k_scale = torch.empty(sizes[1] // 4, dtype=torch.float32, device="cuda")
        self.v8 = torch.empty(sizes[2], dtype=torch.uint8, device="cuda")
        h = ctypes.c_void_p()
        ptrs = [ctypes.c_void_p(t.data_ptr()) for t in (self.k8, self.k_scale, self.v8)]
        if tokens is None:
            _check(lib().spl_sage_kv_create(eng._h, ws._h, *ptrs, ctypes.byref(h)))
        else:
            _check(lib().spl_sage_kv_create_gathered(eng._h, ws._h, tokens, *ptrs, ctypes.byref(h)))
        self._h = h

    def tensors(self):
        return [self.k8, self.k_scale, self.v8]

    def close(self):
        if self._h:
            lib().spl_sage_kv_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def quantize_noalloc(head_dim: int, shape: Shape, q: Tensor, k: Tensor, v: Tensor, q8, q_scale, k8, k_scale, v8,
                     stats, opts: Options | None = None, pv_accum: int = PvAccum.F32, stream=None):
    """Quantises q, k, v into caller-owned CUDA tensors without any device
    allocation (spl_sage_quantize_noalloc; no counterpart in the reference).
    Outputs use the workspace layouts: q8 [b][h][tq_pad][D] i8, q_scale
    [b][h][tq_pad/16] f32, k8 [b][g][tk_pad][D] i8, k_scale [b][g][tk_pad/64]
    f32, v8 [b][g][D][tk_pad] E4M3 bytes, stats [b][g][4][D] f32.  Dense keys
    only; the library's fixed scratch bounds batch * kv_heads *
    ceil(tokens/128) * 4 * D to 1,048,576.  The C ABI cannot see the
    outputs' sizes, so every output is checked here (a CUDA tensor of at
    least its layout's bytes) before the call."""
    b, h, g, t, d = shape.batch, shape.heads, shape.kv, shape.tokens, head_dim
    tq_pad = (t + 127) // 128 * 128
    tk_pad = (t + 63) // 64 * 64
    part = b * g * (tq_pad // 128) * 4 * d
    if part > NOALLOC_SCRATCH_FLOATS:  # the library's own check, made before the outputs' sizes are looked at
        raise SageError(ERR_INVALID, f"quantize_noalloc: batch x kv_heads x ceil(tokens/128) x 4 x head_dim = {part} "
                                     f"floats exceeds its fixed scratch of {NOALLOC_SCRATCH_FLOATS} floats; use a "
                                     "workspace (SageAttention.prepare)")
    need = {"q8": b * h * tq_pad * d, "q_scale": 4 * b * h * (tq_pad // 16), "k8": b * g * tk_pad * d,
            "k_scale": 4 * b * g * (tk_pad // 64), "v8": b * g * d * tk_pad, "stats": 4 * b * g * 4 * d}
    for name, t_out in (("q8", q8), ("q_scale", q_scale), ("k8", k8), ("k_scale", k_scale), ("v8", v8),
                        ("stats", stats)):
        if not getattr(t_out, "is_cuda", False):
            raise SageError(ERR_INVALID, f"quantize_noalloc: {name} must be a CUDA tensor")
        have = t_out.numel() * t_out.element_size()
        if have < need[name]:
            raise SageError(ERR_INVALID,
                            f"quantize_noalloc: {name} holds {have} bytes, the shape needs {need[name]}")
    sh = _Shape(shape.batch, shape.heads, shape.kv, shape.tokens, int(shape.causal), 0)
    o = (opts or Options())._c()
    ptr = (lambda t: ctypes.c_void_p(t.data_ptr()))
    _check(lib().spl_sage_quantize_noalloc(_stream_ptr(stream), head_dim, pv_accum, ctypes.byref(sh), q._c(), k._c(),
                                           v._c(), ctypes.byref(o), ptr(q8), ptr(q_scale), ptr(k8), ptr(k_scale),
                                           ptr(v8), ptr(stats)))


def rope_table_1d(base: float, head_dim: int, positions: int):
    """A Llama-style 1-D RoPE table (f32 numpy [positions][D/2][2])."""
    import numpy as np
    out = np.empty((positions, head_dim // 2, 2), np.float32)
    _check(lib().spl_sage_rope_table_1d(base, head_dim, positions, out.ctypes.data_as(ctypes.c_void_p)))
    return out


class RopeLayout:
    """Which channels rotate together (qkv.rs:36-61): channel c pairs with
    c ^ half and reads angle row pair(c) = (c / 2·half)·half + c % half.
    VGGT: half 16 (channels 0-31 by row position, 32-63 by column); DINOv3:
    half 32; a 1-D (Llama) table over D channels: half D/2.  The QKV GEMMs
    take `half` as their `rope_half` argument."""
    VGGT = 16
    DINOV3 = 32

    @staticmethod
    def one_d(head_dim: int) -> int:
        return head_dim // 2

    @staticmethod
    def pair(half: int, c: int) -> int:
        return (c // (2 * half)) * half + c % half


class RopeTable:
    """cos / sin per (token of a frame, pair), as the QKV epilogue reads
    them: `cos_sin` f32 [frame_len][D/2][2] (RopeTable, qkv.rs:63-131).
    Angles are taken in f64 and their cos / sin stored as f32."""

    def __init__(self, half: int, cos_sin):
        self.half = half
        self.cos_sin = cos_sin
        self.frame_len = cos_sin.shape[0]

    @classmethod
    def from_angles(cls, half: int, frame_len: int, pairs: int, angle):
        """qkv.rs:75-96: `angle(token, pair)` in radians."""
        import numpy as np
        a = np.array([[angle(t, p) for p in range(pairs)] for t in range(frame_len)], np.float64).reshape(
            frame_len, pairs)
        return cls(half, np.stack([np.cos(a), np.sin(a)], -1).astype(np.float32))

    @classmethod
    def vggt(cls, grid_h: int, grid_w: int, special: int, base: float = 100.0):
        """qkv.rs:98-110: `special` leading tokens unrotated, then a grid at
        positions (y + 1, x + 1); pair i of each 16-pair half at frequency
        base^(-i/16) (D = 64)."""
        def angle(t, p):
            if t < special:
                return 0.0
            y, x = divmod(t - special, grid_w)
            return float((y + 1) if p < 16 else (x + 1)) * base ** (-(p % 16) / 16.0)
        return cls.from_angles(RopeLayout.VGGT, special + grid_h * grid_w, 32, angle)

    @classmethod
    def dinov3(cls, grid_h: int, grid_w: int, special: int, base: float = 100.0):
        """qkv.rs:112-128: patch coordinates normalised to [-1, 1] per axis,
        period base^(j/16) for pair j of each axis (D = 64)."""
        def angle(t, p):
            if t < special:
                return 0.0
            y, x = divmod(t - special, grid_w)
            coord = (y + 0.5) / grid_h * 2.0 - 1.0 if p < 16 else (x + 0.5) / grid_w * 2.0 - 1.0
            return 2.0 * math.pi * coord / base ** ((p % 16) / 16.0)
        return cls.from_angles(RopeLayout.DINOV3, special + grid_h * grid_w, 32, angle)

    @classmethod
    def one_d(cls, base: float, head_dim: int, positions: int):
        """Llama-style 1-D positions 0..positions-1, frequency
        base^(-p/(D/2)) for pair p (spl_sage_rope_table_1d)."""
        return cls(RopeLayout.one_d(head_dim), rope_table_1d(base, head_dim, positions))


def flops(plan: Plan, head_dim: int) -> float:
    """mod.rs:905-910: 4 * B * H * Tq * Tk * D."""
    return 4.0 * plan.shape.batch * plan.shape.heads * plan.shape.tokens * plan.tk * head_dim


def causal_flops(batch: int, heads: int, n: int, head_dim: int) -> float:
    """Algorithmic FLOPs of causal attention: 4 * B * H * D * N (N + 1) / 2."""
    return 4.0 * batch * heads * head_dim * n * (n + 1) / 2
