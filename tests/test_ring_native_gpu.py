"""The ring driven inside the library (spl_sage_ring_create / _forward over a
caller's NCCL communicator): at one rank, byte-identical to the Python ring
(sota-papers-lab_b200/ring.py, the same kernels in the same order) and
within the attention gate of single-GPU causal attention; at two ranks
(when two GPUs are visible), two processes with a real NCCL communicator,
their zig-zag shards put back together against single-GPU causal
attention."""
from __future__ import annotations

import ctypes
import importlib
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import sagetest as st
from oracle import oracle as O

pytestmark = pytest.mark.gpu
sage = importlib.import_module("sota-papers-lab_b200")
ring = importlib.import_module("sota-papers-lab_b200.ring")


def _qkv(b, t, h, g, d, seed):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(b, t, h, d, generator=gen).to(torch.bfloat16)
    k = (torch.randn(b, t, g, d, generator=gen) + 2 * torch.randn(1, 1, g, d, generator=gen)).to(torch.bfloat16)
    v = torch.randn(b, t, g, d, generator=gen).to(torch.bfloat16)
    return q, k, v


def _single_gpu(eng, q, k, v):
    b, t, h, d = q.shape
    g = k.shape[2]
    ws = eng.workspace(sage.Shape(b, h, t, g, True))
    out = torch.zeros(b, t, h, d, dtype=torch.bfloat16, device="cuda")
    sq, skv = sage.Strides.bthd(t, h, d), sage.Strides.bthd(t, g, d)
    eng.forward(ws, sage.Tensor(q.cuda().contiguous(), sq), sage.Tensor(k.cuda().contiguous(), skv),
                sage.Tensor(v.cuda().contiguous(), skv), sage.Tensor(out, sq))
    torch.cuda.synchronize()
    assert eng.status(ws) == 0
    ws.close()
    return out


def _f32(t):
    return O.bf16_to_f32(t.view(torch.int16).cpu().numpy().view(np.uint16))


@pytest.mark.parametrize("schedule", ["ring", "gather"])
def test_native_ring_one_rank_equals_python_ring(schedule):
    b, t, h, g, d = 2, 1024, 8, 2, 128
    q, k, v = (x.cuda() for x in _qkv(b, t, h, g, d, seed=3))
    eng = sage.SageAttention(torch.cuda.current_stream(), d)
    sq, skv = sage.Strides.bthd(t, h, d), sage.Strides.bthd(t, g, d)
    args = (sage.Tensor(q, sq), sage.Tensor(k, skv), sage.Tensor(v, skv))
    nat = sage.NativeRing(eng, b, h, g, t, 0, 1, schedule=schedule)
    out_n = torch.zeros(b, t, h, d, dtype=torch.bfloat16, device="cuda")
    for _ in range(2):  # twice: the ring's buffers carry no state between calls
        nat.forward(*args, sage.Tensor(out_n, sq))
    py = ring.RingAttention(eng, b, h, g, t, 0, 1, d, schedule=schedule)
    out_p = torch.zeros_like(out_n)
    py.forward(*args, sage.Tensor(out_p, sq))
    torch.cuda.synchronize()
    assert torch.equal(out_n, out_p)
    single = _single_gpu(eng, q, k, v)
    e = O.errors(_f32(out_n), _f32(single))
    assert st.attention_gate(e), e
    nat.close()
    py.close()
    with pytest.raises(sage.SageError):
        sage.NativeRing(eng, b, h, g, 1000, 0, 1)  # not two chunks of whole tiles
    with pytest.raises(sage.SageError):
        sage.NativeRing(eng, b, h, g, t, 0, 1, schedule="tree")


class _UniqueId(ctypes.Structure):
    _fields_ = [("internal", ctypes.c_byte * 128)]


def _rank(rank, world, uid_q, res_q, shape, schedule="ring"):
    torch.cuda.set_device(rank)
    nccl = ctypes.CDLL("libnccl.so.2")
    if rank == 0:
        uid = _UniqueId()
        assert nccl.ncclGetUniqueId(ctypes.byref(uid)) == 0
        for _ in range(world - 1):
            uid_q.put(bytes(uid.internal))
    else:
        uid = _UniqueId()
        ctypes.memmove(uid.internal, uid_q.get(timeout=120), 128)
    comm = ctypes.c_void_p()
    assert nccl.ncclCommInitRank(ctypes.byref(comm), world, uid, rank) == 0
    b, t_all, h, g, d = shape
    t = t_all // world
    q, k, v = _qkv(b, t_all, h, g, d, seed=11)
    qs, ks, vs = (ring.shard_zigzag(x, rank, world).cuda() for x in (q, k, v))
    eng = sage.SageAttention(torch.cuda.current_stream(), d)
    nat = sage.NativeRing(eng, b, h, g, t, rank, world, schedule=schedule)
    out = torch.zeros(b, t, h, d, dtype=torch.bfloat16, device="cuda")
    sq, skv = sage.Strides.bthd(t, h, d), sage.Strides.bthd(t, g, d)
    nat.forward(sage.Tensor(qs, sq), sage.Tensor(ks, skv), sage.Tensor(vs, skv), sage.Tensor(out, sq),
                comm=comm.value)
    torch.cuda.synchronize()
    nat.close()
    nccl.ncclCommDestroy(comm)
    res_q.put((rank, out.view(torch.int16).cpu().numpy()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("schedule", ["ring", "gather"])
def test_native_ring_two_ranks_over_nccl(schedule):
    world, shape = 2, (1, 4096, 8, 2, 128)
    ctx = mp.get_context("spawn")
    uid_q, res_q = ctx.Queue(), ctx.Queue()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    procs = [ctx.Process(target=_rank, args=(r, world, uid_q, res_q, shape, schedule)) for r in range(world)]
    for p in procs:
        p.start()
    outs = {}
    for _ in range(world):
        r, o = res_q.get(timeout=300)
        outs[r] = torch.from_numpy(o).view(torch.bfloat16)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    full = ring.unshard_zigzag([outs[r] for r in range(world)], world, dim=1)
    b, t, h, g, d = shape
    q, k, v = _qkv(b, t, h, g, d, seed=11)
    single = _single_gpu(sage.SageAttention(torch.cuda.current_stream(), d), q, k, v)
    e = O.errors(_f32(full), _f32(single))
    assert st.attention_gate(e), e


def _py_rank(rank, world, port, res_q, shape, schedule):
    import datetime

    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        b, t_all, h, g, d = shape
        t = t_all // world
        q, k, v = _qkv(b, t_all, h, g, d, seed=13)
        qs, ks, vs = (ring.shard_zigzag(x, rank, world).cuda() for x in (q, k, v))
        eng = sage.SageAttention(torch.cuda.current_stream(), d)
        rg = ring.RingAttention(eng, b, h, g, t, rank, world, d, schedule=schedule)
        out = torch.zeros(b, t, h, d, dtype=torch.bfloat16, device="cuda")
        sq, skv = sage.Strides.bthd(t, h, d), sage.Strides.bthd(t, g, d)
        for _ in range(2):
            rg.forward(sage.Tensor(qs, sq), sage.Tensor(ks, skv), sage.Tensor(vs, skv), sage.Tensor(out, sq))
        torch.cuda.synchronize()
        assert eng.status(rg.ws) == 0
        rg.close()
        res_q.put((rank, out.view(torch.int16).cpu().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("schedule", ["gather", "ring"])
def test_python_cp_two_ranks_over_nccl(schedule):
    """RingAttention over torch.distributed NCCL on two GPUs, both schedules:
    the zig-zag shards put back together against single-GPU causal
    attention."""
    import socket
    world, shape = 2, (1, 4096, 8, 2, 128)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    res_q = ctx.Queue()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    procs = [ctx.Process(target=_py_rank, args=(r, world, port, res_q, shape, schedule)) for r in range(world)]
    for p in procs:
        p.start()
    outs = {}
    for _ in range(world):
        r, o = res_q.get(timeout=300)
        outs[r] = torch.from_numpy(o).view(torch.bfloat16)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    full = ring.unshard_zigzag([outs[r] for r in range(world)], world, dim=1)
    b, t, h, g, d = shape
    q, k, v = _qkv(b, t, h, g, d, seed=13)
    single = _single_gpu(sage.SageAttention(torch.cuda.current_stream(), d), q, k, v)
    e = O.errors(_f32(full), _f32(single))
    print(f"{schedule} at two ranks vs single GPU: {e}")
    assert st.attention_gate(e), e
