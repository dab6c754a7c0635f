"""Host logic of the context-parallel ring (sota-papers-lab_b200/ring.py), on
CPU: the zig-zag schedule, the sharding helpers and, with world_size 2 on
gloo, the K/V exchange and the statistics combination the GPU run uses."""
from __future__ import annotations

import importlib
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ring = importlib.import_module("sota-papers-lab_b200.ring")


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_schedule_covers_every_visible_chunk_pair_once(world):
    for rank in range(world):
        seen = []
        for src, pairs in ring.ring_schedule(rank, world):
            for p in pairs:
                cq = ring.zigzag_chunks(rank, world)[p.q_local]
                ck = ring.zigzag_chunks(src, world)[p.k_local]
                assert ck <= cq
                assert p.causal == (ck == cq)
                seen.append((cq, ck))
        want = [(cq, ck) for cq in ring.zigzag_chunks(rank, world) for ck in range(2 * world) if ck <= cq]
        assert sorted(seen) == sorted(want)
        # the first step attends the rank's own K/V
        assert ring.ring_schedule(rank, world)[0][0] == rank


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_segments_cover_the_scheduled_pairs(world):
    """One launch per step: each step's segment covers exactly that step's
    chunk pairs, with the same masks."""
    for rank in range(world):
        segs = ring.ring_segments(rank, world)
        sched = ring.ring_schedule(rank, world)
        assert len(segs) == len(sched) == world
        for (src, seg), (src2, pairs) in zip(segs, sched):
            assert src == src2
            assert sorted(ring.segment_pairs(seg), key=str) == sorted(pairs, key=str)
            assert seg.q_chunk + seg.q_chunks <= 2 and seg.k_chunk + seg.k_chunks <= 2
        # the first step covers every local query row (it writes the accumulator)
        assert segs[0][1].q_chunk == 0 and segs[0][1].q_chunks == 2


@pytest.mark.parametrize("world", [2, 4, 8])
def test_zigzag_balances_causal_work(world):
    # key chunks seen per rank, a diagonal chunk counting one half
    work = []
    for rank in range(world):
        w = 0.0
        for _, pairs in ring.ring_schedule(rank, world):
            w += sum(0.5 if p.causal else 1.0 for p in pairs)
        work.append(w)
    assert max(work) == min(work)


@pytest.mark.parametrize("world", [1, 2, 4])
def test_shard_unshard_round_trip(world):
    x = torch.arange(2 * 3 * 16 * world * 4, dtype=torch.float32).view(2, 16 * world, 3, 4)
    parts = [ring.shard_zigzag(x, r, world, dim=1) for r in range(world)]
    assert all(p.shape == (2, 16, 3, 4) for p in parts)
    assert torch.equal(ring.unshard_zigzag(parts, world, dim=1), x)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r = importlib.import_module("sota-papers-lab_b200.ring")
        # the ring's exchange: after s steps each rank holds rank (r - s)'s buffers
        ex = r.nccl_exchange()
        cur = [torch.full((3,), float(rank)), torch.full((2,), 10.0 + rank)]
        nxt = [torch.zeros(3), torch.zeros(2)]
        held = []
        for s, (src, _) in enumerate(r.ring_schedule(rank, world)):
            held.append((src, int(cur[0][0].item()), int(cur[1][0].item()) - 10))
            if s + 1 < world:
                ex(cur, nxt)()
                cur, nxt = nxt, cur
        # statistics: sums added, -min / max maxed
        raw = torch.tensor([[[1.0 + rank], [2.0 * rank], [-(5.0 - rank)], [3.0 * rank]]])  # [1][4][1]
        r.combine_stats(raw, world)
        q.put((rank, held, raw.flatten().tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_exchange_and_statistics_over_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, held, raw = q.get(timeout=120)
        results[rank] = (held, raw)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, (held, raw) in results.items():
        for src, a, b in held:
            assert a == src and b == src  # the K/V of the scheduled source rank
        assert raw[0] == sum(1.0 + r for r in range(world))
        assert raw[1] == sum(2.0 * r for r in range(world))
        assert raw[2] == max(-(5.0 - r) for r in range(world))
        assert raw[3] == max(3.0 * r for r in range(world))


def test_native_schedule_is_the_python_schedule(sage):
    """The ring inside the library (spl_sage_ring_segment, the schedule
    spl_sage_ring_forward follows) attends, at every step of every rank,
    the segment the Python ring attends, for 1 to 8 ranks."""
    C = 384
    for world in range(1, 9):
        for rank in range(world):
            for step, (src, seg) in enumerate(ring.ring_segments(rank, world)):
                flags = (sage.CP_CAUSAL if seg.causal else 0) | (sage.CP_FIRST if step == 0 else 0)
                want = (seg.q_chunk * C, seg.q_chunks * C, seg.k_chunk * C, seg.k_chunks * C, flags)
                assert sage.ring_segment(rank, world, step, C) == want, (world, rank, step)
    for bad in ((0, 0, 0, C), (2, 2, 0, C), (0, 2, 2, C), (0, 2, 0, 0), (-1, 2, 0, C)):
        with pytest.raises(sage.SageError):
            sage.ring_segment(*bad)


class _Buf:
    def __init__(self, tensors):
        self._t = tensors

    def tensors(self):
        return self._t


def _local_kv(rank, world, B, G, C, D):
    """A rank's local K/V buffers whose every key carries its global position
    (k8 and v8 bytes = position % 251, k_scale = global 64-key group)."""
    pos = torch.cat([torch.arange(c * C, (c + 1) * C) for c in ring.zigzag_chunks(rank, world)])  # [2C]
    k8 = (pos % 251).to(torch.uint8).view(1, 1, 2 * C, 1).expand(B, G, 2 * C, D).contiguous()
    v8 = (pos % 251).to(torch.uint8).view(1, 1, 1, 2 * C).expand(B, G, D, 2 * C).contiguous()
    ks = (pos[::64] // 64).to(torch.float32).view(1, 1, 2 * C // 64).expand(B, G, 2 * C // 64).contiguous()
    return [k8.flatten(), ks.flatten(), v8.flatten()]


def _check_whole(whole, world, B, G, C, D):
    n = 2 * world * C
    pos = torch.arange(n)
    k8, ks, v8 = whole
    assert torch.equal(k8.view(B, G, n, D), (pos % 251).to(torch.uint8).view(1, 1, n, 1).expand(B, G, n, D))
    assert torch.equal(v8.view(B, G, D, n), (pos % 251).to(torch.uint8).view(1, 1, 1, n).expand(B, G, D, n))
    assert torch.equal(ks.view(B, G, n // 64), (pos[::64] // 64).to(torch.float32).view(1, 1, -1).expand(B, G, -1))


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_gathered_layout_is_global_key_order(world):
    """layout_gathered puts every rank's two zig-zag chunks at their global
    key positions in the whole-sequence K/V buffer (k8, k_scale, v8)."""
    B, G, C, D = 2, 3, 128, 16
    parts = [torch.cat([_local_kv(r, world, B, G, C, D)[j] for r in range(world)]) for j in range(3)]
    n = 2 * world * C
    whole = [torch.zeros(B * G * n * D, dtype=torch.uint8), torch.zeros(B * G * n // 64),
             torch.zeros(B * G * D * n, dtype=torch.uint8)]
    ring.layout_gathered(parts, _Buf(whole), world, B, G, C, D)
    _check_whole(whole, world, B, G, C, D)


def _gather_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r = importlib.import_module("sota-papers-lab_b200.ring")
        B, G, C, D = 1, 2, 128, 8
        local = _local_kv(rank, world, B, G, C, D)
        staging = [torch.empty(t.numel() * world, dtype=t.dtype) for t in local]
        n = 2 * world * C
        whole = [torch.zeros(B * G * n * D, dtype=torch.uint8), torch.zeros(B * G * n // 64),
                 torch.zeros(B * G * D * n, dtype=torch.uint8)]
        r.gather_kv(_Buf(local), _Buf(whole), staging, world, B, G, C, D)
        _check_whole(whole, world, B, G, C, D)
        q.put((rank, True))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gather_kv_over_gloo(world):
    """The all-gather of the gather schedule with real ranks (gloo): every
    rank ends with the whole sequence's K/V in key order."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(v is True for v in got.values()), got
