"""Context-parallel (ring) SageAttention over several GPUs, one process per
GPU.  No counterpart in the reference, which runs a sequence on one GPU.

The sequence of N tokens is cut into 2P chunks of C = N / (2P) tokens; rank r
holds chunks r and 2P-1-r ("zig-zag", so that every rank has the same causal
work).  Its Q, K and V are those 2C tokens, chunk r first.

1. Every rank quantises its Q and reduces its K/V channel statistics; the
   statistics are combined over all ranks (one all-reduce of sums, one of
   maxima), so every rank smooths and scales K/V with the whole sequence's
   mean and range; then each rank quantises its own K/V.
2. P steps: at step s rank r holds the quantised K/V of rank (r - s) mod P,
   attends its two query chunks to that rank's two key chunks (a pair of
   chunks is skipped when the key chunk lies after the query chunk, causal
   when they are the same chunk, full otherwise) and merges the result into
   an fp32 accumulator by log-sum-exp.  The pairs of a step always form one
   contiguous segment of queries and keys (ring_segments), so a step is one
   launch: step 0 is causal attention over the rank's own 2C tokens (in
   local order, chunk r then chunk 2P-1-r, the causal mask is exactly the
   global one) and writes the accumulator; a later step attends either both
   query chunks to the sender's first key chunk (sender before r) or the
   second query chunk to both key chunks (sender after r), unmasked.
   Meanwhile the K/V it holds travels to rank r + 1 and the next arrives
   from rank r - 1 (NCCL send/recv, on NCCL's own stream, double-buffered):
   the transfer of ~2 * C * Hkv * D bytes overlaps the attention of the
   step.  The attention kernels are persistent (one CTA per SM for the
   whole launch), so NCCL's kernel would find no free SM until the step
   ends; the ring therefore runs NCCL in its own group capped at
   NCCL_CTAS CTAs and has the attention leave that many SMs free
   (reserve_sms).
3. The accumulator is converted to bf16.

With P = 1 this is one GPU attending the whole sequence in two chunks.

schedule="gather" replaces step 2: the ranks all-gather their quantised K/V
(about 2 * C * Hkv * D bytes each) into a buffer of the whole sequence in
key order, and each rank attends its two query chunks to it in ONE causal
launch (spl_sage_cp_attend_gathered): no per-step merge into an fp32
accumulator, no per-step launch tail, and the zig-zag split still gives
every rank the same work.  The transfer is not overlapped with attention
(the launch needs every key), but on NVSwitch it takes well under a
millisecond against a step of tens.
"""
from __future__ import annotations

import importlib
from dataclasses import dataclass
from typing import Callable, List, Sequence, Tuple


def zigzag_chunks(rank: int, world: int) -> Tuple[int, int]:
    """The two global chunk indices (of 2 * world) rank holds, in local order."""
    return rank, 2 * world - 1 - rank


@dataclass(frozen=True)
class Pair:
    q_local: int   # 0 or 1: which of this rank's chunks is the query
    k_local: int   # 0 or 1: which of the source rank's chunks is the key
    causal: bool   # same global chunk: causal mask within it


def ring_schedule(rank: int, world: int) -> List[Tuple[int, List[Pair]]]:
    """For each step: the rank whose K/V this rank holds, and the chunk
    pairs to attend.  Across the steps every (query chunk, key chunk) pair
    with the key chunk at or before the query chunk appears exactly once."""
    steps = []
    for s in range(world):
        src = (rank - s) % world
        pairs = []
        for qi, cq in enumerate(zigzag_chunks(rank, world)):
            for ki, ck in enumerate(zigzag_chunks(src, world)):
                if ck > cq:
                    continue
                pairs.append(Pair(qi, ki, ck == cq))
        steps.append((src, pairs))
    return steps


@dataclass(frozen=True)
class Segment:
    q_chunk: int   # first query chunk (local, 0 or 1)
    q_chunks: int  # query chunks (1 or 2)
    k_chunk: int   # first key chunk of the source rank (0 or 1)
    k_chunks: int  # key chunks (1 or 2)
    causal: bool


def ring_segments(rank: int, world: int) -> List[Tuple[int, Segment]]:
    """ring_schedule with each step's chunk pairs as one contiguous segment
    (one attention launch per step)."""
    steps = []
    for s, (src, pairs) in enumerate(ring_schedule(rank, world)):
        if s == 0:
            seg = Segment(0, 2, 0, 2, True)
        elif src < rank:
            seg = Segment(0, 2, 0, 1, False)
        else:
            seg = Segment(1, 1, 0, 2, False)
        steps.append((src, seg))
    return steps


def segment_pairs(seg: Segment) -> List[Pair]:
    """The chunk pairs a segment covers (for a causal segment over both
    chunks: the pairs its local causal mask leaves visible)."""
    out = []
    for qi in range(seg.q_chunk, seg.q_chunk + seg.q_chunks):
        for ki in range(seg.k_chunk, seg.k_chunk + seg.k_chunks):
            if seg.causal and ki > qi:
                continue
            out.append(Pair(qi, ki, seg.causal and ki == qi))
    return out


def shard_zigzag(x, rank: int, world: int, dim: int = 1):
    """This rank's two chunks of a full-sequence tensor, concatenated."""
    import torch
    n = x.shape[dim]
    c = n // (2 * world)
    a, b = zigzag_chunks(rank, world)
    return torch.cat([x.narrow(dim, a * c, c), x.narrow(dim, b * c, c)], dim=dim).contiguous()


def unshard_zigzag(parts: Sequence, world: int, dim: int = 1):
    """Inverse of shard_zigzag over all ranks' outputs."""
    import torch
    c = parts[0].shape[dim] // 2
    chunks = [None] * (2 * world)
    for r, p in enumerate(parts):
        a, b = zigzag_chunks(r, world)
        chunks[a] = p.narrow(dim, 0, c)
        chunks[b] = p.narrow(dim, c, c)
    return torch.cat(chunks, dim=dim)


def nccl_exchange(group=None):
    """send(bufs) to rank + 1 and recv(into) from rank - 1 with torch.distributed
    P2P ops; returns a function (send_bufs, recv_bufs) -> a wait() callable."""
    import torch.distributed as dist

    def exchange(send_bufs, recv_bufs):
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        nxt, prv = (rank + 1) % world, (rank - 1) % world
        if group is not None:
            nxt = dist.get_global_rank(group, nxt)
            prv = dist.get_global_rank(group, prv)
        ops = []
        for t in send_bufs:
            ops.append(dist.P2POp(dist.isend, t, nxt, group))
        for t in recv_bufs:
            ops.append(dist.P2POp(dist.irecv, t, prv, group))
        works = dist.batch_isend_irecv(ops)

        def wait():
            for w in works:
                w.wait()
        return wait
    return exchange


# NCCL kernels of the ring's process group use at most this many CTAs, and
# the attention leaves as many SMs free during the ring steps (measured on
# 8 B200s, C5: 1 CTA + 1 SM 18.0 ms per step; 2 + 2 18.6; 8 + 8 19.3;
# NCCL's default with none free 20.5)
NCCL_CTAS = 1
RESERVED_SMS = NCCL_CTAS


def nccl_ring_group(ranks=None):
    """A new NCCL process group over `ranks` (default all) whose kernels use
    at most NCCL_CTAS CTAs; every rank must call it (a collective)."""
    import torch.distributed as dist
    o = dist.ProcessGroupNCCL.Options()
    o.config.max_ctas = NCCL_CTAS
    o.config.min_ctas = 1
    if ranks is None:
        ranks = list(range(dist.get_world_size()))
    return dist.new_group(ranks, pg_options=o)


def combine_stats(raw, world: int, group=None):
    """raw [b*g, 4, D] summed (entries 0-1) and maxed (2-3) over the ranks."""
    if world == 1:
        return raw
    import torch.distributed as dist
    sums = raw[:, :2].contiguous()
    maxs = raw[:, 2:].contiguous()
    dist.all_reduce(sums, op=dist.ReduceOp.SUM, group=group)
    dist.all_reduce(maxs, op=dist.ReduceOp.MAX, group=group)
    raw[:, :2].copy_(sums)
    raw[:, 2:].copy_(maxs)
    return raw


def gather_kv(local, whole, staging, world: int, batch: int, kv_heads: int, chunk: int, head_dim: int,
              group=None):
    """All-gather every rank's quantised K/V buffer `local` (its chunks r and
    2P-1-r, local order) and lay the result out in `whole` in global key
    order.  staging: three flat CUDA tensors of world x the local sizes (or
    None at world 1)."""
    if world > 1:
        import torch.distributed as dist
        for dst, src in zip(staging, local.tensors()):
            dist.all_gather_into_tensor(dst, src, group=group)
        parts = staging
    else:
        parts = local.tensors()
    layout_gathered(parts, whole, world, batch, kv_heads, chunk, head_dim)


def layout_gathered(parts, whole, world: int, batch: int, kv_heads: int, chunk: int, head_dim: int):
    """The gathered buffers `parts` (every rank's k8, k_scale, v8 one after
    the other, rank order) copied into `whole` in global key order: rank s's
    local chunk 0 is global chunk s, its chunk 1 global chunk 2P-1-s.
    Layouts: k8 [b][g][t][D], k_scale [b][g][t/64], v8 [b][g][D][t], t the
    buffer's keys."""
    import torch
    B, G, C, D, P = batch, kv_heads, chunk, head_dim, world
    dev = parts[0].device
    first = torch.arange(P, device=dev)                 # rank s's chunk s
    second = 2 * P - 1 - torch.arange(P, device=dev)    # rank s's chunk 2P-1-s
    # per tensor: the gathered view [P][b][g]..[2][C].., whole's view, the
    # dimension of the local chunk index in the first, of the chunk in the second
    views = (((P, B, G, 2, C, D), (B, G, 2 * P, C, D), 3, 2),
             ((P, B, G, 2, C // 64), (B, G, 2 * P, C // 64), 3, 2),
             ((P, B, G, D, 2, C), (B, G, D, 2 * P, C), 4, 3))
    for src, dst, (sv, dv, cdim, gdim) in zip(parts, whole.tensors(), views):
        x, y = src.view(*sv), dst.view(*dv)
        for c, idx in ((0, first), (1, second)):
            y.index_copy_(gdim, idx, x.select(cdim, c).movedim(0, gdim))


def _torch_stream(stream):
    """The torch stream object of an engine stream (a torch stream, a raw
    cudaStream_t as an int, or None for the legacy default stream)."""
    import torch
    if stream is None:
        return torch.cuda.default_stream()
    if isinstance(stream, int):
        return torch.cuda.ExternalStream(stream) if stream else torch.cuda.default_stream()
    return stream


class RingAttention:
    """Ring attention of one rank.  Holds the workspace (this rank's tokens),
    two K/V buffers (the one being attended, the one being received) and the
    fp32 accumulator; reuse it for every call of the same shape.

    group: the process group of the ring's NCCL calls; by default (world > 1
    with torch.distributed initialised) the ring makes its own with
    nccl_ring_group(), so construct the ring on every rank together.
    reserved_sms: SMs the attention leaves free during the steps (default
    RESERVED_SMS when there is a transfer, else 0); it must cover the CTAs
    of the group's NCCL kernels."""

    def __init__(self, eng, batch: int, heads: int, kv_heads: int, local_tokens: int, rank: int, world: int,
                 head_dim: int, reserved_sms: int | None = None, group=None, schedule: str = "ring"):
        import torch
        sage = importlib.import_module("sota-papers-lab_b200")
        if local_tokens % 256:
            raise sage.SageError(1, "each rank's tokens must be two chunks of whole 128-token tiles")
        if schedule not in ("ring", "gather"):
            raise sage.SageError(1, f"unknown context-parallel schedule {schedule!r}")
        self.sage, self.eng = sage, eng
        self.schedule = schedule
        self.rank, self.world = rank, world
        self.B, self.H, self.G, self.T, self.D = batch, heads, kv_heads, local_tokens, head_dim
        self.C = local_tokens // 2
        # SMs left free during the ring steps (none without a transfer
        # overlapping the attention)
        default_reserved = RESERVED_SMS if world > 1 and schedule == "ring" else 0
        self.reserved_sms = default_reserved if reserved_sms is None else reserved_sms
        self.group, self._own_group = group, False
        if group is None and world > 1 and schedule == "ring":
            import torch.distributed as dist
            if dist.is_available() and dist.is_initialized() and dist.get_backend() == "nccl":
                self.group, self._own_group = nccl_ring_group(), True
        # the segments launch through an engine of their own on the same
        # stream that leaves the reserved SMs free, so the caller's engine is
        # never changed (other threads may use it meanwhile)
        self.seg_eng = eng
        if self.reserved_sms:
            self.seg_eng = sage.SageAttention(eng.stream, head_dim, eng.config)
            self.seg_eng.reserve_sms(self.reserved_sms)
        self.ws = eng.workspace(sage.Shape(batch, heads, local_tokens, kv_heads, False))
        self.kv = [sage.KvBuffer(eng, self.ws)] + ([sage.KvBuffer(eng, self.ws)] if schedule == "ring" else [])
        self.kv_all, self.staging = None, None
        if schedule == "gather":
            self.kv_all = sage.KvBuffer(eng, self.ws, tokens=local_tokens * world)
            if world > 1:
                self.staging = [torch.empty(t.numel() * world, dtype=t.dtype, device=t.device)
                                for t in self.kv[0].tensors()]
        self.raw = torch.empty(batch * kv_heads, 4, head_dim, dtype=torch.float32, device="cuda")
        self.acc = torch.empty(batch, local_tokens, heads, head_dim, dtype=torch.float32, device="cuda")
        self.lse = torch.empty(batch, heads, local_tokens, dtype=torch.float32, device="cuda")

    def forward(self, q, k, v, out, *, exchange: Callable | None = None, group=None, opts=None,
                combine: Callable | None = None):
        """q, k, v, out: this rank's tokens (sage.Tensor views); exchange: the
        K/V transfer (default NCCL P2P over `group`, default the ring's own);
        combine: the statistics reduction (default all-reduce over `group`).

        torch.distributed orders its collectives and P2P calls against
        torch's current stream only, so the body runs with the engine's
        stream made current: the statistics all-reduce and the K/V exchange
        then follow the kernels that produce what they send."""
        import torch
        with torch.cuda.stream(_torch_stream(self.eng.stream)):
            self._forward(q, k, v, out, exchange, group, opts, combine)

    def _forward(self, q, k, v, out, exchange, group, opts, combine):
        if self.schedule == "gather":
            return self._forward_gather(q, k, v, out, group, opts, combine)
        P, r = self.world, self.rank
        if group is None:
            group = self.group
        self.eng.cp_prepare(self.ws, q, k, v, self.raw, opts)
        if combine is not None:
            combine(self.raw)
        else:
            combine_stats(self.raw, P, group)
        self.eng.cp_quantize_kv(self.ws, k, v, self.raw, self.T * P, self.kv[0], opts)
        if exchange is None and P > 1:
            exchange = nccl_exchange(group)
        cur = 0
        for s, (src, seg) in enumerate(ring_segments(r, P)):
            wait = None
            if s + 1 < P:
                wait = exchange(self.kv[cur].tensors(), self.kv[1 - cur].tensors())
            self.attend_segment(self.kv[cur], seg, first=s == 0)
            if wait is not None:
                wait()
                cur = 1 - cur
        self.eng.cp_finish(self.ws, self.acc, out)

    def _forward_gather(self, q, k, v, out, group, opts, combine):
        P, r = self.world, self.rank
        self.eng.cp_prepare(self.ws, q, k, v, self.raw, opts)
        if combine is not None:
            combine(self.raw)
        else:
            combine_stats(self.raw, P, group)
        self.eng.cp_quantize_kv(self.ws, k, v, self.raw, self.T * P, self.kv[0], opts)
        gather_kv(self.kv[0], self.kv_all, self.staging, P, self.B, self.G, self.C, self.D, group)
        self.attend_gathered(out)

    def attend_gathered(self, out):
        a, b = zigzag_chunks(self.rank, self.world)
        self.eng.cp_attend_gathered(self.ws, self.kv_all, a * self.C, b * self.C, out)

    def attend_segment(self, kv, seg: Segment, first: bool):
        C = self.C
        self.seg_eng.cp_attend(self.ws, kv, seg.q_chunk * C, seg.q_chunks * C, seg.k_chunk * C, seg.k_chunks * C,
                               seg.causal, self.acc, self.lse, first=first)

    def close(self):
        for kv in self.kv:
            kv.close()
        if self.kv_all is not None:
            self.kv_all.close()
            self.kv_all = None
        self.ws.close()
        if self.seg_eng is not self.eng:
            self.seg_eng.close()
            self.seg_eng = self.eng
        if self._own_group:
            import torch.distributed as dist
            dist.destroy_process_group(self.group)
            self._own_group, self.group = False, None


def emulate_ring(rings: Sequence[RingAttention], qs, ks, vs, outs, opts=None):
    """All ranks of a ring in one process on one GPU (for tests): the
    statistics are combined and the K/V "exchanged" by copies, in the same
    order as the multi-GPU run."""
    import torch
    P = len(rings)
    for i, rg in enumerate(rings):
        rg.eng.cp_prepare(rg.ws, qs[i], ks[i], vs[i], rg.raw, opts)
    total = torch.stack([rg.raw for rg in rings])
    comb = torch.cat([total[:, :, :2].sum(0), total[:, :, 2:].amax(0)], dim=1)
    for i, rg in enumerate(rings):
        rg.raw.copy_(comb)
        rg.eng.cp_quantize_kv(rg.ws, ks[i], vs[i], rg.raw, rg.T * P, rg.kv[0], opts)
    for i, rg in enumerate(rings):
        for s, (src, seg) in enumerate(ring_segments(i, P)):
            rg.attend_segment(rings[src].kv[0], seg, first=s == 0)
        rg.eng.cp_finish(rg.ws, rg.acc, outs[i])


def emulate_gather(rings: Sequence[RingAttention], qs, ks, vs, outs, opts=None):
    """All ranks of a gather-schedule job in one process on one GPU (for
    tests): the statistics combined and the quantised K/V "all-gathered" by
    a concatenation (what all_gather_into_tensor leaves on every rank), laid
    out in every rank's whole-sequence buffer, then each rank's one launch."""
    import torch
    P = len(rings)
    for i, rg in enumerate(rings):
        rg.eng.cp_prepare(rg.ws, qs[i], ks[i], vs[i], rg.raw, opts)
    total = torch.stack([rg.raw for rg in rings])
    comb = torch.cat([total[:, :, :2].sum(0), total[:, :, 2:].amax(0)], dim=1)
    for i, rg in enumerate(rings):
        rg.raw.copy_(comb)
        rg.eng.cp_quantize_kv(rg.ws, ks[i], vs[i], rg.raw, rg.T * P, rg.kv[0], opts)
    staging = [torch.cat([rings[s].kv[0].tensors()[j] for s in range(P)]) for j in range(3)]
    for i, rg in enumerate(rings):
        layout_gathered(staging, rg.kv_all, P, rg.B, rg.G, rg.C, rg.D)
        rg.attend_gathered(outs[i])
