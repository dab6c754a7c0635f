"""Benchmark of the SageAttention2 hot path on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload C4]

One step = one SageAttention::forward (quantise Q/K/V, then INT8/FP8
attention) over one batch of the workload, through the library's public API.
The default workload is the one BASELINE.json's metric is quoted on: C4,
Llama-3-8B-shaped causal prefill attention (B4, 32 query heads, 8 KV heads,
N=8192, head dim 128).  The metric is effective attention TOPS,
4*B*H*N^2*D / t (the non-causal count, as the metric defines it).

Multi-GPU: one process per GPU (torchrun).  C4 is head-sharded, as the
path's specification asks: the job is the fixed global C4 batch and its 32
(batch, kv head) units are split over the ranks (each rank all 4 sequences
and 8 / N kv heads with their query heads; no communication), so the
scaling is strong.  C1 and C3 give every rank its own batch (weak scaling).
The C4 line also carries `ring_c5`: the C5 context-parallel ring at the same
rank count (strong scaling over NCCL), and `c4_block`: the whole block from
the activations (fused QKV GEMM with Q quantised in its epilogue, K/V
quantiser, attention) on the rank's heads.

Rank 0 prints ONE JSON line.  `--impl reference` times the reference's CPU
path for this op (its f64 attention plus its quantiser, as restated in
oracle/: the reference's Rust cannot be built here) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# (batch, q heads, kv heads, tokens, head dim, causal, k bias std, outlier fraction)
WORKLOADS = {
    "C1": dict(batch=1, heads=8, kv_heads=8, tokens=1024, d=64, causal=False, k_bias=3.0, outliers=0.0,
               desc="C1: single call, B1 H8 N1024 D64, non-causal, K bias N(0,3^2)"),
    "C2": dict(batch=8, heads=16, kv_heads=16, tokens=1370, d=64, causal=False, k_bias=0.0, outliers=0.0,
               layers=24, hidden=1024,
               desc="C2: ViT-L image encoder, 24 layers of fused QKV GEMM 1024->3072 + B8 H16 N1370 D64 "
                    "non-causal attention"),
    "C3": dict(batch=2, heads=24, kv_heads=24, tokens=16384, d=128, causal=False, k_bias=2.0, outliers=0.01,
               desc="C3: DiT, B2 H24 N16384 D128, non-causal, K bias N(0,2^2), 1% outlier tokens x20"),
    "C4": dict(batch=4, heads=32, kv_heads=8, tokens=8192, d=128, causal=True, k_bias=0.0, outliers=0.0,
               qkv=dict(hidden=4096, rope_theta=500000.0),
               desc="C4: Llama-3-8B prefill attention, B4 Hq32 Hkv8 N8192 D128, causal (GQA)"),
    "C5": dict(batch=1, heads=32, kv_heads=8, tokens=131072, d=128, causal=True, k_bias=2.0, outliers=0.0,
               desc="C5: long-context causal attention, B1 Hq32 Hkv8 N131072 D128, K bias N(0,2^2), context-parallel ring"),
}

METRIC = "effective attention TOPS (4*B*H*N^2*D/t) at N=8k, d=128"


def metric_of(name: str) -> str:
    """A workload's metric, the same string in both arms."""
    if name == "C4":
        return METRIC
    if name == "C2":
        return "effective attention TOPS (4*B*H*N^2*D/t), C2, t = whole QKV path of 24 layers"
    return f"effective attention TOPS (4*B*H*N^2*D/t), {name}"


def tensor_peak(eng):
    """The tcgen05 INT8 and FP8 E4M3 dense rates measured by the library's
    probe (best of two runs each, on a GPU not yet heated by the timed loop):
    the burst figures, for kernels timed on their own."""
    i8 = max(eng.tensor_peak(0, 128)[0] for _ in range(2))
    f8 = max(eng.tensor_peak(1, 128)[0] for _ in range(2))
    return i8, f8


def fp16_accumulate_rate(eng):
    """The FP8 E4M3 rate with an FP16 accumulator (SageAttention2++'s PV,
    PvAccum::F16) beside the FP32 one, from the same probe."""
    return max(eng.tensor_peak(3, 128)[0] for _ in range(2))


def effective_flops(w, batch):
    return 4.0 * batch * w["heads"] * w["tokens"] ** 2 * w["d"]


def algorithmic_flops(w, batch):
    n = w["tokens"]
    if w["causal"]:
        return 4.0 * batch * w["heads"] * w["d"] * n * (n + 1) / 2
    return 4.0 * batch * w["heads"] * n * n * w["d"]


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            m = json.load(f)
        return m, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def shard_of(name: str, world: int):
    """(batch, q heads, kv heads) of one rank, and whether the job is
    head-sharded (strong scaling: C4) or batch-replicated (weak)."""
    w = WORKLOADS[name]
    if name == "C4":
        if w["kv_heads"] % world:
            raise SystemExit(f"C4 shards its {w['kv_heads']} kv heads over the ranks: {world} does not divide them")
        return w["batch"], w["heads"] // world, w["kv_heads"] // world, True
    return w["batch"], w["heads"], w["kv_heads"], False


def config_of(name: str, world: int) -> dict:
    """The `config` of a line; the same in both arms."""
    w = WORKLOADS[name]
    B, Hr, Gr, sharded = shard_of(name, world)
    return {"workload": w["desc"], "global_batch": B if sharded else B * world, "seq_len": w["tokens"],
            "q_heads": w["heads"], "kv_heads": w["kv_heads"], "head_dim": w["d"], "causal": w["causal"],
            "parallelism": (f"head-sharded hs{world}: each rank all {B} sequences, {Gr} kv head(s) and its {Hr} "
                            f"query heads" if sharded else f"batch-replicated dp{world}"),
            "l2": "inputs (0.67 GB at C4) exceed the 126 MB L2; no flush"}


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every ~2 ms on a
    background thread while the timed region runs."""

    REASONS = {
        "hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4,
        "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, index):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # NVML missing: report it, do not fail the bench
            self.nv = None
            self.err = str(e)

    def _sample(self):
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for name, bit in self.REASONS.items():
                if r & bit:
                    self.reasons.add(name)
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(0.002)

    def __enter__(self):
        if self.nv is not None:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        # the caller synchronises before leaving the region: one last sample
        # taken here still falls inside it, so short regions get two or more
        if self.nv is not None:
            self._sample()
            self._stop.set()
            self.t.join()

    def summary(self):
        if self.nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable"}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------- inputs

def make_inputs(w, batch, seed, device):
    """Seeded synthetic bf16 Q/K/V [b][t][h][d] on the device: N(0,1) (C4:
    the spread of an N(0,0.02^2)-weight projection of LayerNormed
    activations, std 1.28), K plus a per-channel bias, optional outlier
    tokens."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    t, d = w["tokens"], w["d"]
    std = 1.28 if w["desc"].startswith("C4") else 1.0
    q = torch.randn(batch, t, w["heads"], d, generator=g, device=device) * std
    k = torch.randn(batch, t, w["kv_heads"], d, generator=g, device=device) * std
    v = torch.randn(batch, t, w["kv_heads"], d, generator=g, device=device) * std
    if w["k_bias"]:
        k += torch.randn(1, 1, w["kv_heads"], d, generator=g, device=device) * w["k_bias"]
    if w["outliers"]:
        n_out = max(1, int(w["outliers"] * t))
        idx = torch.randperm(t, generator=g, device=device)[:n_out]
        q[:, idx] *= 20
        k[:, idx] *= 20
    return q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)


# ---------------------------------------------------------------- our arm

def run_layers(args, rank, world, local_rank):
    """C2: per step, 24 ViT-L layers, each the block's whole QKV path up to
    the attention output: fused QKV GEMM (x [B*N][1024] LayerNorm-normalised
    N(0,1), W [3072][1024] ~ N(0, 0.02^2) with bias, a distinct W per
    layer) with the quantiser (spl_sage_qkv_gemm_quant), then the attention.
    Batch sharding over ranks (weak scaling)."""
    import torch
    import torch.distributed as dist
    sage = importlib.import_module("sota-papers-lab_b200")
    w = WORKLOADS[args.workload]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B, H, N, D, Lr, Hd = w["batch"], w["heads"], w["tokens"], w["d"], w["layers"], w["hidden"]
    stream = torch.cuda.current_stream()
    g = torch.Generator(device=dev)
    g.manual_seed(777 + rank)
    x = torch.randn(B * N, Hd, generator=g, device=dev)
    x = ((x - x.mean(1, keepdim=True)) / x.std(1, keepdim=True)).to(torch.bfloat16)
    ws_w = [(torch.randn(3 * H * D, Hd, generator=g, device=dev) * 0.02).to(torch.bfloat16) for _ in range(Lr)]
    ws_b = [(torch.randn(3 * H * D, generator=g, device=dev) * 0.02).to(torch.bfloat16) for _ in range(Lr)]
    q = torch.empty(B, N, H, D, dtype=torch.bfloat16, device=dev)
    k, v = torch.empty_like(q), torch.empty_like(q)
    out = torch.empty_like(q)
    eng = sage.SageAttention(stream, D)
    ws = eng.workspace(sage.Shape(B, H, N, H, False))
    to = sage.Tensor(out, sage.Strides.bthd(N, H, D))

    def layer(i):
        eng.qkv_gemm_quant(ws, x, ws_w[i], ws_b[i], None, q, k, v)
        eng.attend(ws, to)

    def barrier():
        if world > 1:
            dist.barrier()

    peaks_hw = tensor_peak(eng) if rank == 0 else (0.0, 0.0)
    for _ in range(args.warmup):
        for i in range(Lr):
            layer(i)
    torch.cuda.synchronize()
    word = eng.status(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            for i in range(Lr):
                layer(i)
        e1.record(stream)
        torch.cuda.synchronize()
    # attention alone, for the share
    a0.record(stream)
    for _ in range(args.steps):
        for i in range(Lr):
            eng.attend(ws, to)
    a1.record(stream)
    torch.cuda.synchronize()
    barrier()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    attn_ms = a0.elapsed_time(a1) / (args.steps * Lr)

    # the projection alone (bf16 q/k/v out, no quantiser) against the
    # library's linear on the same operands (bias, one [B*N][3072] output, no
    # head scatter), each over the 24 layers' weights
    def per_layer(call):
        for i in range(Lr):
            call(i)
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(args.steps):
            for i in range(Lr):
                call(i)
        g1.record(stream)
        torch.cuda.synchronize()
        return g0.elapsed_time(g1) / (args.steps * Lr)

    gemm_ms = per_layer(lambda i: eng.qkv_gemm(x, ws_w[i], ws_b[i], None, q, k, v, batch=B, tokens=N, heads=H))
    y_lib = torch.empty(B * N, 3 * H * D, dtype=torch.bfloat16, device=dev)
    lib_ms = per_layer(lambda i: torch.addmm(ws_b[i], x, ws_w[i].t(), out=y_lib))
    del y_lib

    # end to end: each step's activations up from pinned host memory, the 24
    # layers, the last layer's attention output back to the host.  As a
    # serving loop runs it: uploads on one stream into two alternating
    # device buffers, the layers on the engine's stream, downloads of each
    # step's last attention output (its own buffer per step parity) on a
    # third, so one step's copies overlap its neighbours' layers; events
    # order every reuse of a buffer.
    xh = x.cpu().pin_memory()
    oh = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    xs = [torch.empty_like(x) for _ in range(2)]
    lasts = [torch.empty_like(out) for _ in range(2)]
    to_last = [sage.Tensor(t_, sage.Strides.bthd(N, H, D)) for t_ in lasts]
    up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731 (ordering only)
    e_steps = max(1, args.steps)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    up.wait_event(e0)
    down.wait_event(e0)
    done_x, done_dl = [None, None], [None, None]
    for s_ in range(e_steps):
        p_ = s_ & 1
        with torch.cuda.stream(up):
            if done_x[p_] is not None:
                up.wait_event(done_x[p_])  # step s - 2 has finished reading xs[p]
            xs[p_].copy_(xh, non_blocking=True)
            up_done = ev()
            up_done.record(up)
        stream.wait_event(up_done)
        for i in range(Lr - 1):
            eng.qkv_gemm_quant(ws, xs[p_], ws_w[i], ws_b[i], None, q, k, v)
            eng.attend(ws, to)
        eng.qkv_gemm_quant(ws, xs[p_], ws_w[Lr - 1], ws_b[Lr - 1], None, q, k, v)
        if done_dl[p_] is not None:
            stream.wait_event(done_dl[p_])  # step s - 2's output is on the host
        eng.attend(ws, to_last[p_])
        done_x[p_] = ev()
        done_x[p_].record(stream)
        with torch.cuda.stream(down):
            down.wait_event(done_x[p_])
            oh[p_].copy_(lasts[p_], non_blocking=True)
            done_dl[p_] = ev()
            done_dl[p_].record(down)
    for d_ in done_dl:
        if d_ is not None:
            stream.wait_event(d_)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item()) / e_steps
    word |= eng.status(ws)
    if rank != 0:
        return None
    step_ms = ms_max / args.steps
    eff = Lr * effective_flops(w, B * world)
    i8_peak, f8_peak = peaks_hw
    peak = min(i8_peak, f8_peak)
    alg = algorithmic_flops(w, B)
    return {
        "metric": metric_of(args.workload),
        "value": round(eff / (step_ms * 1e-3) / 1e12, 2), "unit": "TOPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 GEMM, int8/e4m3 attention (fp32 accumulate)",
        "data": "synthetic (seeded torch.randn on device, LayerNorm-normalised activations)",
        "config": {"workload": w["desc"], "global_batch": B * world, "seq_len": N, "heads": H, "head_dim": D,
                   "layers": Lr, "parallelism": f"batch-sharded dp{world}",
                   "l2": "each layer's weights (6 MB) and activations (22 MB in, 67 MB q/k/v) differ; no flush"},
        "roofline": {"bound": "tensor", "kernel": "sp_attn (D=64)", "achieved": round(alg / (attn_ms * 1e-3) / 1e12, 1),
                     "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(alg / (attn_ms * 1e-3) / 1e12 / peak, 4),
                     "traffic": None, "attn_ms_per_layer": round(attn_ms, 4),
                     "layer_ms": round(step_ms / Lr, 4),
                     "peak_source": "measured in this run by the tcgen05 probe (lower of INT8, FP8 E4M3)"},
        "qkv_gemm": {"kernel": "sp_qkv_gemm_2sm (bias, bf16 q/k/v scattered per head)",
                     "shape": f"[{B * N}x{Hd}] x [{3 * H * D}x{Hd}]^T", "ms": round(gemm_ms, 4),
                     "achieved": round(2.0 * B * N * Hd * 3 * H * D / (gemm_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                     "library_addmm_ms": round(lib_ms, 4),
                     "library": "torch.addmm(bias, x, W^T) into one [B*N][3*H*D] bf16 output (cuBLASLt)",
                     "library_ms_over_ours": round(lib_ms / gemm_ms, 3)},
        "e2e": {"value": round(eff / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TOPS", "ms_per_step": round(e2e_ms, 3),
                "h2d_bytes_per_step": x.numel() * x.element_size(),
                "d2h_bytes_per_step": out.numel() * out.element_size(),
                "api": "qkv_gemm_quant + attend via libsplsage C ABI, 24 layers per step, pinned host buffers; "
                       "uploads, layers and downloads of consecutive steps overlapped on three streams"},
        "gpu_launches": 4 * Lr * args.steps,  # per layer: GEMM, quantiser (sp_prep, sp_quant_kv_stream), attention
        "clocks": clk.summary(),
        "device_error_word": word,
    }


def ring_measure(rank, world, local_rank, steps, warmup, reserve_sms=None, e2e=True, schedule="gather"):
    """The C5 ring (sota-papers-lab_b200/ring.py) on this rank: one long
    causal sequence split over the ranks (zig-zag chunks), K/V passed around
    a ring.  Device time of `steps` forwards (CUDA events on the launching
    stream, max over ranks) and, with e2e, the same through pinned host
    buffers.  Every rank calls it together."""
    import torch
    import torch.distributed as dist
    sage = importlib.import_module("sota-papers-lab_b200")
    ring = importlib.import_module("sota-papers-lab_b200.ring")
    w = WORKLOADS["C5"]
    dev = torch.device("cuda", local_rank)
    B, H, G, N, D = w["batch"], w["heads"], w["kv_heads"], w["tokens"], w["d"]
    T = N // world
    stream = torch.cuda.current_stream()
    # this rank's two chunks of one synthetic sequence: N(0,1) tokens, the
    # per-channel K bias shared by all ranks
    g = torch.Generator(device=dev)
    g.manual_seed(4321 + rank)
    q = torch.randn(B, T, H, D, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(B, T, G, D, generator=g, device=dev)
    v = torch.randn(B, T, G, D, generator=g, device=dev).to(torch.bfloat16)
    gb = torch.Generator(device=dev)
    gb.manual_seed(99)
    k = (k + torch.randn(1, 1, G, D, generator=gb, device=dev) * w["k_bias"]).to(torch.bfloat16)
    out = torch.empty(B, T, H, D, dtype=torch.bfloat16, device=dev)
    eng = sage.SageAttention(stream, D)
    rg = ring.RingAttention(eng, B, H, G, T, rank, world, D, reserved_sms=reserve_sms, schedule=schedule)
    sq, skv = sage.Strides.bthd(T, H, D), sage.Strides.bthd(T, G, D)
    tq, tk, tv, to = sage.Tensor(q, sq), sage.Tensor(k, skv), sage.Tensor(v, skv), sage.Tensor(out, sq)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(ms):
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(warmup):
        rg.forward(tq, tk, tv, to)
    torch.cuda.synchronize()
    word = eng.status(rg.ws)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        e0.record(stream)
        for _ in range(steps):
            rg.forward(tq, tk, tv, to)
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    res = {"ms_per_step": max_over_ranks(e0.elapsed_time(e1)) / steps, "clocks": clk.summary(),
           "reserved_sms": rg.reserved_sms, "nccl_ctas": ring.NCCL_CTAS, "schedule": schedule,
           "h2d": sum(x.numel() * x.element_size() for x in (q, k, v)), "d2h": out.numel() * out.element_size()}
    if e2e:
        # this rank's Q/K/V from pinned host memory, the ring, the rank's
        # output back to the host
        qh, kh, vh = (x.cpu().pin_memory() for x in (q, k, v))
        oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        e_steps = max(1, min(steps, 3))
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(e_steps):
            q.copy_(qh, non_blocking=True); k.copy_(kh, non_blocking=True); v.copy_(vh, non_blocking=True)
            rg.forward(tq, tk, tv, to)
            oh.copy_(out, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        res["e2e_ms"] = max_over_ranks(e0.elapsed_time(e1)) / e_steps
    word |= eng.status(rg.ws)
    res["device_error_word"] = word
    rg.close()
    eng.close()
    return res


def run_ring(args, rank, world, local_rank):
    """C5: one long causal sequence split over the ranks (zig-zag chunks),
    K/V passed around a ring (sota-papers-lab_b200/ring.py).  Strong
    scaling: the whole job is one sequence whatever the rank count."""
    import torch
    sage = importlib.import_module("sota-papers-lab_b200")
    w = WORKLOADS[args.workload]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B, H, G, N, D = w["batch"], w["heads"], w["kv_heads"], w["tokens"], w["d"]
    peaks_hw = tensor_peak(sage.SageAttention(torch.cuda.current_stream(), D)) if rank == 0 else (0.0, 0.0)
    r = ring_measure(rank, world, local_rank, args.steps, args.warmup, args.reserve_sms, schedule=args.cp_schedule)
    if rank != 0:
        return None
    step_ms, e2e_ms = r["ms_per_step"], r["e2e_ms"]
    value = effective_flops(w, B) / (step_ms * 1e-3) / 1e12
    alg_per_rank = algorithmic_flops(w, B) / world
    achieved = alg_per_rank / (step_ms * 1e-3) / 1e12
    i8_peak, f8_peak = peaks_hw
    peak = min(i8_peak, f8_peak)
    return {
        "metric": metric_of(args.workload), "value": round(value, 2),
        "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8/e4m3 (fp32 accumulate; bf16 in/out)", "data": "synthetic (seeded torch.randn on device)",
        "config": {"workload": w["desc"], "global_batch": B,
                   "seq_len": N, "q_heads": H, "kv_heads": G, "head_dim": D, "causal": True,
                   "parallelism": cp_description(world, r),
                   "l2": "inputs exceed the 126 MB L2; no flush"},
        "roofline": {"bound": "tensor", "kernel": "whole ring step per GPU (quantiser, segment attention, merge)",
                     "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "traffic": None,
                     "peak_source": "measured in this run by the tcgen05 probe (lower of INT8, FP8 E4M3)",
                     "algorithmic_flops_per_gpu": alg_per_rank},
        "e2e": {"value": round(effective_flops(w, B) / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TOPS",
                "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": r["h2d"] * world,
                "d2h_bytes_per_step": r["d2h"] * world,
                "api": "RingAttention.forward via libsplsage C ABI, pinned host buffers (every rank its own chunks)"},
        # per forward: prepare 2, K/V quantiser 2, one segment per ring step, finish 1
        "gpu_launches": (5 + world) * args.steps,
        "clocks": r["clocks"],
        "device_error_word": r["device_error_word"],
    }


def cp_description(world, r):
    if r["schedule"] == "gather":
        return (f"cp{world}: zig-zag chunks; the quantised K/V of all ranks all-gathered over NCCL into the whole "
                f"sequence, then one causal attention launch per rank over it")
    return (f"cp{world}: zig-zag chunks, one attention launch per ring step, K/V ring over NCCL send/recv in a "
            f"group capped at {r['nccl_ctas']} CTA(s), {r['reserved_sms']} SM(s) left free for it")


def ring_c5_summary(rank, world, local_rank, peak):
    """The `ring_c5` object of the C4 line: the C5 context-parallel job at
    this rank count, with both schedules (all-gather, the default, and the
    send/recv ring)."""
    w = WORKLOADS["C5"]
    steps = 3
    runs = {sch: ring_measure(rank, world, local_rank, steps, 3, e2e=False, schedule=sch)
            for sch in ("gather", "ring")}
    if rank != 0:
        return None
    alg_per_rank = algorithmic_flops(w, w["batch"]) / world
    r = runs["gather"]
    tops = lambda x: round(effective_flops(w, w["batch"]) / (x["ms_per_step"] * 1e-3) / 1e12, 2)
    return {"workload": w["desc"], "n_gpus": world, "scaling": "strong", "steps": steps, "warmup": 3,
            "ms_per_step": round(r["ms_per_step"], 4), "value": tops(r), "unit": "TOPS",
            "roofline_frac_per_gpu": round(alg_per_rank / (r["ms_per_step"] * 1e-3) / 1e12 / peak, 4) if peak else None,
            "parallelism": cp_description(world, r),
            "send_recv_ring": {"ms_per_step": round(runs["ring"]["ms_per_step"], 4), "value": tops(runs["ring"]),
                               "parallelism": cp_description(world, runs["ring"]),
                               "device_error_word": runs["ring"]["device_error_word"]},
            "timing": "CUDA events on the launching stream, max over ranks", "clocks": r["clocks"],
            "device_error_word": r["device_error_word"]}


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    sage = importlib.import_module("sota-papers-lab_b200")
    w = WORKLOADS[args.workload]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    N, D = w["tokens"], w["d"]
    B, H, G, sharded = shard_of(args.workload, world)  # this rank's share
    wr = dict(w, heads=H, kv_heads=G)
    stream = torch.cuda.current_stream()
    q, k, v = make_inputs(wr, B, 1234 + rank, dev)
    out = torch.empty(B, N, H, D, dtype=torch.bfloat16, device=dev)
    eng = sage.SageAttention(stream, D)
    ws = eng.workspace(sage.Shape(B, H, N, G, w["causal"]))
    sq, skv = sage.Strides.bthd(N, H, D), sage.Strides.bthd(N, G, D)
    tq, tk, tv = sage.Tensor(q, sq), sage.Tensor(k, skv), sage.Tensor(v, skv)
    to = sage.Tensor(out, sq)
    opts = sage.Options()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(ms):
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    peaks_hw = tensor_peak(eng) if rank == 0 else (0.0, 0.0)
    f16acc = fp16_accumulate_rate(eng) if rank == 0 else 0.0
    for _ in range(args.warmup):
        eng.forward(ws, tq, tk, tv, to, opts)
    torch.cuda.synchronize()
    eng.status(ws)

    # device-timed region: K forwards, inputs resident in HBM (Q/K/V/out are
    # 0.67 GB at C4 on one GPU, larger than the 126 MB L2, so no flush)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        start.record(stream)
        for i in range(args.steps):
            ev[i][0].record(stream)
            eng.prepare(ws, tq, tk, tv, opts)
            ev[i][1].record(stream)
            eng.attend(ws, to)
            ev[i][2].record(stream)
        stop.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms_max = max_over_ranks(start.elapsed_time(stop))
    prep_ms = [a.elapsed_time(b) for a, b, _ in ev]
    attn_ms = [b.elapsed_time(c) for _, b, c in ev]
    word = eng.status(ws)

    # the CPU leg (one GPU only): the reference's CPU path timed on a sample
    # of these very inputs, and this run's output checked on the sample
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_leg(wr, B, q, k, v, out, nthreads=os.cpu_count() or 1)

    # end to end through the public API with host buffers, pipelined as a
    # serving loop would run it: step i's Q/K/V go up from pinned memory on
    # one copy stream while step i-1 computes and step i-2's output comes
    # down on another (two device buffer sets; PCIe copies both ways at
    # once).  Every step copies its own inputs and its result inside the
    # timed region, which runs from the first upload to the last download.
    qh, kh, vh = (x.cpu().pin_memory() for x in (q, k, v))
    oh = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    bufs = [(q, k, v, out), (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(out))]
    views = [(sage.Tensor(a, sq), sage.Tensor(bb, skv), sage.Tensor(cc, skv), sage.Tensor(oo, sq))
             for a, bb, cc, oo in bufs]
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def run_e2e(n, first=None):
        down = [None, None]
        for i in range(n):
            sb = i % 2
            if down[sb] is not None:  # step i-2 computed and downloaded: set sb is free
                h2d_s.wait_event(down[sb])
            if i == 0 and first is not None:
                first.record(h2d_s)
            with torch.cuda.stream(h2d_s):
                for dst, src in zip(bufs[sb][:3], (qh, kh, vh)):
                    dst.copy_(src, non_blocking=True)
            up = torch.cuda.Event()
            up.record(h2d_s)
            stream.wait_event(up)
            tq_, tk_, tv_, to_ = views[sb]
            eng.forward(ws, tq_, tk_, tv_, to_, opts)
            done = torch.cuda.Event()
            done.record(stream)
            d2h_s.wait_event(done)
            with torch.cuda.stream(d2h_s):
                oh[sb].copy_(bufs[sb][3], non_blocking=True)
            down[sb] = torch.cuda.Event()
            down[sb].record(d2h_s)

    run_e2e(3)
    torch.cuda.synchronize()
    e_steps = max(2, min(args.steps, 10))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    run_e2e(e_steps, first=e0)
    e1.record(d2h_s)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / e_steps
    word |= eng.status(ws)
    h2d = sum(x.numel() * x.element_size() for x in (q, k, v)) * world
    d2h = out.numel() * out.element_size() * world
    del bufs, views, qh, kh, vh, oh

    block = qkv = qkv8 = ring_sub = None
    if w.get("qkv") and not args.no_extras:
        block = c4_block_time(eng, wr, B, dev, stream, rank, world, max_over_ranks)
        qkv = qkv_gemm_time(eng, w, dev, stream) if rank == 0 else None
        qkv8 = qkv_fp8_time(eng, w, dev, stream) if rank == 0 else None
        del q, k, v, out, ws
        torch.cuda.empty_cache()
        peak_sub = min(peaks_hw) if rank == 0 else 0.0
        ring_sub = ring_c5_summary(rank, world, local_rank, peak_sub)

    if rank != 0:
        return None
    peaks, peak_src = load_peaks()
    cfg = config_of(args.workload, world)
    step_ms = ms_max / args.steps
    value = effective_flops(w, cfg["global_batch"]) / (step_ms * 1e-3) / 1e12
    attn_avg = statistics.mean(attn_ms)
    alg = algorithmic_flops(wr, B)  # one attention launch: this rank's heads
    achieved = alg / (attn_avg * 1e-3) / 1e12
    # The INT8 / FP8 dense tcgen05 rates are not in MEASURED_PEAKS.json: they
    # are measured here by the library's probe (one CTA per SM issuing
    # back-to-back M128 N128 MMAs); the slower of the two is the denominator.
    i8_peak, f8_peak = peaks_hw
    peak = min(i8_peak, f8_peak)
    if qkv is not None:
        qkv["peak"] = peaks["bf16_tflops"]
        qkv["frac"] = round(qkv["achieved"] / peaks["bf16_tflops"], 4)
        if "bf16_tflops_sustained" in peaks:
            qkv["frac_of_sustained"] = round(qkv["achieved"] / peaks["bf16_tflops_sustained"], 4)
        qkv["peak_source"] = f"{peak_src} bf16_tflops (cuBLAS bf16 burst)"
    traffic = None
    tf = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(tf) and world == 1:
        with open(tf) as f:
            traffic = json.load(f).get(args.workload)
    line = {
        "metric": metric_of(args.workload),
        "value": round(value, 2), "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "strong" if sharded else "weak",
        "vs_baseline": None, "dtype": "int8/e4m3 (fp32 accumulate; bf16 in/out)",
        "data": "synthetic (seeded torch.randn on device)", "config": cfg,
        "roofline": {"bound": "tensor", "kernel": "sp_attn (tcgen05 kind::i8 QK + kind::f8f6f4 PV)",
                     "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "peak_source": f"measured in this run by the tcgen05 probe: INT8 {i8_peak:.0f} TOPS, FP8 E4M3 "
                                    f"{f8_peak:.0f} TFLOPS (the lower); for context 2 x {peak_src} cuBLAS bf16 = "
                                    f"{2 * peaks['bf16_tflops']:.0f}",
                     "frac_of_2x_measured_bf16": round(achieved / (2 * peaks["bf16_tflops"]), 4),
                     "algorithmic_flops_per_launch": alg, "attn_ms_avg": round(attn_avg, 4),
                     "prepare_ms_avg": round(statistics.mean(prep_ms), 4),
                     "fp8_rate_with_fp16_accumulator": round(f16acc, 1)},
        "e2e": {"value": round(effective_flops(w, cfg["global_batch"]) / (e2e_ms * 1e-3) / 1e12, 2),
                "unit": "TOPS", "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "api": "SageAttention.forward via libsplsage C ABI, pinned host buffers; uploads, compute and "
                       "downloads of consecutive steps overlapped on three streams (every rank its own share)"},
        "gpu_launches": 3 * args.steps,  # per step: the quantiser (sp_prep, sp_quant_kv_stream), the attention
        "clocks": clk.summary(),
        "device_error_word": word,
    }
    if cpu is not None:
        line["cpu_baseline"], line["parity"] = cpu
    if block is not None:
        line["c4_block"] = block
    if qkv is not None:
        line["qkv_gemm"] = qkv
    if qkv8 is not None:
        qkv8["peak"] = round(f8_peak, 1)
        qkv8["frac"] = round(qkv8["achieved"] / f8_peak, 4)
        qkv8["peak_source"] = "FP8 E4M3 tcgen05 rate measured in this run by the probe"
        qkv8["ln_frac_of_hbm"] = round(qkv8["ln_gbs"] / peaks["hbm_gbs"], 4)
        gc = qkv8["gemm_clocks"]
        if gc.get("sm_mhz") and gc.get("sm_max_mhz"):
            # the probe's rate is a burst at the maximum clock; the GEMM runs
            # long enough to meet the power cap: its rate at the clock it ran at
            qkv8["frac_of_peak_at_its_clock"] = round(qkv8["frac"] * gc["sm_max_mhz"] / gc["sm_mhz"], 4)
        lib = qkv8["library_fp8_gemm"]
        if "ms" in lib:  # > 1: ours (with its RoPE / bf16 scatter epilogue) is faster
            lib["library_ms_over_ours"] = round(lib["ms"] / qkv8["gemm_ms"], 3)
        line["qkv_fp8"] = qkv8
    if ring_sub is not None:
        line["ring_c5"] = ring_sub
    return line


def c4_block_time(eng, wr, B, dev, stream, rank, world, max_over_ranks, iters=5):
    """The C4 block on this rank's heads, from the activations: x [B*N][4096]
    (LayerNorm-normalised N(0,1)) -> the fused QKV GEMM (W [(Hq+2Hkv)*128]
    [4096] ~ N(0, 0.02^2), RoPE theta 5e5) with Q quantised in its epilogue
    and no bf16 Q written (spl_sage_qkv_gemm_quant) -> the K/V quantiser ->
    causal attention.  Also the same block unfused (GEMM writing bf16 Q, K, V,
    then the whole quantiser), so the removed Q round trip shows.  CUDA
    events, max over ranks."""
    import torch
    sage = importlib.import_module("sota-papers-lab_b200")
    H, G, N, D = wr["heads"], wr["kv_heads"], wr["tokens"], wr["d"]
    hidden = wr["qkv"]["hidden"]
    n_out = (H + 2 * G) * D
    g = torch.Generator(device=dev)
    g.manual_seed(97 + rank)
    x = torch.randn(B * N, hidden, generator=g, device=dev)
    x = ((x - x.mean(1, keepdim=True)) / x.std(1, keepdim=True)).to(torch.bfloat16)
    wt = (torch.randn(n_out, hidden, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    rope = torch.from_numpy(sage.rope_table_1d(wr["qkv"]["rope_theta"], D, N)).to(dev)
    q = torch.empty(B, N, H, D, dtype=torch.bfloat16, device=dev)
    k = torch.empty(B, N, G, D, dtype=torch.bfloat16, device=dev)
    v = torch.empty_like(k)
    out = torch.empty_like(q)
    ws = eng.workspace(sage.Shape(B, H, N, G, True))
    sq, skv = sage.Strides.bthd(N, H, D), sage.Strides.bthd(N, G, D)
    to = sage.Tensor(out, sq)

    def fused():
        eng.qkv_gemm_quant(ws, x, wt, None, rope, None, k, v, rope_half=D // 2, frame_len=N)

    def unfused():
        eng.qkv_gemm(x, wt, None, rope, q, k, v, batch=B, tokens=N, heads=H, kv_heads=G, rope_half=D // 2,
                     frame_len=N)
        eng.prepare(ws, sage.Tensor(q, sq), sage.Tensor(k, skv), sage.Tensor(v, skv))

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) / iters)

    t_block = timed(lambda: (fused(), eng.attend(ws, to)))
    t_fused = timed(fused)
    t_unfused = timed(unfused)
    word = eng.status(ws)
    del x, wt, q, k, v, out
    ws.close()
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    full = WORKLOADS["C4"]
    gemm_flops = 2.0 * B * N * hidden * (full["heads"] + 2 * full["kv_heads"]) * D  # whole job
    attn_flops = algorithmic_flops(full, B)
    return {"what": "x -> fused QKV GEMM (Q to INT8 in its epilogue, no bf16 Q) -> K/V quantiser -> causal "
                    "attention, this rank's heads; whole-job rates",
            "ms": round(t_block, 4),
            "value": round(effective_flops(full, B) / (t_block * 1e-3) / 1e12, 2), "unit": "TOPS",
            "tflops_gemm_plus_attention": round((gemm_flops + attn_flops) / (t_block * 1e-3) / 1e12, 1),
            "gemm_quant_ms": round(t_fused, 4), "unfused_gemm_then_quantiser_ms": round(t_unfused, 4),
            "q_round_trip_bytes_removed": B * N * full["heads"] * D * 2 // world * 2,
            "gpu_launches_per_block": 4, "device_error_word": word}  # GEMM, sp_prep, sp_quant_kv_stream, attention


def qkv_gemm_time(eng, w, dev, stream, iters=30):
    """The block's fused QKV projection (row a1 + a2) at the workload's
    shape: x [B*N][hidden] -> q, k, v with bias and RoPE, timed with CUDA
    events (x + w = 0.32 GB at C4, larger than L2)."""
    import torch
    B, H, G, N, D = w["batch"], w["heads"], w["kv_heads"], w["tokens"], w["d"]
    hidden = w["qkv"]["hidden"]
    n_out = (H + 2 * G) * D
    g = torch.Generator(device=dev)
    g.manual_seed(99)
    x = torch.randn(B * N, hidden, generator=g, device=dev).to(torch.bfloat16)
    wt = (torch.randn(n_out, hidden, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    sage = importlib.import_module("sota-papers-lab_b200")
    rope = torch.from_numpy(sage.rope_table_1d(w["qkv"]["rope_theta"], D, N)).to(dev)
    q = torch.empty(B, N, H, D, dtype=torch.bfloat16, device=dev)
    k = torch.empty(B, N, G, D, dtype=torch.bfloat16, device=dev)
    v = torch.empty_like(k)
    call = lambda: eng.qkv_gemm(x, wt, None, rope, q, k, v, batch=B, tokens=N, heads=H, kv_heads=G,
                                rope_half=D // 2, frame_len=N)
    for _ in range(3):
        call()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with ClockSampler(torch.device(dev).index or 0) as clk:
        e0.record(stream)
        for _ in range(iters):
            call()
        e1.record(stream)
        torch.cuda.synchronize()
    assert eng.engine_status() == 0
    ms = e0.elapsed_time(e1) / iters
    flops = 2.0 * B * N * hidden * n_out
    return {"kernel": "sp_qkv_gemm_2sm (tcgen05 kind::f16 on SM pairs, cta_group::2; bias + RoPE + bf16 epilogue)",
            "shape": f"[{B * N}x{hidden}] x [{n_out}x{hidden}]^T", "ms": round(ms, 4),
            "achieved": round(flops / (ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "bound": "tensor",
            "clocks": clk.summary()}


def qkv_fp8_time(eng, w, dev, stream, iters=30):
    """The FP8 QKV side of the reference's FP8 block (row f1): LN1 of the
    bf16 activations to per-token E4M3 (spl_sage_layer_norm_fp8) and the FP8
    QKV GEMM with token / channel scales, RoPE and bf16 out fused
    (spl_sage_qkv_gemm_fp8), at the workload's shape; weights E4M3 with one
    scale per output channel."""
    import torch
    B, H, G, N, D = w["batch"], w["heads"], w["kv_heads"], w["tokens"], w["d"]
    hidden = w["qkv"]["hidden"]
    n_out = (H + 2 * G) * D
    g = torch.Generator(device=dev)
    g.manual_seed(98)
    x = torch.randn(B * N, hidden, generator=g, device=dev).to(torch.bfloat16)
    gamma = 1.0 + 0.1 * torch.randn(hidden, generator=g, device=dev)
    beta = 0.1 * torch.randn(hidden, generator=g, device=dev)
    wt = torch.randn(n_out, hidden, generator=g, device=dev) * 0.02
    w_scale = (wt.abs().amax(dim=1) / 448.0).clamp_min(1e-12)
    w8 = (wt / w_scale[:, None]).to(torch.float8_e4m3fn).view(torch.uint8)
    del wt
    sage = importlib.import_module("sota-papers-lab_b200")
    rope = torch.from_numpy(sage.rope_table_1d(w["qkv"]["rope_theta"], D, N)).to(dev)
    x8 = torch.empty(B * N, hidden, dtype=torch.uint8, device=dev)
    xs = torch.empty(B * N, dtype=torch.float32, device=dev)
    q = torch.empty(B, N, H, D, dtype=torch.bfloat16, device=dev)
    k = torch.empty(B, N, G, D, dtype=torch.bfloat16, device=dev)
    v = torch.empty_like(k)
    ln = lambda: eng.layer_norm_fp8(x, gamma, beta, 1e-6, x8, xs)
    gemm = lambda: eng.qkv_gemm_fp8(x8, xs, w8, w_scale, None, rope, q, k, v, batch=B, tokens=N, heads=H,
                                    kv_heads=G, rope_half=D // 2, frame_len=N)
    times, clocks = {}, {}
    for name, call in (("ln", ln), ("gemm", gemm)):
        for _ in range(3):
            call()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        with ClockSampler(torch.device(dev).index or 0) as clk:
            e0.record(stream)
            for _ in range(iters):
                call()
            e1.record(stream)
            torch.cuda.synchronize()
        times[name] = e0.elapsed_time(e1) / iters
        clocks[name] = clk.summary()
    assert eng.engine_status() == 0
    flops = 2.0 * B * N * hidden * n_out
    lib = library_fp8_gemm_time(x8, xs, w8, w_scale, iters, flops)
    ln_bytes = B * N * hidden * (2 + 1) + B * N * 4  # bf16 in, E4M3 out, scales
    return {"kernels": "sp_ln_fp8 (LN1 -> per-token E4M3) + sp_qkv_gemm_2sm<FP8> (tcgen05 kind::f8f6f4 on SM "
                       "pairs, token/channel scales + RoPE + bf16 epilogue)",
            "shape": f"[{B * N}x{hidden}] x [{n_out}x{hidden}]^T", "ln_ms": round(times["ln"], 4),
            "ln_gbs": round(ln_bytes / (times["ln"] * 1e-3) / 1e9, 1), "gemm_ms": round(times["gemm"], 4),
            "achieved": round(flops / (times["gemm"] * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "bound": "tensor",
            "gemm_clocks": clocks["gemm"], "library_fp8_gemm": lib}


def library_fp8_gemm_time(x8, xs, w8, w_scale, iters, flops):
    """The same E4M3 product through torch._scaled_mm (a library FP8 GEMM,
    cuBLASLt or torch's own kernels) on the same operands, bf16 out: with
    the token / channel scales when the library takes them, else with one
    scale per operand (the plain GEMM, no epilogue).  A comparison on the
    same GPU, not part of the path."""
    import torch
    a = x8.view(torch.float8_e4m3fn)
    b = w8.view(torch.float8_e4m3fn).t()  # [hidden][n_out], column-major
    one = torch.ones((), dtype=torch.float32, device=x8.device)
    forms = (("per-token x per-channel scales", lambda: torch._scaled_mm(
                 a, b, scale_a=xs[:, None].contiguous(), scale_b=w_scale[None, :].contiguous(),
                 out_dtype=torch.bfloat16)),
             ("one scale per operand", lambda: torch._scaled_mm(a, b, scale_a=one, scale_b=one,
                                                                 out_dtype=torch.bfloat16)))
    for form, call in forms:
        try:
            for _ in range(3):
                call()
            torch.cuda.synchronize()
        except Exception as e:  # the library lacks this form on this build
            last = f"{type(e).__name__}: {str(e).splitlines()[0][:120]}"
            continue
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(torch.cuda.current_device()) as clk:
            e0.record()
            for _ in range(iters):
                call()
            e1.record()
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        return {"call": "torch._scaled_mm", "scales": form, "ms": round(ms, 4),
                "achieved": round(flops / (ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "clocks": clk.summary()}
    return {"call": "torch._scaled_mm", "unavailable": last}


# ---------------------------------------------------------------- CPU arms

def cpu_sample_time(w, chunks, heads_sample, nthreads, seed=7):
    """Times the CPU port of the reference's path on a bounded sample of the
    workload and extrapolates it to the whole job: batch item 0,
    `heads_sample` query heads (and their kv heads), `chunks` seeded random
    runs of 64 query rows for the f64 attention, the full sequence for the
    quantiser.  Returns (seconds for the full job, sample description)."""
    from oracle import oracle as O
    N, D, H, G = w["tokens"], w["d"], w["heads"], w["kv_heads"]
    rng = np.random.default_rng(seed)
    hs = min(heads_sample, H)
    gs = max(1, hs * G // H)
    q = O.f32_to_bf16(rng.normal(size=(1, N, hs, D)).astype(np.float32))
    k = O.f32_to_bf16(rng.normal(size=(1, N, gs, D)).astype(np.float32))
    v = O.f32_to_bf16(rng.normal(size=(1, N, gs, D)).astype(np.float32))
    g = O.make_geom(1, hs, gs, N, D, O.bthd_strides(N, hs, D), O.bthd_strides(N, gs, D), O.bthd_strides(N, gs, D))
    t0 = time.perf_counter()
    O.prepare(q, k, v, g)
    t_quant = time.perf_counter() - t0
    run = min(64, N)
    starts = rng.choice(max(1, N - run + 1), size=chunks, replace=True)
    pairs_sample = 0
    t0 = time.perf_counter()
    for r0 in starts:
        r0 = int(r0)
        O.attention_bthd(q, k, v, g, causal=w["causal"], rows=(r0, r0 + run), nthreads=nthreads)
        pairs_sample += sum((r + 1) if w["causal"] else N for r in range(r0, r0 + run))
    t_attn = time.perf_counter() - t0
    pairs_full = (N * (N + 1) // 2 if w["causal"] else N * N) * w["batch"] * H
    full = t_attn * pairs_full / (pairs_sample * hs) + t_quant * (w["batch"] * H) / hs
    desc = (f"oracle port (f64 attention + bit-exact quantiser, C -O2, {nthreads} threads): batch 0, {hs} q heads / "
            f"{gs} kv heads, {chunks} random runs of {run} query rows for the attention, the full sequence for the "
            f"quantiser; measured {t_attn + t_quant:.2f} s, extrapolated by (causal) key-pair count and head count")
    return full, desc


def cpu_leg(w, batch, q, k, v, out, nthreads, chunks=96, heads_sample=8, parity_runs=8, seed=7):
    """The CPU baseline on a bounded sample of the bench's own inputs, and
    the parity of this run's output on the same sample.  The reference's CPU
    path (the oracle port: bit-exact quantiser + f64 attention, C, all host
    threads) runs on batch item 0 and its first `heads_sample` query heads
    (with their kv heads): the quantiser over the whole sequence, the
    attention on `chunks` seeded runs of 64 query rows; its time is
    extrapolated to the whole job by (causal) key-pair and head count.  The
    GPU output of the first `parity_runs` runs is compared with that f64
    attention and with the oracle's restatement of the reference kernel's
    online arithmetic (or_sage_online, 64-key blocks) on the quantised sample.
    Returns (cpu_baseline, parity)."""
    from oracle import oracle as O
    N, D, H, G = w["tokens"], w["d"], w["heads"], w["kv_heads"]
    hs = min(heads_sample, H)
    gs = max(1, hs * G // H)
    bits = lambda t: t.contiguous().view(__import__("torch").int16).cpu().numpy().view(np.uint16)
    qs, ks, vs = bits(q[0:1, :, :hs]), bits(k[0:1, :, :gs]), bits(v[0:1, :, :gs])
    ours_all = O.bf16_to_f32(bits(out[0:1, :, :hs]))
    g = O.make_geom(1, hs, gs, N, D, O.bthd_strides(N, hs, D), O.bthd_strides(N, gs, D), O.bthd_strides(N, gs, D))
    t0 = time.perf_counter()
    quant = O.prepare(qs, ks, vs, g)
    t_quant = time.perf_counter() - t0
    rng = np.random.default_rng(seed)
    run = min(64, N)
    starts = [int(r) for r in rng.choice(max(1, N - run + 1), size=chunks, replace=True)]
    pairs_sample = 0
    t_attn = 0.0
    got, f64, ref = [], [], []
    for i, r0 in enumerate(starts):
        t0 = time.perf_counter()
        ex = O.attention_bthd(qs, ks, vs, g, causal=w["causal"], rows=(r0, r0 + run), nthreads=nthreads)
        t_attn += time.perf_counter() - t0
        pairs_sample += sum((r + 1) if w["causal"] else N for r in range(r0, r0 + run))
        if i < parity_runs:
            got.append(ours_all[:, r0:r0 + run])
            f64.append(ex[:, r0:r0 + run])
            on = O.sage_online(quant, g, block=O.REF_BLOCK, causal=w["causal"], rows=(r0, r0 + run),
                               nthreads=nthreads)
            ref.append(on[:, r0:r0 + run])
    pairs_full = (N * (N + 1) // 2 if w["causal"] else N * N) * batch * H
    full = t_attn * pairs_full / (pairs_sample * hs) + t_quant * (batch * H) / hs
    value = effective_flops(w, batch) / full / 1e12
    desc = (f"oracle port (f64 attention + bit-exact quantiser, C -O2, {nthreads} threads) on the bench's own "
            f"inputs: batch 0, {hs} q heads / {gs} kv heads, {chunks} seeded runs of {run} query rows for the "
            f"attention, the full sequence for the quantiser; measured {t_attn + t_quant:.2f} s, extrapolated by "
            f"(causal) key-pair count and head count")
    cpu = {"value": value, "unit": "TOPS", "cores": nthreads, "kind": "port", "sample": desc}
    got, f64, ref = (np.ascontiguousarray(np.concatenate(a, axis=1)) for a in (got, f64, ref))
    e64, eref = O.errors(got, f64), O.errors(got, ref)
    rnd = lambda e: {k2: round(float(e[k2]), 6) for k2 in ("cos", "rel_l1", "rel_l2")}
    parity = {"rows": f"{len(starts[:parity_runs])} runs of {run} query rows x {hs} q heads of batch 0 of the "
                      f"timed output",
              "vs_f64": rnd(e64), "vs_reference_kernel_arithmetic": rnd(eref),
              "gate": "vs the reference kernel's arithmetic: cos >= 0.9995, rel-L1 <= 1e-2",
              "gate_ok": bool(eref["cos"] >= 0.9995 and eref["rel_l1"] <= 1e-2)}
    return cpu, parity


def cpu_qkv_sample_time(w, rows, nthreads, seed=7):
    """Times the CPU port of one layer's QKV GEMM + prologue (f64, the
    oracle's restatement of host::linear and qkv::reference) on `rows`
    seeded rows and extrapolates it to the layer's B*N rows.  Returns
    (seconds for the layer, sample description)."""
    from oracle import oracle as O
    H, D, Hd, M = w["heads"], w["d"], w["hidden"], w["batch"] * w["tokens"]
    rng = np.random.default_rng(seed)
    x = O.f32_to_bf16(rng.normal(size=(rows, Hd)).astype(np.float32))
    wt = O.f32_to_bf16((0.02 * rng.normal(size=(3 * H * D, Hd))).astype(np.float32))
    bias = O.f32_to_bf16((0.02 * rng.normal(size=3 * H * D)).astype(np.float32))
    t0 = time.perf_counter()
    O.qkv_reference(x, wt, bias, None, tokens=rows, hq=H, hkv=H, d=D, nthreads=nthreads)
    t = time.perf_counter() - t0
    return t * M / rows, f"QKV GEMM + prologue in f64 on {rows} of {M} rows, measured {t:.2f} s, scaled by rows"


def run_reference(args, rank, world):
    if rank != 0:
        return None
    w = WORKLOADS[args.workload]
    nthreads = os.cpu_count() or 1
    times = []
    desc = ""
    for i in range(args.warmup + args.steps):
        full, desc = cpu_sample_time(w, chunks=8, heads_sample=8, nthreads=nthreads, seed=7 + i)
        if "layers" in w:
            # C2: each layer's QKV GEMM (host::linear in f64) before its
            # attention, as the arm on the GPU times the whole QKV path
            t_gemm, gdesc = cpu_qkv_sample_time(w, rows=256, nthreads=nthreads, seed=7 + i)
            full = w["layers"] * (full + t_gemm)
            desc = f"{w['layers']} layers of [{gdesc}] + [{desc}]"
        if i >= args.warmup:
            times.append(full)
    t = statistics.median(times)
    # the same job as our arm's line at this rank count (its config)
    cfg = config_of(args.workload, world) if args.workload not in ("C2", "C5") else {
        "workload": w["desc"], "global_batch": w["batch"], "seq_len": w["tokens"], "parallelism": "host cores"}
    jobs = cfg["global_batch"] / w["batch"]
    t *= jobs
    value = w.get("layers", 1) * effective_flops(w, cfg["global_batch"]) / t / 1e12
    sharded = args.workload in ("C4", "C5")
    return {
        "impl": "reference", "metric": metric_of(args.workload),
        "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "strong" if sharded else "weak",
        "vs_baseline": None, "dtype": "f64 (reference CPU path)", "data": "synthetic (seeded numpy normal)",
        "config": cfg,
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": nthreads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="C4", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="C4: leave out the c4_block, qkv_gemm, qkv_fp8 and ring_c5 measurements (quick runs, profiling)")
    ap.add_argument("--cp-schedule", default="gather", choices=["gather", "ring"],
                    help="C5: all-gather the quantised K/V (default) or pass it around a send/recv ring")
    ap.add_argument("--reserve-sms", type=int, default=None,
                    help="C5: SMs the attention leaves to NCCL during ring steps (default: the ring's own)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    import datetime

    import torch
    import torch.distributed as dist
    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        runner = {"C5": run_ring, "C2": run_layers}.get(args.workload, run_ours)
        line = runner(args, rank, world, local_rank)
        if line is not None and world == 1 and not args.no_cpu_baseline and "cpu_baseline" not in line:
            full, desc = cpu_sample_time(WORKLOADS[args.workload], chunks=96, heads_sample=8,
                                         nthreads=os.cpu_count() or 1)
            v = effective_flops(WORKLOADS[args.workload], WORKLOADS[args.workload]["batch"]) / full / 1e12
            line["cpu_baseline"] = {"value": v, "unit": "TOPS", "cores": os.cpu_count() or 1, "kind": "port",
                                    "sample": desc}
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
