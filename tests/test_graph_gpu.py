"""The op under CUDA-graph capture, as the reference's callers run it: the
VGGT engine captures its trunk into a CUDA graph (apps/image-to-3d/src/vggt/
mod.rs:393-422) with the Sage workspaces made outside capture
(trunk/sched.rs:120-147).  Here the FP8 block (LN1 -> per-token E4M3 -> FP8
QKV GEMM with RoPE -> quantised causal GQA attention -> per-token E4M3 ->
FP8 output projection) and the bf16 QKV GEMM -> attention chain are captured
once on the engine's stream into a torch CUDA graph; replays on new inputs
give the bytes of the same calls made eagerly."""
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu
sage = importlib.import_module("sota-papers-lab_b200")

B, T, HID, HQ, HKV, D = 1, 1000, 1024, 8, 2, 128
N = (HQ + 2 * HKV) * D


def _e4m3_rows(w):
    """Per-row E4M3 weights (amax / 448) as uint8 bytes, and their scales."""
    scale = (w.abs().amax(dim=1) / 448.0).clamp_min(1e-12)
    return (w / scale[:, None]).to(torch.float8_e4m3fn).view(torch.uint8).contiguous(), scale.float().contiguous()


class Block:
    """Device buffers of one block; the workspace is made here, outside any
    capture, as the reference's scheduler does."""

    def __init__(self, eng):
        dev = "cuda"
        g = torch.Generator(device=dev).manual_seed(7)
        self.eng = eng
        self.ws = eng.workspace(sage.Shape(B, HQ, T, HKV, True))
        self.x = torch.zeros(B * T, HID, dtype=torch.bfloat16, device=dev)
        self.gamma = 1.0 + 0.1 * torch.randn(HID, generator=g, device=dev)
        self.beta = 0.1 * torch.randn(HID, generator=g, device=dev)
        self.w8, self.w_scale = _e4m3_rows(0.02 * torch.randn(N, HID, generator=g, device=dev))
        self.w = (0.02 * torch.randn(N, HID, generator=g, device=dev)).to(torch.bfloat16)
        self.bias = (0.1 * torch.randn(N, generator=g, device=dev)).to(torch.bfloat16)
        self.p8, _ = _e4m3_rows(0.02 * torch.randn(HID, HQ * D, generator=g, device=dev))
        self.rope = torch.from_numpy(sage.rope_table_1d(500000.0, D, T)).to(dev)
        self.x8 = torch.zeros(B * T, HID, dtype=torch.uint8, device=dev)
        self.t0 = torch.zeros(B * T, device=dev)
        self.q = torch.zeros(B, T, HQ, D, dtype=torch.bfloat16, device=dev)
        self.k = torch.zeros(B, T, HKV, D, dtype=torch.bfloat16, device=dev)
        self.v = torch.zeros(B, T, HKV, D, dtype=torch.bfloat16, device=dev)
        self.o = torch.zeros(B, T, HQ, D, dtype=torch.bfloat16, device=dev)
        self.o8 = torch.zeros(B * T, HQ * D, dtype=torch.uint8, device=dev)
        self.t1 = torch.zeros(B * T, device=dev)
        self.y = torch.zeros(B * T, HID, dtype=torch.bfloat16, device=dev)
        sq, skv = sage.Strides.bthd(T, HQ, D), sage.Strides.bthd(T, HKV, D)
        self.views = (sage.Tensor(self.q, sq), sage.Tensor(self.k, skv), sage.Tensor(self.v, skv),
                      sage.Tensor(self.o, sq))
        self.shape = dict(batch=B, tokens=T, heads=HQ, kv_heads=HKV, rope_half=D // 2, frame_len=T)

    def fp8_block(self):
        e = self.eng
        e.layer_norm_fp8(self.x, self.gamma, self.beta, 1e-6, self.x8, self.t0)
        e.qkv_gemm_fp8(self.x8, self.t0, self.w8, self.w_scale, self.bias, self.rope, self.q, self.k, self.v,
                       **self.shape)
        e.forward(self.ws, *self.views)
        e.rows_fp8(self.o.view(B * T, HQ * D), self.o8, self.t1)
        e.linear_fp8(self.o8, None, self.p8, None, None, self.y)  # scales deferred, as block.rs does

    def bf16_chain(self):
        self.eng.qkv_gemm(self.x, self.w, self.bias, self.rope, self.q, self.k, self.v, **self.shape)
        self.eng.forward(self.ws, *self.views)

    def outputs(self, chain):
        """Copies of what the chain writes (q, k, v, o first)."""
        ts = (self.q, self.k, self.v, self.o)
        if chain == "fp8_block":
            ts += (self.x8, self.t0, self.o8, self.t1, self.y)
        return [t.clone() for t in ts]


def _fill(blk, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    # a residual stream with per-channel offsets
    blk.x.copy_(2.0 * torch.randn(B * T, HID, generator=g, device="cuda") +
                torch.randn(HID, generator=g, device="cuda"))


@pytest.mark.parametrize("chain", ["fp8_block", "bf16_chain"])
def test_chain_replays_from_a_cuda_graph(chain):
    s = torch.cuda.Stream()
    eng = sage.SageAttention(s, D)
    blk = Block(eng)
    run = getattr(blk, chain)
    eager = {}
    with torch.cuda.stream(s):
        for seed in (1, 2):
            _fill(blk, seed)
            run()
            eager[seed] = blk.outputs(chain)
    s.synchronize()
    assert eng.status(blk.ws) == 0 and eng.engine_status() == 0
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        run()
    for seed in (2, 1, 2):
        with torch.cuda.stream(s):
            _fill(blk, seed)
            graph.replay()
            got = blk.outputs(chain)
        s.synchronize()
        for a, b in zip(got, eager[seed]):
            assert torch.equal(a, b)
    assert not torch.equal(eager[1][3], eager[2][3])  # the inputs matter
    assert eng.status(blk.ws) == 0 and eng.engine_status() == 0
    del graph
