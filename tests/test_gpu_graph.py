"""The ops are graph-capturable (no host sync, no allocation in the kernels' C ABI, grids that
depend only on the batch size): the decode-step chain (Qwen3, 256 tokens) is captured once in a
CUDA graph and replayed on fresh inputs, and every replay must equal the eager run bit for bit.
This is the launch-latency answer for the small-T regime (reference docs/ROADMAP.md:42)."""

from __future__ import annotations

import pytest
import torch

import svllm_ops

pytestmark = pytest.mark.gpu


def fill(bufs, seed):
    g = torch.Generator(device=bufs["x"].device).manual_seed(seed)
    for name in ("x", "r", "q", "k", "gate", "up"):
        bufs[name].normal_(generator=g)
    bufs["ids"].random_(0, 151936, generator=g)
    bufs["pos"].random_(0, 4096, generator=g)


def chain(b):
    emb = svllm_ops.embedding(b["ids"], b["table"])
    svllm_ops.add_rms_norm(b["x"], b["r"], b["w"], 1e-6)
    svllm_ops.qk_norm_rope(b["q"], b["k"], b["qw"], b["kw"], b["pos"], 1e-6, 1e6)
    y = svllm_ops.silu_and_mul(b["gate"], b["up"])
    return emb, y


def test_decode_chain_replays_in_a_cuda_graph(cuda):
    T = 256
    bf = dict(device=cuda, dtype=torch.bfloat16)
    b = {"table": torch.randn(151936, 1024, **bf) * 0.02, "x": torch.empty(T, 1024, **bf),
         "r": torch.empty(T, 1024, **bf), "w": torch.ones(1024, **bf),
         "q": torch.empty(T, 16, 128, **bf), "k": torch.empty(T, 8, 128, **bf),
         "qw": torch.ones(128, **bf), "kw": torch.ones(128, **bf),
         "gate": torch.empty(T, 3072, **bf), "up": torch.empty(T, 3072, **bf),
         "ids": torch.empty(T, device=cuda, dtype=torch.int32),
         "pos": torch.empty(T, device=cuda, dtype=torch.int64)}

    fill(b, 0)
    chain(b)  # warm-up outside capture: caches the rope table and the launch shapes
    torch.cuda.synchronize()

    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        fill(b, 1)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            g_emb, g_y = chain(b)
    torch.cuda.synchronize()

    for seed in (2, 3, 4):
        fill(b, seed)
        inputs = {k: v.clone() for k, v in b.items() if k != "table"}
        graph.replay()
        torch.cuda.synchronize()
        got = {"emb": g_emb.clone(), "y": g_y.clone(), "x": b["x"].clone(), "r": b["r"].clone(),
               "q": b["q"].clone(), "k": b["k"].clone()}
        eager = dict(inputs, table=b["table"])
        e_emb, e_y = chain(eager)
        torch.cuda.synchronize()
        assert torch.equal(got["emb"], e_emb) and torch.equal(got["y"], e_y)
        for name in ("x", "r", "q", "k"):
            assert torch.equal(got[name], eager[name]), name
    del graph
