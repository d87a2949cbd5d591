"""The row-sharded multi-rank path on CPU: two gloo ranks each run the chain on their rows
(svllm_dist.split_rows) through svllm_ops' CPU backend, all-gather the output shards
(svllm_dist.all_gather_rows, the validation collective) and rank 0 checks the gathered result
against the oracle on the whole batch. No GPU: the same plumbing bench.py runs over NCCL."""

from __future__ import annotations

import os
import socket
import sys
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import ORACLE_DIR, PKG_PY

T_TOTAL = 37  # odd, so the shards differ by one row


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(7)

    def randn(*shape, scale=1.0, shift=0.0):
        return (torch.randn(shape, generator=g) * scale + shift).to(torch.bfloat16)

    return {
        "table": randn(500, 256, scale=0.02),
        "ids": torch.randint(0, 500, (T_TOTAL,), generator=g, dtype=torch.int32),
        "x": randn(T_TOTAL, 256), "r": randn(T_TOTAL, 256), "w": randn(256, scale=0.1, shift=1),
        "q": randn(T_TOTAL, 4, 64), "k": randn(T_TOTAL, 2, 64),
        "qw": randn(64, scale=0.1, shift=1), "kw": randn(64, scale=0.1, shift=1),
        "pos": torch.randint(0, 4096, (T_TOTAL,), generator=g),
        "gate": randn(T_TOTAL, 384), "up": randn(T_TOTAL, 384),
    }


def _rank_main(rank: int, world: int, port: int, out_path: str) -> None:
    sys.path[:0] = [str(PKG_PY), str(ORACLE_DIR)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    import svllm_dist
    import svllm_ops

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = _inputs()
        b, e = svllm_dist.split_rows(T_TOTAL, world, rank)
        s = {k: (v[b:e].clone() if v.shape[0] == T_TOTAL else v) for k, v in full.items()}
        emb = svllm_ops.embedding(s["ids"], s["table"])
        svllm_ops.add_rms_norm(s["x"], s["r"], s["w"], 1e-6)
        svllm_ops.qk_norm_rope(s["q"], s["k"], s["qw"], s["kw"], s["pos"], 1e-6, 1e6)
        y = svllm_ops.silu_and_mul(s["gate"], s["up"])
        gathered = {name: svllm_dist.all_gather_rows(t, T_TOTAL) for name, t in
                    dict(emb=emb, x=s["x"], r=s["r"], q=s["q"], k=s["k"], y=y).items()}
        if rank == 0:
            torch.save({k: v.view(torch.int16) for k, v in gathered.items()}, out_path)
    finally:
        dist.destroy_process_group()


def test_split_rows_covers_every_row_once():
    sys.path.insert(0, str(PKG_PY))
    import svllm_dist

    for total in (0, 1, 7, 1_048_576, 70_001):
        for world in (1, 2, 3, 4, 8):
            ranges = [svllm_dist.split_rows(total, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            assert max(e - b for b, e in ranges) - min(e - b for b, e in ranges) <= 1
    with pytest.raises(ValueError):
        svllm_dist.split_rows(10, 2, 2)


def test_two_gloo_ranks_match_the_oracle():
    import oracle

    port = _free_port()
    with tempfile.TemporaryDirectory() as tmp:
        out_path = os.path.join(tmp, "gathered.pt")
        mp.start_processes(_rank_main, args=(2, port, out_path), nprocs=2, join=True,
                           start_method="spawn")
        got = {k: v.numpy().view(np.uint16) for k, v in torch.load(out_path).items()}

    full = _inputs()

    def bits(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    emb, bad = oracle.embedding(full["ids"].numpy(), bits(full["table"]))
    ox, orr = oracle.add_rms_norm(bits(full["x"]), bits(full["r"]), bits(full["w"]), 1e-6)
    inv = oracle.inv_freq(1e6, 64)
    oq, ok = oracle.qk_norm_rope(bits(full["q"]), bits(full["k"]), bits(full["qw"]),
                                 bits(full["kw"]), full["pos"].numpy(), 1e-6, inv)
    oy = oracle.silu_and_mul(bits(full["gate"]), bits(full["up"]))
    from conftest import ulp_diff_bf16

    assert bad == 0 and np.array_equal(got["emb"], emb)
    assert np.array_equal(got["r"], orr)
    assert ulp_diff_bf16(got["x"], ox).max() <= 1
    assert ulp_diff_bf16(got["q"], oq).max() <= 2 and ulp_diff_bf16(got["k"], ok).max() <= 2
    assert ulp_diff_bf16(got["y"], oy).max() <= 2
