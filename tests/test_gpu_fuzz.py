"""Seeded random shapes, row strides and alignments for every op, through the C ABI, against
references on the same GPU that must agree bit for bit:

  * rms_norm / add_rms_norm (bf16): the reference's own CUDA rms_norm kernel (oracle/_ref) on
    the same rows, after a LibTorch add for the fused op; fp32: the CPU oracle, 1e-5 relative.
  * qk_norm_rope / rope (bf16): the reference kernel on the [tokens * heads, head_dim] view for
    the q/k norm, then Hugging Face's rotary formula as torch ops.
  * silu_and_mul (bf16): F.silu(gate) * up; fp32: the CPU oracle, 1e-5 relative.
  * embedding: index_select. argmax: torch.argmax.

Each case draws its sizes across the launch regimes (row-block and bulk norms, direct and table
SiLU, the cluster splits of argmax), strides with padding between rows, and, for some cases,
rows that start off a 16-byte boundary (the plain-load kernels)."""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
import svllm_capi as capi
from conftest import assert_rel_f32, to_bits
from test_gpu_parity import torch_rope

pytestmark = pytest.mark.gpu

CASES = 16


def rng(op: str, case: int) -> np.random.Generator:
    return np.random.default_rng([sum(map(ord, op)), case])


def rows_of(r: np.random.Generator, rows: int, cols: int, dtype, device, pad: int, offset: int,
            scale: float = 1.0) -> torch.Tensor:
    """[rows, cols] with row stride cols + pad, starting `offset` elements into its buffer."""
    stride = cols + pad
    flat = torch.from_numpy(r.standard_normal(offset + rows * stride).astype(np.float32) * scale)
    flat = flat.to(device=device, dtype=dtype)
    return flat[offset:].view(rows, stride)[:, :cols]


@pytest.fixture(autouse=True)
def _clear_device_error(cuda):
    capi.read_device_error(0, reset=True)
    yield
    torch.cuda.synchronize()
    assert capi.read_device_error(0, reset=True) == 0


@pytest.mark.parametrize("case", range(CASES))
def test_norms(cuda, case):
    r = rng("norm", case)
    dt = torch.bfloat16 if case % 4 else torch.float32
    hidden = int(r.choice([64, 96, 128, 256, 768, 1000, 1024, 2048, 4096, 4100, 6144]))
    rows = int(r.choice([1, 3, 17, 200, 1000, 5000, 12000]))
    unaligned = case % 5 == 3
    pad = 0 if unaligned else int(r.choice([0, 8, 64]))
    offset = 1 if unaligned else 0
    x = rows_of(r, rows, hidden, dt, cuda, pad, offset)
    res = rows_of(r, rows, hidden, dt, cuda, pad, offset)
    w = rows_of(r, 1, hidden, dt, cuda, 0, 0, 0.1)[0] + 1
    eps = 1e-6
    ref = oracle.reference_module()
    what = f"{rows}x{hidden} pad {pad} offset {offset} {dt}"
    if case % 2:
        out = rows_of(r, rows, hidden, dt, cuda, pad, offset)
        capi.rms_norm(out, x, w, eps)
        if dt == torch.bfloat16:
            assert torch.equal(out, ref.rms_norm(x.contiguous(), w, eps)), what
        else:
            assert_rel_f32(out, oracle.rms_norm(to_bits(x), to_bits(w), eps), 1e-5, what)
    else:
        s = x + res  # the residual add as torch computes it
        x_in, res_in = to_bits(x), to_bits(res)
        capi.add_rms_norm(x, res, w, eps)
        assert torch.equal(res, s), what
        if dt == torch.bfloat16:
            assert torch.equal(x, ref.rms_norm(s.contiguous(), w, eps)), what
        else:
            ox, _ = oracle.add_rms_norm(x_in, res_in, to_bits(w), eps)
            assert_rel_f32(x, ox, 1e-5, what)


@pytest.mark.parametrize("case", range(CASES))
def test_rotary(cuda, case):
    r = rng("rope", case)
    d = int(r.choice([64, 128, 128, 256]))
    hq, hk = [(16, 8), (32, 8), (8, 1), (4, 4)][int(r.integers(4))]
    tokens = int(r.choice([1, 5, 64, 300, 2000, 9000]))
    norm = case % 2 == 0
    # q and k as views of one qkv projection, maybe off a 16-byte boundary
    offset = 1 if case % 5 == 4 else 0
    qkv = rows_of(r, tokens, (hq + 2 * hk) * d, torch.bfloat16, cuda, 0, offset)
    q = qkv[:, : hq * d].view(tokens, hq, d)
    k = qkv[:, hq * d:(hq + hk) * d].view(tokens, hk, d)
    pos = torch.from_numpy(r.integers(0, 32768, tokens)).to(cuda)
    scaling = (32.0, 1.0, 4.0, 8192) if case % 3 == 0 else None
    inv = oracle.inv_freq(5e5 if scaling else 1e6, d, scaling)
    invt = torch.from_numpy(inv)
    what = f"{tokens} tokens, heads {hq}/{hk}, d {d}, norm {norm}, offset {offset}"
    if norm:
        ref = oracle.reference_module()
        qw = rows_of(r, 1, d, torch.bfloat16, cuda, 0, 0, 0.1)[0] + 1
        kw = rows_of(r, 1, d, torch.bfloat16, cuda, 0, 0, 0.1)[0] + 1

        def heads(x):
            # the [tokens * heads, head_dim] rows the reference kernel normalises, at the same
            # 16-byte alignment as ours (it vectorises exactly when the rows are aligned)
            buf = torch.empty(offset + x.numel(), dtype=x.dtype, device=x.device)
            view = buf[offset:].view(-1, d)
            view.copy_(x.reshape(-1, d))
            return view

        eq = torch_rope(ref.rms_norm(heads(q), qw, 1e-6).view(q.shape), pos, invt)
        ek = torch_rope(ref.rms_norm(heads(k), kw, 1e-6).view(k.shape), pos, invt)
        capi.qk_norm_rope(q, k, qw, kw, pos, 1e-6, inv)
    else:
        eq, ek = torch_rope(q, pos, invt), torch_rope(k, pos, invt)
        capi.rope(q, k, pos, inv)
    assert torch.equal(q, eq) and torch.equal(k, ek), what


@pytest.mark.parametrize("case", range(CASES))
def test_silu_and_mul(cuda, case):
    r = rng("silu", case)
    dt = torch.bfloat16 if case % 4 else torch.float32
    inter = int(r.choice([64, 1000, 3072, 8192, 3001]))
    rows = int(r.choice([1, 7, 100, 1500, 4000]))
    halves = case % 3 == 1  # gate and up as the halves of one gate_up projection
    if halves:
        gate_up = rows_of(r, rows, 2 * inter, dt, cuda, 0, 0, 3.0)
        gate, up = gate_up[:, :inter], gate_up[:, inter:]
    else:
        offset = 1 if case % 5 == 2 else 0
        gate = rows_of(r, rows, inter, dt, cuda, 0, offset, 3.0)
        up = rows_of(r, rows, inter, dt, cuda, 0, offset)
    out = torch.empty(rows, inter, dtype=dt, device=cuda)
    capi.silu_and_mul(out, gate, up)
    what = f"{rows}x{inter} halves {halves} {dt}"
    if dt == torch.bfloat16:
        assert torch.equal(out, F.silu(gate) * up), what
    else:
        assert_rel_f32(out, oracle.silu_and_mul(to_bits(gate), to_bits(up)), 1e-5, what)


@pytest.mark.parametrize("case", range(CASES))
def test_embedding(cuda, case):
    r = rng("embedding", case)
    dt = torch.bfloat16 if case % 4 else torch.float32
    vocab = int(r.choice([10, 1000, 151936]))
    hidden = int(r.choice([64, 1000, 1024, 2048]))
    tokens = int(r.choice([1, 33, 500, 20000]))
    table = rows_of(r, vocab, hidden, dt, cuda, 0, 0)
    ids = torch.from_numpy(r.integers(0, vocab, tokens)).to(cuda)
    if case % 2:
        ids = ids.to(torch.int32)
    out = torch.empty(tokens, hidden, dtype=dt, device=cuda)
    capi.embedding(out, ids, table)
    assert torch.equal(out, table.index_select(0, ids.long()))


@pytest.mark.parametrize("case", range(CASES))
def test_argmax(cuda, case):
    r = rng("argmax", case)
    dt = torch.bfloat16 if case % 4 else torch.float32
    vocab = int(r.choice([7, 1000, 32000, 128256, 151936]))
    rows = int(r.choice([1, 9, 50, 100, 300, 700, 1500]))
    pad = int(r.choice([0, 8]))
    logits = rows_of(r, rows, vocab, dt, cuda, pad, 0, 3.0)
    # ties at the maximum in some rows
    tie_rows = torch.from_numpy(r.integers(0, rows, max(1, rows // 4))).to(cuda)
    logits[tie_rows] = logits[tie_rows].clamp(max=1.0)
    ids = torch.empty(rows, dtype=torch.int64, device=cuda)
    capi.argmax(ids, logits)
    assert torch.equal(ids, torch.argmax(logits, dim=-1)), f"{rows}x{vocab} pad {pad} {dt}"
