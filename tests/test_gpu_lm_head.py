"""The LM head fused with greedy sampling (svllm_lm_head_argmax_bf16), through the C ABI.

Reference: torch.matmul(hidden, weight.T) in bf16 on the same GPU (cuBLAS: fp32 accumulation,
one rounding to bf16) and torch.argmax. The fused kernel accumulates in fp32 in its own order
(tcgen05), so a logit may round to the neighbouring bf16 value: the bar is every logit within
one bf16 ulp of cuBLAS's and > 99% identical; the ids equal the argmax of the kernel's own
logits exactly, and cuBLAS's argmax wherever its two largest logits are more than two ulps
apart."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import svllm_capi as capi
from conftest import assert_bf16_within_ulp

pytestmark = pytest.mark.gpu


def run(hidden, weight, with_logits=True):
    rows, vocab = hidden.shape[0], weight.shape[0]
    ids = torch.empty(rows, dtype=torch.int64, device=hidden.device)
    ws = torch.zeros(max(rows, 1), dtype=torch.int64, device=hidden.device)
    logits = (torch.empty(rows, vocab, dtype=torch.bfloat16, device=hidden.device)
              if with_logits else None)
    capi.lm_head_argmax(ids, hidden, weight, ws, logits)
    torch.cuda.synchronize()
    assert int(ws.abs().sum()) == 0, "the workspace must be zero again after the call"
    return ids, logits


def check(hidden, weight):
    ids, logits = run(hidden, weight)
    # against the exact product in fp32: each logit is the fp32 sum rounded once to bf16, so it
    # is within one bf16 ulp of the fp32 value plus the fp32 accumulation's own error
    # (K * 2^-24 of the sum of |terms|, K = hidden size)
    h32, w32 = hidden.float(), weight.float()
    exact = torch.matmul(h32, w32.t())
    terms = torch.matmul(h32.abs(), w32.abs().t())
    bound = 2.0 ** -8 * exact.abs() + hidden.shape[1] * 2.0 ** -24 * terms
    assert bool(((logits.float() - exact).abs() <= bound).all()), "logits vs the fp32 product"
    top2 = exact.topk(2, dim=-1).values
    clear32 = (top2[:, 0] - top2[:, 1]) > 2 * bound.max(dim=-1).values
    assert torch.equal(ids[clear32], torch.argmax(exact, dim=-1)[clear32]), "ids vs fp32 argmax"
    ref = torch.matmul(hidden, weight.t())
    exact = assert_bf16_within_ulp(logits, ref, 1, "logits vs cuBLAS")
    assert exact > 0.99, f"only {exact:.4%} of the logits identical to cuBLAS's"
    assert torch.equal(ids, torch.argmax(logits, dim=-1)), "ids vs the kernel's own logits"
    top2 = ref.float().topk(2, dim=-1).values
    ulp = torch.finfo(torch.bfloat16).eps * top2[:, 0].abs().clamp(min=1e-30)
    clear = (top2[:, 0] - top2[:, 1]) > 2 * ulp
    assert torch.equal(ids[clear], torch.argmax(ref, dim=-1)[clear]), "ids vs cuBLAS's argmax"
    return ids


def make(rows, vocab, hidden_size, cuda, seed, scale=1.0):
    g = torch.Generator(device=cuda).manual_seed(seed)
    h = torch.randn(rows, hidden_size, device=cuda, generator=g).bfloat16()
    w = (torch.randn(vocab, hidden_size, device=cuda, generator=g) * scale).bfloat16()
    return h, w


@pytest.mark.parametrize("rows, vocab, hidden_size", [
    (5, 1000, 64),          # one k-block, one partial tile
    (1, 151936, 1024),      # Qwen3-0.6B decode, one sequence
    (8, 151936, 1024),
    (64, 151936, 1024),
    (130, 128256, 2048),    # Llama-3.2-1B, two row tiles
    (300, 1000, 1024),
    (1024, 151936, 1024),   # eight row tiles
    (3, 4097, 200),         # ragged vocabulary and hidden size (k tail read as zeros)
], ids=str)
def test_matches_cublas_and_argmax(cuda, rows, vocab, hidden_size):
    h, w = make(rows, vocab, hidden_size, cuda, seed=rows + vocab, scale=0.05)
    check(h, w)


def test_strided_rows(cuda):
    """hidden rows as a view of a wider buffer, the weight with padded rows."""
    g = torch.Generator(device=cuda).manual_seed(3)
    hb = torch.randn(40, 1024 + 64, device=cuda, generator=g).bfloat16()
    wb = (torch.randn(5000, 1024 + 32, device=cuda, generator=g) * 0.05).bfloat16()
    check(hb[:, :1024], wb[:, :1024])


def test_ties_and_nan(cuda):
    """Equal logits: the first index wins; a NaN in a row's hidden state makes every logit NaN
    and the answer index 0 (the first NaN)."""
    h, w = make(4, 3000, 128, cuda, seed=5, scale=0.01)
    big = h[0].float() * 4
    for n in (7, 100, 2999):
        w[n] = big.bfloat16()  # row 0's three largest logits, equal
    h[2, 17] = float("nan")
    ids, logits = run(h, w)
    assert ids[0].item() == 7
    assert ids[2].item() == 0 and torch.isnan(logits[2]).all()
    assert torch.equal(ids, torch.argmax(logits, dim=-1))


def test_without_logits_and_repeated_calls(cuda):
    """No logits output; the same workspace across calls (it is left zero)."""
    h, w = make(33, 151936, 1024, cuda, seed=9, scale=0.05)
    ws = torch.zeros(33, dtype=torch.int64, device=cuda)
    first = torch.empty(33, dtype=torch.int64, device=cuda)
    second = torch.empty_like(first)
    capi.lm_head_argmax(first, h, w, ws)
    capi.lm_head_argmax(second, h, w, ws)
    torch.cuda.synchronize()
    assert torch.equal(first, second) and int(ws.abs().sum()) == 0
    ids, _ = run(h, w)
    assert torch.equal(first, ids)


def test_rejects_bad_arguments(cuda):
    h, w = make(4, 100, 64, cuda, seed=1)
    ids = torch.empty(4, dtype=torch.int64, device=cuda)
    small = torch.zeros(2, dtype=torch.int64, device=cuda)
    with pytest.raises(capi.CapiError):
        capi.lm_head_argmax(ids, h, w, small)  # workspace for 2 rows, 4 asked
    hb = torch.randn(4 * 64 + 1, device=cuda).bfloat16()[1:].view(4, 64)  # off 16 bytes
    with pytest.raises(capi.CapiError):
        capi.lm_head_argmax(ids, hb, w, torch.zeros(4, dtype=torch.int64, device=cuda))
