"""The decode-sized linear layer (svllm_decode_linear_bf16, up to 16 token rows), through the C
ABI.

Reference: the same product in fp32 on the GPU (x.float() @ w.float().T), rounded once to bf16.
The kernel accumulates in fp32 in its own order (mma.sync over K chunks, the warps' partial sums
added in shared memory). Two fp32 sums of the same K products differ by at most
2 K 2^-24 sum_k |x_k w_k| (the worst-case bound of recursive summation, for each of them), and
each is then rounded to bf16: the bar per element is |ours - ref| <= 2^-7 |ref| (one bf16
rounding step) + 2 K 2^-24 sum_k |x_k w_k|, and more than 99% of the elements identical."""

from __future__ import annotations

import pytest
import torch

import svllm_capi as capi

pytestmark = pytest.mark.gpu


def make(rows, out_features, in_features, cuda, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    x = torch.randn(rows, in_features, device=cuda, generator=g).bfloat16()
    w = (torch.randn(out_features, in_features, device=cuda, generator=g) * 0.02).bfloat16()
    return x, w


def check(x, w, out=None):
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0], dtype=torch.bfloat16, device=x.device)
    capi.decode_linear(out, x, w)
    ref = (x.float() @ w.float().t()).bfloat16().float()
    mag = x.float().abs() @ w.float().abs().t()
    torch.cuda.synchronize()
    bar = 2.0 ** -7 * ref.abs() + 2 * x.shape[1] * 2.0 ** -24 * mag
    err = (out.float() - ref).abs()
    bad = err > bar
    assert not bad.any(), (f"{int(bad.sum())} of {bad.numel()} outputs off the bar (worst "
                           f"{float((err - bar).max()):.3g} past it)")
    exact = float((out.float() == ref).float().mean())
    assert exact > 0.99, f"only {exact:.4%} identical to the rounded fp32 product"
    return out


@pytest.mark.parametrize("rows", [1, 5, 8, 9, 16], ids=lambda r: f"rows{r}")
@pytest.mark.parametrize("out_features, in_features", [
    (4096, 1024),   # Qwen3-0.6B qkv
    (1024, 2048),   # Qwen3-0.6B o_proj
    (6144, 1024),   # Qwen3-0.6B gate_up
    (1024, 3072),   # Qwen3-0.6B down
    (3072, 2048),   # Llama-3.2-1B qkv
    (2048, 8192),   # Llama-3.2-1B down
], ids=lambda v: str(v))
def test_matches_fp32(cuda, rows, out_features, in_features):
    x, w = make(rows, out_features, in_features, cuda, seed=rows * 7 + out_features + in_features)
    check(x, w)


@pytest.mark.parametrize("rows, out_features, in_features", [
    (3, 1000, 200),    # ragged rows, a K tail inside the last chunk of 32
    (7, 4097, 64),     # two chunks, a partial last row tile
    (16, 130, 8),      # one 16-byte piece of K
    (2, 128, 4096),
    (11, 24, 13000),   # 16 warps, several register rounds each
], ids=str)
def test_ragged_shapes(cuda, rows, out_features, in_features):
    x, w = make(rows, out_features, in_features, cuda, seed=rows + out_features)
    check(x, w)


def test_strided_operands_and_output(cuda):
    """x a view of a wider buffer (the attention output inside a bigger row), the weight with
    padded rows, the output written into the leading columns of a wider buffer."""
    g = torch.Generator(device=cuda).manual_seed(11)
    xb = torch.randn(9, 2048 + 64, device=cuda, generator=g).bfloat16()
    wb = (torch.randn(1024, 2048 + 32, device=cuda, generator=g) * 0.02).bfloat16()
    outb = torch.full((9, 1024 + 40), 3.0, dtype=torch.bfloat16, device=cuda)
    check(xb[:, :2048], wb[:, :2048], outb[:, :1024])
    assert (outb[:, 1024:] == 3.0).all(), "columns past out_features must be untouched"


def test_deterministic_and_error_word(cuda):
    x, w = make(13, 1024, 3072, cuda, seed=5)
    capi.read_device_error(0, reset=True)
    first = check(x, w)
    second = check(x, w)
    assert torch.equal(first, second), "the warps' partial sums are added in a fixed order"
    assert capi.read_device_error(0, reset=True) == 0


def test_rejects_what_it_does_not_take(cuda):
    """Unsupported shapes are refused with a status (the model forward then calls its GEMM)."""
    x, w = make(17, 256, 128, cuda, seed=1)
    out = torch.empty(17, 256, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(capi.CapiError):
        capi.decode_linear(out, x, w)  # more rows than a decode batch
    xb = torch.randn(4 * 128 + 1, device=cuda).bfloat16()[1:].view(4, 128)  # off 16 bytes
    with pytest.raises(capi.CapiError):
        capi.decode_linear(out[:4], xb, w)
    g = torch.Generator(device=cuda).manual_seed(13)
    xk = torch.randn(5, 104, device=cuda, generator=g).bfloat16()[:, :100]
    wk = torch.randn(300, 104, device=cuda, generator=g).bfloat16()[:, :100]
    with pytest.raises(capi.CapiError):  # K not a multiple of 8: no whole 16-byte pieces
        capi.decode_linear(torch.empty(5, 300, dtype=torch.bfloat16, device=cuda), xk, wk)
    empty = torch.empty(0, 128, dtype=torch.bfloat16, device=cuda)
    capi.decode_linear(out[:0], empty, w)  # no rows: nothing launched
