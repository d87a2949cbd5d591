"""Paged decode attention (svllm_paged_decode_attention_bf16) against the same attention in
torch: the request's rows gathered through its block table, softmax(scale * q k^T) v in fp32.
The kernel reads bf16, computes in fp32 and stores bf16, so the bar is one bf16 rounding of the
output plus the fp32 noise of a different summation order: |ours - ref| <= 2^-7 * max|ref| of
the request and head (about 2 bf16 ulps of the largest output), per element."""

from __future__ import annotations

import pytest
import torch

import svllm_capi as capi

pytestmark = pytest.mark.gpu


def reference(q, k_cache, v_cache, tables, seq_lens, scale):
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    num_heads, num_kv = q.shape[1], k_cache.shape[2]
    group = num_heads // num_kv
    bs = k_cache.shape[1]
    for b in range(q.shape[0]):
        n = int(seq_lens[b])
        j = torch.arange(n, device=q.device)
        slots = tables[b].long()[j // bs] * bs + j % bs
        k = k_cache.view(-1, num_kv, k_cache.shape[-1])[slots].float()  # [n, Hk, D]
        v = v_cache.view(-1, num_kv, v_cache.shape[-1])[slots].float()
        for h in range(num_heads):
            s = (k[:, h // group] @ q[b, h].float()) * scale
            p = torch.softmax(s, dim=0)
            out[b, h] = p @ v[:, h // group]
    return out


def make_case(cuda, seqs, heads, kv_heads, dim, max_len, bs, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    max_blocks = (max_len + bs - 1) // bs
    num_blocks = seqs * max_blocks + 3
    k_cache = torch.randn(num_blocks, bs, kv_heads, dim, device=cuda, generator=g).bfloat16()
    v_cache = torch.randn(num_blocks, bs, kv_heads, dim, device=cuda, generator=g).bfloat16()
    perm = torch.randperm(num_blocks, device=cuda, generator=g)[: seqs * max_blocks]
    tables = perm.view(seqs, max_blocks).to(torch.int32)
    q = torch.randn(seqs, heads, dim, device=cuda, generator=g).bfloat16()
    return q, k_cache, v_cache, tables


@pytest.mark.parametrize("seqs, heads, kv_heads, dim, max_len, bs", [
    (1, 16, 8, 128, 1, 16),       # one cached token
    (1, 16, 8, 128, 700, 16),     # one request: the context split over a cluster
    (3, 16, 8, 128, 2000, 16),
    (64, 16, 8, 128, 513, 16),    # Qwen3-0.6B decode batch
    (5, 32, 8, 64, 300, 16),      # Llama-3.2-1B
    (4, 8, 1, 128, 900, 16),      # eight query heads per KV head
    (3, 16, 4, 128, 777, 16),     # four query heads per KV head
    (2, 4, 4, 64, 5000, 16),      # no grouping, long contexts (16-warp CTAs)
    (1, 16, 8, 128, 4096, 16),    # one long request: 16-warp CTAs at head dim 128
    (3, 16, 8, 128, 333, 1),      # one row per page
    (3, 16, 8, 128, 1000, 12),    # pages that tiles of 16 rows straddle
    (2, 16, 8, 64, 1500, 3),
    (3, 16, 8, 128, 1300, 256),   # large pages
], ids=str)
def test_matches_torch(cuda, seqs, heads, kv_heads, dim, max_len, bs):
    g = torch.Generator(device=cuda).manual_seed(seqs * 1000 + max_len + bs)
    max_blocks = (max_len + bs - 1) // bs
    num_blocks = seqs * max_blocks + 3
    k_cache = torch.randn(num_blocks, bs, kv_heads, dim, device=cuda, generator=g).bfloat16()
    v_cache = torch.randn(num_blocks, bs, kv_heads, dim, device=cuda, generator=g).bfloat16()
    # blocks handed out in a random order, tables padded with block 0 past each context
    perm = torch.randperm(num_blocks, device=cuda, generator=g)[: seqs * max_blocks]
    tables = perm.view(seqs, max_blocks).to(torch.int32)
    seq_lens = torch.randint(1, max_len + 1, (seqs,), device=cuda, generator=g,
                             dtype=torch.int32)
    seq_lens[0] = max_len
    # q as the leading columns of a wider qkv row, as the model passes it
    qkv = torch.randn(seqs, (heads + 2 * kv_heads) * dim, device=cuda, generator=g).bfloat16()
    q = qkv[:, : heads * dim].view(seqs, heads, dim)
    scale = dim ** -0.5
    out = torch.empty(seqs, heads, dim, dtype=torch.bfloat16, device=cuda)
    capi.read_device_error(0, reset=True)
    capi.paged_decode_attention(out, q, k_cache, v_cache, tables, seq_lens, max_len, scale)
    ref = reference(q, k_cache, v_cache, tables, seq_lens, scale)
    torch.cuda.synchronize()
    assert capi.read_device_error(0, reset=True) == 0
    bar = 2.0 ** -7 * ref.abs().amax(dim=-1, keepdim=True)
    assert ((out.float() - ref).abs() <= bar).all()


def test_rejects_unsupported_shapes(cuda):
    q = torch.zeros(1, 6, 128, dtype=torch.bfloat16, device=cuda)  # 6 / 2 = 3 heads per group
    cache = torch.zeros(2, 16, 2, 128, dtype=torch.bfloat16, device=cuda)
    tables = torch.zeros(1, 1, dtype=torch.int32, device=cuda)
    lens = torch.ones(1, dtype=torch.int32, device=cuda)
    out = torch.empty_like(q)
    with pytest.raises(capi.CapiError):
        capi.paged_decode_attention(out, q, cache, cache, tables, lens, 16, 0.1)


def test_empty_requests_and_bad_entries(cuda):
    """A request of length 0 gets zeros; a table entry outside the cache or a length past the
    table raises the bad-index bit (the kernel reads block 0 / stops at the table's end) and
    leaves the other requests exact."""
    seqs, heads, kv, dim, bs, max_len = 4, 16, 8, 128, 16, 200
    q, k_cache, v_cache, tables = make_case(cuda, seqs, heads, kv, dim, max_len, bs, seed=7)
    lens = torch.tensor([0, 200, 37, 150], dtype=torch.int32, device=cuda)
    out = torch.full((seqs, heads, dim), 7.0, dtype=torch.bfloat16, device=cuda)
    capi.read_device_error(0, reset=True)
    capi.paged_decode_attention(out, q, k_cache, v_cache, tables, lens, max_len, dim ** -0.5)
    ref = reference(q, k_cache, v_cache, tables, lens, dim ** -0.5)
    torch.cuda.synchronize()
    assert capi.read_device_error(0, reset=True) == 0
    assert (out[0] == 0).all()
    bar = 2.0 ** -7 * ref[1:].abs().amax(dim=-1, keepdim=True)
    assert ((out[1:].float() - ref[1:]).abs() <= bar).all()

    bad = tables.clone()
    bad[2, 1] = k_cache.shape[0]          # one past the last block
    bad_lens = lens.clone()
    bad_lens[3] = tables.shape[1] * bs + 5  # past the block table
    capi.paged_decode_attention(out, q, k_cache, v_cache, bad, bad_lens, max_len, dim ** -0.5)
    torch.cuda.synchronize()
    assert capi.read_device_error(0, reset=True) == capi.DEVERR_BAD_INDEX
    assert ((out[1].float() - ref[1]).abs() <= bar[0]).all()  # request 1 untouched by the others
