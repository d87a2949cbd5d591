"""svllm_ops' fused layer ops against torch composites of the Hugging Face formulas, on CPU (the
OpenMP backend) and CUDA (the sm_100a kernels, marked gpu), in the reference's op-test style
(parametrized shapes, seeded inputs, its bf16 tolerance) plus argument checks."""

from __future__ import annotations

import pytest
import svllm_ops
import torch
import torch.nn.functional as F
from conftest import assert_close_bf16, random_bf16, random_t

QWEN_EPS = 1e-6
LLAMA3 = (8.0, 1.0, 4.0, 8192)


def hf_rms_norm(x, w, eps):
    """Qwen3RMSNorm: fp32 normalise, round to x's dtype, multiply by the weight."""
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return w * (xf * torch.rsqrt(var + eps)).to(x.dtype)


def hf_rope(x, pos, inv_freq):
    """apply_rotary_pos_emb on [T, H, D] with Hugging Face's fp32 angles and bf16 cos/sin."""
    freqs = pos.float()[:, None] * inv_freq.to(x.device)[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().to(x.dtype)[:, None, :], emb.sin().to(x.dtype)[:, None, :]
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos + rot * sin


# ---------------------------------------------------------------------------------------------
# add_rms_norm

@pytest.mark.parametrize("shape", [(1, 1024), (7, 1024), (300, 1024), (5, 2048), (3, 4100),
                                   (0, 1024)], ids=str)
def test_add_rms_norm(device, shape):
    x = random_bf16(*shape, device=device, seed=3)
    r = random_bf16(*shape, device=device, seed=4)
    w = random_t(shape[-1], device=device, seed=5, scale=0.1, shift=1.0)
    expected_r = x + r
    expected_x = hf_rms_norm(expected_r, w, QWEN_EPS)
    svllm_ops.add_rms_norm(x, r, w, QWEN_EPS)
    assert torch.equal(r, expected_r), "the residual add is one bf16 rounding: bit-exact"
    assert_close_bf16(x, expected_x)


def test_add_rms_norm_rejects_mismatch():
    x = torch.ones(2, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="do not match"):
        svllm_ops.add_rms_norm(x, torch.ones(2, 4, dtype=torch.bfloat16),
                               torch.ones(8, dtype=torch.bfloat16), 1e-6)
    with pytest.raises(RuntimeError, match="expected bf16"):
        svllm_ops.add_rms_norm(x.float(), x, torch.ones(8, dtype=torch.bfloat16), 1e-6)
    with pytest.raises(RuntimeError, match="unsupported device"):
        m = torch.ones(2, 8, dtype=torch.bfloat16, device="meta")
        svllm_ops.add_rms_norm(m, m, torch.ones(8, dtype=torch.bfloat16, device="meta"), 1e-6)


# ---------------------------------------------------------------------------------------------
# qk_norm_rope (Qwen3) and rope (Llama)

@pytest.mark.parametrize("T, pos_dtype", [(1, torch.int64), (7, torch.int32), (64, torch.int64)])
def test_qk_norm_rope(device, T, pos_dtype):
    q = random_bf16(T, 16, 128, device=device, seed=6)
    k = random_bf16(T, 8, 128, device=device, seed=7)
    qw = random_t(128, device=device, seed=8, scale=0.1, shift=1.0)
    kw = random_t(128, device=device, seed=9, scale=0.1, shift=1.0)
    g = torch.Generator().manual_seed(10)
    pos = torch.randint(0, 32768, (T,), generator=g).to(device=device, dtype=pos_dtype)
    inv = svllm_ops.rope_inv_freq(1e6, 128)
    eq = hf_rope(hf_rms_norm(q, qw, QWEN_EPS), pos, inv)
    ek = hf_rope(hf_rms_norm(k, kw, QWEN_EPS), pos, inv)
    svllm_ops.qk_norm_rope(q, k, qw, kw, pos, QWEN_EPS, 1e6)
    assert_close_bf16(q, eq, atol=2e-2)
    assert_close_bf16(k, ek, atol=2e-2)


@pytest.mark.parametrize("factor", [8.0, 32.0])
def test_llama3_rope(device, factor):
    T = 33
    q = random_bf16(T, 32, 64, device=device, seed=11)
    k = random_bf16(T, 8, 64, device=device, seed=12)
    pos = torch.arange(T, device=device) * 61
    scaling = svllm_ops.Llama3RopeScaling(factor, 1.0, 4.0, 8192)
    inv = svllm_ops.rope_inv_freq(5e5, 64, scaling)
    eq, ek = hf_rope(q, pos, inv), hf_rope(k, pos, inv)
    svllm_ops.rope(q, k, pos, 5e5, scaling)
    assert_close_bf16(q, eq, atol=2e-2)
    assert_close_bf16(k, ek, atol=2e-2)


def test_rope_on_views_of_a_fused_qkv_tensor(device):
    T, hq, hk, d = 9, 16, 8, 128
    qkv = random_bf16(T, (hq + 2 * hk) * d, device=device, seed=13)
    q = qkv[:, : hq * d].view(T, hq, d)
    k = qkv[:, hq * d:(hq + hk) * d].view(T, hk, d)
    v_before = qkv[:, (hq + hk) * d:].clone()
    pos = torch.arange(T, device=device)
    inv = svllm_ops.rope_inv_freq(1e6, d)
    eq, ek = hf_rope(q.clone(), pos, inv), hf_rope(k.clone(), pos, inv)
    svllm_ops.rope(q, k, pos, 1e6)
    assert_close_bf16(q, eq, atol=2e-2)
    assert_close_bf16(k, ek, atol=2e-2)
    assert torch.equal(qkv[:, (hq + hk) * d:], v_before), "v must be untouched"


def test_rope_inv_freq_is_hugging_face_bit_for_bit():
    from conftest import golden

    g = golden()
    assert torch.equal(svllm_ops.rope_inv_freq(1e6, 128),
                       torch.from_numpy(g["inv_freq/qwen3"]))
    for factor, name in ((8.0, "llama3"), (32.0, "llama3_f32x")):
        s = svllm_ops.Llama3RopeScaling(factor, 1.0, 4.0, 8192)
        assert torch.equal(svllm_ops.rope_inv_freq(5e5, 64, s), torch.from_numpy(g[f"inv_freq/{name}"]))


def test_rope_rejects_bad_inputs():
    q = torch.ones(2, 4, 8, dtype=torch.bfloat16)
    k = torch.ones(2, 2, 8, dtype=torch.bfloat16)
    pos = torch.arange(2)
    with pytest.raises(RuntimeError, match="expected bf16"):
        svllm_ops.rope(q.float(), k, pos, 1e4)
    with pytest.raises(RuntimeError, match="int32 or int64"):
        svllm_ops.rope(q, k, pos.float(), 1e4)
    with pytest.raises(RuntimeError, match="positions for"):
        svllm_ops.rope(q, k, torch.arange(3), 1e4)
    with pytest.raises(RuntimeError, match="do not match"):
        svllm_ops.rope(q, torch.ones(2, 2, 6, dtype=torch.bfloat16), pos, 1e4)
    with pytest.raises(RuntimeError, match="even"):
        svllm_ops.rope(torch.ones(2, 4, 7, dtype=torch.bfloat16),
                       torch.ones(2, 2, 7, dtype=torch.bfloat16), pos, 1e4)
    with pytest.raises(RuntimeError, match="contiguous heads"):
        svllm_ops.rope(torch.ones(2, 8, 4, dtype=torch.bfloat16).transpose(1, 2), k, pos, 1e4)
    with pytest.raises(RuntimeError, match="unsupported device"):
        m = lambda t: t.to("meta")  # noqa: E731
        svllm_ops.rope(m(q), m(k), m(pos), 1e4)


# ---------------------------------------------------------------------------------------------
# silu_and_mul

@pytest.mark.parametrize("shape", [(1, 3072), (7, 3072), (130, 8192), (3, 3001), (0, 3072),
                                   (2, 3, 256)], ids=str)
def test_silu_and_mul(device, shape):
    gate = random_bf16(*shape, device=device, seed=14) * 3
    up = random_bf16(*shape, device=device, seed=15)
    expected = F.silu(gate) * up
    out = svllm_ops.silu_and_mul(gate, up)
    assert out.shape == gate.shape and out.is_contiguous()
    assert_close_bf16(out, expected)


def test_silu_and_mul_on_halves_of_a_gate_up_projection(device):
    gate_up = random_bf16(17, 2 * 3072, device=device, seed=16)
    gate, up = gate_up[:, :3072], gate_up[:, 3072:]
    assert_close_bf16(svllm_ops.silu_and_mul(gate, up), F.silu(gate) * up)


def test_silu_and_mul_rejects_bad_inputs():
    a = torch.ones(2, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="expected bf16"):
        svllm_ops.silu_and_mul(a.float(), a)
    with pytest.raises(RuntimeError, match="does not match"):
        svllm_ops.silu_and_mul(a, torch.ones(2, 4, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="contiguous last"):
        svllm_ops.silu_and_mul(torch.ones(8, 2, dtype=torch.bfloat16).t(), a)


# ---------------------------------------------------------------------------------------------
# embedding

@pytest.mark.parametrize("ids_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("shape", [(1,), (37,), (4, 9), (0,)], ids=str)
def test_embedding(device, ids_dtype, shape):
    vocab, hidden = 1000, 1024
    table = random_t(vocab, hidden, device=device, seed=17, scale=0.02)
    g = torch.Generator().manual_seed(18)
    ids = torch.randint(0, vocab, shape, generator=g).to(device=device, dtype=ids_dtype)
    out = svllm_ops.embedding(ids, table)
    assert out.shape == (*shape, hidden)
    assert torch.equal(out, F.embedding(ids.long(), table)), "the gather is bit-exact"


def test_embedding_out_of_range_ids_fail_on_cpu():
    table = torch.ones(10, 16, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="ids outside"):
        svllm_ops.embedding(torch.tensor([1, 10, -1]), table)


def test_embedding_rejects_bad_inputs():
    table = torch.ones(10, 16, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="int32 or int64"):
        svllm_ops.embedding(torch.tensor([1.0]), table)
    with pytest.raises(RuntimeError, match="bf16 table"):
        svllm_ops.embedding(torch.tensor([1]), table.float())
    with pytest.raises(RuntimeError, match="vocab, hidden"):
        svllm_ops.embedding(torch.tensor([1]), torch.ones(16, dtype=torch.bfloat16))


# ---------------------------------------------------------------------------------------------
# rotary + paged-KV cache write

def _paged_slots(T, num_blocks, block_size, device, seed):
    """Tokens laid out block by block over a random permutation of cache blocks, a few padded."""
    g = torch.Generator().manual_seed(seed)
    blocks = torch.randperm(num_blocks, generator=g)[: (T + block_size - 1) // block_size]
    t = torch.arange(T)
    slots = blocks[t // block_size] * block_size + t % block_size
    slots[::7] = -1  # padding tokens write nothing
    return slots.to(device)


@pytest.mark.parametrize("with_norm", [True, False], ids=["qk_norm_rope_cache", "rope_cache"])
def test_rope_cache(device, with_norm):
    T, hq, hk, d, blocks, bs = 37, 16, 8, 128, 20, 16
    qkv = random_bf16(T, (hq + 2 * hk) * d, device=device, seed=20)
    q = qkv[:, : hq * d].view(T, hq, d)
    k = qkv[:, hq * d:(hq + hk) * d].view(T, hk, d)
    v = qkv[:, (hq + hk) * d:].view(T, hk, d)
    qw = random_t(d, device=device, seed=21, scale=0.1, shift=1.0)
    kw = random_t(d, device=device, seed=22, scale=0.1, shift=1.0)
    pos = torch.arange(T, device=device) * 3
    slots = _paged_slots(T, blocks, bs, device, seed=23)
    k_cache = torch.full((blocks, bs, hk, d), 5.0, dtype=torch.bfloat16, device=device)
    v_cache = torch.full((blocks, bs, hk, d), 7.0, dtype=torch.bfloat16, device=device)
    inv = svllm_ops.rope_inv_freq(1e6, d)
    if with_norm:
        eq = hf_rope(hf_rms_norm(q, qw, QWEN_EPS), pos, inv)
        ek = hf_rope(hf_rms_norm(k, kw, QWEN_EPS), pos, inv)
    else:
        eq, ek = hf_rope(q.clone(), pos, inv), hf_rope(k.clone(), pos, inv)
    ev = v.clone()
    if with_norm:
        svllm_ops.qk_norm_rope_cache(q, k, v, qw, kw, pos, slots, k_cache, v_cache, QWEN_EPS, 1e6)
    else:
        svllm_ops.rope_cache(q, k, v, pos, slots, k_cache, v_cache, 1e6)
    assert_close_bf16(q, eq, atol=2e-2)
    assert_close_bf16(k, ek, atol=2e-2)
    flat_k, flat_v = k_cache.view(-1, hk, d), v_cache.view(-1, hk, d)
    written = slots >= 0
    assert torch.equal(flat_k[slots[written]], k[written]), "cache holds the rotated k"
    assert torch.equal(flat_v[slots[written]], ev[written]), "cache holds v"
    untouched = torch.ones(blocks * bs, dtype=torch.bool, device=device)
    untouched[slots[written]] = False
    assert (flat_k[untouched] == 5.0).all() and (flat_v[untouched] == 7.0).all()


def test_rope_cache_rejects_bad_caches():
    q, k = torch.ones(2, 4, 8, dtype=torch.bfloat16), torch.ones(2, 2, 8, dtype=torch.bfloat16)
    pos, slots = torch.arange(2), torch.tensor([0, 1])
    good = torch.zeros(4, 2, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="caches must be"):
        svllm_ops.rope_cache(q, k, k.clone(), pos, slots, torch.zeros(4, 3, 8, dtype=torch.bfloat16),
                             good, 1e4)
    with pytest.raises(RuntimeError, match="slot_mapping"):
        svllm_ops.rope_cache(q, k, k.clone(), pos, slots.int(), good, good.clone(), 1e4)
    with pytest.raises(RuntimeError, match="slots past"):
        svllm_ops.rope_cache(q, k, k.clone(), pos, torch.tensor([0, 4]), good, good.clone(), 1e4)


@pytest.mark.parametrize("shape", [(5, 2 * 3072), (2, 3, 2 * 512), (2 * 256,)], ids=str)
def test_silu_and_mul_on_one_gate_up_tensor(device, shape):
    gate_up = random_bf16(*shape, device=device, seed=24)
    inter = shape[-1] // 2
    out = svllm_ops.silu_and_mul(gate_up)
    assert out.shape == (*shape[:-1], inter)
    assert torch.equal(out, svllm_ops.silu_and_mul(gate_up[..., :inter].contiguous(),
                                                   gate_up[..., inter:].contiguous()))
    assert_close_bf16(out, F.silu(gate_up[..., :inter]) * gate_up[..., inter:])
    with pytest.raises(RuntimeError, match="even last dimension"):
        svllm_ops.silu_and_mul(gate_up[..., :-1])


# ---------------------------------------------------------------------------------------------
# greedy sampling

@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
@pytest.mark.parametrize("shape", [(1, 151936), (7, 1000), (3, 4, 700), (2, 17)], ids=str)
def test_argmax(device, dtype, shape):
    logits = random_t(*shape, dtype=dtype, device=device, seed=25)
    assert torch.equal(svllm_ops.argmax(logits), torch.argmax(logits, dim=-1))


def test_argmax_ties_nan_and_infinities(device):
    logits = torch.zeros(4, 5000, dtype=torch.bfloat16, device=device)
    logits[0, [17, 300, 4999]] = 3.0           # a tie: the first index wins
    logits[1, 123] = float("nan")              # NaN beats any number
    logits[1, 4000] = float("nan")
    logits[1, 10] = float("inf")
    logits[2, :] = float("-inf")               # all -inf: index 0
    logits[3, 4999] = 1.0                      # the last element
    assert svllm_ops.argmax(logits).tolist() == [17, 123, 0, 4999]


def test_greedy_sample_with_a_tied_lm_head(device):
    hidden = random_bf16(6, 256, device=device, seed=26)
    table = random_t(3000, 256, device=device, seed=27, scale=0.02)
    logits = hidden @ table.t()
    assert torch.equal(svllm_ops.greedy_sample(hidden, table), torch.argmax(logits, dim=-1))


def test_argmax_rejects_bad_inputs():
    with pytest.raises(RuntimeError, match="bf16 or fp32"):
        svllm_ops.argmax(torch.zeros(2, 3, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="contiguous last"):
        svllm_ops.argmax(torch.zeros(8, 2).t())
