"""Five whole workloads, end to end through svllm_ops on the GPU.

  fp32       Qwen3 shapes, fp32, T=256 (through the C ABI's fp32 entry points: svllm_ops is bf16
             only, like the reference) against the C/OpenMP oracle, 1e-5 relative.
  decode     Qwen3, bf16, 256 single-token sequences, positions uniform in [0, 4096).
  prefill    Qwen3 packed prefill, 64 sequences of uniform [128, 2048] tokens, positions
             0..len-1.
  llama      Llama-3.2-1B shapes, T=16384 = 8 x 2048, llama3 rope scaling at factor 32 and 8
             (the model's config.json).
  sweep      the 1,048,576-token bandwidth sweep at full size.

At full size the bf16 checks are the size-independent ones: bit-identity with the reference's own
rms_norm kernel (oracle/_ref) on the same GPU, bit-identity with the torch composites that call
the same CUDA math functions, the exact gather, plus a sample of rows against the CPU oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
import svllm_capi as capi
import svllm_ops
from conftest import assert_bf16_within_ulp, assert_rel_f32, rope_within_rounding, to_bits

pytestmark = pytest.mark.gpu

QWEN = dict(hidden=1024, heads=16, kv_heads=8, head_dim=128, inter=3072, vocab=151936, eps=1e-6,
            theta=1e6)
LLAMA = dict(hidden=2048, heads=32, kv_heads=8, head_dim=64, inter=8192, vocab=128256, eps=1e-5,
             theta=5e5)


def rand(shape, device, gen, dtype=torch.bfloat16, scale=1.0, shift=0.0):
    t = torch.empty(shape, device=device, dtype=torch.float32).normal_(shift, scale, generator=gen)
    return t.to(dtype)


def torch_rope(x, pos, inv):
    freqs = pos.float()[:, None] * inv.to(x.device)[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().to(x.dtype)[:, None, :], emb.sin().to(x.dtype)[:, None, :]
    half = x.shape[-1] // 2
    return x * cos + torch.cat((-x[..., half:], x[..., :half]), dim=-1) * sin


def make(cfg, T, device, seed, pos=None, pos_hi=4096):
    gen = torch.Generator(device=device).manual_seed(seed)
    d = cfg["head_dim"]
    inp = {
        "table": rand((cfg["vocab"], cfg["hidden"]), device, gen, scale=0.02),
        "ids": torch.randint(0, cfg["vocab"], (T,), device=device, generator=gen,
                             dtype=torch.int32),
        "x": rand((T, cfg["hidden"]), device, gen), "r": rand((T, cfg["hidden"]), device, gen),
        "w": rand((cfg["hidden"],), device, gen, scale=0.1, shift=1.0),
        "q": rand((T, cfg["heads"], d), device, gen), "k": rand((T, cfg["kv_heads"], d), device, gen),
        "qw": rand((d,), device, gen, scale=0.1, shift=1.0),
        "kw": rand((d,), device, gen, scale=0.1, shift=1.0),
        "gate": rand((T, cfg["inter"]), device, gen), "up": rand((T, cfg["inter"]), device, gen),
    }
    inp["pos"] = pos if pos is not None else torch.randint(0, pos_hi, (T,), device=device,
                                                           generator=gen)
    return inp


def check_chain_bf16(inp, cfg, qk_norm=True, scaling=None, sample_rows=512):
    """Runs the chain through svllm_ops and checks it against the reference kernel / torch
    composites on the same GPU (every row) and the CPU oracle (a sample of rows)."""
    ref = oracle.reference_module()
    assert ref is not None, "oracle/_ref was not built"
    d, eps = cfg["head_dim"], cfg["eps"]
    T = inp["ids"].shape[0]
    rows = torch.linspace(0, T - 1, min(sample_rows, T)).long().unique().to(inp["ids"].device)
    per_token = ("x", "r", "q", "k", "gate", "up")
    host = {k: to_bits(inp[k][rows]) for k in per_token}
    host.update({k: to_bits(inp[k]) for k in ("w", "qw", "kw")})
    host["pos"] = inp["pos"][rows].cpu().numpy()
    host["ids"] = inp["ids"][rows].cpu().numpy()

    # embedding
    emb = svllm_ops.embedding(inp["ids"], inp["table"])
    assert torch.equal(emb, inp["table"][inp["ids"].long()])
    # add + RMSNorm: the reference's path is a LibTorch add then its rms_norm kernel
    summed = inp["x"] + inp["r"]
    expect_x = ref.rms_norm(summed, inp["w"], eps)
    svllm_ops.add_rms_norm(inp["x"], inp["r"], inp["w"], eps)
    assert torch.equal(inp["r"], summed)
    assert torch.equal(inp["x"], expect_x)
    del summed, expect_x
    # q/k norm + rope, or rope alone
    sc = svllm_ops.Llama3RopeScaling(*scaling) if scaling else None
    inv = svllm_ops.rope_inv_freq(cfg["theta"], d, sc)
    if qk_norm:
        eq = torch_rope(ref.rms_norm(inp["q"].reshape(-1, d), inp["qw"], eps).view(inp["q"].shape),
                        inp["pos"], inv)
        ek = torch_rope(ref.rms_norm(inp["k"].reshape(-1, d), inp["kw"], eps).view(inp["k"].shape),
                        inp["pos"], inv)
        svllm_ops.qk_norm_rope(inp["q"], inp["k"], inp["qw"], inp["kw"], inp["pos"], eps,
                               cfg["theta"], sc)
    else:
        eq, ek = torch_rope(inp["q"], inp["pos"], inv), torch_rope(inp["k"], inp["pos"], inv)
        svllm_ops.rope(inp["q"], inp["k"], inp["pos"], cfg["theta"], sc)
    assert torch.equal(inp["q"], eq) and torch.equal(inp["k"], ek)
    del eq, ek
    # SiLU * up
    y = svllm_ops.silu_and_mul(inp["gate"], inp["up"])
    assert torch.equal(y, F.silu(inp["gate"]) * inp["up"])

    # sampled rows against the CPU oracle
    o_emb, bad = oracle.embedding(host["ids"], to_bits(inp["table"]))
    assert bad == 0 and np.array_equal(to_bits(emb[rows]), o_emb)
    ox, orr = oracle.add_rms_norm(host["x"], host["r"], host["w"], eps)
    assert np.array_equal(to_bits(inp["r"][rows]), orr)
    assert_bf16_within_ulp(inp["x"][rows], ox, 2, "add_rms_norm vs oracle")
    invn = inv.numpy()
    if qk_norm:
        oq, ok = oracle.qk_norm_rope(host["q"], host["k"], host["qw"], host["kw"], host["pos"],
                                     eps, invn)
    else:
        oq, ok = oracle.rope(host["q"], host["k"], host["pos"], invn)
    # every sampled element within one rounding of each rotation term, and > 99% bit-exact
    if qk_norm:
        pre_q = oracle.rms_norm(host["q"].reshape(-1, d), host["qw"], eps).reshape(host["q"].shape)
        pre_k = oracle.rms_norm(host["k"].reshape(-1, d), host["kw"], eps).reshape(host["k"].shape)
    else:
        pre_q, pre_k = host["q"], host["k"]
    assert rope_within_rounding(to_bits(inp["q"][rows]), oq, pre_q).all()
    assert rope_within_rounding(to_bits(inp["k"][rows]), ok, pre_k).all()
    assert (to_bits(inp["q"][rows]) == oq).mean() > 0.99
    assert (to_bits(inp["k"][rows]) == ok).mean() > 0.99
    oy = oracle.silu_and_mul(host["gate"], host["up"])
    assert_bf16_within_ulp(y[rows], oy, 2, "silu_and_mul vs oracle")


def test_qwen3_fp32_t256(cuda):
    cfg, T = QWEN, 256
    g = torch.Generator().manual_seed(0)
    f = lambda *s, scale=1.0, shift=0.0: (torch.randn(s, generator=g) * scale + shift)  # noqa
    table = f(cfg["vocab"], cfg["hidden"], scale=0.02)
    ids = torch.randint(0, cfg["vocab"], (T,), generator=g, dtype=torch.int32)
    x, r, w = f(T, 1024), f(T, 1024), f(1024, scale=0.1, shift=1.0)
    q, k = f(T, 16, 128), f(T, 8, 128)
    qw, kw = f(128, scale=0.1, shift=1.0), f(128, scale=0.1, shift=1.0)
    pos = torch.arange(T)
    gate, up = f(T, 3072), f(T, 3072)
    inv = oracle.inv_freq(1e6, 128)
    o_emb, _ = oracle.embedding(ids.numpy(), table.numpy())
    ox, orr = oracle.add_rms_norm(x.numpy(), r.numpy(), w.numpy(), 1e-6)
    oq, ok = oracle.qk_norm_rope(q.numpy(), k.numpy(), qw.numpy(), kw.numpy(), pos.numpy(), 1e-6,
                                 inv)
    oy = oracle.silu_and_mul(gate.numpy(), up.numpy())

    dv = {n: t.to(cuda) for n, t in dict(table=table, ids=ids, x=x, r=r, w=w, q=q, k=k, qw=qw,
                                          kw=kw, pos=pos, gate=gate, up=up).items()}
    emb = torch.empty(T, 1024, device=cuda)
    capi.embedding(emb, dv["ids"], dv["table"])
    capi.add_rms_norm(dv["x"], dv["r"], dv["w"], 1e-6)
    capi.qk_norm_rope(dv["q"], dv["k"], dv["qw"], dv["kw"], dv["pos"], 1e-6, inv)
    y = torch.empty(T, 3072, device=cuda)
    capi.silu_and_mul(y, dv["gate"], dv["up"])
    assert np.array_equal(emb.cpu().numpy(), o_emb)
    assert np.array_equal(dv["r"].cpu().numpy(), orr)
    assert_rel_f32(dv["x"], ox, 1e-5, "x")
    pre_q = oracle.rms_norm(q.numpy().reshape(-1, 128), qw.numpy(), 1e-6).reshape(q.shape)
    pre_k = oracle.rms_norm(k.numpy().reshape(-1, 128), kw.numpy(), 1e-6).reshape(k.shape)

    def pair(pre):
        p = np.abs(pre.astype(np.float64))
        m = p[..., :64] + p[..., 64:]
        return np.concatenate([m, m], axis=-1)

    assert_rel_f32(dv["q"], oq, 1e-5, "q", scale=pair(pre_q))
    assert_rel_f32(dv["k"], ok, 1e-5, "k", scale=pair(pre_k))
    assert_rel_f32(y, oy, 1e-5, "silu")


def test_qwen3_decode(cuda):
    inp = make(QWEN, 256, cuda, seed=1, pos_hi=4096)
    check_chain_bf16(inp, QWEN)


def test_qwen3_packed_prefill(cuda):
    g = torch.Generator().manual_seed(2)
    lens = torch.randint(128, 2049, (64,), generator=g)
    pos = torch.cat([torch.arange(int(n)) for n in lens]).to(cuda)
    inp = make(QWEN, int(lens.sum()), cuda, seed=2, pos=pos)
    check_chain_bf16(inp, QWEN)


@pytest.mark.parametrize("factor", [32.0, 8.0])
def test_llama_packed_batch(cuda, factor):
    pos = torch.arange(2048, device=cuda).repeat(8)
    inp = make(LLAMA, 16384, cuda, seed=3, pos=pos)
    check_chain_bf16(inp, LLAMA, qk_norm=False, scaling=(factor, 1.0, 4.0, 8192))


def test_full_size_sweep(cuda):
    inp = make(QWEN, 1 << 20, cuda, seed=4, pos_hi=32768)
    check_chain_bf16(inp, QWEN, sample_rows=2048)
    torch.cuda.synchronize()
    assert svllm_ops.read_device_error(0, True) == 0
