"""Writes the golden fixtures in tests/golden/ (run here, where the reference checkout and
Hugging Face transformers are importable; the fixtures travel, this script's inputs do not).

Two sources pin the oracle:
  * the reference's own rms_norm (its OpenMP CPU kernel, src/ops/cpu/rms_norm.cpp:13-44, built
    from its sources into oracle/_ref by oracle/build.py), on the reference test's shapes
    (tests/python/test_rms_norm.py:9-17) and seeds (tests/python/conftest.py:29-32);
  * Hugging Face modules, the formulas the reference commits to for the ops it has not written
    yet (docs/design-spec.md:105-106): Qwen3RMSNorm, the decoder layer's residual add,
    Qwen3RotaryEmbedding / LlamaRotaryEmbedding (llama3 scaling) with apply_rotary_pos_emb,
    the SiLU MLP gate, and nn.functional.embedding, on seeded inputs at Qwen3-0.6B and
    Llama-3.2-1B shapes (tests/cpp/data/*/config.json), bf16 and fp32, a few tokens each.

Usage: python tests/golden/make_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "oracle"))

import oracle  # noqa: E402  (oracle/oracle.py: loads the reference build in oracle/_ref)

QWEN = dict(hidden=1024, heads=16, kv_heads=8, head_dim=128, inter=3072, vocab=151936,
            eps=1e-6, theta=1e6)
LLAMA = dict(hidden=2048, heads=32, kv_heads=8, head_dim=64, inter=8192, vocab=128256,
             eps=1e-5, theta=5e5, scaling=(8.0, 1.0, 4.0, 8192))


def randn(*shape, seed: int, dtype=torch.bfloat16) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(dtype)


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 as uint16 bit patterns, fp32 as float32, ints as they are."""
    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def rms_norm_reference(out: dict) -> None:
    ref = oracle.reference_module()
    if ref is None:
        raise SystemExit("oracle/_ref is not built: run python oracle/build.py first")
    shapes = [(1, 128), (4, 64), (7, 1024), (2, 5, 2048), (3, 4100), (2, 16384)]
    for i, shape in enumerate(shapes):
        x = randn(*shape, seed=0)
        w = randn(shape[-1], seed=1)
        y = ref.rms_norm(x, w, 1e-6)
        out[f"rms_norm/{i}/x"] = bits(x)
        out[f"rms_norm/{i}/w"] = bits(w)
        out[f"rms_norm/{i}/y"] = bits(y)


def hf_ops(out: dict) -> None:
    from transformers import LlamaConfig, Qwen3Config
    from transformers.activations import ACT2FN
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    from transformers.models.qwen3.modeling_qwen3 import (
        Qwen3RMSNorm,
        Qwen3RotaryEmbedding,
        apply_rotary_pos_emb,
    )

    qcfg = Qwen3Config(hidden_size=QWEN["hidden"], head_dim=QWEN["head_dim"],
                       num_attention_heads=QWEN["heads"], num_key_value_heads=QWEN["kv_heads"],
                       rope_theta=QWEN["theta"], rms_norm_eps=QWEN["eps"],
                       intermediate_size=QWEN["inter"], vocab_size=QWEN["vocab"],
                       max_position_embeddings=40960)
    f, lo, hi, orig = LLAMA["scaling"]
    lcfg = LlamaConfig(hidden_size=LLAMA["hidden"], head_dim=LLAMA["head_dim"],
                       num_attention_heads=LLAMA["heads"], num_key_value_heads=LLAMA["kv_heads"],
                       rope_theta=LLAMA["theta"], rms_norm_eps=LLAMA["eps"],
                       intermediate_size=LLAMA["inter"], vocab_size=LLAMA["vocab"],
                       max_position_embeddings=131072,
                       rope_scaling={"rope_type": "llama3", "factor": f, "low_freq_factor": lo,
                                     "high_freq_factor": hi,
                                     "original_max_position_embeddings": orig})
    qrot = Qwen3RotaryEmbedding(qcfg)
    lrot = LlamaRotaryEmbedding(lcfg)
    out["inv_freq/qwen3"] = bits(qrot.inv_freq.float())
    out["inv_freq/llama3"] = bits(lrot.inv_freq.float())
    # The same rule at the BASELINE factor 32, through the same function.
    lcfg32 = LlamaConfig(hidden_size=LLAMA["hidden"], head_dim=LLAMA["head_dim"],
                         num_attention_heads=LLAMA["heads"],
                         num_key_value_heads=LLAMA["kv_heads"], rope_theta=LLAMA["theta"],
                         max_position_embeddings=131072,
                         rope_scaling={"rope_type": "llama3", "factor": 32.0,
                                       "low_freq_factor": lo, "high_freq_factor": hi,
                                       "original_max_position_embeddings": orig})
    out["inv_freq/llama3_f32x"] = bits(LlamaRotaryEmbedding(lcfg32).inv_freq.float())

    for dt_name, dt in (("bf16", torch.bfloat16), ("f32", torch.float32)):
        # add + RMSNorm (decoder layer): residual = x + residual; x = norm(residual)
        T, H = 4, QWEN["hidden"]
        x = randn(T, H, seed=10, dtype=dt)
        r = randn(T, H, seed=11, dtype=dt)
        w = (1 + 0.1 * randn(H, seed=12, dtype=torch.float32)).to(dt)
        norm = Qwen3RMSNorm(H, eps=QWEN["eps"]).to(dt)
        with torch.no_grad():
            norm.weight.copy_(w)
            r_new = x + r
            y = norm(r_new)
        for k, v in dict(x=x, r=r, w=w, r_out=r_new, y=y).items():
            out[f"add_rms_norm/{dt_name}/{k}"] = bits(v)

        # Qwen3 q/k norm + RoPE
        T = 6
        q = randn(T, QWEN["heads"], QWEN["head_dim"], seed=20, dtype=dt)
        k = randn(T, QWEN["kv_heads"], QWEN["head_dim"], seed=21, dtype=dt)
        qw = (1 + 0.1 * randn(QWEN["head_dim"], seed=22, dtype=torch.float32)).to(dt)
        kw = (1 + 0.1 * randn(QWEN["head_dim"], seed=23, dtype=torch.float32)).to(dt)
        pos = torch.tensor([0, 1, 7, 255, 4095, 32767], dtype=torch.int64)
        qn = Qwen3RMSNorm(QWEN["head_dim"], eps=QWEN["eps"]).to(dt)
        kn = Qwen3RMSNorm(QWEN["head_dim"], eps=QWEN["eps"]).to(dt)
        with torch.no_grad():
            qn.weight.copy_(qw)
            kn.weight.copy_(kw)
            cos, sin = qrot(q, pos[None, :])
            # HF layout is [batch, heads, seq, head_dim]
            qh = qn(q).transpose(0, 1)[None]
            kh = kn(k).transpose(0, 1)[None]
            qe, ke = apply_rotary_pos_emb(qh, kh, cos, sin)
        for name, v in dict(q=q, k=k, qw=qw, kw=kw, pos=pos, q_out=qe[0].transpose(0, 1),
                            k_out=ke[0].transpose(0, 1)).items():
            out[f"qk_norm_rope/{dt_name}/{name}"] = bits(v)

        # Llama RoPE (llama3 scaling), no q/k norm
        q = randn(T, LLAMA["heads"], LLAMA["head_dim"], seed=30, dtype=dt)
        k = randn(T, LLAMA["kv_heads"], LLAMA["head_dim"], seed=31, dtype=dt)
        pos = torch.tensor([0, 3, 100, 2047, 8191, 65535], dtype=torch.int64)
        with torch.no_grad():
            cos, sin = lrot(q, pos[None, :])
            qe, ke = apply_rotary_pos_emb(q.transpose(0, 1)[None], k.transpose(0, 1)[None], cos,
                                          sin)
        for name, v in dict(q=q, k=k, pos=pos, q_out=qe[0].transpose(0, 1),
                            k_out=ke[0].transpose(0, 1)).items():
            out[f"rope_llama3/{dt_name}/{name}"] = bits(v)

        # SiLU(gate) * up, Qwen3 intermediate
        g = randn(2, QWEN["inter"], seed=40, dtype=dt) * 3
        u = randn(2, QWEN["inter"], seed=41, dtype=dt)
        with torch.no_grad():
            y = ACT2FN["silu"](g) * u
        for name, v in dict(gate=g, up=u, y=y).items():
            out[f"silu_and_mul/{dt_name}/{name}"] = bits(v)

    # Embedding gather (bit-exact), a small table with the Qwen3 hidden size
    table = (0.02 * randn(96, QWEN["hidden"], seed=50, dtype=torch.float32)).to(torch.bfloat16)
    gen = torch.Generator().manual_seed(51)
    ids = torch.randint(0, 96, (33,), generator=gen, dtype=torch.int64)
    out["embedding/table"] = bits(table)
    out["embedding/ids"] = bits(ids)
    out["embedding/y"] = bits(F.embedding(ids, table))


def main() -> int:
    out: dict[str, np.ndarray] = {}
    rms_norm_reference(out)
    hf_ops(out)
    path = HERE / "golden.npz"
    np.savez_compressed(path, **out)
    print(f"wrote {len(out)} arrays to {path} ({path.stat().st_size} bytes)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
