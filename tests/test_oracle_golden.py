"""The oracle, pinned before it is trusted (CPU only).

rms_norm is pinned against the reference's own OpenMP kernel, built from its sources into
oracle/_ref and recorded in tests/golden/golden.npz on the reference test's shapes. The ops the
reference has not written yet are pinned against Hugging Face modules run on seeded inputs
(tests/golden/make_golden.py). bf16 tolerances: the reference sums squares in fp32 in SIMD order
and the oracle in double, and torch's CPU cos/sin/exp are not the C library's, so a bf16 output
may sit one rounding step away; most are bit-identical and the tests say how many.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import assert_bf16_within_ulp, assert_rel_f32, bf16_values, golden

G = golden()


@pytest.mark.parametrize("i", range(6))
def test_rms_norm_matches_reference_cpu_kernel(i):
    x, w, y = G[f"rms_norm/{i}/x"], G[f"rms_norm/{i}/w"], G[f"rms_norm/{i}/y"]
    out = oracle.rms_norm(x, w, 1e-6)
    exact = assert_bf16_within_ulp(out, y, 1, f"rms_norm shape {x.shape}")
    assert exact > 0.99


@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_add_rms_norm_matches_hf_decoder_layer(dt):
    g = {k.split("/")[-1]: v for k, v in G.items() if k.startswith(f"add_rms_norm/{dt}/")}
    y, r = oracle.add_rms_norm(g["x"], g["r"], g["w"], 1e-6)
    if dt == "bf16":
        assert np.array_equal(r, g["r_out"]), "residual add must be bit-exact"
        assert_bf16_within_ulp(y, g["y"], 1, "add_rms_norm")
    else:
        assert np.array_equal(r, g["r_out"])
        assert_rel_f32(y, g["y"], 1e-5, "add_rms_norm f32")


def _rope_bound_ok(out, ref, pre):
    """|out - ref| <= one bf16 rounding of each rotation term + one of the result."""
    o, r = bf16_values(out).astype(np.float64), bf16_values(ref).astype(np.float64)
    p = bf16_values(pre).astype(np.float64)
    half = p.shape[-1] // 2
    mag = np.abs(p[..., :half]) + np.abs(p[..., half:])
    mag = np.concatenate([mag, mag], axis=-1)
    return np.abs(o - r) <= 2.0 ** -7 * mag + 2.0 ** -8 * np.abs(r) + 1e-30


@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_qk_norm_rope_matches_hf(dt):
    g = {k.split("/")[-1]: v for k, v in G.items() if k.startswith(f"qk_norm_rope/{dt}/")}
    inv = G["inv_freq/qwen3"]
    q, k = oracle.qk_norm_rope(g["q"], g["k"], g["qw"], g["kw"], g["pos"], 1e-6, inv)
    if dt == "bf16":
        qn = oracle.rms_norm(g["q"].reshape(-1, 128), g["qw"], 1e-6).reshape(g["q"].shape)
        kn = oracle.rms_norm(g["k"].reshape(-1, 128), g["kw"], 1e-6).reshape(g["k"].shape)
        assert _rope_bound_ok(q, g["q_out"], qn).all()
        assert _rope_bound_ok(k, g["k_out"], kn).all()
        assert (q == g["q_out"]).mean() > 0.99
    else:
        assert_rel_f32(q, g["q_out"], 1e-5, "q f32")
        assert_rel_f32(k, g["k_out"], 1e-5, "k f32")


@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_llama3_rope_matches_hf(dt):
    g = {k.split("/")[-1]: v for k, v in G.items() if k.startswith(f"rope_llama3/{dt}/")}
    inv = G["inv_freq/llama3"]
    q, k = oracle.rope(g["q"], g["k"], g["pos"], inv)
    if dt == "bf16":
        assert _rope_bound_ok(q, g["q_out"], g["q"]).all()
        assert _rope_bound_ok(k, g["k_out"], g["k"]).all()
        assert (q == g["q_out"]).mean() > 0.99
    else:
        assert_rel_f32(q, g["q_out"], 1e-5, "q f32")
        assert_rel_f32(k, g["k_out"], 1e-5, "k f32")


@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_silu_and_mul_matches_hf(dt):
    g = {k.split("/")[-1]: v for k, v in G.items() if k.startswith(f"silu_and_mul/{dt}/")}
    y = oracle.silu_and_mul(g["gate"], g["up"])
    if dt == "bf16":
        exact = assert_bf16_within_ulp(y, g["y"], 2, "silu_and_mul")
        assert exact > 0.99
    else:
        assert_rel_f32(y, g["y"], 1e-5, "silu_and_mul f32")


def test_embedding_matches_torch_bit_exact():
    y, bad = oracle.embedding(G["embedding/ids"], G["embedding/table"])
    assert bad == 0
    assert np.array_equal(y, G["embedding/y"])


def test_embedding_bad_ids_zero_rows():
    table = G["embedding/table"]
    ids = np.array([0, -1, table.shape[0], 5], dtype=np.int32)
    y, bad = oracle.embedding(ids, table)
    assert bad == 2
    assert not y[1].any() and not y[2].any()
    assert np.array_equal(y[3], table[5])


@pytest.mark.parametrize("name, args", [
    ("qwen3", (1e6, 128, None)),
    ("llama3", (5e5, 64, (8.0, 1.0, 4.0, 8192))),
    ("llama3_f32x", (5e5, 64, (32.0, 1.0, 4.0, 8192))),
])
def test_inv_freq_restatement_matches_hf(name, args):
    """The C restatement uses the C library's powf where torch uses its own fp32 pow; they may
    disagree by one fp32 ulp on a rare entry. The op layer uses torch itself (bit-exact)."""
    ref = G[f"inv_freq/{name}"]
    ours = oracle.inv_freq(*args)
    rel = np.abs(ours.astype(np.float64) - ref) / ref
    assert rel.max() <= 2.0 ** -23
    assert (ours == ref).mean() >= 0.95
