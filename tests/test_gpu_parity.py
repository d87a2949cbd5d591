"""Parity of the sm_100a kernels, called through the C ABI (svllm_capi), with the oracle
(oracle/, the C/OpenMP restatement) on the same seeded inputs, for bf16 and fp32, across the
bulk-copy path, the plain-load path (unaligned or odd sizes), strided rows and the edge cases.

Bars (one bf16 ulp against the reference kernel, 1e-5 relative for fp32; written per test):
  * embedding: bit-exact.
  * fp32 outputs: within 1e-5 relative of the oracle.
  * bf16 norms: bit-identical to the reference's own CUDA rms_norm kernel (oracle/_ref, same
    GPU; for add_rms_norm after the exact residual add, for the q/k norm on the [tokens * heads,
    head_dim] view); within 2 bf16 ulp of the CPU oracle (which sums in double and uses
    1 / sqrtf where the kernels replay the reference's fp32 tree and rsqrtf: a normalised value
    one step apart can move the weighted output two), bit-exact for the residual add.
  * rotary outputs: within one bf16 rounding of each rotation term of the oracle (the C
    library's cosf/sinf are not CUDA's), and bit-exact against the torch composite on the same
    GPU, which calls the same CUDA functions.
  * SiLU-mul: within 2 ulp of the oracle (expf differs by an fp32 ulp between the two libraries,
    which can move the rounded SiLU by one step) and bit-exact against torch on the GPU.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
import svllm_capi as capi
from conftest import (assert_bf16_within_ulp, assert_rel_f32, bf16_values, from_bits, random_t,
                      rope_within_rounding, to_bits)

pytestmark = pytest.mark.gpu

DTYPES = [torch.bfloat16, torch.float32]


def ids_of(dt):
    return "bf16" if dt == torch.bfloat16 else "f32"


def np_of(t: torch.Tensor) -> np.ndarray:
    return to_bits(t)


def check(ours: torch.Tensor, ref: np.ndarray, dt, max_ulp: int, what: str, min_exact=0.99):
    if dt == torch.bfloat16:
        exact = assert_bf16_within_ulp(ours, ref, max_ulp, what)
        assert exact >= min_exact, f"{what}: only {exact:.4%} bit-exact"
    else:
        assert_rel_f32(ours, ref, 1e-5, what)


@pytest.fixture(autouse=True)
def _clear_device_error(cuda):
    capi.read_device_error(0, reset=True)
    yield
    torch.cuda.synchronize()
    assert capi.read_device_error(0, reset=True) & capi.DEVERR_WAIT_TIMEOUT == 0


# ---------------------------------------------------------------------------------------------
# rms_norm

RMS_SHAPES = [(1, 128), (4, 64), (7, 1024), (50, 2048), (3, 4100), (2, 16384), (300, 1024),
              (4096, 128), (2049, 1024), (1000, 768), (33, 4096),
              # above 64 rows per SM: the bulk-copy kernels
              (10000, 1024), (12000, 128), (10000, 2048), (10000, 768), (10000, 4096)]


@pytest.mark.parametrize("dt", DTYPES, ids=ids_of)
@pytest.mark.parametrize("shape", RMS_SHAPES, ids=str)
def test_rms_norm(cuda, dt, shape):
    x = random_t(*shape, dtype=dt, device=cuda, seed=1)
    w = random_t(shape[-1], dtype=dt, device=cuda, seed=2, scale=0.1, shift=1.0)
    out = torch.empty_like(x)
    capi.rms_norm(out, x, w, 1e-6)
    ref = oracle.rms_norm(np_of(x), np_of(w), 1e-6)
    check(out, ref, dt, 2, f"rms_norm {shape}")
    if dt == torch.bfloat16:
        assert torch.equal(out, oracle.reference_module().rms_norm(x, w, 1e-6))


@pytest.mark.parametrize("dt", DTYPES, ids=ids_of)
def test_rms_norm_strided_and_unaligned(cuda, dt):
    rows, hidden = 37, 1024
    big = random_t(rows, hidden + 8, dtype=dt, device=cuda, seed=3)
    x = big[:, :hidden]  # row stride hidden + 8: still 16-byte aligned rows
    w = random_t(hidden, dtype=dt, device=cuda, seed=4)
    out_big = torch.zeros(rows, hidden + 16, dtype=dt, device=cuda)
    out = out_big[:, 8:8 + hidden]
    capi.rms_norm(out, x, w, 1e-5)
    ref = oracle.rms_norm(np_of(x.contiguous()), np_of(w), 1e-5)
    check(out.contiguous(), ref, dt, 2, "strided")
    assert not out_big[:, :8].any() and not out_big[:, 8 + hidden:].any(), "wrote outside rows"
    # one element in: rows lose 16-byte alignment, the plain-load path runs
    flat = random_t(rows * hidden + 1, dtype=dt, device=cuda, seed=5)
    xu = flat[1:].view(rows, hidden)
    outu = torch.empty_like(xu)
    capi.rms_norm(outu, xu, w, 1e-5)
    check(outu, oracle.rms_norm(np_of(xu), np_of(w), 1e-5), dt, 2, "unaligned")


# ---------------------------------------------------------------------------------------------
# add_rms_norm

@pytest.mark.parametrize("dt", DTYPES, ids=ids_of)
@pytest.mark.parametrize("shape", [(1, 1024), (7, 1024), (1000, 1024), (513, 2048), (5, 4100),
                                   (64, 128), (10000, 1024), (10000, 2048), (12000, 128)], ids=str)
def test_add_rms_norm(cuda, dt, shape):
    x = random_t(*shape, dtype=dt, device=cuda, seed=6)
    r = random_t(*shape, dtype=dt, device=cuda, seed=7)
    w = random_t(shape[-1], dtype=dt, device=cuda, seed=8, scale=0.1, shift=1.0)
    ref_x, ref_r = oracle.add_rms_norm(np_of(x), np_of(r), np_of(w), 1e-6)
    summed = x + r
    capi.add_rms_norm(x, r, w, 1e-6)
    assert np.array_equal(np_of(r), ref_r), "residual + x must be bit-exact"
    check(x, ref_x, dt, 2, f"add_rms_norm {shape}")
    if dt == torch.bfloat16:  # the reference's path: a LibTorch add, then its rms_norm kernel
        assert torch.equal(x, oracle.reference_module().rms_norm(summed, w, 1e-6))


# ---------------------------------------------------------------------------------------------
# rotary embedding

rope_bound_ok = rope_within_rounding


def torch_rope(x, pos, inv):
    """Hugging Face's rotary embedding as torch ops, on x's device."""
    freqs = pos.float()[:, None] * inv.to(x.device)[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().to(x.dtype)[:, None, :], emb.sin().to(x.dtype)[:, None, :]
    half = x.shape[-1] // 2
    return x * cos + torch.cat((-x[..., half:], x[..., :half]), dim=-1) * sin


def _positions(T, hi, dtype, cuda, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, hi, (T,), generator=g).to(device=cuda, dtype=dtype)


@pytest.mark.parametrize("dt", DTYPES, ids=ids_of)
@pytest.mark.parametrize("T, hq, hk, d, pos_dtype", [
    (1, 16, 8, 128, torch.int64), (7, 16, 8, 128, torch.int32), (256, 16, 8, 128, torch.int64),
    (2000, 16, 8, 128, torch.int64), (300, 32, 8, 64, torch.int32), (40, 8, 2, 256, torch.int64),
    (20, 4, 2, 96, torch.int64), (11, 4, 1, 32, torch.int32),
], ids=str)
def test_qk_norm_rope(cuda, dt, T, hq, hk, d, pos_dtype):
    q = random_t(T, hq, d, dtype=dt, device=cuda, seed=9)
    k = random_t(T, hk, d, dtype=dt, device=cuda, seed=10)
    qw = random_t(d, dtype=dt, device=cuda, seed=11, scale=0.1, shift=1.0)
    kw = random_t(d, dtype=dt, device=cuda, seed=12, scale=0.1, shift=1.0)
    pos = _positions(T, 32768, pos_dtype, cuda, 13)
    inv = oracle.inv_freq(1e6, d)
    rq, rk = oracle.qk_norm_rope(np_of(q), np_of(k), np_of(qw), np_of(kw), np_of(pos).astype(
        np.int64 if pos_dtype == torch.int64 else np.int32), 1e-6, inv)
    pre_q = oracle.rms_norm(np_of(q).reshape(-1, d), np_of(qw), 1e-6).reshape(q.shape)
    pre_k = oracle.rms_norm(np_of(k).reshape(-1, d), np_of(kw), 1e-6).reshape(k.shape)
    if dt == torch.bfloat16:
        # the reference's path on the same GPU: its rms_norm kernel on the head view, then the
        # Hugging Face rotary composite
        ref = oracle.reference_module()
        invt = torch.from_numpy(inv)
        eq = torch_rope(ref.rms_norm(q.reshape(-1, d), qw, 1e-6).view(q.shape), pos, invt)
        ek = torch_rope(ref.rms_norm(k.reshape(-1, d), kw, 1e-6).view(k.shape), pos, invt)
    capi.qk_norm_rope(q, k, qw, kw, pos, 1e-6, inv)
    if dt == torch.bfloat16:
        assert torch.equal(q, eq) and torch.equal(k, ek), "reference kernel + torch rotary"
        assert rope_bound_ok(q, rq, pre_q).all() and rope_bound_ok(k, rk, pre_k).all()
        assert (np_of(q) == rq).mean() > 0.99
    else:
        half = d // 2

        def pair_scale(pre):
            p = np.abs(np.asarray(pre, dtype=np.float64))
            m = p[..., :half] + p[..., half:]
            return np.concatenate([m, m], axis=-1)

        assert_rel_f32(q, rq, 1e-5, "q", scale=pair_scale(pre_q))
        assert_rel_f32(k, rk, 1e-5, "k", scale=pair_scale(pre_k))


@pytest.mark.parametrize("dt", DTYPES, ids=ids_of)
@pytest.mark.parametrize("factor", [8.0, 32.0])
def test_llama3_rope(cuda, dt, factor):
    T, hq, hk, d = 1000, 32, 8, 64
    q = random_t(T, hq, d, dtype=dt, device=cuda, seed=14)
    k = random_t(T, hk, d, dtype=dt, device=cuda, seed=15)
    pos = (torch.arange(T, device=cuda) % 2048)
    inv = oracle.inv_freq(5e5, d, (factor, 1.0, 4.0, 8192))
    invt = torch.from_numpy(inv)
    eq, ek = torch_rope(q, pos, invt), torch_rope(k, pos, invt)
    rq, rk = oracle.rope(np_of(q), np_of(k), np_of(pos), inv)
    pq, pk = np_of(q).copy(), np_of(k).copy()
    capi.rope(q, k, pos, inv)
    if dt == torch.bfloat16:
        # same GPU, same cosf/sinf as the torch composite: bit-exact
        assert torch.equal(q, eq) and torch.equal(k, ek)
        assert rope_bound_ok(q, rq, pq).all() and rope_bound_ok(k, rk, pk).all()
    else:
        assert_rel_f32(q, rq, 1e-5, "q")
        assert_rel_f32(k, rk, 1e-5, "k")
        torch.testing.assert_close(q, eq, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dt", DTYPES, ids=ids_of)
def test_rope_on_strided_views(cuda, dt):
    T, hq, hk, d = 129, 16, 8, 128
    qkv = random_t(T, (hq + 2 * hk) * d, dtype=dt, device=cuda, seed=16)
    q = qkv[:, : hq * d].view(T, hq, d)
    k = qkv[:, hq * d:(hq + hk) * d].view(T, hk, d)
    v_before = qkv[:, (hq + hk) * d:].clone()
    pos = torch.arange(T, device=cuda, dtype=torch.int32) * 7
    inv = oracle.inv_freq(1e6, d)
    rq, rk = oracle.rope(np_of(q.contiguous()), np_of(k.contiguous()), np_of(pos), inv)
    capi.rope(q, k, pos, inv)
    check(q.contiguous(), rq, dt, 1, "q view", min_exact=0.99)
    check(k.contiguous(), rk, dt, 1, "k view", min_exact=0.99)
    assert torch.equal(qkv[:, (hq + hk) * d:], v_before)


# ---------------------------------------------------------------------------------------------
# silu_and_mul

@pytest.mark.parametrize("dt", DTYPES, ids=ids_of)
@pytest.mark.parametrize("shape", [(1, 3072), (7, 3072), (1000, 3072), (33, 8192), (3, 3001),
                                   (5, 64)], ids=str)
def test_silu_and_mul(cuda, dt, shape):
    gate = random_t(*shape, dtype=dt, device=cuda, seed=17, scale=3.0)
    up = random_t(*shape, dtype=dt, device=cuda, seed=18)
    out = torch.empty_like(gate)
    capi.silu_and_mul(out, gate, up)
    ref = oracle.silu_and_mul(np_of(gate), np_of(up))
    check(out, ref, dt, 2, f"silu_and_mul {shape}")
    if dt == torch.bfloat16:
        assert torch.equal(out, F.silu(gate) * up), "same GPU, same expf: bit-exact with torch"


@pytest.mark.parametrize("dt", DTYPES, ids=ids_of)
def test_silu_and_mul_halves(cuda, dt):
    rows, inter = 77, 3072
    gate_up = random_t(rows, 2 * inter, dtype=dt, device=cuda, seed=19, scale=2.0)
    gate, up = gate_up[:, :inter], gate_up[:, inter:]
    out = torch.empty(rows, inter, dtype=dt, device=cuda)
    capi.silu_and_mul(out, gate, up)
    check(out, oracle.silu_and_mul(np_of(gate.contiguous()), np_of(up.contiguous())), dt, 2,
          "halves")


# ---------------------------------------------------------------------------------------------
# embedding

@pytest.mark.parametrize("dt", DTYPES, ids=ids_of)
@pytest.mark.parametrize("T, vocab, hidden, ids_dtype", [
    (1, 151936, 1024, torch.int32), (33, 151936, 1024, torch.int64),
    (5000, 151936, 1024, torch.int32), (777, 128256, 2048, torch.int64),
    (100, 1000, 1001, torch.int32),  # odd row size: plain path
], ids=str)
def test_embedding(cuda, dt, T, vocab, hidden, ids_dtype):
    table = random_t(vocab, hidden, dtype=dt, device=cuda, seed=20, scale=0.02)
    g = torch.Generator().manual_seed(21)
    ids = torch.randint(0, vocab, (T,), generator=g).to(device=cuda, dtype=ids_dtype)
    out = torch.empty(T, hidden, dtype=dt, device=cuda)
    capi.embedding(out, ids, table)
    assert torch.equal(out, table[ids.long()])
    ref, bad = oracle.embedding(np_of(ids), np_of(table))
    assert bad == 0 and np.array_equal(np_of(out), ref)


def test_embedding_bad_ids_zero_rows_and_raise_the_error_word(cuda):
    vocab, hidden = 4000, 1024
    table = random_t(vocab, hidden, device=cuda, seed=22)
    ids = torch.tensor([3, -1, vocab, 17, vocab + 1000, 0], device=cuda, dtype=torch.int64)
    out = torch.full((6, hidden), 7.0, dtype=torch.bfloat16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    capi.embedding(out, ids, table, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & capi.DEVERR_BAD_INDEX
    for i, good in enumerate([True, False, False, True, False, True]):
        if good:
            assert torch.equal(out[i], table[ids[i]])
        else:
            assert not out[i].any()
    # with no err pointer the library's own word records it
    capi.embedding(out, ids, table)
    assert capi.read_device_error(0, reset=True) & capi.DEVERR_BAD_INDEX


# Batches with at least half a token per table row take the vocabulary-bucket walk (the gather
# visits its tokens once per L2-sized slice of the table); these tables span 2 to 24 slices.
@pytest.mark.parametrize("vocab, hidden, T, dt, ids_dtype", [
    (8192, 1024, 16384, torch.bfloat16, torch.int32),
    (8192, 1024, 4096, torch.bfloat16, torch.int64),  # half a token per row
    (151936, 1024, 131072, torch.bfloat16, torch.int32),  # one rank's share of the 1M sweep
    (20000, 2048, 40000, torch.bfloat16, torch.int64),
    (4096, 1024, 9000, torch.float32, torch.int32),
    (151936, 1024, 300000, torch.bfloat16, torch.int32),
], ids=str)
def test_embedding_vocabulary_buckets(cuda, vocab, hidden, T, dt, ids_dtype):
    table = random_t(vocab, hidden, dtype=dt, device=cuda, seed=24, scale=0.02)
    g = torch.Generator().manual_seed(25)
    ids = torch.randint(0, vocab, (T,), generator=g).to(device=cuda, dtype=ids_dtype)
    out = torch.empty(T, hidden, dtype=dt, device=cuda)
    capi.embedding(out, ids, table)
    assert torch.equal(out, table[ids.long()])
    assert capi.read_device_error(0, reset=True) == 0


def test_embedding_vocabulary_buckets_bad_ids_and_strided_rows(cuda):
    vocab, hidden, T = 8192, 1024, 20000
    table = random_t(vocab, hidden, device=cuda, seed=26)
    g = torch.Generator().manual_seed(27)
    ids = torch.randint(0, vocab, (T,), generator=g)
    bad = torch.randperm(T, generator=g)[:50]
    ids[bad] = torch.tensor([-1, vocab, vocab + 7, -(2 ** 40), 2 ** 40]).repeat(10)
    ids = ids.to(cuda)
    big = torch.full((T, hidden + 64), 3.0, dtype=torch.bfloat16, device=cuda)
    out = big[:, 64:]
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    capi.embedding(out, ids, table, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == capi.DEVERR_BAD_INDEX
    good = (ids >= 0) & (ids < vocab)
    assert torch.equal(out[good], table[ids[good]])
    assert not out[~good].any()
    assert bool((big[:, :64] == 3.0).all())


def test_embedding_strided_output_rows(cuda):
    vocab, hidden, T = 5000, 1024, 300
    table = random_t(vocab, hidden, device=cuda, seed=23)
    ids = torch.randint(0, vocab, (T,), device=cuda)
    big = torch.zeros(T, hidden + 64, dtype=torch.bfloat16, device=cuda)
    out = big[:, 32:32 + hidden]
    capi.embedding(out, ids, table)
    assert torch.equal(out, table[ids])
    assert not big[:, :32].any() and not big[:, 32 + hidden:].any()


# ---------------------------------------------------------------------------------------------
# pipeline shapes do not change results

# The pipeline shape comes from the library's defaults, or from the SVLLM_PIPELINE environment
# variable read once per process; each override runs in a fresh interpreter.
PIPELINE_PROBE = r"""
import hashlib, sys
sys.path[:0] = sys.argv[1:]
import torch
import svllm_capi as capi
from conftest import random_t
cuda = torch.device("cuda", 0)
x = random_t(12000, 1024, device=cuda, seed=24)  # enough rows for the bulk-copy kernel
w = random_t(1024, device=cuda, seed=25)
gate = random_t(2000, 3072, device=cuda, seed=26)  # chunks of the tuned size, not shrunk
up = random_t(2000, 3072, device=cuda, seed=27)
q = random_t(5000, 16, 128, device=cuda, seed=28)
k = random_t(5000, 8, 128, device=cuda, seed=29)
pos = torch.arange(5000, device=cuda) * 7
inv = torch.tensor([1e6 ** (-2 * i / 128) for i in range(64)], dtype=torch.float32)
table = random_t(4000, 1024, device=cuda, seed=30)
ids = torch.randint(0, 4000, (9000,), generator=torch.Generator().manual_seed(31)).to(cuda)
xs = random_t(40000, 128, device=cuda, seed=32)  # short rows: half again as many warps
ws = random_t(128, device=cuda, seed=33)
out, sout, eout = torch.empty_like(x), torch.empty_like(gate), torch.empty(9000, 1024, dtype=torch.bfloat16, device=cuda)
souts = torch.empty_like(xs)
capi.rms_norm(out, x, w, 1e-6)
capi.rms_norm(souts, xs, ws, 1e-6)
capi.silu_and_mul(sout, gate, up)
capi.rope(q, k, pos, inv)
capi.embedding(eout, ids, table)
torch.cuda.synchronize()
h = hashlib.sha256()
for t in (out, souts, sout, q, k, eout):
    h.update(t.view(torch.int16).cpu().numpy().tobytes())
print(h.hexdigest())
"""


def pipeline_digest(spec: str | None) -> str:
    import os
    import subprocess
    import sys

    from conftest import ORACLE_DIR, PKG_PY, REPO_ROOT

    env = dict(os.environ)
    env.pop("SVLLM_PIPELINE", None)
    if spec is not None:
        env["SVLLM_PIPELINE"] = spec
    proc = subprocess.run([sys.executable, "-c", PIPELINE_PROBE, str(REPO_ROOT / "tests"),
                           str(PKG_PY), str(ORACLE_DIR)], capture_output=True, text=True,
                          env=env, timeout=600)
    assert proc.returncode == 0, proc.stderr[-3000:]
    return proc.stdout.strip().splitlines()[-1]


# (4096, 2, 12): short rows take half again as many warps, capped at the kernels' 16
@pytest.mark.parametrize("unit, stages, warps",
                         [(2048, 2, 1), (4096, 3, 8), (16384, 4, 2), (4096, 2, 12)])
def test_pipeline_shape_does_not_change_results(cuda, unit, stages, warps):
    spec = ",".join(f"{op}={unit}:{stages}:{warps}"
                    for op in ("rms_norm", "silu_and_mul", "rope", "embedding"))
    assert pipeline_digest(spec) == pipeline_digest(None)


def test_malformed_pipeline_entries_are_ignored(cuda):
    """Entries that do not parse, name no op, or are out of range leave the defaults in force;
    a valid entry beside them still applies (results are the same either way)."""
    spec = ("rms_norm=abc,no_such_op=4096:2:8,silu_and_mul=100:2:8,rope=4096:99:8,"
            "embedding=4096:1:8,rms_norm=4096:2:17,add_rms_norm,=,embedding=0:3:4")
    assert pipeline_digest(spec) == pipeline_digest(None)


def test_silu_table_path_is_exhaustively_identical(cuda):
    """Every one of the 65536 bf16 gate patterns (NaNs and infinities included) through the
    table path (a batch large enough to take it) and through the direct path (one row, too small
    for the table) gives the same bits, and the same bits as torch's silu * up on the GPU."""
    patterns = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    reps = 640  # 640 * 65536 elements: above the table path's threshold on a B200
    gate = patterns.to(cuda).repeat(reps).view(reps, 65536)
    up = random_t(reps, 65536, device=cuda, seed=30)
    out = torch.empty_like(gate)
    capi.silu_and_mul(out, gate, up)
    small = torch.empty(1, 65536, dtype=torch.bfloat16, device=cuda)
    capi.silu_and_mul(small, gate[:1], up[:1])
    expect = F.silu(gate) * up
    bits = lambda t: t.view(torch.int16)  # noqa: E731  (NaN == NaN as bit patterns)
    assert torch.equal(bits(out[:1]), bits(small)), "table path != direct path"
    assert torch.equal(bits(out), bits(expect)), "table path != torch silu * up"


# ---------------------------------------------------------------------------------------------
# rotary + paged-KV cache write, through the C ABI

@pytest.mark.parametrize("dt", DTYPES, ids=ids_of)
@pytest.mark.parametrize("with_norm, hq, hk, d", [(True, 16, 8, 128), (False, 32, 8, 64),
                                                  (True, 4, 2, 96)], ids=str)
def test_rope_cache(cuda, dt, with_norm, hq, hk, d):
    T, block_size = 1500, 16
    num_blocks = (T + block_size - 1) // block_size + 5
    qkv = random_t(T, (hq + 2 * hk) * d, dtype=dt, device=cuda, seed=40)
    q = qkv[:, : hq * d].view(T, hq, d)
    k = qkv[:, hq * d:(hq + hk) * d].view(T, hk, d)
    v = qkv[:, (hq + hk) * d:].view(T, hk, d)
    qw = random_t(d, dtype=dt, device=cuda, seed=41, scale=0.1, shift=1.0)
    kw = random_t(d, dtype=dt, device=cuda, seed=42, scale=0.1, shift=1.0)
    pos = _positions(T, 32768, torch.int64, cuda, 43)
    g = torch.Generator().manual_seed(44)
    perm = torch.randperm(num_blocks, generator=g)
    t = torch.arange(T)
    slots = (perm[t // block_size] * block_size + t % block_size)
    slots[::11] = -1
    slots = slots.to(cuda)
    k_cache = torch.zeros(num_blocks, block_size, hk, d, dtype=dt, device=cuda)
    v_cache = torch.zeros_like(k_cache)
    inv = oracle.inv_freq(1e6, d)
    qn, kn = np_of(q.contiguous()), np_of(k.contiguous())
    if with_norm:
        rq, rk = oracle.qk_norm_rope(qn, kn, np_of(qw), np_of(kw), np_of(pos), 1e-6, inv)
    else:
        rq, rk = oracle.rope(qn, kn, np_of(pos), inv)
    v_before = v.clone()
    if with_norm:
        capi.qk_norm_rope_cache(q, k, v, qw, kw, pos, slots, k_cache, v_cache, 1e-6, inv)
    else:
        capi.rope_cache(q, k, v, pos, slots, k_cache, v_cache, inv)
    torch.cuda.synchronize()
    written = slots >= 0
    flat_k = k_cache.view(-1, hk, d)
    flat_v = v_cache.view(-1, hk, d)
    s_w = slots[written]
    # the cache rows are exactly the kernel's own rotated k and the untouched v
    assert torch.equal(flat_k[s_w], k[written])
    assert torch.equal(flat_v[s_w], v_before[written])
    mask = torch.ones(flat_k.shape[0], dtype=torch.bool, device=cuda)
    mask[s_w] = False
    assert not flat_k[mask].any() and not flat_v[mask].any(), "a slot not in slot_mapping changed"
    if dt == torch.bfloat16:
        # every element within one rounding of each rotation term, and > 99% bit-exact
        if with_norm:
            pre_q = oracle.rms_norm(qn.reshape(-1, d), np_of(qw), 1e-6).reshape(qn.shape)
            pre_k = oracle.rms_norm(kn.reshape(-1, d), np_of(kw), 1e-6).reshape(kn.shape)
        else:
            pre_q, pre_k = qn, kn
        assert rope_bound_ok(np_of(q.contiguous()), rq, pre_q).all()
        assert rope_bound_ok(np_of(k.contiguous()), rk, pre_k).all()
        assert (np_of(q.contiguous()) == rq).mean() > 0.99
        assert (np_of(k.contiguous()) == rk).mean() > 0.99
    else:
        half = d // 2

        def pair(x):
            p = np.abs(np.asarray(x, dtype=np.float64))
            m = p[..., :half] + p[..., half:]
            return np.concatenate([m, m], axis=-1)

        pre_q = oracle.rms_norm(qn.reshape(-1, d), np_of(qw), 1e-6).reshape(qn.shape) \
            if with_norm else qn
        assert_rel_f32(q.contiguous(), rq, 1e-5, "q", scale=pair(pre_q))


def test_rope_cache_matches_rope_then_copy(cuda):
    """The fused op equals qk_norm_rope followed by a scatter of k and v into the cache."""
    T, hq, hk, d = 777, 16, 8, 128
    base = random_t(T, (hq + 2 * hk) * d, device=cuda, seed=45)
    qw = random_t(d, device=cuda, seed=46, scale=0.1, shift=1.0)
    kw = random_t(d, device=cuda, seed=47, scale=0.1, shift=1.0)
    pos = _positions(T, 4096, torch.int32, cuda, 48)
    slots = torch.randperm(T + 100, device=cuda)[:T]
    inv = oracle.inv_freq(1e6, d)

    def split(t):
        return (t[:, : hq * d].view(T, hq, d), t[:, hq * d:(hq + hk) * d].view(T, hk, d),
                t[:, (hq + hk) * d:].view(T, hk, d))

    a, b = base.clone(), base.clone()
    qa, ka, va = split(a)
    qb, kb, vb = split(b)
    kc = torch.zeros(T + 100, hk, d, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    capi.qk_norm_rope_cache(qa, ka, va, qw, kw, pos, slots, kc, vc, 1e-6, inv)
    capi.qk_norm_rope(qb, kb, qw, kw, pos, 1e-6, inv)
    kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
    kc2[slots], vc2[slots] = kb, vb
    assert torch.equal(a, b) and torch.equal(kc, kc2) and torch.equal(vc, vc2)


def test_rope_cache_slot_past_the_cache(cuda):
    T, hk, d = 4, 2, 64
    q = random_t(T, 4, d, device=cuda, seed=49)
    k = random_t(T, hk, d, device=cuda, seed=50)
    v = random_t(T, hk, d, device=cuda, seed=51)
    kc = torch.zeros(8, hk, d, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    slots = torch.tensor([0, 8, 3, 100], device=cuda)
    capi.rope_cache(q, k, v, torch.arange(T, device=cuda), slots, kc, vc, oracle.inv_freq(1e4, d))
    assert capi.read_device_error(0, reset=True) & capi.DEVERR_BAD_INDEX
    assert torch.equal(kc[0], k[0]) and torch.equal(vc[3], v[2])
    assert not kc[[1, 2, 4, 5, 6, 7]].any()


# ---------------------------------------------------------------------------------------------
# greedy sampling (argmax), through the C ABI, against numpy's argmax (first maximum; NaN wins)

@pytest.mark.parametrize("dt", DTYPES, ids=ids_of)
@pytest.mark.parametrize("rows, vocab", [(1, 151936), (256, 151936), (1024, 128256), (3, 1001),
                                         (64, 8), (5, 1024), (37, 151936), (73, 151936),
                                         (2000, 32000)], ids=str)
def test_argmax(cuda, dt, rows, vocab):
    logits = random_t(rows, vocab, dtype=dt, device=cuda, seed=60, scale=3.0)
    ids = torch.empty(rows, dtype=torch.int64, device=cuda)
    capi.argmax(ids, logits)
    want = np.argmax(logits.float().cpu().numpy(), axis=-1)
    assert np.array_equal(ids.cpu().numpy(), want)
    assert torch.equal(ids, torch.argmax(logits, dim=-1))


def test_argmax_strided_rows_and_edge_values(cuda):
    big = random_t(40, 5000 + 8, device=cuda, seed=61)
    logits = big[:, :5000]  # row stride 5008
    logits[0, 4999] = 100.0
    logits[1, :] = 0.0
    logits[1, [7, 4000]] = 5.0
    logits[2, 333] = float("nan")
    logits[3, :] = float("-inf")
    ids = torch.empty(40, dtype=torch.int64, device=cuda)
    capi.argmax(ids, logits)
    assert ids[:4].tolist() == [4999, 7, 333, 0]
    assert torch.equal(ids[4:], torch.argmax(logits[4:], dim=-1))


@pytest.mark.parametrize("dt", DTYPES, ids=ids_of)
@pytest.mark.parametrize("rows, vocab", [(4, 151936), (40, 151936), (100, 151936),
                                         (200, 151937), (400, 151936), (700, 151936),
                                         (1100, 151936)], ids=str)
def test_argmax_edge_rows_every_split(cuda, dt, rows, vocab):
    """Row counts that give one row to 8 and 4 CTAs of a cluster, and to one CTA of 512, 256,
    192 and 128 threads (148 SMs); the odd vocabulary takes the element-wise path. Planted rows: every element tied, a row of -inf, ties across the
    slice boundaries of the CTAs sharing a row, a maximum in the last element, and NaNs after
    the maximum (the first NaN wins)."""
    logits = random_t(rows, vocab, dtype=dt, device=cuda, seed=62, scale=2.0)
    logits[0, :] = 1.0
    logits[1, :] = float("-inf")
    logits[2, vocab // 8 - 1] = 50.0
    logits[2, vocab // 2] = 50.0
    logits[2, vocab - 1] = 50.0
    logits[3, vocab - 1] = 60.0
    if rows > 4:
        logits[4, 10] = 70.0
        logits[4, vocab // 3] = float("nan")
        logits[4, vocab - 2] = float("nan")
    ids = torch.empty(rows, dtype=torch.int64, device=cuda)
    capi.argmax(ids, logits)
    want = [0, 0, vocab // 8 - 1, vocab - 1] + ([vocab // 3] if rows > 4 else [])
    assert ids[:len(want)].tolist() == want
    assert torch.equal(ids, torch.argmax(logits, dim=-1))
