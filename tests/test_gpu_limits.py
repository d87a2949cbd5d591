"""Sizes at the edges: more rows than an int32 grid index can count (the reference's kernel
rejects them, src/ops/cuda/rms_norm.cu:104-108; these kernels index rows in 64 bits), and the
smallest batches (one token, one row) that take the decode-sized launch shapes."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import svllm_capi as capi
from conftest import assert_bf16_within_ulp, random_t, rope_within_rounding, to_bits

pytestmark = pytest.mark.gpu


def test_rms_norm_beyond_int32_rows(cuda):
    rows, hidden = (1 << 31) + 7, 8  # 34 GB in, 34 GB out
    free, _ = torch.cuda.mem_get_info()
    if free < 2 * rows * hidden * 2 + (8 << 30):
        pytest.skip("needs ~80 GB of free device memory")
    x = torch.empty(rows, hidden, device=cuda, dtype=torch.bfloat16).normal_()
    w = random_t(hidden, device=cuda, seed=1, scale=0.1, shift=1.0)
    out = torch.empty_like(x)
    capi.rms_norm(out, x, w, 1e-6)
    torch.cuda.synchronize()
    sample = torch.cat([torch.arange(0, 64), torch.arange((1 << 31) - 64, (1 << 31) + 7)])
    sample = sample.to(cuda)
    ref = oracle.rms_norm(to_bits(x[sample]), to_bits(w), 1e-6)
    assert_bf16_within_ulp(out[sample], ref, 2, "rows past 2^31")
    assert capi.read_device_error(0, reset=True) == 0
    del x, out
    torch.cuda.empty_cache()


@pytest.mark.parametrize("op", ["rms_norm", "add_rms_norm", "qk_norm_rope", "silu_and_mul",
                                "embedding"])
def test_single_token(cuda, op):
    if op in ("rms_norm", "add_rms_norm"):
        x = random_t(1, 1024, device=cuda, seed=2)
        r = random_t(1, 1024, device=cuda, seed=3)
        w = random_t(1024, device=cuda, seed=4)
        if op == "rms_norm":
            out = torch.empty_like(x)
            capi.rms_norm(out, x, w, 1e-6)
            ref = oracle.rms_norm(to_bits(x), to_bits(w), 1e-6)
            assert_bf16_within_ulp(out, ref, 2, op)
        else:
            ox, orr = oracle.add_rms_norm(to_bits(x), to_bits(r), to_bits(w), 1e-6)
            capi.add_rms_norm(x, r, w, 1e-6)
            assert np.array_equal(to_bits(r), orr)
            assert_bf16_within_ulp(x, ox, 2, op)
    elif op == "qk_norm_rope":
        q, k = random_t(1, 16, 128, device=cuda, seed=5), random_t(1, 8, 128, device=cuda, seed=6)
        qw, kw = random_t(128, device=cuda, seed=7), random_t(128, device=cuda, seed=8)
        pos = torch.tensor([40959], device=cuda)
        inv = oracle.inv_freq(1e6, 128)
        oq, ok = oracle.qk_norm_rope(to_bits(q), to_bits(k), to_bits(qw), to_bits(kw),
                                     pos.cpu().numpy(), 1e-6, inv)
        pre_q = oracle.rms_norm(to_bits(q).reshape(-1, 128), to_bits(qw), 1e-6).reshape(16, 128)
        pre_k = oracle.rms_norm(to_bits(k).reshape(-1, 128), to_bits(kw), 1e-6).reshape(8, 128)
        capi.qk_norm_rope(q, k, qw, kw, pos, 1e-6, inv)
        # every element within one rounding of each rotation term of the oracle, > 98% exact
        assert rope_within_rounding(to_bits(q)[0], oq[0], pre_q).all()
        assert rope_within_rounding(to_bits(k)[0], ok[0], pre_k).all()
        assert (to_bits(q) == oq).mean() > 0.98 and (to_bits(k) == ok).mean() > 0.98
    elif op == "silu_and_mul":
        g, u = random_t(1, 3072, device=cuda, seed=9), random_t(1, 3072, device=cuda, seed=10)
        out = torch.empty_like(g)
        capi.silu_and_mul(out, g, u)
        assert_bf16_within_ulp(out, oracle.silu_and_mul(to_bits(g), to_bits(u)), 2, op)
    else:
        table = random_t(151936, 1024, device=cuda, seed=11)
        ids = torch.tensor([151935], device=cuda, dtype=torch.int32)
        out = torch.empty(1, 1024, device=cuda, dtype=torch.bfloat16)
        capi.embedding(out, ids, table)
        assert torch.equal(out[0], table[-1])
