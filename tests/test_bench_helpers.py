"""bench.py's workload definitions, on CPU: the packed-prefill sequences (config 2: 64 seeded
sequences of 128-2048 tokens, each at positions 0..len-1), the Llama packing (config 3), the
algorithmic bytes per token in bf16 and fp32, and the op names per model."""

from __future__ import annotations

import sys

import numpy as np

from conftest import REPO_ROOT

sys.path.insert(0, str(REPO_ROOT))
import bench  # noqa: E402


def test_prefill_is_64_packed_sequences_at_positions_from_zero():
    _, total, spec = bench.WORKLOADS["prefill"]
    assert total is None and spec[0] == "sequences"
    lengths = bench.sequence_lengths(spec)
    assert len(lengths) == 64 and lengths.min() >= 128 and lengths.max() <= 2048
    T = bench.workload_total("prefill")
    assert T == int(lengths.sum()) and 60_000 < T < 80_000  # "about 70k token rows"
    pos = bench.global_positions(spec, T)
    starts = np.concatenate([[0], np.cumsum(lengths)[:-1]])
    assert (pos[starts] == 0).all()
    assert np.array_equal(pos[starts[1] - 1], lengths[0] - 1)
    assert bench.workload_total("prefill", 1000) == 1000


def test_llama_is_8_sequences_of_2048():
    _, total, spec = bench.WORKLOADS["llama"]
    pos = bench.global_positions(spec, total)
    assert total == 16384 and pos.max() == 2047 and (pos.reshape(8, 2048) == np.arange(2048)).all()


def test_bytes_per_token():
    q, l = bench.QWEN3, bench.LLAMA
    assert sum(bench.op_bytes(q).values()) == 43020
    assert sum(bench.op_bytes(l).values()) == 83980
    assert sum(bench.op_bytes(q, elem=4).values()) == 86028
    assert bench.op_names(l) == ["embedding", "add_rms_norm", "rope", "silu_and_mul"]
    assert bench.op_names(dict(q, kv_cache=True))[2] == "qk_norm_rope_cache"
    assert bench.op_bytes(dict(q, kv_cache=True))["qk_norm_rope_cache"] == 12296 + 3 * 2048 + 8
