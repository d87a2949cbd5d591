"""The C ABI library on the host (no GPU needed): it loads, exports every entry point that
include/svllm_kernels.h declares, rejects bad arguments before touching CUDA, and its host-side
inverse-frequency helper agrees with the oracle and with Hugging Face."""

from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest

import oracle
import svllm_capi as capi
from conftest import REPO_ROOT, golden

HEADER = REPO_ROOT / "include" / "svllm_kernels.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(svllm_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_op_set():
    names = declared_functions()
    for op in ("rms_norm", "add_rms_norm", "qk_norm_rope", "rope", "silu_and_mul", "embedding"):
        assert f"svllm_{op}_bf16" in names and f"svllm_{op}_f32" in names


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports_every_declared_symbol(name):
    assert hasattr(capi.lib(), name), f"{name} is declared but not exported"


def test_version_and_status_strings():
    assert capi.version() == "0.1.0"
    lib = capi.lib()
    assert lib.svllm_status_string(0) == b"ok"
    for status in range(1, 6):
        assert lib.svllm_status_string(status) not in (b"ok", b"unknown status")
    assert lib.svllm_status_string(99) == b"unknown status"


INVALID = 1


@pytest.mark.parametrize("call", [
    lambda L: L.svllm_rms_norm_bf16(8, 8, 8, 1, 0, 0, 0, 1e-6, None),        # hidden 0
    lambda L: L.svllm_rms_norm_bf16(8, 8, 8, -1, 16, 16, 16, 1e-6, None),    # negative rows
    lambda L: L.svllm_rms_norm_f32(8, 8, 8, 2, 16, 8, 16, 1e-6, None),       # stride < hidden
    lambda L: L.svllm_rms_norm_bf16(None, 8, 8, 2, 16, 16, 16, 1e-6, None),  # null out
    lambda L: L.svllm_add_rms_norm_bf16(8, None, 8, 2, 16, 16, 16, 1e-6, None),
    lambda L: L.svllm_qk_norm_rope_bf16(8, 8, 8, 8, 8, 0, 4, 2, 1, 7, 14, 7, 1e-6, 8, None),
    lambda L: L.svllm_qk_norm_rope_bf16(8, 8, 8, 8, 8, 2, 4, 2, 1, 8, 16, 8, 1e-6, 8, None),
    lambda L: L.svllm_rope_bf16(8, 8, 8, 0, 4, 2, 1, 1026, 2052, 1026, 8, None),  # head_dim>512
    lambda L: L.svllm_rope_f32(8, 8, 8, 0, 4, 2, 1, 8, 16, 8, None, None),  # no inv_freq
    lambda L: L.svllm_silu_and_mul_bf16(8, 8, 8, 2, 0, 0, 0, 0, None),
    lambda L: L.svllm_silu_and_mul_f32(8, 8, 8, 2, 16, 16, 8, 16, None),
    lambda L: L.svllm_embedding_bf16(8, 8, 5, 8, 4, 10, 16, 16, 16, None, None),  # bad id type
    lambda L: L.svllm_embedding_bf16(8, 8, 0, 8, 4, 0, 16, 16, 16, None, None),   # vocab 0
    lambda L: L.svllm_rope_inv_freq(1e6, 7, None, 8),
    lambda L: L.svllm_rope_inv_freq(-1.0, 8, None, 8),
    # decode linear: in_features 0; out_stride < out_features; null x
    lambda L: L.svllm_decode_linear_bf16(256, 64, 256, 1, 0, 64, 256, 64, 64, None),
    lambda L: L.svllm_decode_linear_bf16(256, 32, 256, 1, 64, 64, 256, 64, 64, None),
    lambda L: L.svllm_decode_linear_bf16(256, 64, None, 1, 64, 64, 256, 64, 64, None),
    # paged decode attention: 6 heads over 4 KV heads; max_seq_len past the table; null q
    lambda L: L.svllm_paged_decode_attention_bf16(256, 256, 768, 256, 256, 4, 16, 256, 2, 256,
                                                  1, 6, 4, 128, 16, 0.1, None),
    lambda L: L.svllm_paged_decode_attention_bf16(256, 256, 2048, 256, 256, 4, 16, 256, 2, 256,
                                                  1, 16, 8, 128, 33, 0.1, None),
    lambda L: L.svllm_paged_decode_attention_bf16(256, None, 2048, 256, 256, 4, 16, 256, 2, 256,
                                                  1, 16, 8, 128, 32, 0.1, None),
    # fused LM head + argmax: vocabulary 0; a workspace of 8 bytes for 2 rows
    lambda L: L.svllm_lm_head_argmax_bf16(256, 2, 64, 64, 256, 0, 64, 256, None, 0, 256, 16, None),
    lambda L: L.svllm_lm_head_argmax_bf16(256, 2, 64, 64, 256, 100, 64, 256, None, 0, 256, 8,
                                          None),
    lambda L: L.svllm_lm_head_argmax_static_bf16(256, 2, 64, 64, 256, 100, 64, 256, 256, 50,
                                                 None),  # logits_stride < vocab
], ids=lambda c: "")
def test_bad_arguments_are_rejected_without_a_gpu(call):
    assert call(capi.lib()) == INVALID


UNSUPPORTED, TOO_LARGE = 3, 2


@pytest.mark.parametrize("call, status", [
    # 17 token rows: more than a decode batch, the caller's GEMM takes it
    (lambda L: L.svllm_decode_linear_bf16(256, 64, 256, 17, 64, 64, 256, 64, 64, None),
     UNSUPPORTED),
    # in_features not a multiple of 8
    (lambda L: L.svllm_decode_linear_bf16(256, 64, 256, 2, 60, 64, 256, 64, 64, None),
     UNSUPPORTED),
    # head_dim 96; three query heads per KV head
    (lambda L: L.svllm_paged_decode_attention_bf16(256, 256, 1536, 256, 256, 4, 16, 256, 2, 256,
                                                   1, 16, 8, 96, 32, 0.1, None), UNSUPPORTED),
    (lambda L: L.svllm_paged_decode_attention_bf16(256, 256, 768, 256, 256, 4, 16, 256, 2, 256,
                                                   1, 6, 2, 128, 32, 0.1, None), UNSUPPORTED),
    # the allocation-free LM head takes at most 4096 rows
    (lambda L: L.svllm_lm_head_argmax_static_bf16(256, 4097, 64, 64, 256, 100, 64, 256, None, 0,
                                                  None), TOO_LARGE),
], ids=lambda c: "")
def test_shapes_without_a_kernel_are_refused_without_a_gpu(call, status):
    assert call(capi.lib()) == status


def test_empty_batches_are_a_no_op_without_a_gpu():
    lib = capi.lib()
    assert lib.svllm_rms_norm_bf16(None, None, None, 0, 1024, 1024, 1024, 1e-6, None) == 0
    assert lib.svllm_add_rms_norm_f32(None, None, None, 0, 1024, 1024, 1024, 1e-6, None) == 0
    assert lib.svllm_silu_and_mul_bf16(None, None, None, 0, 3072, 3072, 3072, 3072, None) == 0
    assert lib.svllm_embedding_bf16(None, None, 0, None, 0, 10, 16, 16, 16, None, None) == 0
    assert lib.svllm_decode_linear_bf16(None, 1024, None, 0, 1024, 1024, None, 1024, 1024,
                                        None) == 0
    assert lib.svllm_paged_decode_attention_bf16(None, None, 2048, None, None, 4, 16, None, 2,
                                                 None, 0, 16, 8, 128, 32, 0.1, None) == 0
    assert lib.svllm_lm_head_argmax_bf16(None, 0, 64, 64, None, 100, 64, None, None, 0, None, 0,
                                         None) == 0
    inv = (ctypes.c_float * 64)()
    assert lib.svllm_rope_bf16(None, None, None, 0, 0, 16, 8, 128, 2048, 1024,
                               ctypes.cast(inv, ctypes.c_void_p), None) == 0


@pytest.mark.parametrize("theta, head_dim, scaling, name", [
    (1e6, 128, None, "qwen3"),
    (5e5, 64, (8.0, 1.0, 4.0, 8192), "llama3"),
    (5e5, 64, (32.0, 1.0, 4.0, 8192), "llama3_f32x"),
])
def test_inv_freq_helper(theta, head_dim, scaling, name):
    ours = np.array(capi.inv_freq(theta, head_dim, scaling), dtype=np.float32)
    # the C helper and the C restatement use the same C library powf: bit-identical
    assert np.array_equal(ours, oracle.inv_freq(theta, head_dim, scaling))
    hf = golden()[f"inv_freq/{name}"]
    assert np.abs(ours.astype(np.float64) - hf).max() <= 2.0 ** -23 * np.abs(hf).max()
