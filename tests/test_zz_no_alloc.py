"""svllm_lm_head_argmax_static_bf16: the LM head and greedy sampling for callers that cannot
allocate device memory (a host program driving the C ABI through an FFI without a CUDA
allocator of its own). Its per-row scratch is an array inside the library, so the test passes
no workspace; it calls the entry point through the C ABI twice in a row, on different inputs,
and checks ids and logits against svllm_lm_head_argmax_bf16 given a zeroed workspace (the same
kernels: identical results). This file is collected last."""

from __future__ import annotations

import ctypes

import pytest
import torch

import svllm_capi as capi

pytestmark = pytest.mark.gpu

MAX_ROWS = 4096
SVLLM_ERR_TOO_LARGE = 2  # include/svllm_kernels.h


def static_call(ids, hidden, weight, logits=None) -> int:
    lib = capi.lib()
    rows, hidden_size, hidden_stride = hidden.shape[0], hidden.shape[1], hidden.stride(0)
    stream = torch.cuda.current_stream().cuda_stream
    return lib.svllm_lm_head_argmax_static_bf16(
        hidden.data_ptr(), rows, hidden_size, hidden_stride, weight.data_ptr(), weight.shape[0],
        weight.stride(0), ids.data_ptr(), logits.data_ptr() if logits is not None else None,
        logits.stride(0) if logits is not None else 0, ctypes.c_void_p(stream))


@pytest.mark.parametrize("with_logits", [True, False], ids=["ids+logits", "ids-only"])
@pytest.mark.parametrize("rows", [7, 300])  # both orientations of the kernel
def test_matches_the_workspace_entry_point_on_two_calls(cuda, rows, with_logits):
    """Two calls in a row on different inputs; ids-only is the decode use (no logits kept)."""
    vocab, hidden_size = 20000, 1024
    for call in range(2):
        g = torch.Generator(device=cuda).manual_seed(100 * rows + call + (7 if with_logits else 0))
        hidden = torch.randn(rows, hidden_size, device=cuda, generator=g).bfloat16()
        weight = (torch.randn(vocab, hidden_size, device=cuda, generator=g) * 0.05).bfloat16()
        ids = torch.empty(rows, dtype=torch.int64, device=cuda)
        logits = (torch.empty(rows, vocab, dtype=torch.bfloat16, device=cuda) if with_logits
                  else None)
        assert static_call(ids, hidden, weight, logits) == 0
        want_ids = torch.empty_like(ids)
        want_logits = torch.empty_like(logits) if with_logits else None
        workspace = torch.zeros(rows, dtype=torch.int64, device=cuda)
        capi.lm_head_argmax(want_ids, hidden, weight, workspace, want_logits)
        torch.cuda.synchronize()
        assert torch.equal(ids, want_ids), f"call {call}"
        if with_logits:
            assert torch.equal(logits, want_logits), f"call {call}"
            assert torch.equal(ids, torch.argmax(logits, dim=-1))


def test_rejects_more_rows_than_the_scratch_holds(cuda):
    hidden = torch.zeros(MAX_ROWS + 1, 64, dtype=torch.bfloat16, device=cuda)
    weight = torch.zeros(16, 64, dtype=torch.bfloat16, device=cuda)
    ids = torch.empty(MAX_ROWS + 1, dtype=torch.int64, device=cuda)
    assert static_call(ids, hidden, weight) == SVLLM_ERR_TOO_LARGE
