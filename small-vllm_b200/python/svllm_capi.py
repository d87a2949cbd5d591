"""ctypes binding of the C ABI in include/svllm_kernels.h (lib/libsvllm_kernels.so).

This is the binding a Python caller of the C ABI would write; the LibTorch op layer (svllm_ops)
is the reference-compatible front end, and this module is the thin one: raw device pointers,
sizes, strides and the current CUDA stream, taken from torch tensors for convenience. Every call
raises CapiError on a non-zero status. There is no CPU path: loading fails loudly if the library
is missing.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent.parent / "lib" / "libsvllm_kernels.so"

INDEX_I32 = 0
INDEX_I64 = 1
DEVERR_BAD_INDEX = 1
DEVERR_WAIT_TIMEOUT = 2

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_F = ctypes.c_float
_I = ctypes.c_int


class Llama3Scaling(ctypes.Structure):
    """svllm_llama3_scaling; the reference's Llama3RopeScaling (src/model/config.h:10-15)."""

    _fields_ = [("factor", ctypes.c_double), ("low_freq_factor", ctypes.c_double),
                ("high_freq_factor", ctypes.c_double),
                ("original_max_position_embeddings", ctypes.c_int64)]


class CapiError(RuntimeError):
    pass


# name -> argument types; every function returns int status
SIGNATURES = {
    "svllm_rms_norm_bf16": [_P, _P, _P, _I64, _I64, _I64, _I64, _F, _P],
    "svllm_rms_norm_f32": [_P, _P, _P, _I64, _I64, _I64, _I64, _F, _P],
    "svllm_add_rms_norm_bf16": [_P, _P, _P, _I64, _I64, _I64, _I64, _F, _P],
    "svllm_add_rms_norm_f32": [_P, _P, _P, _I64, _I64, _I64, _I64, _F, _P],
    "svllm_qk_norm_rope_bf16": [_P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _F,
                                _P, _P],
    "svllm_qk_norm_rope_f32": [_P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _F,
                               _P, _P],
    "svllm_rope_bf16": [_P, _P, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P],
    "svllm_rope_f32": [_P, _P, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P],
    "svllm_rope_inv_freq": [ctypes.c_double, _I64, _P, _P],
    "svllm_qk_norm_rope_cache_bf16": [_P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _I64, _I64, _I64,
                                      _I64, _I64, _I64, _I64, _I64, _F, _P, _P],
    "svllm_qk_norm_rope_cache_f32": [_P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _I64, _I64, _I64,
                                     _I64, _I64, _I64, _I64, _I64, _F, _P, _P],
    "svllm_rope_cache_bf16": [_P, _P, _P, _P, _I, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                              _I64, _I64, _P, _P],
    "svllm_rope_cache_f32": [_P, _P, _P, _P, _I, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                             _I64, _I64, _P, _P],
    "svllm_silu_and_mul_bf16": [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P],
    "svllm_silu_and_mul_f32": [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P],
    "svllm_embedding_bf16": [_P, _P, _I, _P, _I64, _I64, _I64, _I64, _I64, _P, _P],
    "svllm_embedding_f32": [_P, _P, _I, _P, _I64, _I64, _I64, _I64, _I64, _P, _P],
    "svllm_argmax_bf16": [_P, _I64, _I64, _I64, _P, _P],
    "svllm_argmax_f32": [_P, _I64, _I64, _I64, _P, _P],
    "svllm_lm_head_argmax_bf16": [_P, _I64, _I64, _I64, _P, _I64, _I64, _P, _P, _I64, _P, _I64,
                                  _P],
    "svllm_lm_head_argmax_static_bf16": [_P, _I64, _I64, _I64, _P, _I64, _I64, _P, _P, _I64, _P],
    "svllm_paged_decode_attention_bf16": [_P, _P, _I64, _P, _P, _I64, _I64, _P, _I64, _P, _I64,
                                          _I64, _I64, _I64, _I64, ctypes.c_float, _P],
    "svllm_decode_linear_bf16": [_P, _I64, _P, _I64, _I64, _I64, _P, _I64, _I64, _P],
    "svllm_read_device_error": [_I, _I, _P],
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise CapiError(f"{LIB_PATH} is missing: build it with small-vllm_b200/build.py")
        _lib = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(_lib, name)
            fn.argtypes = args
            fn.restype = _I
        _lib.svllm_status_string.argtypes = [_I]
        _lib.svllm_status_string.restype = ctypes.c_char_p
        _lib.svllm_version.argtypes = []
        _lib.svllm_version.restype = ctypes.c_char_p
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().svllm_status_string(status).decode()
        raise CapiError(f"{what}: {msg} (status {status})")


def _stream(stream=None) -> int | None:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream or None


def _bf16_or_f32(t) -> str:
    import torch

    if t.dtype == torch.bfloat16:
        return "bf16"
    if t.dtype == torch.float32:
        return "f32"
    raise CapiError(f"unsupported dtype {t.dtype}")


def _index_type(t) -> int:
    import torch

    if t.dtype == torch.int64:
        return INDEX_I64
    if t.dtype == torch.int32:
        return INDEX_I32
    raise CapiError(f"unsupported index dtype {t.dtype}")


def _rows(t) -> tuple[int, int, int]:
    """(rows, row length, row stride) of a tensor whose last dim is contiguous."""
    if t.stride(-1) != 1:
        raise CapiError("the last dimension must be contiguous")
    n = t.shape[-1]
    rows = t.numel() // n if n else 0
    stride = t.stride(-2) if t.dim() >= 2 else n
    return rows, n, stride


def rms_norm(out, x, weight, eps: float, stream=None) -> None:
    rows, hidden, xs = _rows(x)
    _, _, os_ = _rows(out)
    fn = getattr(lib(), f"svllm_rms_norm_{_bf16_or_f32(x)}")
    check(fn(out.data_ptr(), x.data_ptr(), weight.data_ptr(), rows, hidden, os_, xs, eps,
             _stream(stream)), "rms_norm")


def add_rms_norm(x, residual, weight, eps: float, stream=None) -> None:
    rows, hidden, xs = _rows(x)
    _, _, rs = _rows(residual)
    fn = getattr(lib(), f"svllm_add_rms_norm_{_bf16_or_f32(x)}")
    check(fn(x.data_ptr(), residual.data_ptr(), weight.data_ptr(), rows, hidden, xs, rs, eps,
             _stream(stream)), "add_rms_norm")


def inv_freq(theta: float, head_dim: int, scaling: tuple | None = None):
    """Hugging Face's fp32 table from the C helper, as a list of floats."""
    out = (ctypes.c_float * (head_dim // 2))()
    sc = Llama3Scaling(*scaling) if scaling is not None else None
    check(lib().svllm_rope_inv_freq(theta, head_dim, ctypes.byref(sc) if sc else None,
                                    ctypes.cast(out, _P)), "rope_inv_freq")
    return list(out)


def _inv_array(inv):
    arr = (ctypes.c_float * len(inv))(*[float(v) for v in inv])
    return arr


def qk_norm_rope(q, k, q_weight, k_weight, positions, eps: float, inv, stream=None) -> None:
    """q [T, Hq, D], k [T, Hk, D] (token stride free), in place; inv: head_dim/2 floats."""
    arr = _inv_array(inv)
    fn = getattr(lib(), f"svllm_qk_norm_rope_{_bf16_or_f32(q)}")
    check(fn(q.data_ptr(), k.data_ptr(), q_weight.data_ptr(), k_weight.data_ptr(),
             positions.data_ptr(), _index_type(positions), q.shape[0], q.shape[1], k.shape[1],
             q.shape[2], q.stride(0), k.stride(0), eps, ctypes.cast(arr, _P), _stream(stream)),
          "qk_norm_rope")


def rope(q, k, positions, inv, stream=None) -> None:
    arr = _inv_array(inv)
    fn = getattr(lib(), f"svllm_rope_{_bf16_or_f32(q)}")
    check(fn(q.data_ptr(), k.data_ptr(), positions.data_ptr(), _index_type(positions),
             q.shape[0], q.shape[1], k.shape[1], q.shape[2], q.stride(0), k.stride(0),
             ctypes.cast(arr, _P), _stream(stream)), "rope")


def qk_norm_rope_cache(q, k, v, q_weight, k_weight, positions, slot_mapping, k_cache, v_cache,
                       eps: float, inv, stream=None) -> None:
    """qk_norm_rope plus the paged-KV write; caches are [num_slots, Hk, D] (or a
    [blocks, block_size, Hk, D] tensor, flattened)."""
    arr = _inv_array(inv)
    num_slots = k_cache.numel() // (k.shape[1] * k.shape[2])
    fn = getattr(lib(), f"svllm_qk_norm_rope_cache_{_bf16_or_f32(q)}")
    check(fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), q_weight.data_ptr(), k_weight.data_ptr(),
             positions.data_ptr(), _index_type(positions), slot_mapping.data_ptr(),
             k_cache.data_ptr(), v_cache.data_ptr(), num_slots, q.shape[0], q.shape[1],
             k.shape[1], q.shape[2], q.stride(0), k.stride(0), v.stride(0), eps,
             ctypes.cast(arr, _P), _stream(stream)), "qk_norm_rope_cache")


def rope_cache(q, k, v, positions, slot_mapping, k_cache, v_cache, inv, stream=None) -> None:
    arr = _inv_array(inv)
    num_slots = k_cache.numel() // (k.shape[1] * k.shape[2])
    fn = getattr(lib(), f"svllm_rope_cache_{_bf16_or_f32(q)}")
    check(fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), positions.data_ptr(),
             _index_type(positions), slot_mapping.data_ptr(), k_cache.data_ptr(),
             v_cache.data_ptr(), num_slots, q.shape[0], q.shape[1], k.shape[1], q.shape[2],
             q.stride(0), k.stride(0), v.stride(0), ctypes.cast(arr, _P), _stream(stream)),
          "rope_cache")


def silu_and_mul(out, gate, up, stream=None) -> None:
    rows, inter, gs = _rows(gate)
    _, _, us = _rows(up)
    _, _, os_ = _rows(out)
    fn = getattr(lib(), f"svllm_silu_and_mul_{_bf16_or_f32(gate)}")
    check(fn(out.data_ptr(), gate.data_ptr(), up.data_ptr(), rows, inter, os_, gs, us,
             _stream(stream)), "silu_and_mul")


def embedding(out, ids, table, err=None, stream=None) -> None:
    vocab, hidden = table.shape
    _, _, os_ = _rows(out)
    fn = getattr(lib(), f"svllm_embedding_{_bf16_or_f32(table)}")
    check(fn(out.data_ptr(), ids.data_ptr(), _index_type(ids), table.data_ptr(), ids.numel(),
             vocab, hidden, os_, table.stride(0), err.data_ptr() if err is not None else None,
             _stream(stream)), "embedding")


def argmax(out_ids, logits, stream=None) -> None:
    rows, vocab, stride = _rows(logits)
    fn = getattr(lib(), f"svllm_argmax_{_bf16_or_f32(logits)}")
    check(fn(logits.data_ptr(), rows, vocab, stride, out_ids.data_ptr(), _stream(stream)),
          "argmax")


def lm_head_argmax(out_ids, hidden, weight, workspace, logits=None, stream=None) -> None:
    """out_ids[r] = argmax_n bf16(hidden[r] . weight[n]); workspace: int64 [>= rows], zero."""
    rows, hidden_size, hidden_stride = _rows(hidden)
    vocab, _, weight_stride = _rows(weight)
    check(lib().svllm_lm_head_argmax_bf16(
        hidden.data_ptr(), rows, hidden_size, hidden_stride, weight.data_ptr(), vocab,
        weight_stride, out_ids.data_ptr(), logits.data_ptr() if logits is not None else None,
        logits.stride(0) if logits is not None else 0, workspace.data_ptr(),
        workspace.numel() * workspace.element_size(), _stream(stream)), "lm_head_argmax")


def paged_decode_attention(out, q, k_cache, v_cache, block_tables, seq_lens, max_seq_len: int,
                           scale: float, stream=None) -> None:
    """out [S, Hq, D] = decode attention of q [S, Hq, D] over the paged caches."""
    num_seqs, num_heads, head_dim = q.shape
    num_blocks, block_size, num_kv_heads, _ = k_cache.shape
    check(lib().svllm_paged_decode_attention_bf16(
        out.data_ptr(), q.data_ptr(), q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
        num_blocks, block_size, block_tables.data_ptr(), block_tables.shape[1],
        seq_lens.data_ptr(), num_seqs, num_heads, num_kv_heads, head_dim, max_seq_len, scale,
        _stream(stream)), "paged_decode_attention")


def decode_linear(out, x, weight, stream=None) -> None:
    """out [R, N] = x [R, K] . weight [N, K]^T for R <= 16 (bf16, fp32 accumulation)."""
    rows, in_features, x_stride = _rows(x)
    out_features, _, weight_stride = _rows(weight)
    check(lib().svllm_decode_linear_bf16(
        out.data_ptr(), out.stride(0), x.data_ptr(), rows, in_features, x_stride,
        weight.data_ptr(), out_features, weight_stride, _stream(stream)), "decode_linear")


def read_device_error(device: int = 0, reset: bool = True) -> int:
    flags = ctypes.c_int(0)
    check(lib().svllm_read_device_error(device, 1 if reset else 0, ctypes.byref(flags)),
          "read_device_error")
    return flags.value



def version() -> str:
    return lib().svllm_version().decode()
