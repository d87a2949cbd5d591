"""ctypes front end of the oracle (TEST INFRASTRUCTURE; never part of the product).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module. It
wraps oracle/libsvllm_oracle.so (the C/OpenMP restatement in oracle/svllm_oracle.c) for numpy
arrays, and loads the reference's own rms_norm built from its sources into oracle/_ref/.

bf16 arrays are numpy uint16 bit patterns. Every function works on copies it returns, except
where noted, so callers keep their inputs.
"""

from __future__ import annotations

import ctypes
import importlib.util
import sys
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "libsvllm_oracle.so"
REF_DIR = ORACLE_DIR / "_ref"

_lib: ctypes.CDLL | None = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_F = ctypes.c_float
_I = ctypes.c_int


def lib() -> ctypes.CDLL:
    """Loads (building if needed) the oracle library."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            sys.path.insert(0, str(ORACLE_DIR))
            import build as oracle_build  # oracle/build.py

            oracle_build.build_oracle()
        _lib = ctypes.CDLL(str(LIB_PATH))
        sigs = {
            "orc_rms_norm_bf16": [_P, _P, _P, _I64, _I64, _F],
            "orc_rms_norm_f32": [_P, _P, _P, _I64, _I64, _F],
            "orc_add_rms_norm_bf16": [_P, _P, _P, _I64, _I64, _F],
            "orc_add_rms_norm_f32": [_P, _P, _P, _I64, _I64, _F],
            "orc_qk_norm_rope_bf16": [_P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _F, _P],
            "orc_qk_norm_rope_f32": [_P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _F, _P],
            "orc_rope_bf16": [_P, _P, _P, _I, _I64, _I64, _I64, _I64, _P],
            "orc_rope_f32": [_P, _P, _P, _I, _I64, _I64, _I64, _I64, _P],
            "orc_inv_freq": [ctypes.c_double, _I64, ctypes.c_double, ctypes.c_double,
                             ctypes.c_double, _I64, _P],
            "orc_silu_and_mul_bf16": [_P, _P, _P, _I64, _I64],
            "orc_silu_and_mul_f32": [_P, _P, _P, _I64, _I64],
            "orc_embedding": [_P, _P, _I, _P, _I64, _I64, _I64],
            "orc_set_num_threads": [_I],
        }
        for name, args in sigs.items():
            fn = getattr(_lib, name)
            fn.argtypes = args
            fn.restype = _I64 if name == "orc_embedding" else _I
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def _is_bf16(a: np.ndarray) -> bool:
    return a.dtype == np.uint16


# ---------------------------------------------------------------------------------------------
# bf16 helpers (uint16 bit patterns)

def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits, NaN kept quiet."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), rounded)


# ---------------------------------------------------------------------------------------------
# ops

def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    hidden = x.shape[-1]
    rows = x.size // hidden if hidden else 0
    dt = x.dtype
    xc, wc = _c(x, dt), _c(w, dt)
    out = np.empty_like(xc)
    fn = lib().orc_rms_norm_bf16 if _is_bf16(x) else lib().orc_rms_norm_f32
    fn(_ptr(out), _ptr(xc), _ptr(wc), rows, hidden, eps)
    return out


def add_rms_norm(x: np.ndarray, residual: np.ndarray, w: np.ndarray, eps: float,
                 inplace: bool = False):
    """Returns (normed x, updated residual); with inplace (contiguous inputs) x and residual
    themselves are updated, as the timed CPU baseline does."""
    hidden = x.shape[-1]
    rows = x.size // hidden if hidden else 0
    dt = x.dtype
    if inplace:
        xc, rc = x, residual
    else:
        xc, rc = _c(x, dt).copy(), _c(residual, dt).copy()
    wc = _c(w, dt)
    fn = lib().orc_add_rms_norm_bf16 if _is_bf16(x) else lib().orc_add_rms_norm_f32
    fn(_ptr(xc), _ptr(rc), _ptr(wc), rows, hidden, eps)
    return xc, rc


def qk_norm_rope(q, k, q_weight, k_weight, positions, eps, inv_freq, inplace: bool = False):
    """q [T, Hq, D], k [T, Hk, D]; returns rotated copies (or, with inplace and contiguous
    inputs, rotates q and k themselves). Weights None means rope alone."""
    dt = q.dtype
    qc, kc = (q, k) if inplace else (_c(q, dt).copy(), _c(k, dt).copy())
    pos = np.ascontiguousarray(positions)
    pos_i64 = 1 if pos.dtype == np.int64 else 0
    if not pos_i64:
        pos = _c(pos, np.int32)
    inv = _c(inv_freq, np.float32)
    T, hq, d = qc.shape
    hk = kc.shape[1]
    if q_weight is None:
        fn = lib().orc_rope_bf16 if _is_bf16(q) else lib().orc_rope_f32
        rc = fn(_ptr(qc), _ptr(kc), _ptr(pos), pos_i64, T, hq, hk, d, _ptr(inv))
    else:
        fn = lib().orc_qk_norm_rope_bf16 if _is_bf16(q) else lib().orc_qk_norm_rope_f32
        rc = fn(_ptr(qc), _ptr(kc), _ptr(_c(q_weight, dt)), _ptr(_c(k_weight, dt)), _ptr(pos),
                pos_i64, T, hq, hk, d, eps, _ptr(inv))
    if rc != 0:
        raise ValueError(f"oracle rope: unsupported head_dim {d}")
    return qc, kc


def rope(q, k, positions, inv_freq, inplace: bool = False):
    return qk_norm_rope(q, k, None, None, positions, 0.0, inv_freq, inplace)


def inv_freq(theta: float, head_dim: int, scaling: tuple | None = None) -> np.ndarray:
    """Hugging Face's fp32 table; scaling = (factor, low, high, original_max_positions)."""
    out = np.empty(head_dim // 2, dtype=np.float32)
    f, lo, hi, orig = scaling if scaling is not None else (0.0, 0.0, 0.0, 0)
    if lib().orc_inv_freq(theta, head_dim, f, lo, hi, orig, _ptr(out)) != 0:
        raise ValueError("oracle inv_freq: bad head_dim")
    return out


def silu_and_mul(gate: np.ndarray, up: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
    """Returns silu(gate) * up, written into `out` when given (contiguous, gate's shape)."""
    dt = gate.dtype
    g, u = _c(gate, dt), _c(up, dt)
    if out is None:
        out = np.empty_like(g)
    inter = g.shape[-1]
    rows = g.size // inter if inter else 0
    fn = lib().orc_silu_and_mul_bf16 if _is_bf16(gate) else lib().orc_silu_and_mul_f32
    fn(_ptr(out), _ptr(g), _ptr(u), rows, inter)
    return out


def embedding(ids: np.ndarray, table: np.ndarray,
              out: np.ndarray | None = None) -> tuple[np.ndarray, int]:
    """Returns (rows, number of ids outside [0, vocab)); rows go into `out` when given."""
    ids_c = np.ascontiguousarray(ids)
    is64 = 1 if ids_c.dtype == np.int64 else 0
    if not is64:
        ids_c = _c(ids_c, np.int32)
    tab = np.ascontiguousarray(table)
    if out is None:
        out = np.empty(ids_c.shape + (tab.shape[1],), dtype=tab.dtype)
    bad = lib().orc_embedding(_ptr(out), _ptr(ids_c), is64, _ptr(tab), ids_c.size, tab.shape[0],
                              tab.shape[1] * tab.itemsize)
    return out, int(bad)


def set_num_threads(n: int) -> int:
    """Threads of the oracle's OpenMP loops; returns the count in force."""
    return int(lib().orc_set_num_threads(int(n)))


# ---------------------------------------------------------------------------------------------
# the reference's own rms_norm, built from its sources

def reference_module():
    """The reference's rms_norm (torch extension in oracle/_ref), or None if it was not built."""
    candidates = sorted(REF_DIR.glob("svllm_ref_ops*.so"))
    if not candidates:
        return None
    import torch  # noqa: F401  (libtorch must be loaded first)

    spec = importlib.util.spec_from_file_location("svllm_ref_ops", candidates[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod
