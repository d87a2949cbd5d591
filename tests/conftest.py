"""Shared fixtures: import paths, seeded inputs, bf16 comparison helpers.

Mirrors the reference's tests/python/conftest.py: a `device` fixture that runs a test on CPU and
CUDA (the CUDA case marked `gpu`), seeded CPU generators so inputs are identical on every device
(conftest.py:29-32), and the reference's bf16 tolerance, rtol = 2 * bf16 eps, atol = 1e-5
(conftest.py:35-45). The product is imported from small-vllm_b200/python (svllm_ops, the
LibTorch op layer; svllm_capi, the ctypes binding of the C ABI); the oracle from oracle/.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch  # loads libtorch before svllm_ops, which links against it

REPO_ROOT = Path(__file__).resolve().parents[1]
PKG_PY = REPO_ROOT / "small-vllm_b200" / "python"
ORACLE_DIR = REPO_ROOT / "oracle"
GOLDEN = REPO_ROOT / "tests" / "golden" / "golden.npz"
for p in (PKG_PY, ORACLE_DIR):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

BF16_EPS = torch.finfo(torch.bfloat16).eps


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def cuda_ok() -> bool:
    return torch.cuda.is_available()


@pytest.fixture(params=["cpu", pytest.param("cuda", marks=pytest.mark.gpu)])
def device(request) -> torch.device:
    """Run the test once per device the ops have a kernel for."""
    if request.param == "cuda" and not cuda_ok():
        pytest.skip("needs a GPU")
    return torch.device(request.param)


@pytest.fixture
def cuda() -> torch.device:
    if not cuda_ok():
        pytest.skip("needs a GPU")
    return torch.device("cuda", 0)


def random_bf16(*shape: int, device: torch.device | str = "cpu", seed: int = 0) -> torch.Tensor:
    """Seeded standard-normal bf16 values, identical on every device for a given seed."""
    generator = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=generator).to(device=device, dtype=torch.bfloat16)


def random_t(*shape: int, dtype=torch.bfloat16, device="cpu", seed: int = 0, scale: float = 1.0,
             shift: float = 0.0) -> torch.Tensor:
    generator = torch.Generator().manual_seed(seed)
    t = torch.randn(shape, generator=generator) * scale + shift
    return t.to(device=device, dtype=dtype)


def assert_close_bf16(actual: torch.Tensor, expected: torch.Tensor, *, rtol: float = 2 * BF16_EPS,
                      atol: float = 1e-5) -> None:
    """The reference's bf16 tolerance: two bf16 rounding steps, relative."""
    assert actual.dtype == torch.bfloat16, f"expected a bf16 output, got {actual.dtype}"
    torch.testing.assert_close(actual, expected, rtol=rtol, atol=atol)


# ---------------------------------------------------------------------------------------------
# bf16 bit-level comparisons (numpy uint16 bit patterns or torch bf16 tensors)

def to_bits(t) -> np.ndarray:
    if isinstance(t, torch.Tensor):
        t = t.detach().cpu().contiguous()
        if t.dtype == torch.bfloat16:
            return t.view(torch.int16).numpy().view(np.uint16)
        return t.numpy()
    return np.asarray(t)


def from_bits(a: np.ndarray, device="cpu") -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return torch.from_numpy(a.copy()).to(device)


def bf16_key(bits: np.ndarray) -> np.ndarray:
    """Maps bf16 bit patterns to integers whose difference counts representable steps (ulps)."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.int32)
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


def ulp_diff_bf16(a, b) -> np.ndarray:
    return np.abs(bf16_key(to_bits(a)) - bf16_key(to_bits(b)))


def bf16_values(bits) -> np.ndarray:
    return (np.asarray(to_bits(bits), dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def assert_bf16_within_ulp(actual, expected, max_ulp: int, what: str = "") -> float:
    """Every element within max_ulp bf16 steps; returns the fraction that is bit-exact."""
    d = ulp_diff_bf16(actual, expected)
    if d.size == 0:
        return 1.0
    worst = int(d.max())
    assert worst <= max_ulp, (
        f"{what}: {int((d > max_ulp).sum())} of {d.size} elements differ by more than {max_ulp} "
        f"bf16 ulp (worst {worst})")
    return float((d == 0).mean())


def rope_within_rounding(out, ref, pre) -> np.ndarray:
    """Per element: a rotated bf16 output within one bf16 rounding of each rotation term of the
    reference (2^-7 of |x_i| + |x_{i+d/2}| of the pre-rotation values `pre`) plus one rounding of
    the result (2^-8 of |ref|). The rotation cancels, so a result near zero can be many of its
    own ulps off and still this close; the CPU oracle's cosf/sinf are the C library's, not
    CUDA's. Arguments: bf16 bit patterns (or tensors) with the head dimension last."""
    o = bf16_values(out).astype(np.float64)
    r = bf16_values(ref).astype(np.float64)
    p = bf16_values(pre).astype(np.float64)
    half = p.shape[-1] // 2
    mag = np.abs(p[..., :half]) + np.abs(p[..., half:])
    mag = np.concatenate([mag, mag], axis=-1)
    return np.abs(o - r) <= 2.0 ** -7 * mag + 2.0 ** -8 * np.abs(r) + 1e-30


def assert_rel_f32(actual, expected, rtol: float = 1e-5, what: str = "", scale=None) -> None:
    """fp32: |a - e| <= rtol * max(|e|, s) per element (the fp32 ops' 1e-5 relative bar),
    where s is the magnitude the element was computed from: by default the RMS of its row (the
    last axis), so a value that cancels to near zero is held to the row's scale, not its own."""
    a = np.asarray(to_bits(actual), dtype=np.float64)
    e = np.asarray(to_bits(expected), dtype=np.float64)
    if scale is None:
        scale = np.sqrt((e ** 2).mean(axis=-1, keepdims=True)) if e.ndim else np.abs(e)
    bound = rtol * np.maximum(np.abs(e), scale)
    bad = np.abs(a - e) > bound
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} fp32 elements off by more "
                           f"than {rtol} relative (worst {np.abs(a - e)[bad].max()})")


def golden() -> dict[str, np.ndarray]:
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}
