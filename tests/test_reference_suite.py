"""The reference's own op-API tests, run unmodified against small-vllm_b200's svllm_ops.

small-vLLM's tests/python/conftest.py, test_rms_norm.py and test_bindings.py (with the
pyproject.toml whose version test_bindings.py checks) are copied byte for byte by oracle/build.py
into oracle/_ref/reference_tests/, in the reference's own layout, and run here in a fresh
interpreter with SVLLM_BUILD_DIR pointing at small-vllm_b200/ (the reference's conftest.py:10-13
puts $SVLLM_BUILD_DIR/python on sys.path, where small-vllm_b200's svllm_ops lives). The CPU run hides
the GPU, so the reference's CUDA cases skip as they do on a CPU machine; the GPU run needs every
case, CUDA included, to pass. tests/test_cmake_build.py runs the same suite against the module
that the CMake target builds.
"""

from __future__ import annotations

import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

from conftest import ORACLE_DIR, REPO_ROOT

REF_TESTS = ORACLE_DIR / "_ref" / "reference_tests"
PKG = REPO_ROOT / "small-vllm_b200"


def staged() -> bool:
    return (REF_TESTS / "tests" / "python" / "test_rms_norm.py").exists()


def run_reference_suite(build_dir: Path, hide_gpu: bool) -> tuple[int, dict[str, int], str]:
    """Runs the staged reference tests against the svllm_ops in build_dir/python; returns the
    exit code, the outcome counts and the output."""
    env = dict(os.environ, SVLLM_BUILD_DIR=str(build_dir), PYTHONDONTWRITEBYTECODE="1")
    if hide_gpu:
        env["CUDA_VISIBLE_DEVICES"] = ""
    proc = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-rs", "-p", "no:cacheprovider",
         str(REF_TESTS / "tests" / "python")],
        cwd=REF_TESTS, env=env, capture_output=True, text=True, timeout=900)
    out = proc.stdout + proc.stderr
    counts = {k: 0 for k in ("passed", "failed", "skipped", "error", "errors")}
    tail = out.strip().splitlines()[-1] if out.strip() else ""
    for num, what in re.findall(r"(\d+) (passed|failed|skipped|errors?)", tail):
        counts[what] = int(num)
    return proc.returncode, counts, out


@pytest.mark.skipif(not staged(), reason="the reference's tests are not staged in oracle/_ref")
def test_reference_suite_passes_on_cpu():
    rc, counts, out = run_reference_suite(PKG, hide_gpu=True)
    assert rc == 0, out[-3000:]
    # 7 shapes + unaligned rows on CPU, 5 invalid-input cases, the version check; the 8 CUDA
    # cases skip for want of a GPU, as in the reference's own CPU runs
    assert counts["passed"] == 14 and counts["skipped"] == 8, out[-3000:]
    assert counts["failed"] == 0


@pytest.mark.gpu
@pytest.mark.skipif(not staged(), reason="the reference's tests are not staged in oracle/_ref")
def test_reference_suite_passes_on_cuda():
    rc, counts, out = run_reference_suite(PKG, hide_gpu=False)
    assert rc == 0, out[-3000:]
    assert counts["passed"] == 22 and counts["skipped"] == 0, out[-3000:]
