"""The CMake target (small-vllm_b200/CMakeLists.txt) builds the same library and module as
build.py, and the module it builds works.

Configures with -DSVLLM_B200_OPS=ON in a temporary directory with the image's default compilers
(CXX included), builds, and checks that
  * CMake compiled exactly the sources build.py compiles (kernels, op layer, model, binding);
  * the module imports from the CMake build tree, with the same attributes as build.py's;
  * its CPU ops give the same bits as build.py's module on seeded inputs;
  * the reference's own op-API tests pass against it (when staged in oracle/_ref).
About a minute of compiling (nvcc for sm_100a and the C++ op layer); no GPU needed.
"""

from __future__ import annotations

import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from conftest import REPO_ROOT

PKG = REPO_ROOT / "small-vllm_b200"

# Computed in a fresh interpreter against whichever svllm_ops is first on sys.path: module
# facts plus the bits of a few CPU ops on seeded inputs.
PROBE = r"""
import hashlib, json, sys
sys.path.insert(0, sys.argv[1])
import torch
import svllm_ops as m
g = torch.Generator().manual_seed(7)
def r(*s, scale=1.0, shift=0.0):
    return (torch.randn(s, generator=g) * scale + shift).to(torch.bfloat16)
x, res, w = r(9, 1024), r(9, 1024), r(1024, scale=0.1, shift=1.0)
q, k, qw, kw = r(9, 16, 128), r(9, 8, 128), r(128, scale=0.1, shift=1.0), r(128, scale=0.1, shift=1.0)
pos = torch.arange(9, dtype=torch.int64) * 1000
gate, up = r(9, 3072), r(9, 3072)
table, ids = r(500, 1024), torch.randint(0, 500, (9,), generator=g)
outs = [m.rms_norm(x, w, 1e-6)]
m.add_rms_norm(x, res, w, 1e-6); outs += [x, res]
m.qk_norm_rope(q, k, qw, kw, pos, 1e-6, 1e6); outs += [q, k]
outs += [m.silu_and_mul(gate, up), m.embedding(ids, table)]
h = hashlib.sha256(b"".join(o.contiguous().view(torch.int16).numpy().tobytes() for o in outs))
print(json.dumps({"file": m.__file__, "version": m.__version__, "cuda": m.built_with_cuda,
                  "attrs": sorted(a for a in dir(m) if not a.startswith("__")),
                  "digest": h.hexdigest()}))
"""


def probe(python_dir: Path) -> dict:
    proc = subprocess.run([sys.executable, "-c", PROBE, str(python_dir)], capture_output=True,
                          text=True, timeout=300, env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert proc.returncode == 0, proc.stderr[-3000:]
    return json.loads(proc.stdout.strip().splitlines()[-1])


@pytest.fixture(scope="module")
def cmake_build(tmp_path_factory) -> Path:
    if shutil.which("cmake") is None or shutil.which("nvcc") is None and not Path(
            "/usr/local/cuda/bin/nvcc").exists():
        pytest.skip("cmake or nvcc not available")
    build = tmp_path_factory.mktemp("cmake") / "b200"
    env = dict(os.environ)
    env.setdefault("CUDACXX", str(Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) /
                                  "bin" / "nvcc"))
    cfg = subprocess.run(["cmake", "-S", str(PKG), "-B", str(build), "-DSVLLM_B200_OPS=ON",
                          f"-DPython_EXECUTABLE={sys.executable}"],
                         capture_output=True, text=True, env=env, timeout=600)
    assert cfg.returncode == 0, cfg.stdout[-3000:] + cfg.stderr[-3000:]
    jobs = str(max(1, min(16, os.cpu_count() or 1)))
    out = subprocess.run(["cmake", "--build", str(build), "-j", jobs], capture_output=True,
                         text=True, env=env, timeout=1800)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    return build


def test_cmake_compiles_the_sources_build_py_compiles(cmake_build):
    sys.path.insert(0, str(PKG))
    try:
        import build as build_py  # small-vllm_b200/build.py
    finally:
        sys.path.remove(str(PKG))
    built = {p.name[:-2]  # "norm.cu.o" -> "norm.cu"
             for target in ("svllm_kernels", "svllm_ops")
             for p in (cmake_build / "CMakeFiles" / f"{target}.dir").rglob("*.o")}
    want = {p.name for p in build_py.kernel_sources() + build_py.op_sources()}
    # object names are per-source basenames (cpu/rms_norm.cpp and rms_norm.cpp share one)
    assert built == want
    assert (cmake_build / "lib" / "libsvllm_kernels.so").exists()


def test_cmake_module_imports_and_matches_build_py(cmake_build):
    ours = probe(cmake_build / "python")
    theirs = probe(PKG / "python")
    assert Path(ours["file"]).parent == cmake_build / "python"
    assert Path(theirs["file"]).parent == PKG / "python"
    assert ours["version"] == theirs["version"] == "0.1.0"
    assert ours["cuda"] and theirs["cuda"]
    assert ours["attrs"] == theirs["attrs"]
    assert ours["digest"] == theirs["digest"]


def test_cmake_module_passes_the_reference_suite(cmake_build):
    from test_reference_suite import run_reference_suite, staged

    if not staged():
        pytest.skip("the reference's tests are not staged in oracle/_ref")
    rc, counts, out = run_reference_suite(cmake_build, hide_gpu=True)
    assert rc == 0 and counts["passed"] == 14, out[-3000:]
