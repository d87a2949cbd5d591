"""Build recipe for the oracle (TEST INFRASTRUCTURE; never part of the product).

1. oracle/libsvllm_oracle.so: the C/OpenMP restatement in oracle/svllm_oracle.c, compiled with
   -ffp-contract=off so every multiply and add rounds on its own, as the formulas say.
2. oracle/_ref/svllm_ref_ops*.so: the reference's own rms_norm (its op API, OpenMP CPU kernel and
   CUDA kernel, src/ops/rms_norm.cpp, src/ops/cpu/rms_norm.cpp, src/ops/cuda/rms_norm.cu), compiled
   from the sources where they lie under the reference checkout, for sm_100a, with the binding
   oracle/ref_binding.cpp. Only built when the reference checkout is present (this container);
   the built file travels with the tree. Outputs go to oracle/_ref/ only.
3. oracle/_ref/reference_tests/: the reference's own Python tests of the op API, unmodified
   (tests/python/conftest.py, test_rms_norm.py, test_bindings.py, and the pyproject.toml whose
   version test_bindings.py checks), copied in the reference's layout so that they run against
   small-vllm_b200's svllm_ops with SVLLM_BUILD_DIR pointing at it (tests/test_reference_suite.py).

The reference checkout is given by --reference or the SVLLM_REFERENCE environment variable;
without either, only the restatement is built.

Usage: python oracle/build.py [--force] [--reference PATH]
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

ORACLE = Path(__file__).resolve().parent
REF_OUT = ORACLE / "_ref"
ORACLE_LIB = ORACLE / "libsvllm_oracle.so"
REF_TESTS = REF_OUT / "reference_tests"
# The reference's test files run unmodified, in its layout (REPO_ROOT = tests/python/../..).
REF_TEST_FILES = ["pyproject.toml", "tests/python/conftest.py", "tests/python/test_rms_norm.py",
                  "tests/python/test_bindings.py"]
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def _stale(target: Path, deps: list[Path]) -> bool:
    return not target.exists() or any(d.stat().st_mtime > target.stat().st_mtime for d in deps)


def build_oracle(force: bool = False) -> Path:
    src = ORACLE / "svllm_oracle.c"
    if force or _stale(ORACLE_LIB, [src, Path(__file__)]):
        _run(["/usr/bin/gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-ffp-contract=off",
              "-fPIC", "-shared", "-o", str(ORACLE_LIB), str(src), "-lm"])
    return ORACLE_LIB


def build_reference(reference: Path, force: bool = False) -> Path | None:
    """Compiles the reference's rms_norm (CPU + CUDA) into oracle/_ref/. None if absent."""
    src_dir = reference / "src"
    sources = [src_dir / "ops" / "rms_norm.cpp", src_dir / "ops" / "cpu" / "rms_norm.cpp",
               src_dir / "ops" / "cuda" / "rms_norm.cu"]
    if not all(s.exists() for s in sources):
        return None
    import torch
    from torch.utils import cpp_extension

    REF_OUT.mkdir(parents=True, exist_ok=True)
    ext = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    target = REF_OUT / f"svllm_ref_ops{ext}"
    deps = [*sources, ORACLE / "ref_binding.cpp", Path(__file__)]
    if not force and not _stale(target, deps):
        return target

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    common = [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DSVLLM_CUDA", f"-I{src_dir}",
              f"-I{sysconfig.get_paths()['include']}", f"-I{CUDA_HOME / 'include'}",
              "-DTORCH_EXTENSION_NAME=svllm_ref_ops", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    for key in ("COMPILER_TYPE", "STDLIB", "BUILD_ABI"):
        val = getattr(torch._C, f"_PYBIND11_{key}", None)
        if val:
            common.append(f'-DPYBIND11_{key}="{val}"')
    common += [f"-I{inc}" for inc in cpp_extension.include_paths()]
    cxx = "/usr/bin/g++"
    objs = []
    cpp_units = [(sources[0], "ref_ops_rms_norm.o"), (sources[1], "ref_cpu_rms_norm.o"),
                 (ORACLE / "ref_binding.cpp", "ref_binding.o")]
    for src, name in cpp_units:
        obj = REF_OUT / name
        _run([cxx, "-O3", "-std=c++20", "-fPIC", "-fopenmp", *common, "-c", str(src), "-o", str(obj)])
        objs.append(obj)
    cu_obj = REF_OUT / "ref_cuda_rms_norm.o"
    _run([str(CUDA_HOME / "bin" / "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a", "-O3",
          "-std=c++20", "-Xcompiler", "-fPIC", f"-ccbin={cxx}", *common, "-c", str(sources[2]),
          "-o", str(cu_obj)])
    objs.append(cu_obj)
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    _run([cxx, "-shared", "-fopenmp", *map(str, objs), f"-L{torch_lib}", "-lc10", "-ltorch",
          "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", f"-L{CUDA_HOME / 'lib64'}",
          "-lcudart_static", "-ldl", "-lrt", "-lpthread", f"-Wl,-rpath,{torch_lib}", "-o",
          str(target)])
    for obj in objs:
        obj.unlink()
    return target


def stage_reference_tests(reference: Path) -> Path | None:
    """Copies the reference's op-API tests, byte for byte, into oracle/_ref/reference_tests/."""
    import shutil

    if not all((reference / f).exists() for f in REF_TEST_FILES):
        return None
    for f in REF_TEST_FILES:
        dst = REF_TESTS / f
        dst.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(reference / f, dst)
    return REF_TESTS


def reference_dir(explicit: Path | None = None) -> Path | None:
    """The reference checkout: the explicit path, else $SVLLM_REFERENCE, else None."""
    if explicit is not None:
        return explicit
    env = os.environ.get("SVLLM_REFERENCE")
    return Path(env) if env else None


def build(force: bool = False, reference: Path | None = None) -> None:
    build_oracle(force)
    reference = reference_dir(reference)
    if reference is not None and reference.exists():
        build_reference(reference, force)
        stage_reference_tests(reference)


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--reference", type=Path, default=None,
                        help="the reference checkout (default: $SVLLM_REFERENCE)")
    args = parser.parse_args()
    build(args.force, args.reference)
    return 0


if __name__ == "__main__":
    sys.exit(main())
