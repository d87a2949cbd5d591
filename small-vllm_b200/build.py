"""Builds the small-vLLM B200 layer-op library in place.

Products (all inside this directory, so they travel with the source tree):
  lib/libsvllm_kernels.so   the sm_100a CUDA kernels behind the C ABI in include/svllm_kernels.h
  python/svllm_ops*.so      the LibTorch op layer, the model forward that calls it, and the
                            pybind11 module `svllm_ops` (the reference's binding name,
                            bindings/svllm_ops.cpp:11), linked to the library above

Usage: python small-vllm_b200/build.py [--force] [--jobs N]
Only sources newer than their outputs are rebuilt. nvcc cross-compiles for sm_100a without a
GPU. The op layer is compiled with the C++ compiler against the installed torch.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB_DIR = PKG / "lib"
PY_DIR = PKG / "python"
INCLUDE = REPO / "include"
KERNEL_LIB = LIB_DIR / "libsvllm_kernels.so"
VERSION = "0.1.0"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *GENCODE,
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-ffp-contract=off",
    f"-I{INCLUDE}",
    f"-I{CSRC / 'kernels'}",
]


def _newer(target: Path, deps: list[Path]) -> bool:
    """True when target is missing or older than any dependency."""
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n"
                           f"{proc.stdout}\n{proc.stderr}")


def kernel_sources() -> list[Path]:
    """The CUDA sources of libsvllm_kernels.so (CMakeLists.txt globs the same files)."""
    return sorted((CSRC / "kernels").glob("*.cu"))


def op_sources() -> list[Path]:
    """The C++ sources of the svllm_ops module: the op layer, the model forward and the binding
    (CMakeLists.txt globs the same files)."""
    return (sorted((CSRC / "ops").rglob("*.cpp")) + sorted((CSRC / "model").glob("*.cpp")) +
            sorted((CSRC / "bindings").glob("*.cpp")))


def build_kernels(force: bool, jobs: int, verbose_ptxas: bool = False) -> Path:
    """Compiles csrc/kernels/*.cu for sm_100a and links libsvllm_kernels.so."""
    kdir = CSRC / "kernels"
    sources = kernel_sources()
    headers = sorted(kdir.glob("*.cuh")) + sorted(kdir.glob("*.h")) + [INCLUDE / "svllm_kernels.h"]
    obj_dir = BUILD / "kernels"
    obj_dir.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)

    def compile_one(src: Path) -> Path:
        obj = obj_dir / (src.stem + ".o")
        if force or _newer(obj, [src, *headers, Path(__file__)]):
            extra = ["-Xptxas", "-v"] if verbose_ptxas else []
            _run([NVCC, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)])
        return obj

    with ThreadPoolExecutor(max_workers=jobs) as pool:
        objs = list(pool.map(compile_one, sources))
    if force or _newer(KERNEL_LIB, objs):
        _run([NVCC, *GENCODE, "-shared", "-o", str(KERNEL_LIB), *map(str, objs)])
    return KERNEL_LIB


def _torch_flags() -> tuple[list[str], list[str]]:
    import torch
    from torch.utils import cpp_extension

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cflags = [
        "-O3",
        "-std=c++17",
        "-fPIC",
        "-fopenmp",
        "-ffp-contract=off",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-DTORCH_EXTENSION_NAME=svllm_ops",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        "-DSVLLM_CUDA",
        f'-DSVLLM_VERSION="{VERSION}"',
        f"-I{sysconfig.get_paths()['include']}",
        f"-I{CUDA_HOME / 'include'}",
        f"-I{INCLUDE}",
        f"-I{CSRC}",
    ]
    for key in ("COMPILER_TYPE", "STDLIB", "BUILD_ABI"):
        val = getattr(torch._C, f"_PYBIND11_{key}", None)
        if val:
            cflags.append(f'-DPYBIND11_{key}="{val}"')
    for inc in cpp_extension.include_paths():
        cflags.append(f"-I{inc}")
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    ldflags = [
        "-shared",
        "-fopenmp",
        f"-L{torch_lib}",
        "-lc10",
        "-ltorch",
        "-ltorch_cpu",
        "-ltorch_python",
        "-lc10_cuda",
        "-ltorch_cuda",
        f"-L{LIB_DIR}",
        "-lsvllm_kernels",
        "-Wl,-rpath,$ORIGIN/../lib",
        f"-Wl,-rpath,{torch_lib}",
    ]
    return cflags, ldflags


def build_ops(force: bool, jobs: int) -> Path:
    """Compiles the LibTorch op layer and the pybind11 module svllm_ops."""
    # The system g++ ships OpenMP's spec files; a toolchain on CXX may not.
    cxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else os.environ.get("CXX", "g++")
    sources = op_sources()
    headers = (sorted((CSRC / "ops").rglob("*.h")) + sorted((CSRC / "model").glob("*.h")) +
               [INCLUDE / "svllm_kernels.h"])
    obj_dir = BUILD / "ops"
    obj_dir.mkdir(parents=True, exist_ok=True)
    PY_DIR.mkdir(parents=True, exist_ok=True)
    cflags, ldflags = _torch_flags()

    def compile_one(src: Path) -> Path:
        rel = src.relative_to(CSRC).with_suffix(".o")
        obj = obj_dir / str(rel).replace(os.sep, "__")
        if force or _newer(obj, [src, *headers, Path(__file__)]):
            _run([cxx, *cflags, "-c", str(src), "-o", str(obj)])
        return obj

    with ThreadPoolExecutor(max_workers=jobs) as pool:
        objs = list(pool.map(compile_one, sources))
    ext = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    target = PY_DIR / f"svllm_ops{ext}"
    if force or _newer(target, [*objs, KERNEL_LIB]):
        _run([cxx, *map(str, objs), *ldflags, "-o", str(target)])
    return target


def build(force: bool = False, jobs: int | None = None) -> None:
    jobs = jobs or max(1, min(16, os.cpu_count() or 1))
    build_kernels(force, jobs)
    build_ops(force, jobs)


def clean() -> None:
    for path in (BUILD, LIB_DIR):
        if path.exists():
            shutil.rmtree(path)
    for so in PY_DIR.glob("svllm_ops*.so"):
        so.unlink()


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true", help="rebuild everything")
    parser.add_argument("--jobs", type=int, default=None)
    parser.add_argument("--kernels-only", action="store_true")
    parser.add_argument("--ptxas-verbose", action="store_true",
                        help="print registers / spills / shared memory per kernel")
    parser.add_argument("--clean", action="store_true")
    args = parser.parse_args()
    if args.clean:
        clean()
        return 0
    jobs = args.jobs or max(1, min(16, os.cpu_count() or 1))
    if args.ptxas_verbose:
        build_kernels(True, jobs, verbose_ptxas=True)
    elif args.kernels_only:
        build_kernels(args.force, jobs)
    else:
        build(args.force, jobs)
    return 0


if __name__ == "__main__":
    sys.exit(main())
