"""Build recipes for the native parts of tvarant_b200.

Two shared objects are produced in-tree, next to this file:

* ``lib/libtvarant_cuda.so`` — the C ABI of ``include/tvarant.h``: runtime,
  kernels (sm_100a, compiled by nvcc with ``-gencode arch=compute_100a,
  code=sm_100a``), NVRTC pointwise JIT and the NCCL wrapper.  It links the
  CUDA runtime statically and has no PyTorch dependency.
* ``_C.so`` — the PyTorch extension that registers the ``tvarant``
  PrivateUse1 device and its ATen kernels; it contains no CUDA code and calls
  the C ABI above.

Builds are incremental (object files are rebuilt when a source or header is
newer) and run compilers in parallel.  Usage, from the repository root:
``python tvarant_b200/build.py [--force] [--clean]`` (run as a script: importing the
package needs the extension this builds).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
EXT_SRC = CSRC / "ext"
BUILD = ROOT / "_build"
LIB_DIR = PKG / "lib"
CUDA_LIB = LIB_DIR / "libtvarant_cuda.so"
EXT_LIB = PKG / "_C.so"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]

CUDA_SOURCES = [
    "runtime.cu",
    "elementwise.cu",
    "select.cu",
    "reduce.cu",
    "gemm.cu",
    "gemm_epilogue.cu",
    "gemm_simt.cu",
    "gemm_skinny.cu",
    "gemm_tc.cu",
    "gemm_ws.cu",
    "attention.cu",
    "attention_decode.cu",
    "pointwise_jit.cu",
    "nccl.cu",
    "nvls.cu",
    "llama_ops.cu",
]

EXT_SOURCES = [
    "Module.cpp",
    "Runtime.cpp",
    "Allocator.cpp",
    "Guard.cpp",
    "Hooks.cpp",
    "Generator.cpp",
    "Ops.cpp",
    "LlmOps.cpp",
    "ExtendedOps.cpp",
    "CustomOps.cpp",
    "Collectives.cpp",
    "Attention.cpp",
    "Select.cpp",
    "LlamaOps.cpp",
]


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stdout}")
    if proc.stdout.strip() and os.environ.get("TVARANT_BUILD_VERBOSE"):
        print(proc.stdout)


def _newest(paths) -> float:
    t = 0.0
    for p in paths:
        try:
            t = max(t, Path(p).stat().st_mtime)
        except FileNotFoundError:
            pass
    return t


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    return _newest(deps) > target.stat().st_mtime


def _cuda_headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "tvarant.h"]


def build_cuda_library(jobs: int | None = None, force: bool = False) -> Path:
    """Compiles the CUDA sources and links ``lib/libtvarant_cuda.so``."""
    obj_dir = BUILD / "cuda"
    obj_dir.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    headers = _cuda_headers()
    flags = [
        "-O3",
        "-std=c++17",
        "-lineinfo",
        *ARCH_FLAGS,
        "-Xcompiler",
        "-fPIC",
        "-Xcompiler",
        "-fvisibility=hidden",
        "-I",
        str(ROOT / "include"),
        "--expt-relaxed-constexpr",
    ]
    if os.environ.get("TVARANT_PTXAS_VERBOSE"):
        flags += ["-Xptxas", "-v"]

    def compile_one(name: str) -> Path:
        src = CSRC / name
        obj = obj_dir / (name + ".o")
        if force or _stale(obj, [src, *headers]):
            _run([NVCC, *flags, "-c", str(src), "-o", str(obj)])
        return obj

    with ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(compile_one, CUDA_SOURCES))
    if force or _stale(CUDA_LIB, objs):
        _run(
            [
                NVCC,
                "-shared",
                *ARCH_FLAGS,
                "-cudart=static",
                "-o",
                str(CUDA_LIB),
                *map(str, objs),
                "-lnvrtc",
                "-ldl",
                "-lpthread",
                "-lrt",
                "-L",
                str(CUDA_HOME / "lib64"),
                "-Xlinker",
                f"-rpath={CUDA_HOME / 'lib64'}",
            ]
        )
    return CUDA_LIB


def _torch_flags():
    import torch
    from torch.utils import cpp_extension

    includes = cpp_extension.include_paths()
    libdirs = cpp_extension.library_paths()
    py_inc = sysconfig.get_paths()["include"]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    return includes, libdirs, py_inc, abi


def build_extension(jobs: int | None = None, force: bool = False) -> Path:
    """Compiles the PyTorch extension ``_C.so`` (host C++ only)."""
    includes, libdirs, py_inc, abi = _torch_flags()
    obj_dir = BUILD / "ext"
    obj_dir.mkdir(parents=True, exist_ok=True)
    headers = sorted(EXT_SRC.glob("*.h")) + [ROOT / "include" / "tvarant.h"]
    # The system compiler links the shared libstdc++ that PyTorch and
    # libtvarant_cuda.so use; a toolchain that links a private static copy
    # would export a second libstdc++ from _C.so.
    cxx = os.environ.get("TVARANT_CXX") or ("/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++")
    flags = [
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-fvisibility=hidden",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-DTORCH_EXTENSION_NAME=_C",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        "-Wno-unused-parameter",
        "-I",
        str(ROOT / "include"),
        "-I",
        str(EXT_SRC),
        "-isystem",
        py_inc,
    ]
    for inc in includes:
        flags += ["-isystem", inc]

    def compile_one(name: str) -> Path:
        src = EXT_SRC / name
        obj = obj_dir / (name + ".o")
        if force or _stale(obj, [src, *headers]):
            _run([cxx, *flags, "-c", str(src), "-o", str(obj)])
        return obj

    with ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(compile_one, EXT_SOURCES))
    if force or _stale(EXT_LIB, [*objs, CUDA_LIB]):
        link = [cxx, "-shared", "-Wl,--exclude-libs,ALL", "-o", str(EXT_LIB), *map(str, objs)]
        for d in libdirs:
            link += ["-L", d, f"-Wl,-rpath,{d}"]
        link += [
            "-L",
            str(LIB_DIR),
            "-ltvarant_cuda",
            "-Wl,-rpath,$ORIGIN/lib",
            "-lc10",
            "-ltorch",
            "-ltorch_cpu",
            "-ltorch_python",
        ]
        _run(link)
    return EXT_LIB


def build(force: bool = False) -> None:
    """Builds everything: the CUDA library first, then the extension."""
    build_cuda_library(force=force)
    build_extension(force=force)


def clean() -> None:
    shutil.rmtree(BUILD, ignore_errors=True)
    for p in (CUDA_LIB, EXT_LIB):
        if p.exists():
            p.unlink()


if __name__ == "__main__":
    if "--clean" in sys.argv:
        clean()
    build(force="--force" in sys.argv)
