"""Build recipe for the oracle libraries (test infrastructure only).

* ``oracle/liboracle.so`` — the C restatement in ``oracle/oracle.c``.
* ``oracle/_ref/libtvr_ref.so`` — the reference simulator's own kernels,
  compiled straight from the reference checkout's sources
  (``csrc/kernels/host/HostKernels.cpp`` and ``csrc/jit/Jit.cpp``) with the
  reference's own compiler flags (its setup.py uses ``-std=c++17 -fPIC -O3``),
  plus the C wrapper ``oracle/ref_capi.cpp`` and the ``TORCH_CHECK`` stand-in
  in ``oracle/shim``.  Only built where the reference checkout exists; the
  built file travels with the repository snapshot.

Usage: ``python oracle/build.py [--reference DIR]``.  Without ``--reference``
the checkout is ``$TVARANT_REFERENCE_DIR``, else ``../reference`` relative to
the repository root.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"
LIB = HERE / "liboracle.so"
REF_LIB = REF_OUT / "libtvr_ref.so"
# The reference checkout: $TVARANT_REFERENCE_DIR, else a directory named
# "reference" beside this repository's root.
DEFAULT_REFERENCE = Path(os.environ.get("TVARANT_REFERENCE_DIR",
                                        str(HERE.parent.parent / "reference")))


def _run(cmd):
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(map(str, cmd))}\n{proc.stdout}")


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps if Path(d).exists())


def build_oracle(force: bool = False) -> Path:
    src = HERE / "oracle.c"
    if force or _stale(LIB, [src]):
        _run(["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off",
              "-fvisibility=hidden", str(src), "-o", str(LIB), "-lm"])
    return LIB


def build_reference(reference: Path = DEFAULT_REFERENCE, force: bool = False) -> Path | None:
    csrc = reference / "csrc"
    sources = [csrc / "kernels" / "host" / "HostKernels.cpp", csrc / "jit" / "Jit.cpp"]
    if not all(s.exists() for s in sources):
        return REF_LIB if REF_LIB.exists() else None
    REF_OUT.mkdir(exist_ok=True)
    wrapper = HERE / "ref_capi.cpp"
    shim = HERE / "shim"
    deps = [*sources, wrapper, shim / "c10" / "util" / "Exception.h",
            csrc / "kernels" / "host" / "HostKernels.h", csrc / "jit" / "Jit.h"]
    if force or _stale(REF_LIB, deps):
        _run(["g++", "-std=c++17", "-fPIC", "-O3", "-Wno-unused-parameter", "-shared",
              "-I", str(shim), "-I", str(csrc), "-I", str(csrc / "kernels" / "host"),
              *map(str, sources), str(wrapper), "-o", str(REF_LIB)])
    return REF_LIB


def build(force: bool = False) -> None:
    build_oracle(force)
    ref = DEFAULT_REFERENCE
    if "--reference" in sys.argv:
        ref = Path(sys.argv[sys.argv.index("--reference") + 1])
    build_reference(ref, force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
