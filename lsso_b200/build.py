"""Build ``lsso_equilibrium_sm100.so`` in-tree with nvcc for sm_100a.

Usage: ``python -m lsso_b200.build [--force]``.  The library is a plain C-ABI
shared object (no libtorch): CUDA runtime linked statically, kernels compiled
for ``sm_100a`` only.  The result lands in ``lsso_b200/lib/`` so that it
travels with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
LIBDIR = PACKAGE / "lib"
LIBRARY_NAME = "lsso_equilibrium_sm100.so"
SOURCES = ("mixer.cu", "linear.cu", "tokens.cu", "solve.cu", "peer.cu", "capi.cu")
HEADERS = ("mixer.h", "mixer_common.cuh", "tc.cuh", "linear.h", "peer.h")
ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")


def library_path() -> Path:
    return LIBDIR / LIBRARY_NAME


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.is_file():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc was not found; set CUDA_HOME")
    return found


def _inputs() -> list[Path]:
    return [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [ROOT / "include" / "lsso_equilibrium.h"]


def is_stale() -> bool:
    target = library_path()
    if not target.is_file():
        return True
    built = target.stat().st_mtime
    return any(p.stat().st_mtime > built for p in _inputs())


LAST_BUILD = {"compiled": False, "seconds": 0.0}


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library unless it is up to date; return its path.

    ``LAST_BUILD["compiled"]`` says whether this call ran nvcc (False: the
    existing library was newer than every source and was reused).
    """
    import time

    target = library_path()
    LAST_BUILD.update(compiled=False, seconds=0.0)
    if not force and not is_stale():
        return target
    start = time.perf_counter()
    LIBDIR.mkdir(parents=True, exist_ok=True)
    tmp = target.with_suffix(".so.tmp")
    command = [
        _nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared", "-cudart", "static",
        "-I", str(ROOT / "include"), "-o", str(tmp),
        *[str(CSRC / s) for s in SOURCES],
    ]
    if verbose:
        print(" ".join(command))
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    os.replace(tmp, target)
    LAST_BUILD.update(compiled=True, seconds=time.perf_counter() - start)
    return target


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True)
    print(path)
