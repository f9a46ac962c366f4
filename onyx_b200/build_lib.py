"""Compile the sm_100a CUDA library ``libonyx_b200.so`` in-tree with nvcc.

The library is the product's only compute path; it is built here (cross-compiled, no GPU
needed) and loaded by :mod:`onyx_b200._lib` through its C ABI (``include/onyx_b200.h``).
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libonyx_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "onyx_b200.h"]
    return any(p.stat().st_mtime > mtime for p in deps)


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: cannot build libonyx_b200.so")
    return found


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and not _stale():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [
        nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-shared",
        "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
        "-I", str(ROOT / "include"),
        *(extra or []),
        *[str(s) for s in sources()],
        "-o", str(tmp),
    ]
    if verbose:
        print(" ".join(cmd))
    env = dict(os.environ)
    subprocess.run(cmd, check=True, env=env)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    import sys

    print(build(force="--force" in sys.argv, verbose=True,
                extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None))
