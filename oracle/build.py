"""Build recipe for the C oracle -- TEST INFRASTRUCTURE ONLY.

Compiles ``oracle/oracle_cpu.c`` with gcc and OpenMP into ``oracle/_build/liboracle_cpu.so``.
The reference (bayareahomelander/Onyx) contains no C/C++ for this path -- its native
code is two Rust crates and there is no Rust toolchain here -- so there is no
``oracle/_ref`` build; the oracle is the restatement in ``oracle_cpu.c``.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

_HERE = Path(__file__).resolve().parent


def build(verbose: bool = False) -> Path:
    out_dir = _HERE / "_build"
    out_dir.mkdir(exist_ok=True)
    out = out_dir / "liboracle_cpu.so"
    src = _HERE / "oracle_cpu.c"
    if out.exists() and out.stat().st_mtime >= src.stat().st_mtime:
        return out
    tmp = out.with_suffix(".so.tmp")
    cmd = [
        "gcc", "-O2", "-std=gnu11", "-fPIC", "-shared", "-fopenmp",
        "-fno-fast-math", "-ffp-contract=off",
        str(src), "-o", str(tmp), "-lm",
    ]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    tmp.replace(out)
    return out


if __name__ == "__main__":
    print(build(verbose=True))
