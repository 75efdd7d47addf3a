"""Build recipe for the oracle's C restatement (test infrastructure only).

    python -m oracle.build        # -> oracle/_build/libk3oracle.so

The reference project is Python + an MSL string compiled by MLX at run time; it has no
C/C++ sources, so there is nothing of the reference itself to compile into
``oracle/_ref``. Only this package's own restatement is built.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent


def build(force: bool = False) -> Path:
    out = HERE / "_build" / "libk3oracle.so"
    src = HERE / "matvec_ref.c"
    if out.exists() and not force and out.stat().st_mtime >= src.stat().st_mtime:
        return out
    out.parent.mkdir(exist_ok=True)
    tmp = out.with_suffix(f".so.tmp{os.getpid()}")
    # -ffp-contract=off: the fma calls are explicit (as in the MSL body); nothing else fuses.
    cmd = ["gcc", "-O3", "-march=x86-64-v2", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared",
           str(src), "-o", str(tmp), "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print(build(force=True))
