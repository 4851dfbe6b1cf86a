"""Compiles the CPU oracle (oracle/ossa_oracle.c) into oracle/_build/libossa_oracle.so.

Test infrastructure: only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg use the result.  Flags pin IEEE fp32 semantics: no fast-math, no
FMA contraction beyond the explicit fmaf() calls.
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
SRC = ORACLE_DIR / "ossa_oracle.c"
OUT_DIR = ORACLE_DIR / "_build"
LIB = OUT_DIR / "libossa_oracle.so"
CFLAGS = ["-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
          "-fno-fast-math", "-fexcess-precision=standard"]


def _arch_flags() -> list[str]:
    """Hardware FMA makes fmaf() one instruction; results are identical either way
    (fmaf is correctly rounded in software too), only faster."""
    try:
        flags = Path("/proc/cpuinfo").read_text()
    except OSError:
        return []
    return ["-mfma", "-mavx2"] if (" fma " in flags and " avx2 " in flags) else []


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("gcc is required to build the CPU oracle")
    OUT_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *CFLAGS, *_arch_flags(), str(SRC), "-o", str(tmp), "-lm"]
    res = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    if res.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + res.stdout.decode(errors="replace"))
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
