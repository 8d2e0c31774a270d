"""Build recipe for the CPU oracle (test infrastructure only).

Compiles oracle/kvoff_oracle.c with gcc into oracle/_build/libkvoff_oracle.so.
IEEE semantics matter: no -ffast-math, no FMA contraction. The reference
project is pure Python (torch), so there is no reference source to compile
into oracle/_ref; the reference itself pins this oracle through the golden
fixtures under tests/golden/.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
SOURCE = ORACLE_DIR / "kvoff_oracle.c"
LIBRARY = ORACLE_DIR / "_build" / "libkvoff_oracle.so"
# -mavx2 lets the fast port's loops vectorize (both the build container and the
# GPU hosts have AVX2); IEEE semantics are unaffected.
FLAGS = ["-O3", "-mavx2", "-fPIC", "-shared", "-fopenmp", "-fno-fast-math", "-ffp-contract=off",
         "-fvisibility=hidden", "-std=c11", "-lm"]


def build(force: bool = False) -> Path:
    if not force and LIBRARY.exists() and LIBRARY.stat().st_mtime >= max(
            SOURCE.stat().st_mtime, Path(__file__).stat().st_mtime):
        return LIBRARY
    LIBRARY.parent.mkdir(exist_ok=True)
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = ["gcc", str(SOURCE), "-o", str(tmp), *FLAGS]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{result.stderr}")
    tmp.replace(LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force=True))
