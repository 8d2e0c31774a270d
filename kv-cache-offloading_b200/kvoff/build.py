"""Build libkvoff.so (sm_100a) in-tree with nvcc.

The shared library is written next to this file so that it travels with the
source tree; nothing is installed into site-packages. The build is skipped
when the library is newer than every source and header.

    python -m kvoff.build [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
SOURCE_DIR = PACKAGE_DIR.parent / "csrc"
INCLUDE_DIR = PACKAGE_DIR.parents[1] / "include"
LIBRARY = PACKAGE_DIR / "libkvoff.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
# No --use_fast_math: the FP8 codec depends on IEEE division, multiplication
# and denormals (no flush-to-zero) to match the reference bit for bit.
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "-shared",
    "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3",
    "-ftz=false", "-prec-div=true", "-prec-sqrt=true", "-fmad=true",
]


def sources() -> list[Path]:
    return sorted([*SOURCE_DIR.glob("*.cu"), *SOURCE_DIR.glob("*.cpp")])


def _inputs() -> list[Path]:
    return [*sources(), *SOURCE_DIR.glob("*.h"), *SOURCE_DIR.glob("*.cuh"),
            *INCLUDE_DIR.glob("*.h"), Path(__file__)]


def up_to_date() -> bool:
    if not LIBRARY.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in _inputs())


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    default = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if default.exists():
        return str(default)
    raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every CUDA/C++ source of the extension into LIBRARY."""
    if not force and up_to_date():
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE_DIR}",
           *map(str, sources()), "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    if verbose:
        print(result.stderr, file=sys.stderr)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose))
