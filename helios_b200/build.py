"""Build libhelios_b200.so in-tree with nvcc for sm_100a.

    python -m helios_b200.build            # compile if sources are newer than the library
    python -m helios_b200.build --force    # always compile

The library lands in ``helios_b200/_lib/`` and is what ``helios_b200._native``
loads; it is built here (nvcc cross-compiles without a GPU) and travels with the
source tree to the GPU machine.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libhelios_b200.so"
MAIN = CSRC / "helios_b200.cu"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "--expt-relaxed-constexpr", "--extended-lambda",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-shared",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu*")) + [ROOT / "include" / "helios_b200.h"]


def stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    return any(src.stat().st_mtime > built for src in sources())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and not stale():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, *(extra or []), "-o", str(tmp), str(MAIN)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    args = sys.argv[1:]
    extra = [a for a in args if a not in ("--force", "-v")]
    print(build(force="--force" in args, verbose="-v" in args, extra=extra))
