"""Build the sm_100a shared library ``libpe_b200.so`` in-tree with nvcc.

    python -m packed_encoders_b200.build        # or packed_encoders_b200.build.build()

The library is a plain C-ABI shared object (include/pe_b200_attn.h); CUDA runtime is linked
statically so the .so only needs the NVIDIA driver at run time.
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
LIB = PKG / "libpe_b200.so"
SOURCES = [CSRC / "attn_fwd.cu", CSRC / "noalloc.cu"]
HEADERS = [ROOT / "include" / "pe_b200_attn.h", *sorted(CSRC.glob("*.cuh"))]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O2,-Wall",
    "-Xptxas", "-warn-spills",
    "-shared",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    built = LIB.stat().st_mtime
    return all(src.stat().st_mtime <= built for src in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"), *map(str, SOURCES), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
