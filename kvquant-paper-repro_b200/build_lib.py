"""Builds the kvquant_b200 C-ABI shared library for sm_100a (in-tree).

Output: kvquant/_lib/libkvquant_b200.so next to the Python package that loads
it. The library is one translation unit (csrc/kvq_lib.cu); it is compiled
without --use_fast_math because the quantize kernels must reproduce the
reference's IEEE fp32 normalization bit for bit.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "csrc" / "kvq_lib.cu"
OUT = HERE / "kvquant" / "_lib" / "libkvquant_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    return sorted((HERE / "csrc").glob("*.cu*")) + sorted((HERE.parent / "include").glob("*.h"))


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    nvcc = os.environ.get("NVCC", "nvcc")
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
           "-shared", "-o", str(tmp), str(SRC)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
