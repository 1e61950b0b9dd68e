"""Build libfaquant_b200.so in-tree with nvcc for sm_100a.

``python faquant-public_b200/build.py`` (or ``__graft_entry__.build()``) compiles
``csrc/faquant_b200.cu`` -- the single translation unit that includes every
kernel -- into ``faquant_b200/libfaquant_b200.so`` next to the Python package that
loads it. nvcc cross-compiles without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "faquant_b200" / "libfaquant_b200.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [
        HERE.parent / "include" / "faquant_b200.h"
    ]


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    built = OUT.stat().st_mtime
    return all(src.stat().st_mtime <= built for src in sources())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    cmd = [
        nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC,-O3", "-shared", "-o", str(OUT) + ".tmp", str(CSRC / "faquant_b200.cu"),
    ]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, cwd=str(CSRC), capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    if verbose or ptxas_info:
        print(proc.stdout, proc.stderr, sep="\n", flush=True)
    os.replace(str(OUT) + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas-info" in sys.argv)
