"""Builds ironmule_b200/libimspec.so from ironmule_b200/csrc/*.cu for sm_100a (in-tree, so the built
library travels with the source tree). Cross-compiles without a GPU.

    python -m ironmule_b200.build          # or: python ironmule_b200/build.py
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
LIB = HERE / "libimspec.so"
STAMP = HERE / ".libimspec.stamp"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _digest() -> str:
    h = hashlib.sha256()
    for path in sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h")):
        h.update(path.name.encode())
        h.update(path.read_bytes())
    h.update(" ".join(ARCH + FLAGS).encode())
    return h.hexdigest()


def up_to_date() -> bool:
    return LIB.exists() and STAMP.exists() and STAMP.read_text().strip() == _digest()


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    cmd = [NVCC, *ARCH, *FLAGS, f"-I{INCLUDE}", *map(str, sources()), "-o", str(LIB) + ".tmp"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    STAMP.write_text(_digest())
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
