"""Builds ``libkda_b200.so`` (the C ABI of ``include/kda_b200.h``) in-tree.

``python -m sophia_b200.build`` compiles every CUDA source of the package for
sm_100a with nvcc directly; the shared library lands next to this file so it
travels with the source tree.  No torch types cross the ABI, so the library
does not link against libtorch.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libkda_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the KDA CUDA library cannot be built")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def build(verbose: bool = False, force: bool = False) -> Path:
    srcs = sources()
    deps = srcs + sorted(CSRC.glob("*.cuh")) + [PKG.parent / "include" / "kda_b200.h"]
    if LIB.exists() and not force:
        newest = max(p.stat().st_mtime for p in deps)
        if LIB.stat().st_mtime >= newest:
            return LIB
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17",
           "-Xcompiler", "-fPIC", "-shared", "-o", str(LIB) + ".tmp",
           *[str(s) for s in srcs]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
