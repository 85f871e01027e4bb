"""Build the sm_100a kernel library in-tree: pdum_dsl_b200/libpdb_sm100.so.

One nvcc invocation over ``csrc/*.cu`` with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``; the CUDA runtime
is linked statically so the library does not depend on which libcudart the
host process (e.g. torch) loaded.  The TMA encoder is reached through the
driver entry-point API, so there is no link-time dependency on libcuda.
Usage: ``python -m pdum_dsl_b200.build [--force] [--verbose]``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
LIB = PKG / "libpdb_sm100.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the sm_100a kernel library cannot be built")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-I", str(INCLUDE), "-I", str(CSRC), "-o", str(tmp), *map(str, sources())]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    jobs = str(min(8, os.cpu_count() or 1))
    cmd[1:1] = ["--threads", jobs]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
