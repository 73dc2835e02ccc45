"""Build `libscunet_b200.so` in-tree with nvcc for sm_100a.

    python scunet-rs_b200/build.py [--force]

One translation unit (`csrc/scunet_b200.cu`) holds every kernel and the C ABI;
cudart is linked statically and the driver API is reached through
`cudaGetDriverEntryPoint`, so the library loads on a machine without a GPU driver
(the CPU test suite checks its exported symbols there).
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libscunet_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", "-ldl",
]


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [HERE.parent / "include" / "scunet_b200.h"]


def up_to_date():
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(s.stat().st_mtime <= t for s in sources())


def build(force=False, verbose=False):
    if not force and up_to_date():
        return LIB
    cmd = [NVCC, *FLAGS, "-o", str(LIB), str(CSRC / "scunet_b200.cu")]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
