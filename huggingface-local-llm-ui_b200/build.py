"""Build libb2q.so (CUDA for sm_100a) in-tree with nvcc.

The library is a single translation unit (csrc/b2q_api.cu includes the
kernels and the model code) exposing the C ABI of include/b2q.h.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libb2q.so"
LIB_CHECKS = HERE / "libb2q_checks.so"
INCLUDE = HERE.parent / "include"

NVCC_FLAGS = [
    "-O3", "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
    "-shared",
]


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
                  + list(INCLUDE.glob("*.h")))


def lib_path(checks: bool = False) -> Path:
    """libb2q.so, or libb2q_checks.so: the debug-bounds build (-DB2Q_CHECKS,
    the kernels' index and layout checks compiled in; loaded when the
    environment sets B2Q_CHECKS=1)."""
    return LIB_CHECKS if checks else LIB


def up_to_date(checks: bool = False) -> bool:
    lib = lib_path(checks)
    if not lib.exists():
        return False
    t = lib.stat().st_mtime
    return all(s.stat().st_mtime <= t for s in sources())


def build(force: bool = False, verbose: bool = False, checks: bool = False) -> Path:
    """Compile libb2q.so (or, with `checks`, libb2q_checks.so) if a source is
    newer than it.  Safe when several processes (tensor-parallel ranks) call
    it at once: they serialise on a lock file, the first one compiles, the
    others find it up to date."""
    lib = lib_path(checks)
    if not force and up_to_date(checks):
        return lib
    import fcntl
    with open(lib.with_suffix(".so.lock"), "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            if not force and up_to_date(checks):
                return lib
            nvcc = os.environ.get("NVCC", "nvcc")
            tmp = lib.with_suffix(f".so.tmp{os.getpid()}")
            cmd = [nvcc, *NVCC_FLAGS, *(["-DB2Q_CHECKS"] if checks else []), "-o", str(tmp),
                   str(CSRC / "b2q_api.cu"), "-ldl"]
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
            os.replace(tmp, lib)
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, checks="--checks" in sys.argv))
