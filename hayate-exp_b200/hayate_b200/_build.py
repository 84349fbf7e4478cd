"""Build ``libhayate_b200.so`` from ``csrc/`` with nvcc for sm_100a (in-tree).

``python -m hayate_b200._build`` (or ``__graft_entry__.build()``) compiles every
``csrc/*.cu`` into one shared library next to this file. No GPU is needed: nvcc
cross-compiles for ``sm_100a``. The build is skipped when the library is newer
than every source and header.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PACKAGE_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC_DIR = os.path.join(os.path.dirname(PACKAGE_DIR), "csrc")
REPO_ROOT = os.path.dirname(os.path.dirname(PACKAGE_DIR))
INCLUDE_DIR = os.path.join(REPO_ROOT, "include")
LIB_NAME = "libhayate_b200.so"
LIB_PATH = os.path.join(PACKAGE_DIR, LIB_NAME)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O2",
    "-shared",
]


def nvcc_path() -> str:
    for candidate in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and os.path.exists(candidate):
            return candidate
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build hayate_b200")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC_DIR, "*.cu")))


def _inputs() -> list[str]:
    return sources() + sorted(glob.glob(os.path.join(CSRC_DIR, "*.cuh"))) + sorted(
        glob.glob(os.path.join(INCLUDE_DIR, "*.h"))) + [os.path.abspath(__file__)]


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    built = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(path) <= built for path in _inputs())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compile the library if needed and return its path."""
    if not force and up_to_date():
        return LIB_PATH
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", INCLUDE_DIR, "-o", LIB_PATH + ".tmp", *sources()]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    if verbose or ptxas_info:
        print(proc.stderr, file=sys.stderr)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas-info" in sys.argv))
