"""Builds libgollek_kernels.so (sm_100a) in-tree with nvcc.

    python -m gollek_b200.build            # build if sources changed
    python -m gollek_b200.build --force -v # rebuild, print ptxas register/spill report
"""
from __future__ import annotations

import argparse
import fcntl
import glob
import os
import shutil
import subprocess
import sys
import time

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB_DIR = os.path.join(PKG, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libgollek_kernels.so")
HEADER = os.path.join(ROOT, "include", "gollek_kernels.h")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))) + [HEADER]


def stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(s) > t for s in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    """Builds the library if its sources are newer (or `force`).  Safe to call from several
    processes at once (the ranks of one job): one builds under an exclusive file lock while
    the others wait, then find it fresh; the new file replaces the old one atomically."""
    if not force and not stale():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    with open(os.path.join(LIB_DIR, ".build.lock"), "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if not force and not stale():
            return LIB_PATH
        return _build_locked(verbose)


def _build_locked(verbose: bool) -> str:
    tmp = f"{LIB_PATH}.{os.getpid()}.tmp"
    # The output carries the build's start time, so a source edited while nvcc runs still
    # reads as newer than the library.
    start = time.time()
    cmd = [
        nvcc_path(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-shared",
        "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
        "--expt-relaxed-constexpr",
        "-I", os.path.join(ROOT, "include"),
        "-o", tmp, os.path.join(CSRC, "gollek_kernels.cu"),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    env = dict(os.environ)
    # nvcc's host compiler: prefer the system g++ (the environment's CXX may lack libgomp
    # or differ from what libstdc++ on the GPU box expects).
    if os.path.exists("/usr/bin/g++"):
        cmd[1:1] = ["-ccbin", "/usr/bin/g++"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    if r.returncode != 0:
        if os.path.exists(tmp):
            os.remove(tmp)
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libgollek_kernels.so")
    if verbose:
        sys.stderr.write(r.stderr)
    os.utime(tmp, (start, start))
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
