"""Build libfa_b200.so in-tree with nvcc for sm_100a.

    python -m cs348k_fast_attention_grammar_b200.build [--force] [--verbose]

The library is a plain C-ABI shared object (no torch types in its
signatures), so it is compiled by nvcc directly rather than as a torch
extension.  It links the CUDA runtime statically and needs no libcuda at link
time (tensor maps are encoded through cudaGetDriverEntryPoint).
"""

from __future__ import annotations

import argparse
import fcntl
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_NAME = "libfa_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
SOURCES = ["common.cu", "attn_fwd.cu", "gemm.cu"]
HEADERS = ["sm100_ptx.cuh", "sm100_tmem_wide.cuh", "sm100_2sm.cuh", "fa_internal.h"]
PUBLIC_HEADER = os.path.join(os.path.dirname(PKG_DIR), "include", "fa_b200.h")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def _inputs():
    return ([os.path.join(CSRC, s) for s in SOURCES] +
            [os.path.join(CSRC, h) for h in HEADERS] + [PUBLIC_HEADER])


def is_stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(p) > t for p in _inputs() if os.path.exists(p))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if it is missing or older than its sources.

    Safe when several processes (the ranks of one job) call it at once: an
    exclusive lock on a file beside the library lets one of them compile, the
    others wait and then find the library fresh; each compile writes its own
    temporary file and renames it over the library atomically."""
    if not force and not is_stale():
        return LIB_PATH
    with open(LIB_PATH + ".lock", "a+") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            if not force and not is_stale():
                return LIB_PATH          # another process built it meanwhile
            tmp = f"{LIB_PATH}.{os.getpid()}.tmp"
            cmd = ([nvcc_path()] + ARCH_FLAGS + NVCC_FLAGS +
                   [os.path.join(CSRC, s) for s in SOURCES] + ["-o", tmp])
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
                print(" ".join(cmd), file=sys.stderr)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if verbose or r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode != 0:
                if os.path.exists(tmp):
                    os.unlink(tmp)
                raise RuntimeError(f"nvcc failed with exit code {r.returncode}")
            os.replace(tmp, LIB_PATH)
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
