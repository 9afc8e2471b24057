"""Compile libtackmc.so (the sm_100a kernels and their C ABI) in-tree.

Run as ``python -m tack_b200._build [-v]``.  The library has no PyTorch
dependency: it is plain CUDA C++ with an ``extern "C"`` interface declared in
``include/tackmc.h``, built by nvcc for sm_100a only.
"""

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_PATH = os.path.join(PKG_DIR, "libtackmc.so")

SOURCES = ["tackmc.cu"]
HEADERS = ["mc_tables.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2",
    "-shared",
]


def nvcc_path():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _inputs():
    paths = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    paths.append(os.path.join(REPO_DIR, "include", "tackmc.h"))
    paths.append(os.path.abspath(__file__))
    return paths


def up_to_date():
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(p) <= t for p in _inputs())


def build(verbose=False, force=False, ptxas_info=False):
    """Compile libtackmc.so unless it is newer than all of its inputs."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    cmd += ["-I", os.path.join(REPO_DIR, "include"), "-I", CSRC]
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    cmd += ["-o", tmp]
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or proc.returncode != 0:
        sys.stdout.write(proc.stdout)
        sys.stderr.write(proc.stderr)
    if proc.returncode != 0:
        raise RuntimeError("nvcc failed building libtackmc.so")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    v = "-v" in sys.argv
    build(verbose=v, force=True, ptxas_info=v)
