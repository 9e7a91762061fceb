"""Build the CUDA library in-tree: ``flash_uma_b200/lib/libflashuma_b200.so`` (sm_100a only).

    python -m flash_uma_b200.build [--verbose]      # -Xptxas -v register / spill report

The library is a plain shared object with a C ABI (``include/flash_uma_b200.h``);
Python loads it with ctypes. nvcc cross-compiles without a GPU.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
LIBNAME = "libflashuma_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def lib_path() -> str:
    return os.path.join(LIBDIR, LIBNAME)


def needs_build() -> bool:
    out = lib_path()
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    out = lib_path()
    if not force and not needs_build():
        return out
    os.makedirs(LIBDIR, exist_ok=True)
    tmp = out + ".tmp"
    # --no-undefined: a launcher declared but not defined fails the build instead of the first dlopen
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17",
           "-Xcompiler", "-fPIC", "-shared", "-Xlinker", "--no-undefined", "-I", os.path.join(ROOT, "include"),
           "-o", tmp, *sources()]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose:
        sys.stdout.write(res.stdout + res.stderr)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True))
