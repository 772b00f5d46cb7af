"""Build the in-tree C-ABI library ``hsd_b200/libhsd_b200.so`` for sm_100a.

    python -m hsd_b200.build [--verbose]

Compiles every ``hsd_b200/csrc/*.cu`` with nvcc
(``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``) and links them
into one shared library with the CUDA runtime linked statically, so the
library loads next to PyTorch's own runtime without version coupling.  The
build is incremental: nothing is recompiled when the library is newer than
every source and header.
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
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libhsd_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the hsd_b200 library needs CUDA 12.8+")
    return cand


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _deps())


def build(verbose=False, force=False, jobs=None):
    if not force and up_to_date():
        return LIB
    nvcc = nvcc_path()
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                    "-I", INCLUDE, "-I", CSRC, "--expt-relaxed-constexpr"]
    if verbose:
        flags += ["-Xptxas", "-v"]
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        cmd = [nvcc, "-c", src, "-o", obj] + flags
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                            stderr=subprocess.STDOUT, text=True)))
    failed = False
    for cmd, p in procs:
        out, _ = p.communicate()
        if verbose or p.returncode:
            sys.stderr.write(out)
        if p.returncode:
            failed = True
            sys.stderr.write("FAILED: " + " ".join(cmd) + "\n")
    if failed:
        raise RuntimeError("nvcc failed building hsd_b200")
    tmp = LIB + ".tmp"
    link = [nvcc, "-shared", "-o", tmp] + objs + ARCH + ["-cudart", "static"]
    r = subprocess.run(link, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout)
        raise RuntimeError("nvcc link failed building hsd_b200")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force="--force" in sys.argv)
    print(LIB)
