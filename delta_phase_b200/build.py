"""Build the deltaphase_b200 CUDA library in-tree for sm_100a.

    python -m delta_phase_b200.build          # -> delta_phase_b200/lib/libdeltaphase_b200.so

Each ``csrc/*.cu`` file is compiled by nvcc in parallel and linked into one shared
library with a plain C ABI (``include/deltaphase_b200.h``).  No torch headers are
used: the library depends only on the CUDA runtime.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
OBJDIR = os.path.join(ROOT, "_build", "obj")
LIBNAME = "libdeltaphase_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "-I" + os.path.join(ROOT, "include")]


def nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build deltaphase_b200")
    return exe


def lib_path():
    return os.path.join(LIBDIR, LIBNAME)


def _compile(src, extra):
    obj = os.path.join(OBJDIR, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(verbose=False, extra=()):
    """Compile every csrc/*.cu and link the shared library.  Returns its path."""
    os.makedirs(OBJDIR, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, list(extra)), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log.strip():
                print(log, file=sys.stderr)
    out = lib_path()
    tmp = out + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "shared", *objs, "-o", tmp,
           "-Xlinker", "-rpath,/usr/local/cuda/lib64"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    v = "-v" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas" in sys.argv else []
    print(build(verbose=v or bool(extra), extra=extra))
