"""Build the native library libkvr_b200.so in-tree with nvcc (sm_100a).

    python -m kvr_b200._build          # from rina-1bit-kv_b200/

Every .cu under ../csrc is compiled for ``-gencode arch=compute_100a,code=sm_100a``
and linked into kvr_b200/lib/libkvr_b200.so (C ABI, see include/kvr_b200.h).
Objects are rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)                      # rina-1bit-kv_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIBDIR = os.path.join(PKG, "lib")
OBJDIR = os.path.join(ROOT, "_build")
LIB = os.path.join(LIBDIR, "libkvr_b200.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _compile(src, verbose=False, objdir=None, extra=()):
    obj = os.path.join(objdir or OBJDIR, os.path.basename(src) + ".o")
    newest = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in _headers()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr)
    return obj


# variant -> (library file, extra nvcc flags).  "trace" compiles the
# %globaltimer phase stamps (KVR_TRACE_POINT) into every kernel, for latency
# studies only (phase_trace.py); the product library never has them.
VARIANTS = {"": (LIB, ()), "trace": (os.path.join(LIBDIR, "libkvr_b200_trace.so"), ("-DKVR_TRACE",))}


def build(verbose: bool = False, variant: str = "") -> str:
    lib_path, extra = VARIANTS[variant]
    objdir = OBJDIR if not variant else os.path.join(OBJDIR, variant)
    os.makedirs(objdir, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, objdir, extra), srcs))
    if not os.path.exists(lib_path) or os.path.getmtime(lib_path) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", lib_path, *objs, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return lib_path


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, variant="trace" if "--trace" in sys.argv else ""))
