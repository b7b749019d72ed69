"""Build recipe of libwlq_b200.so (sm_100a only), in-tree.

    python qwen_wlqfastshot_helen_beta_b200/build.py [--force] [--verbose]

(run as a script: importing the package loads the library built here).

Compiles every ``csrc/*.cu`` with nvcc for ``arch=compute_100a,code=sm_100a``
and ``csrc/*.cpp`` with g++, then links one shared library next to this file
with the CUDA runtime linked statically, so the library depends only on the
driver.  Objects go to ``_build/`` beside the sources; the build is
incremental on source / header modification times.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libwlq_b200.so")
INCLUDE = os.path.join(ROOT, "include")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                     "--expt-relaxed-constexpr", "-I", INCLUDE]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-I", INCLUDE, "-I", os.path.join(CUDA_HOME, "include")]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, verbose):
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if not _stale(obj, [src] + _headers()):
        return obj
    if src.endswith(".cu"):
        cmd = [NVCC] + NVCC_FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-c", src, "-o", obj]
    else:
        cmd = ["g++"] + CXX_FLAGS + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile and link libwlq_b200.so; returns its path."""
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    if force:
        for o in glob.glob(os.path.join(OBJ, "*.o")):
            os.remove(o)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if force or _stale(LIB, objs):
        # export the C ABI only (sources are compiled with hidden visibility;
        # the extern "C" entry points are marked visible in wlq_b200.h's users
        # through the version script below)
        vs = os.path.join(OBJ, "exports.map")
        with open(vs, "w") as f:
            f.write("{ global: wlq_*; local: *; };\n")
        cmd = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + \
            ["-Xlinker", f"--version-script={vs}", "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
