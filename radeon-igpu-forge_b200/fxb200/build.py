"""Ahead-of-time build of libfxb200.so (sm_100a) from csrc/*.cu.

The reference compiles its HIP sources at run time with hiprtc
(ml/fxgpu/hip_kernel.py:50-131); this build compiles every CUDA source once,
in parallel, with nvcc for sm_100a and links one shared library with a plain C
ABI (include/fxb200.h). cudart is linked statically and the driver API is
reached through cudaGetDriverEntryPoint, so the library loads on a machine
without libcuda (symbol checks on CPU) and runs wherever the driver is present.

    python -m fxb200.build          # from radeon-igpu-forge_b200/
"""
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(PKG_ROOT, "csrc")
LIB_DIR = os.path.join(PKG_ROOT, "lib")
OBJ_DIR = os.path.join(LIB_DIR, "obj")
LIB_PATH = os.path.join(LIB_DIR, "libfxb200.so")
REPO_ROOT = os.path.dirname(PKG_ROOT)
INCLUDE = os.path.join(REPO_ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
         "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC]


def _nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found (CUDA toolkit required to build libfxb200)")
    return exe


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime():
    ts = [os.path.getmtime(os.path.join(CSRC, f)) for f in os.listdir(CSRC)
          if f.endswith((".cuh", ".h"))]
    ts.append(os.path.getmtime(os.path.join(INCLUDE, "fxb200.h")))
    return max(ts)


def _compile(src, verbose=False):
    obj = os.path.join(OBJ_DIR, src[:-3] + ".o")
    cmd = [_nvcc()] + ARCH + FLAGS + ["-c", os.path.join(CSRC, src), "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force=False, verbose=False, jobs=None):
    """Compile stale objects and relink; returns the library path."""
    os.makedirs(OBJ_DIR, exist_ok=True)
    hdr = _headers_mtime()
    todo, objs = [], []
    for src in _sources():
        obj = os.path.join(OBJ_DIR, src[:-3] + ".o")
        objs.append(obj)
        stale = (force or not os.path.exists(obj)
                 or os.path.getmtime(obj) < max(hdr, os.path.getmtime(os.path.join(CSRC, src))))
        if stale:
            todo.append(src)
    if todo:
        n = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=n) as ex:
            for obj, log in ex.map(lambda s: _compile(s, verbose), todo):
                if verbose and log:
                    sys.stderr.write(log)
    if todo or not os.path.exists(LIB_PATH):
        tmp = LIB_PATH + ".tmp"
        cmd = [_nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(p)
