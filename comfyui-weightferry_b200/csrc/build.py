"""Build the C-ABI library of the B200 kernels (libweightferry_b200.so) in-tree.

Every .cu file of this folder is compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``) and linked
into one shared library with the CUDA runtime linked dynamically, so that the process shares one runtime (and one
stream namespace) with PyTorch. Objects go to ``csrc/_build/``, the library to ``<package>/_lib/``. A file is
recompiled only when it, or a header, is newer than its object.

    python comfyui-weightferry_b200/csrc/build.py [--force] [-j N]
"""

import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
INCLUDE = os.path.join(REPO, "include")
OBJ_DIR = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(PKG, "_lib")
LIB_NAME = "libweightferry_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc():
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the B200 kernels need the CUDA toolkit to build")
    return cand


def _cuda_home(nvcc):
    return os.path.dirname(os.path.dirname(os.path.realpath(nvcc)))


def _cflags():
    return ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                   "-I", INCLUDE, "-I", HERE, "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _headers():
    return glob.glob(os.path.join(HERE, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(src, obj, newest_header):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or newest_header > t


def build(force=False, jobs=None, verbose=False):
    """Compile the library if needed; returns its path."""
    nvcc = _nvcc()
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(HERE, "*.cu")))
    hdrs = _headers()
    newest_header = max((os.path.getmtime(h) for h in hdrs), default=0.0)
    objs, todo = [], []
    for src in sources:
        obj = os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(src, obj, newest_header):
            todo.append((src, obj))

    def compile_one(pair):
        src, obj = pair
        cmd = [nvcc, "-c", src, "-o", obj] + _cflags()
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{res.stdout}\n{res.stderr}")
        return res.stderr

    if todo:
        with ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            for msg in ex.map(compile_one, todo):
                if msg and verbose:
                    print(msg, file=sys.stderr)
    lib = os.path.join(LIB_DIR, LIB_NAME)
    if todo or not os.path.exists(lib) or any(os.path.getmtime(o) > os.path.getmtime(lib) for o in objs):
        cuda_lib = os.path.join(_cuda_home(nvcc), "lib64")
        cmd = [nvcc, "-shared", "-o", lib + ".tmp"] + objs + ARCH + [
            "-cudart", "shared", "-Xlinker", f"-rpath={cuda_lib}"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(lib + ".tmp", lib)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.v))
