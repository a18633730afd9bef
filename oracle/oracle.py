"""Python face of the CPU oracle (wf_oracle.c). TEST INFRASTRUCTURE ONLY: the checker for tests/, smoke() and the
CPU-baseline / reference arm of bench.py. The product package never imports this module.

build() compiles wf_oracle.c with gcc (OpenMP, no floating-point contraction) into oracle/_build/liboracle.so;
the functions below take numpy arrays and call it."""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "wf_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liboracle.so")

F16, BF16, F32 = 0, 1, 2
NP_OUT = {F16: np.uint16, BF16: np.uint16, F32: np.float32}  # bf16 / f16 returned as raw uint16 bits

_lib = None


def build(force=False):
    os.makedirs(OUT_DIR, exist_ok=True)
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", "-O2", "-march=x86-64-v3", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC", "-shared",
           "-fvisibility=hidden", "-o", LIB + ".tmp", SRC, "-lm"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB)
        vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.wfo_dequant_gguf.argtypes = [vp, i64, vp, i64, i32, i32, i32, vp, f32, i32]
        L.wfo_dequant_gguf.restype = i32
        L.wfo_lora_add.argtypes = [vp, vp, i64, i32, f32, i32]
        L.wfo_lora_add.restype = i32
        L.wfo_max_threads.argtypes = []
        L.wfo_max_threads.restype = i32
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def max_threads():
    return lib().wfo_max_threads()


def dequant_gguf(raw, n_values, qtype, mid, out, diff=None, sa=0.0, threads=0):
    """Packed bytes (uint8 array) -> flat output array (uint16 bits for f16 / bf16, float32 for f32)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    dst = np.empty(int(n_values), dtype=NP_OUT[out])
    d = None if diff is None else np.ascontiguousarray(diff, dtype=np.float32).reshape(-1)
    rc = lib().wfo_dequant_gguf(_ptr(raw), raw.size, _ptr(dst), int(n_values), int(qtype), int(mid), int(out),
                                _ptr(d), ctypes.c_float(sa), int(threads))
    if rc != 0:
        raise ValueError(f"oracle dequant rejected the input (status {rc})")
    return dst


def lora_add(diff, w, out, sa, threads=0):
    """In place on w (uint16 bits or float32): w = R(w + R(diff * sa))."""
    diff = np.ascontiguousarray(diff, dtype=np.float32).reshape(-1)
    assert w.flags.c_contiguous and w.size == diff.size
    rc = lib().wfo_lora_add(_ptr(diff), _ptr(w), diff.size, int(out), ctypes.c_float(sa), int(threads))
    if rc != 0:
        raise ValueError(f"oracle lora_add status {rc}")
    return w
