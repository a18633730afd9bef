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
        L.wfo_modulate.argtypes = [vp, vp, vp, vp, i64, i64, i64, i32]
        L.wfo_modulate.restype = None
        L.wfo_ln_modulate.argtypes = [vp, vp, vp, vp, i64, i64, i64, f32, i32, i32]
        L.wfo_ln_modulate.restype = None
        L.wfo_rms_norm_128.argtypes = [vp, vp, vp, i64, f32, i32, i32]
        L.wfo_rms_norm_128.restype = None
        L.wfo_rms_rope128.argtypes = [vp, vp, vp, vp, i64, i64, i64, f32, i32, i32]
        L.wfo_rms_rope128.restype = None
        L.wfo_quant_rows.argtypes = [vp, vp, vp, vp, vp, vp, i64, i64, i64, f32, i32, i32, i32]
        L.wfo_quant_rows.restype = None
        L.wfo_max_threads.argtypes = []
        L.wfo_max_threads.restype = i32
        L.wfo_set_threads.argtypes = [i32]
        L.wfo_set_threads.restype = i32
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def max_threads():
    return lib().wfo_max_threads()


def set_threads(n):
    """OpenMP threads of the oracle's parallel loops on the calling thread; returns the count now in effect."""
    return lib().wfo_set_threads(int(n))


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


# ------------------------------------------------------------------------------------------------ fused block
# bf16 tensors are passed and returned as uint16 bit arrays

def _u16(a):
    return np.ascontiguousarray(a, dtype=np.uint16)


def modulate(x, s1, shift, rows_per_group, threads=0):
    x, s1, shift = _u16(x), _u16(s1), _u16(shift)
    d = x.shape[-1]
    out = np.empty_like(x)
    lib().wfo_modulate(_ptr(x), _ptr(s1), _ptr(shift), _ptr(out), x.size // d, d, int(rows_per_group), threads)
    return out


def ln_modulate(x, s1, shift, rows_per_group, eps, rstd_ulps=0, threads=0):
    x, s1, shift = _u16(x), _u16(s1), _u16(shift)
    k = x.shape[-1]
    out = np.empty_like(x)
    lib().wfo_ln_modulate(_ptr(x), _ptr(s1), _ptr(shift), _ptr(out), x.size // k, k, int(rows_per_group),
                          ctypes.c_float(eps), int(rstd_ulps), threads)
    return out


def rms_norm_128(x, w, eps, rstd_ulps=0, threads=0):
    x, w = _u16(x), _u16(w)
    out = np.empty_like(x)
    lib().wfo_rms_norm_128(_ptr(x), _ptr(w), _ptr(out), x.size // 128, ctypes.c_float(eps), int(rstd_ulps), threads)
    return out


def rms_rope128(x, freqs, w_f32, heads, tokens, eps, rstd_ulps=0, threads=0):
    """x (B, L, H, 128) bf16 bits; freqs float32 (1, L, 1, 64, 2, 2) contiguous; w as float32 values."""
    x = _u16(x)
    f = np.ascontiguousarray(freqs, dtype=np.float32)
    w = np.ascontiguousarray(w_f32, dtype=np.float32)
    out = np.empty_like(x)
    lib().wfo_rms_rope128(_ptr(x), _ptr(f), _ptr(w), _ptr(out), x.size // 128, int(heads), int(tokens),
                          ctypes.c_float(eps), int(rstd_ulps), threads)
    return out


def quant_rows(x, s1=None, shift=None, gelu=None, rows_per_group=1, eps=0.0, pre=0, rotate=True, threads=0):
    """(int8 [rows, K], float32 scales [rows])."""
    x = _u16(x)
    k = x.shape[-1]
    rows = x.size // k
    q = np.empty((rows, k), dtype=np.int8)
    sc = np.empty(rows, dtype=np.float32)
    s1 = _u16(s1) if s1 is not None else None
    shift = _u16(shift) if shift is not None else None
    gelu = _u16(gelu) if gelu is not None else None
    lib().wfo_quant_rows(_ptr(x), _ptr(s1), _ptr(shift), _ptr(gelu), _ptr(q), _ptr(sc), rows, k,
                         int(rows_per_group), ctypes.c_float(eps), int(pre), int(bool(rotate)), threads)
    return q, sc


def rows_match_some_rstd(got, fn, width, max_ulps=2):
    """True per row when `got` equals fn(rstd_ulps=k) bit for bit on that row for some |k| <= max_ulps: the row
    computed with a reciprocal square root within max_ulps of the correctly rounded one (the hardware approximation's
    bound). fn(k) returns the oracle output for shift k."""
    got = np.asarray(got).reshape(-1, width)
    ok = np.zeros(got.shape[0], dtype=bool)
    for k in [0] + [s * m for m in range(1, max_ulps + 1) for s in (1, -1)]:
        ref = np.asarray(fn(k)).reshape(-1, width)
        ok |= np.all(got == ref, axis=1)
        if ok.all():
            break
    return ok
