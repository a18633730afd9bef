"""ctypes binding of the C-ABI library (include/weightferry_b200.h, built by csrc/build.py into _lib/).

There is no CPU fallback: a missing library raises ExtensionMissing, a rejected call raises WFError with the
library's status string. Every launch takes the caller's current CUDA stream, as the reference's kernels do
(enhancers/fused_int8.py:151 passes torch.cuda.current_stream(dev).cuda_stream)."""

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libweightferry_b200.so")

WF_F16, WF_BF16, WF_F32 = 0, 1, 2

_lock = threading.Lock()
_lib = None


class ExtensionMissing(RuntimeError):
    """The CUDA library is not built (run __graft_entry__.build() or comfyui-weightferry_b200/csrc/build.py)."""


class WFError(RuntimeError):
    def __init__(self, status, what):
        self.status = int(status)
        super().__init__(f"{what}: weightferry_b200 status {self.status} ({status_string(self.status)})")


class DequantTask(ctypes.Structure):
    _fields_ = [("src", ctypes.c_void_p), ("dst", ctypes.c_void_p), ("n_values", ctypes.c_int64)]


# (name, restype, argtypes) of every exported function; the CPU test checks the header declares exactly these
SIGNATURES = {
    "wf_version": (ctypes.c_int, []),
    "wf_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "wf_gguf_block_info": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    "wf_dequant_gguf": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "wf_dequant_gguf_batch": (ctypes.c_int, [ctypes.POINTER(DequantTask), ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int, ctypes.c_void_p]),
    "wf_dequant_gguf_lora": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                            ctypes.c_void_p]),
    "wf_lora_add": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float,
                                   ctypes.c_void_p]),
    "wf_modulate": (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 3 + [ctypes.c_void_p]),
    "wf_ln_modulate": (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 3 + [ctypes.c_float,
                                                                                      ctypes.c_void_p]),
    "wf_rms_norm_128": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                       ctypes.c_int64, ctypes.c_float, ctypes.c_void_p]),
    "wf_rms_rope128": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int64] * 4
                       + [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p] + [ctypes.c_int64] * 3
                       + [ctypes.c_float, ctypes.c_void_p]),
    "wf_rms_rope128_pair": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 4
                            + [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
                            + [ctypes.c_int64] * 3 + [ctypes.c_float, ctypes.c_void_p]),
    "wf_quant_rows": (ctypes.c_int, [ctypes.c_void_p] * 6 + [ctypes.c_int64] * 3
                      + [ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "wf_w8a8_gemm": (ctypes.c_int, [ctypes.c_void_p] * 6 + [ctypes.c_int64] * 3 + [ctypes.c_void_p]),
    "wf_w8a8_gemm_residual": (ctypes.c_int, [ctypes.c_void_p] * 6 + [ctypes.c_int64, ctypes.c_void_p]
                              + [ctypes.c_int64] * 3 + [ctypes.c_void_p]),
    "wf_w8a8_gemm_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "wf_w8a8_gemm_set_wait_limit": (ctypes.c_int, [ctypes.c_uint64]),
    "wf_gated_residual": (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 3 + [ctypes.c_void_p]),
    "wf_hbm_probe": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]),
    "wf_w8a8_linear_noalloc": (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 3 + [ctypes.c_void_p]),
}


def _load():
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ExtensionMissing(f"weightferry_b200 CUDA library not built: {LIB_PATH} is missing "
                                   "(run __graft_entry__.build())")
        try:
            import torch  # noqa: F401 -- loads the CUDA runtime the library links against (one runtime per process)
        except ImportError:
            pass
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def lib():
    """The loaded library (raises ExtensionMissing when it is not built)."""
    return _load()


def loaded():
    return _lib is not None


def status_string(status):
    try:
        s = _load().wf_status_string(int(status))
    except ExtensionMissing:
        return "library not loaded"
    return s.decode() if s else "?"


def check(status, what):
    if status != 0:
        raise WFError(status, what)


def stream_of(device):
    """cudaStream_t of the current PyTorch stream on `device` (a torch.device or an index), as an integer for
    ctypes. Read through PyTorch's raw accessor where it exists: the public current_stream() costs a few
    microseconds of Python per call, which a block's dozens of launches would pay each time."""
    import torch
    if isinstance(device, str):
        device = torch.device(device)
    idx = device.index if isinstance(device, torch.device) else device
    if idx is None:
        idx = torch.cuda.current_device()
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return raw(idx)
    return torch.cuda.current_stream(idx).cuda_stream


class _Same:
    """A no-op device guard (the tensor's device is already the current one)."""

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_SAME = _Same()


def on_device(device):
    """Context manager that makes `device` current for a launch: torch.cuda.device(device) when another device is
    current, else a shared no-op (the common case costs one device query)."""
    import torch
    if isinstance(device, str):
        device = torch.device(device)
    idx = device.index if isinstance(device, torch.device) else device
    if idx is None or idx == torch.cuda.current_device():
        return _SAME
    return torch.cuda.device(idx)


def dtype_code(dtype):
    import torch
    return {torch.float16: WF_F16, torch.bfloat16: WF_BF16, torch.float32: WF_F32}[dtype]
