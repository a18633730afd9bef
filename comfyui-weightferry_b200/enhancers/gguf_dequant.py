"""GGUF dequantisation on B200 through the C-ABI kernels (drop-in for enhancers/gguf_dequant.py of ComfyUI-WeightFerry).

The same entry points as the reference, with the same arguments, defaults and "not this case" answers:

* ``dequantize(data, qtype, oshape, mid_dtype, out_dtype)`` (reference :296-326): ComfyUI-GGUF's
  ``dequantize(data, qtype, oshape, dtype=mid_dtype).to(out_dtype)`` for the legacy formats Q4_0 / Q4_1 / Q5_0 /
  Q5_1 / Q8_0 and (WEIGHTFERRY_GGUF_KQUANTS) the K-quants Q2_K .. Q6_K; mid defaults to float16, out to mid. Returns
  a new tensor, or None when this is not that case (another format, CPU data, a dtype outside float16 / bfloat16 /
  float32, bytes that do not match the shape) -- the caller then runs ComfyUI-GGUF's own code, as with the
  reference.
* ``dequantize_lora`` / ``lora_factors`` (:329-406): the dequantisation with plain LoRA patches added by one kernel
  each (w = R_out(w + R_out(diff * (strength * alpha)))), the difference by comfy's own torch.mm in float32.
* ``install(force=False)`` / ``uninstall()`` / ``stats(reset=False)`` (:544-583) patch ComfyUI-GGUF's
  ``ops.dequantize_tensor`` and ``GGMLLayer.get_weight``; the ``_weightferry`` marker keeps install idempotent.

The kernels (csrc/gguf_dequant.cu) reproduce every rounding of the reference's Triton kernels; there is no Triton
and no CPU path here: when the CUDA library is missing, a CUDA tensor raises ExtensionMissing instead of silently
running other code.
"""

import ctypes
import sys
import weakref

import torch

from .. import _ext

# GGML quant type id -> name, bytes per 32-value block, has a minimum m, qh offset (-1: none), quants offset, value
# subtracted from the quant, int8 quants (the reference's interface table, enhancers/gguf_dequant.py:52-54)
_FORMATS = {2: ("Q4_0", 18, False, -1, 2, 8, False), 3: ("Q4_1", 20, True, -1, 4, 0, False),
            6: ("Q5_0", 22, False, 2, 6, 16, False), 7: ("Q5_1", 24, True, 4, 8, 0, False),
            8: ("Q8_0", 34, False, -1, 2, 0, True)}
# K-quants: GGML type id -> name, bytes per block of 256 values (:56)
_KFORMATS = {10: ("Q2_K", 84), 11: ("Q3_K", 110), 12: ("Q4_K", 144), 13: ("Q5_K", 176), 14: ("Q6_K", 210)}
_KQUANTS = None  # None = WEIGHTFERRY_GGUF_KQUANTS; True / False pin it (benchmarks, tests)
_DT = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}
_state = {"orig": None, "ops": None, "orig_gw": None, "stats": {"used": 0, "fallback": 0}}
_LORA = True      # LoRA patches inside the dequantisation too (GGMLLayer.get_weight)
_FACTORS = None   # "pin" / "0"; None = WEIGHTFERRY_GGUF_LORA_FACTORS
_factors = {}     # pinned LoRA factors: id(factor) -> (weakref, key, pinned copy)
_cache = {"pin_freed": False}


def _env_get(name):
    from ..core import env as _env
    return _env.get(name)


def _kquants():
    if _KQUANTS is not None:
        return _KQUANTS
    return _env_get("WEIGHTFERRY_GGUF_KQUANTS") == "1"


def _supported(qtype):
    """Whether this GGML type is dequantised here: the legacy formats; the K-quants with WEIGHTFERRY_GGUF_KQUANTS."""
    q = int(qtype)
    return q in _FORMATS or (q in _KFORMATS and _kquants())


def _raw_bytes(data):
    """data viewed as its flat packed bytes (uint8), or None when it is not contiguous."""
    if not data.is_contiguous():
        return None
    return data.reshape(-1).view(torch.uint8)


def _launch(raw, res, n, qtype, mid, out):
    """One wf_dequant_gguf launch on the current stream of raw's device."""
    lib = _ext.lib()
    with torch.cuda.device(raw.device):
        rc = lib.wf_dequant_gguf(raw.data_ptr(), raw.numel(), res.data_ptr(), n, int(qtype), _DT[mid], _DT[out],
                                 _ext.stream_of(raw.device))
    _ext.check(rc, "wf_dequant_gguf")


def _dequantize_k(data, qtype, oshape, mid, out):
    """dequantize() for a K-quant (_KFORMATS), or None when the data does not match the shape (reference :277-293)."""
    q = int(qtype)
    raw = _raw_bytes(data)
    ts = _KFORMATS[q][1]
    if raw is None or raw.numel() % ts:
        return None
    n = raw.numel() // ts * 256
    if n != int(torch.Size(oshape).numel()):
        return None
    res = torch.empty(tuple(oshape), dtype=out, device=data.device)
    _launch(raw, res, n, q, mid, out)
    return res


def dequantize(data, qtype, oshape, mid_dtype, out_dtype):
    """ComfyUI-GGUF's dequantize(data, qtype, oshape, dtype=mid_dtype).to(out_dtype) for a legacy format (or a K-quant
    with WEIGHTFERRY_GGUF_KQUANTS), or None when this is not that case (other formats, CPU data, dtypes)."""
    if qtype is not None and int(qtype) in _KFORMATS:
        if not _kquants() or not data.is_cuda:
            return None
        mid = mid_dtype if mid_dtype is not None else torch.float16
        out = out_dtype if out_dtype is not None else mid
        if mid not in _DT or out not in _DT:
            return None
        return _dequantize_k(data, qtype, oshape, mid, out)
    fmt = _FORMATS.get(int(qtype)) if qtype is not None else None
    if fmt is None or not data.is_cuda:
        return None
    mid = mid_dtype if mid_dtype is not None else torch.float16
    out = out_dtype if out_dtype is not None else mid
    if mid not in _DT or out not in _DT:
        return None
    ts = fmt[1]
    raw = _raw_bytes(data)
    if raw is None or raw.numel() % ts:
        return None
    n_blocks = raw.numel() // ts
    if n_blocks * 32 != int(torch.Size(oshape).numel()):
        return None
    res = torch.empty(tuple(oshape), dtype=out, device=data.device)
    _launch(raw, res, n_blocks * 32, int(qtype), mid, out)
    return res


def dequantize_many(items, qtype, mid_dtype=None, out_dtype=None):
    """Dequantise a list of (packed CUDA tensor, oshape) of one GGML type in one batched launch (the checkpoint-wide
    sweep; same bits as dequantize() on each). Returns the list of outputs. All tensors on one device."""
    if not items:
        return []
    q = int(qtype)
    if q not in _FORMATS and q not in _KFORMATS:
        raise ValueError(f"GGML type {q} is not dequantised here")
    mid = mid_dtype if mid_dtype is not None else torch.float16
    out = out_dtype if out_dtype is not None else mid
    dev = items[0][0].device
    tasks = (_ext.DequantTask * len(items))()
    outs = []
    for i, (data, oshape) in enumerate(items):
        raw = _raw_bytes(data)
        if raw is None or raw.device != dev:
            raise ValueError("dequantize_many: every tensor must be contiguous and on one device")
        res = torch.empty(tuple(oshape), dtype=out, device=dev)
        tasks[i].src, tasks[i].dst, tasks[i].n_values = raw.data_ptr(), res.data_ptr(), res.numel()
        outs.append(res)
    with torch.cuda.device(dev):
        rc = _ext.lib().wf_dequant_gguf_batch(tasks, len(items), q, _DT[mid], _DT[out], _ext.stream_of(dev))
    _ext.check(rc, "wf_dequant_gguf_batch")
    return outs


# --------------------------------------------------------------------------------------------------------------- LoRA
def lora_factors(patch_list, n_out, n_in):
    """[(up, down, strength * alpha)] when every patch is a plain LoRA that comfy.lora.calculate_weight applies as
    weight += ((strength * alpha) * (up @ down)).type(weight.dtype) on a 2-D weight, else None (reference :329-355:
    no DoRA, mid weight, reshape, offset, function or strength_model; alpha / rank when alpha is given)."""
    out = []
    for p in patch_list:
        if not isinstance(p, tuple) or len(p) != 5:
            return None
        strength, v, strength_model, offset, function = p
        if strength_model != 1.0 or offset is not None or function is not None or type(v).__name__ != "LoRAAdapter":
            return None
        w = getattr(v, "weights", None)
        if not isinstance(w, (tuple, list)) or len(w) < 6 or any(x is not None for x in w[3:6]):
            return None
        up, down, alpha_raw = w[0], w[1], w[2]
        if (not torch.is_tensor(up) or not torch.is_tensor(down) or up.dim() != 2 or down.dim() != 2
                or up.shape[0] != n_out or down.shape[1] != n_in or up.shape[1] != down.shape[0]
                or not isinstance(strength, (int, float)) or isinstance(strength, bool)):
            return None
        if alpha_raw is None:
            alpha = 1.0
        elif isinstance(alpha_raw, (int, float)) and not isinstance(alpha_raw, bool):
            alpha = alpha_raw / down.shape[0]
        else:
            return None
        out.append((up, down, strength * alpha))
    return out


def dequantize_lora(data, qtype, oshape, mid_dtype, out_dtype, loras):
    """ComfyUI-GGUF's get_weight with plain LoRA patches (reference :358-384): dequantise, then add each LoRA's
    difference as comfy.lora.calculate_weight adds it -- the difference by the same torch.mm in float32 (its bits are
    cuBLAS's), the dequantisation and the first LoRA's scale / cast / add in one kernel, each further LoRA in one
    more. None when not that case."""
    if not data.is_cuda or len(oshape) != 2 or not loras or qtype is None:
        return None
    mid = mid_dtype if mid_dtype is not None else torch.float16
    if mid not in _DT or out_dtype not in _DT:
        return None
    q = int(qtype)
    if q in _KFORMATS:
        if not _kquants():
            return None
        ts = _KFORMATS[q][1]
        vpb = 256
    elif q in _FORMATS:
        ts = _FORMATS[q][1]
        vpb = 32
    else:
        return None
    n_out, n_in = int(oshape[0]), int(oshape[1])
    if q in _FORMATS and n_in % 32:
        return None
    raw = _raw_bytes(data)
    n = n_out * n_in
    if raw is None or n % vpb or raw.numel() != n // vpb * ts:
        return None
    res = torch.empty((n_out, n_in), dtype=out_dtype, device=data.device)
    return _add_loras(raw, res, loras, q, mid)


def _add_loras(raw, res, loras, qtype, mid):
    """res = dequant(raw) + each LoRA's difference (the first inside the dequantisation pass, the rest in place)."""
    dev = res.device
    lib = _ext.lib()
    mode = _factor_mode()
    n = res.numel()
    with torch.cuda.device(dev):
        for i, (up, down, sa) in enumerate(loras):
            mat1 = _factor(up, dev, mode)  # comfy's cast_to_device(v[0], device, float32)
            mat2 = _factor(down, dev, mode)
            diff = torch.mm(mat1.flatten(start_dim=1), mat2.flatten(start_dim=1)).contiguous()
            del mat1, mat2
            stream = _ext.stream_of(dev)
            if i == 0:
                rc = lib.wf_dequant_gguf_lora(raw.data_ptr(), raw.numel(), diff.data_ptr(), res.data_ptr(), n, qtype,
                                              _DT[mid], _DT[res.dtype], ctypes.c_float(float(sa)), stream)
                _ext.check(rc, "wf_dequant_gguf_lora")
            else:
                rc = lib.wf_lora_add(diff.data_ptr(), res.data_ptr(), n, _DT[res.dtype], ctypes.c_float(float(sa)),
                                     stream)
                _ext.check(rc, "wf_lora_add")
            del diff
    return res


def _factor_mode():
    if _FACTORS is not None:
        return _FACTORS
    mode = (_env_get("WEIGHTFERRY_GGUF_LORA_FACTORS") or "pin").strip().lower()
    try:  # ComfyUI with pinned memory disabled: no pinned copies here either
        import comfy.model_management as _mm
        from comfy.cli_args import args
        if getattr(_mm, "DISABLE_PINNED_MEMORY", False) or getattr(args, "disable_pinned_memory", False):
            return "0"
    except Exception:  # noqa: BLE001 -- outside ComfyUI
        pass
    return mode if mode == "pin" else "0"


def _version(t):
    try:
        return t._version
    except RuntimeError:  # inference tensors keep no version counter
        return None


def _pin_dropped(i):
    if _factors.pop(i, None) is not None:
        _cache["pin_freed"] = True


def _factor(t, dev, mode):
    """t.to(dev, float32) as comfy casts a LoRA factor. mode "pin": a pinned copy made once per factor (kept while
    the factor lives and its storage / version are unchanged) so the upload does not wait for the GPU queue to drain
    (reference :426-446)."""
    if mode == "0" or t.device.type != "cpu":
        return t.to(dev, torch.float32)
    key = (t.data_ptr(), _version(t), str(dev))
    hit = _factors.get(id(t))
    if hit is not None and hit[0]() is t and hit[1] == key:
        held = hit[2]
    else:
        held = t.pin_memory()
        _factors[id(t)] = (weakref.ref(t, lambda _r, i=id(t): _pin_dropped(i)), key, held)
    return held.to(dev, non_blocking=True).to(torch.float32)


# ------------------------------------------------------------------------------------------------------------ install
def _patched(orig):
    def dequantize_tensor(tensor, dtype=None, dequant_dtype=None):
        qtype = getattr(tensor, "tensor_type", None)
        if qtype is not None and _supported(qtype) and isinstance(tensor, torch.Tensor):
            mid = dtype if dequant_dtype == "target" else dequant_dtype
            if mid is None or isinstance(mid, torch.dtype):
                oshape = getattr(tensor, "tensor_shape", tensor.shape)
                out = dequantize(tensor.data, qtype, oshape, mid, dtype)
                if out is not None:
                    _state["stats"]["used"] += 1
                    return out
        _state["stats"]["fallback"] += 1
        return orig(tensor, dtype, dequant_dtype)
    dequantize_tensor._weightferry = True
    return dequantize_tensor


def _patched_get_weight(orig):
    def get_weight(self, tensor, dtype):
        if tensor is None:
            return None
        pats = getattr(tensor, "patches", None)
        qtype = getattr(tensor, "tensor_type", None)
        if (pats and getattr(self, "patch_dtype", None) is None and qtype is not None and _supported(qtype)
                and isinstance(dtype, torch.dtype) and getattr(tensor, "is_cuda", False)):
            mid = dtype if self.dequant_dtype == "target" else self.dequant_dtype
            if mid is None or isinstance(mid, torch.dtype):
                oshape = getattr(tensor, "tensor_shape", tensor.shape)
                patch_list = []
                for patches, _key in pats:
                    patch_list += list(patches)
                loras = lora_factors(patch_list, *oshape) if len(oshape) == 2 else None
                if loras:
                    out = dequantize_lora(tensor.data, qtype, oshape, mid, dtype, loras)
                    if out is not None:
                        _state["stats"]["lora_used"] = _state["stats"].get("lora_used", 0) + 1
                        return out
                _state["stats"]["lora_fallback"] = _state["stats"].get("lora_fallback", 0) + 1
        return orig(self, tensor, dtype)
    get_weight._weightferry = True
    return get_weight


def install(force=False):
    """Replace ComfyUI-GGUF's ops.dequantize_tensor (and GGMLLayer.get_weight for LoRA) with the B200 kernels, unless
    WEIGHTFERRY_GGUF_TRITON=0 (force: always), when ComfyUI-GGUF is loaded. Idempotent; True when installed. Raises
    ExtensionMissing when the CUDA library is not built (no silent fallback)."""
    from ..utils.logging import log_info
    if not force and _env_get("WEIGHTFERRY_GGUF_TRITON") != "1":
        return False
    ops = next((m for n, m in sys.modules.items() if n.endswith("ComfyUI-GGUF.ops") and m is not None), None)
    if ops is None or not hasattr(ops, "dequantize_tensor"):
        return False
    _ext.lib()  # fail loudly now rather than at the first weight
    if getattr(ops.dequantize_tensor, "_weightferry", False):
        return True
    _state["orig"], _state["ops"] = ops.dequantize_tensor, ops
    ops.dequantize_tensor = _patched(ops.dequantize_tensor)
    layer = getattr(ops, "GGMLLayer", None)
    if _LORA and layer is not None and not getattr(layer.get_weight, "_weightferry", False):
        _state["orig_gw"] = layer.get_weight
        layer.get_weight = _patched_get_weight(layer.get_weight)
    log_info("GGUF dequant on B200: ComfyUI-GGUF's Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0 "
             + ("and Q2_K .. Q6_K " if _kquants() else "") + "dequantisation in one kernel (WEIGHTFERRY_GGUF_TRITON).")
    return True


def uninstall():
    if _state["ops"] is not None and _state.get("orig_gw") is not None:
        _state["ops"].GGMLLayer.get_weight = _state["orig_gw"]
        _state["orig_gw"] = None
    if _state["ops"] is not None and _state["orig"] is not None:
        _state["ops"].dequantize_tensor = _state["orig"]
    _state["orig"] = _state["ops"] = None


def stats(reset=False):
    out = dict(_state["stats"])
    if reset:
        _state["stats"] = {"used": 0, "fallback": 0}
    return out
