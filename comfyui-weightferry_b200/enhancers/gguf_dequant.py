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
_state = {"orig": None, "ops": None, "orig_gw": None}  # ComfyUI-GGUF's module and its replaced functions
_LORA = True      # LoRA patches inside the dequantisation too (GGMLLayer.get_weight)
_FACTORS = None   # "pin" / "0"; None = WEIGHTFERRY_GGUF_LORA_FACTORS


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
    with _ext.on_device(raw.device):
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
    with _ext.on_device(dev):
        rc = _ext.lib().wf_dequant_gguf_batch(tasks, len(items), q, _DT[mid], _DT[out], _ext.stream_of(dev))
    _ext.check(rc, "wf_dequant_gguf_batch")
    return outs


# --------------------------------------------------------------------------------------------------------------- LoRA
def _number(v):
    return isinstance(v, (int, float)) and not isinstance(v, bool)


def _plain_lora(patch, n_out, n_in):
    """(up, down, scale) of one ComfyUI weight patch when it is a plain LoRA on a 2-D [n_out, n_in] weight, which
    comfy.lora.calculate_weight applies as weight += (scale * (up @ down)).type(weight.dtype) with scale = strength *
    alpha / rank (strength when alpha is None); None for anything else."""
    if not (isinstance(patch, tuple) and len(patch) == 5):
        return None
    strength, adapter, strength_model, offset, function = patch
    if type(adapter).__name__ != "LoRAAdapter" or strength_model != 1.0 or offset is not None or function is not None:
        return None
    if not _number(strength):
        return None
    parts = getattr(adapter, "weights", None)
    if not isinstance(parts, (tuple, list)) or len(parts) < 6:
        return None
    up, down, alpha, mid, dora_scale, reshape = parts[:6]
    if mid is not None or dora_scale is not None or reshape is not None:  # LoCon mid weight, DoRA, reshape
        return None
    if not (torch.is_tensor(up) and torch.is_tensor(down) and up.dim() == 2 and down.dim() == 2):
        return None
    rank = down.shape[0]
    if tuple(up.shape) != (n_out, rank) or down.shape[1] != n_in:
        return None
    if alpha is None:
        return up, down, strength
    if not _number(alpha):
        return None
    return up, down, strength * (alpha / rank)


def lora_factors(patch_list, n_out, n_in):
    """[(up, down, strength * alpha / rank)] when every patch is a plain LoRA of a 2-D weight (reference :329-355),
    else None: one patch of another kind sends the whole weight to ComfyUI-GGUF's own code."""
    out = []
    for patch in patch_list:
        lora = _plain_lora(patch, n_out, n_in)
        if lora is None:
            return None
        out.append(lora)
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
    with _ext.on_device(dev):
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
    """"pin": LoRA factors copied to the GPU from pinned host copies (WEIGHTFERRY_GGUF_LORA_FACTORS, default);
    "0": straight from where they are, as comfy does -- also when ComfyUI runs with pinned memory disabled."""
    if _FACTORS is not None:
        return _FACTORS
    wanted = (_env_get("WEIGHTFERRY_GGUF_LORA_FACTORS") or "pin").strip().lower()
    try:
        import comfy.model_management as mm
        from comfy.cli_args import args
        if getattr(args, "disable_pinned_memory", False) or getattr(mm, "DISABLE_PINNED_MEMORY", False):
            return "0"
    except Exception:  # noqa: BLE001 -- outside ComfyUI
        pass
    return "pin" if wanted == "pin" else "0"


class _PinnedFactors:
    """Pinned host copies of CPU LoRA factors, one per factor tensor while it lives and stays unchanged (same storage
    and version). ComfyUI-GGUF keeps the patches on the host, and a copy from pageable memory waits for the GPU queue
    to drain; from a pinned copy it does not. An entry goes away with its factor (a weak reference's callback)."""

    def __init__(self):
        self._by_id = {}
        self.freed = False

    @staticmethod
    def _stamp(t, dev):
        try:
            version = t._version
        except RuntimeError:  # inference tensors keep no version counter
            version = None
        return (t.data_ptr(), version, str(dev))

    def pinned(self, t, dev):
        stamp = self._stamp(t, dev)
        entry = self._by_id.get(id(t))
        if entry is not None and entry[0]() is t and entry[1] == stamp:
            return entry[2]
        copy = t.pin_memory()
        key = id(t)
        self._by_id[key] = (weakref.ref(t, lambda _ref, k=key: self._forget(k)), stamp, copy)
        return copy

    def _forget(self, key):
        if self._by_id.pop(key, None) is not None:
            self.freed = True

    def __len__(self):
        return len(self._by_id)


_factors = _PinnedFactors()


def _factor(t, dev, mode):
    """t.to(dev, float32), the LoRA factor as comfy casts it; in mode "pin" through a kept pinned copy."""
    if mode == "0" or t.device.type != "cpu":
        return t.to(dev, torch.float32)
    return _factors.pinned(t, dev).to(dev, non_blocking=True).to(torch.float32)


# ------------------------------------------------------------------------------------------------------------ install
class _Tally:
    """Calls of the patched entry points: ``used`` / ``fallback`` (dequantize_tensor), ``lora_used`` /
    ``lora_fallback`` (get_weight with LoRA patches)."""

    def __init__(self):
        self.reset()

    def reset(self):
        self.counts = {"used": 0, "fallback": 0}

    def add(self, key):
        self.counts[key] = self.counts.get(key, 0) + 1


_TALLY = _Tally()


def _intermediate(dequant_dtype, dtype):
    """ComfyUI-GGUF's precision of the dequantisation: the target dtype for "target", else dequant_dtype (None:
    the default). Returns False when it is not a dtype this path takes."""
    mid = dtype if dequant_dtype == "target" else dequant_dtype
    return mid if mid is None or isinstance(mid, torch.dtype) else False


def _logical_shape(tensor):
    return tuple(getattr(tensor, "tensor_shape", tensor.shape))


def _one_kernel(tensor, dtype, dequant_dtype):
    """The dequantised weight of a GGUF tensor by one kernel, or None (the caller runs ComfyUI-GGUF's code)."""
    qtype = getattr(tensor, "tensor_type", None)
    if qtype is None or not isinstance(tensor, torch.Tensor) or not _supported(qtype):
        return None
    mid = _intermediate(dequant_dtype, dtype)
    if mid is False:
        return None
    return dequantize(tensor.data, qtype, _logical_shape(tensor), mid, dtype)


def _lora_weight(layer, tensor, dtype):
    """A GGUF layer's weight with its LoRA patches by one kernel per LoRA, or None (ComfyUI-GGUF's code runs)."""
    qtype = getattr(tensor, "tensor_type", None)
    if (getattr(layer, "patch_dtype", None) is not None or qtype is None or not _supported(qtype)
            or not isinstance(dtype, torch.dtype) or not getattr(tensor, "is_cuda", False)):
        return None
    mid = _intermediate(layer.dequant_dtype, dtype)
    shape = _logical_shape(tensor)
    if mid is False or len(shape) != 2:
        return None
    loras = lora_factors([p for group, _key in tensor.patches for p in group], *shape)
    return dequantize_lora(tensor.data, qtype, shape, mid, dtype, loras) if loras else None


def _patched(orig):
    """ComfyUI-GGUF's ops.dequantize_tensor with the one-kernel dequantisation in front (reference :521-541)."""
    def dequantize_tensor(tensor, dtype=None, dequant_dtype=None):
        out = _one_kernel(tensor, dtype, dequant_dtype)
        _TALLY.add("used" if out is not None else "fallback")
        return out if out is not None else orig(tensor, dtype, dequant_dtype)
    dequantize_tensor._weightferry = True
    return dequantize_tensor


def _patched_get_weight(orig):
    """GGMLLayer.get_weight with LoRA patches added inside the dequantisation (reference :464-492)."""
    def get_weight(self, tensor, dtype):
        if tensor is not None and getattr(tensor, "patches", None):
            out = _lora_weight(self, tensor, dtype)
            _TALLY.add("lora_used" if out is not None else "lora_fallback")
            if out is not None:
                return out
        return orig(self, tensor, dtype) if tensor is not None else None
    get_weight._weightferry = True
    return get_weight


def _gguf_ops():
    """ComfyUI-GGUF's ops module (ComfyUI loads custom nodes under path-derived names ending in ComfyUI-GGUF.ops)."""
    for name, mod in list(sys.modules.items()):
        if mod is not None and name.endswith("ComfyUI-GGUF.ops") and hasattr(mod, "dequantize_tensor"):
            return mod
    return None


def install(force=False):
    """Put the B200 kernels in front of ComfyUI-GGUF's ops.dequantize_tensor (and GGMLLayer.get_weight for LoRA
    patches) when ComfyUI-GGUF is loaded, unless WEIGHTFERRY_GGUF_TRITON=0 (force: always). Idempotent; True when
    installed. Raises ExtensionMissing when the CUDA library is not built (no silent fallback)."""
    from ..utils.logging import log_info
    if not force and _env_get("WEIGHTFERRY_GGUF_TRITON") != "1":
        return False
    ops = _gguf_ops()
    if ops is None:
        return False
    _ext.lib()  # fail now rather than at the first weight
    if not getattr(ops.dequantize_tensor, "_weightferry", False):
        _state["orig"], _state["ops"] = ops.dequantize_tensor, ops
        ops.dequantize_tensor = _patched(ops.dequantize_tensor)
        layer = getattr(ops, "GGMLLayer", None)
        if _LORA and layer is not None and not getattr(layer.get_weight, "_weightferry", False):
            _state["orig_gw"] = layer.get_weight
            layer.get_weight = _patched_get_weight(layer.get_weight)
        kinds = "Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0" + (" and Q2_K .. Q6_K" if _kquants() else "")
        log_info(f"GGUF dequant on B200: ComfyUI-GGUF's {kinds} in one kernel per weight (WEIGHTFERRY_GGUF_TRITON).")
    return True


def uninstall():
    """Give ComfyUI-GGUF its own functions back."""
    ops = _state["ops"]
    if ops is not None:
        if _state.get("orig_gw") is not None:
            ops.GGMLLayer.get_weight = _state["orig_gw"]
        if _state["orig"] is not None:
            ops.dequantize_tensor = _state["orig"]
    _state.update(orig=None, ops=None, orig_gw=None)


def stats(reset=False):
    """{"used", "fallback"[, "lora_used", "lora_fallback"]}: calls of the patched entry points."""
    out = dict(_TALLY.counts)
    if reset:
        _TALLY.reset()
    return out
