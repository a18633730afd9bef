"""The int8 (W8A8) linear path of the fused block on B200 (drop-in for enhancers/fused_int8.py of ComfyUI-WeightFerry).

The reference quantises each linear layer's input per token (comfy_kitchen's ConvRot quantiser, or its own Triton
reproduction with a pending operation inside: modulate / LayerNorm + modulate / GELU) and multiplies with
comfy_kitchen's compiled CUTLASS int8 GEMM, whose epilogue rescales by the token's and the output channel's scales
(fused_int8.py:123-206). Here both halves are this package's sm_100a kernels: wf_quant_rows (the quantiser, same
arithmetic as the reference's reproduction) and wf_w8a8_gemm (tcgen05 kind::i8, int32 accumulators in tensor memory,
y = bf16((float(acc) * x_s[m]) * w_s[n])).

Entry points kept from the reference: ``_set_pre`` / ``_clear_pre`` / ``_materialise`` (pending inputs, :28-57),
``_quantise_pre(pre, x_2d, x_q, x_s)`` (:60-75), ``_gelu_table`` (:94-105), ``_int8_quantised`` (:123-188),
``_int8_linear_shared(x, weight, bias)`` (:191-206), ``_int8_linear_residual(x, weight, bias, res)`` (:212-268),
``_shared_forward`` / ``_residual_forward`` / ``_Overrides`` (:271-332). A weight is the reference's
TensorWiseINT8Layout QuantizedTensor (duck-typed: ``_layout_cls``, ``_params``, ``get_plain_tensors``) or a plain
``(w_q int8 [n, k], w_scale)`` pair. ``int8_linear(x, w_q, w_scale)`` is the plain per-token absmax linear of the
BASELINE W8A8 configuration (no rotation).
"""

import atexit

import torch

from .. import _ext
from .fused_kernels import PRE_GELU, PRE_LNMOD, PRE_MOD, PRE_NONE, _get_kernels
from .fused_state import _count, _state, _tls


# ------------------------------------------------------------------------------------------------------ pending inputs
def _key2d(t):
    return (t.data_ptr(), t.numel(), t.shape[-1])


def _set_pre(marker, kind, scale=None, shift=None, norm=None):
    """Register a pending input: the layer that receives ``marker`` quantises kind(marker) itself (mod / gelu;
    lnmod: marker is the block input, norm its LayerNorm)."""
    pre = {"key": _key2d(marker), "kind": kind, "src": marker, "used": False, "mat": None, "norm": norm}
    if kind in ("mod", "lnmod"):
        D = marker.shape[-1]
        groups = scale.numel() // D
        pre["s1"] = (1 + scale).contiguous().view(groups, D)
        pre["shift"] = shift.contiguous().view(groups, D)
        pre["scale5"], pre["shift5"], pre["rows_per_group"] = scale, shift, marker.numel() // D // groups
    _tls.pre = pre
    return pre


def _clear_pre():
    pre = getattr(_tls, "pre", None)
    _tls.pre = None
    return pre


def _materialise(pre):
    if pre["mat"] is None:
        from .fused_block import modulate
        if pre["kind"] == "gelu":
            pre["mat"] = torch.nn.functional.gelu(pre["src"])
        elif pre["kind"] == "lnmod":
            pre["mat"] = modulate(pre["norm"](pre["src"]), pre["scale5"], pre["shift5"])
        else:
            pre["mat"] = modulate(pre["src"], pre["scale5"], pre["shift5"])
    return pre["mat"]


def _quantise_pre(pre, x_2d, x_q, x_s, rotate=True):
    """Fill x_q / x_s with the quantisation of the pending input's real value (its operation inside the kernel)."""
    m, k = x_2d.shape
    quant_row = _get_kernels()["quant_row"][(m,)]
    if pre["kind"] == "gelu":
        quant_row(x_2d, _gelu_table(x_2d.device), x_2d, x_q, x_s, 1, 0.0, K=k, PRE=PRE_GELU, ROTATE=rotate)
    elif pre["kind"] == "lnmod":
        quant_row(x_2d, pre["s1"], pre["shift"], x_q, x_s, pre["rows_per_group"], float(pre["norm"].eps), K=k,
                  PRE=PRE_LNMOD, ROTATE=rotate)
    else:
        quant_row(x_2d, pre["s1"], pre["shift"], x_q, x_s, pre["rows_per_group"], 0.0, K=k, PRE=PRE_MOD,
                  ROTATE=rotate)


_gelu_tables = {}


def _release_gpu_caches():
    _gelu_tables.clear()
    for name in ("pre", "qkv", "res"):
        if getattr(_tls, name, None) is not None:
            setattr(_tls, name, None)


atexit.register(_release_gpu_caches)


def _gelu_table(device):
    """PyTorch's GELU (erf) of every bfloat16 value, indexed by its 16 bits (the quantiser's GELU looks it up, so
    the bits are PyTorch's own)."""
    key = str(device)
    tab = _gelu_tables.get(key)
    if tab is None:
        xs = torch.arange(65536, dtype=torch.int32, device=device).to(torch.int16).view(torch.bfloat16)
        tab = torch.nn.functional.gelu(xs).contiguous()
        _gelu_tables[key] = tab
    return tab


# ---------------------------------------------------------------------------------------------------------- GEMM
def gemm(x_q, w_q, x_s, ws, out=None, acc=None):
    """y = bf16((float(x_q @ w_q^T) * x_s) * ws) on the current stream; x_s [m] or [m, 1], ws [n] float32."""
    m, k = x_q.shape
    n = w_q.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=x_q.device)
    with torch.cuda.device(x_q.device):
        rc = _ext.lib().wf_w8a8_gemm(x_q.data_ptr(), w_q.data_ptr(), x_s.data_ptr(), ws.data_ptr(), out.data_ptr(),
                                     0 if acc is None else acc.data_ptr(), m, n, k, _ext.stream_of(x_q.device))
    _ext.check(rc, "wf_w8a8_gemm")
    return out


def _plain_weight(weight):
    """(w_q int8 [n, k] contiguous, per-channel float32 scales [n], convrot, transposed) of a weight."""
    if isinstance(weight, tuple):
        w_q, w_scale = weight
        convrot, transposed = False, False
    else:
        params = getattr(weight, "_params", None)
        convrot = bool(getattr(params, "convrot", False))
        transposed = bool(getattr(params, "transposed", False))
        layout = getattr(weight, "_layout_type", None) or getattr(weight, "_layout_cls", None)
        getter = getattr(layout, "get_plain_tensors", None) if not isinstance(layout, str) else None
        if getter is None:
            from comfy.quant_ops import TensorWiseINT8Layout  # the reference's layout class
            getter = TensorWiseINT8Layout.get_plain_tensors
        w_q, w_scale = getter(weight)
    w_q = w_q.contiguous()
    n = w_q.shape[0]
    ws = w_scale.reshape(-1).to(torch.float32)
    ws = ws if ws.numel() == n else ws.expand(n)
    return w_q, ws.contiguous(), convrot, transposed


def int8_linear(x, w_q, w_scale, pre=PRE_NONE, s1=None, shift=None, rows_per_group=1, eps=0.0, rotate=False):
    """The W8A8 linear of BASELINE's configuration: per-token int8 quantisation of x (after the optional pending
    operation `pre`) then the int8 GEMM with the rescale epilogue. x bf16 [..., k] on CUDA; returns bf16 [..., n]."""
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    m, k = x2.shape
    n = w_q.shape[0]
    ws = w_scale.reshape(-1).to(torch.float32)
    ws = (ws if ws.numel() == n else ws.expand(n)).contiguous()
    x_q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    x_s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    s = _gelu_table(x.device) if pre == PRE_GELU else s1
    _get_kernels()["quant_row"][(m,)](x2, s, shift, x_q, x_s, rows_per_group, eps, K=k, PRE=pre, ROTATE=rotate)
    out = gemm(x_q, w_q, x_s, ws)
    return out.reshape(*x.shape[:-1], n)


# ------------------------------------------------------------------------------------------------------- int8 linear
def _int8_quantised(x, weight, bias):
    """The quantised input of the int8 linear (reference :123-188), reused while the same input tensor comes back
    (q / k / v); a pending input is quantised with its operation inside. None when this is not the int8 case."""
    cache = getattr(_tls, "qkv", None)
    if cache is None or bias is not None:
        return None
    if not isinstance(weight, tuple) and getattr(weight, "_layout_cls", None) != "TensorWiseINT8Layout":
        return None
    w_q, ws, convrot, transposed = _plain_weight(weight)
    if transposed:
        return None
    x = x.contiguous()
    x_2d = x if x.dim() == 2 else x.reshape(-1, x.shape[-1])
    m, k = x_2d.shape
    n = w_q.shape[0]
    if (x.dtype != torch.bfloat16 or not x.is_cuda or m <= 2 or w_q.shape[1] != k or k % 16 or n % 8
            or (convrot and k % 256)):
        return None
    pre = getattr(_tls, "pre", None)
    is_pre = pre is not None and pre["key"] == _key2d(x_2d)
    if is_pre and pre["kind"] == "lnmod" and (k % 512 or k > 8192):
        _count("ln", False, f"width {k}")
        x_2d = _materialise(pre).reshape(-1, k).contiguous()
        is_pre = False
    key = (x_2d.data_ptr(), tuple(x_2d.shape), tuple(x_2d.stride()), convrot, is_pre)
    if cache.get("key") == key:
        x_q, x_s = cache["q"]
    else:
        x_q = torch.empty((m, k), dtype=torch.int8, device=x.device)
        x_s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
        if is_pre:
            _quantise_pre(pre, x_2d, x_q, x_s, rotate=convrot)
            _count({"gelu": "gelu", "lnmod": "ln"}.get(pre["kind"], "modq"), True)
        else:
            _get_kernels()["quant_row"][(m,)](x_2d, None, None, x_q, x_s, 1, 0.0, K=k, PRE=PRE_NONE, ROTATE=convrot)
        cache["key"], cache["q"] = key, (x_q, x_s)
    return {"x_q": x_q, "x_s": x_s, "w_q": w_q, "ws": ws, "m": m, "n": n, "dev": x.device, "dtype": x.dtype,
            "shape": x.shape}


def _int8_linear_shared(x, weight, bias):
    """The int8 linear with _int8_quantised's input; None when the host's own path applies."""
    q = _int8_quantised(x, weight, bias)
    if q is None:
        return None
    out = gemm(q["x_q"], q["w_q"], q["x_s"], q["ws"])
    return out if x.dim() == 2 else out.reshape(*x.shape[:-1], q["n"])


def gemm_residual(x_q, w_q, x_s, ws, resid, gate, rows_per_group, out=None):
    """out = bf16(resid + gate[row // rows_per_group] * bf16((float(x_q @ w_q^T) * x_s) * ws)) in one launch: the
    GEMM's epilogue adds the gated residual (the bits of gemm() followed by torch.addcmul in bf16). resid / out
    [m, n] bf16, gate [groups, n] bf16, all contiguous; out may be resid."""
    m, k = x_q.shape
    n = w_q.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=x_q.device)
    with torch.cuda.device(x_q.device):
        rc = _ext.lib().wf_w8a8_gemm_residual(x_q.data_ptr(), w_q.data_ptr(), x_s.data_ptr(), ws.data_ptr(),
                                              resid.data_ptr(), gate.data_ptr(), int(rows_per_group), out.data_ptr(),
                                              m, n, k, _ext.stream_of(x_q.device))
    _ext.check(rc, "wf_w8a8_gemm_residual")
    return out


def _int8_linear_residual(x, weight, bias, res):
    """x_res + gate * linear(x) for the block's residual x_res (B, T, H, W, D) and gate (B, T, 1, 1, D), or x_res
    (B, N, D) and gate (B, 1, D) (reference :212-268): one GEMM whose epilogue adds the gated residual, over all the
    (batch, frame) groups at once (each row takes its group's gate row; the reference launches once per group, or once
    for all rows when the gates are equal). None when not possible (the caller runs the plain linear and the block
    its addcmul)."""
    xr, gate = res["x"], res["gate"]
    q = _int8_quantised(x, weight, bias)
    if q is None:
        return None
    m, n = q["m"], q["n"]
    D = xr.shape[-1]
    if xr.dim() == 5:
        B, T, H, W, _ = xr.shape
        if not xr.is_contiguous() or tuple(gate.shape) != (B, T, 1, 1, D):
            return None
        groups, rows = B * T, H * W
    elif xr.dim() == 3:
        groups, rows, _ = xr.shape
        if not xr.is_contiguous() or tuple(gate.shape) != (groups, 1, D):
            return None
    else:
        return None
    if n != D or m != groups * rows or xr.dtype != q["dtype"] or gate.dtype != q["dtype"] or not xr.is_cuda:
        return None
    g2 = gate.reshape(groups, D).contiguous()
    out = torch.empty_like(xr)
    gemm_residual(q["x_q"], q["w_q"], q["x_s"], q["ws"], xr.view(m, D), g2, rows, out=out.view(m, D))
    return out if x.dim() == 2 else out.view(*q["shape"][:-1], n)


def _pending_for(input):
    pre = getattr(_tls, "pre", None)
    is_pre = (pre is not None and torch.is_tensor(input) and input.dim() >= 2
              and pre["key"] == _key2d(input.reshape(-1, input.shape[-1])))
    return pre, is_pre


def _shared_forward(input, weight, bias):
    """The _forward of a linear layer under _Overrides."""
    pre, is_pre = _pending_for(input)
    if is_pre:
        pre["used"] = True
    out = _int8_linear_shared(input, weight, bias)
    if out is None:
        _count("qkv", False, f"weight {type(weight).__name__}, input {getattr(input, 'dtype', None)}")
        if is_pre:
            input = _materialise(pre).reshape(input.shape)
        return torch.nn.functional.linear(input, weight, bias)
    _count("qkv", True)
    return out


def _residual_forward(input, weight, bias):
    """The _forward of a sub-layer's output projection with the block's residual pending (res)."""
    res = getattr(_tls, "res", None)
    if res is not None and not res["done"]:
        pre, is_pre = _pending_for(input)
        out = _int8_linear_residual(input, weight, bias, res)
        if out is not None:
            if is_pre:
                pre["used"] = True
            res["done"] = True
            _count("res", True)
            return out
        _count("res", False, f"input {tuple(input.shape)} {input.dtype}")
    return _shared_forward(input, weight, bias)


class _Overrides:
    """_shared_forward (or the given function) on some linear layers for the duration of a call."""

    def __init__(self, layers):
        pairs = [x if isinstance(x, tuple) else (x, _shared_forward) for x in layers]
        self.layers = [(lin, fn) for lin, fn in pairs if "_forward" not in lin.__dict__]

    def __enter__(self):
        self.outer = getattr(_tls, "qkv", None) is not None
        if not self.outer:
            _tls.qkv = {}
        for lin, fn in self.layers:
            lin._forward = fn
        return self

    def __exit__(self, *exc):
        for lin, _fn in self.layers:
            lin.__dict__.pop("_forward", None)
        if not self.outer:
            _tls.qkv = None
        return False


def parts():
    return _state["parts"]
