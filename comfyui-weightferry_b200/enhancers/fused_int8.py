"""The int8 (W8A8) linear path of the fused block on B200 (the role of enhancers/fused_int8.py in ComfyUI-WeightFerry).

ComfyUI's int8 linear quantises the layer's bf16 input per token (comfy_kitchen's ConvRot quantiser) and multiplies
with comfy_kitchen's int8 GEMM, whose epilogue rescales by the token's and the output channel's scales. The
reference speeds that up three ways (fused_int8.py:19-332), all kept here on this package's sm_100a kernels --
wf_quant_rows (the quantiser) and wf_w8a8_gemm / wf_w8a8_gemm_residual (tcgen05 kind::i8, int32 accumulators in
tensor memory, y = bf16((float(acc) * x_s[m]) * w_s[n])):

* a *pending input*: the block leaves an element-wise step (scale-and-shift, LayerNorm + scale-and-shift, GELU)
  unwritten and hands the next int8 layer its source instead; that layer's quantiser computes the step while it
  reads the row (``Pending``; ``_set_pre`` / ``_clear_pre`` / ``_materialise`` / ``_quantise_pre``);
* *one quantisation for several layers*: q, k and v read the same input, so its int8 copy is made once per
  ``_Overrides`` scope (``_QuantScope``; ``_int8_quantised``);
* the *gated residual* ``x + gate * out`` of a sub-layer inside its output projection's GEMM epilogue, one launch
  for every (batch, frame) group at once (``_int8_linear_residual``).

A layer takes these paths through a per-instance ``_forward`` override, which ComfyUI's Linear calls with the
prepared (input, weight, bias) (``_Overrides``, ``_shared_forward``, ``_residual_forward``). Anything the fused path
does not cover returns None and the layer's own code runs on the real input.

A weight is ComfyUI's TensorWiseINT8Layout QuantizedTensor (duck-typed: ``_layout_cls``, ``_params``,
``get_plain_tensors`` of its layout) or a plain ``(w_q int8 [n, k], w_scale)`` pair. ``int8_linear(x, w_q, w_scale)``
is the plain per-token absmax linear of the BASELINE W8A8 configuration (no rotation).
"""

import atexit
from collections import namedtuple

import torch

from .. import _ext
from .fused_kernels import PRE_GELU, PRE_LNMOD, PRE_MOD, PRE_NONE, _get_kernels
from .fused_state import _count, _state, _tls

_PRE_CODE = {"mod": PRE_MOD, "lnmod": PRE_LNMOD, "gelu": PRE_GELU}
_PART_OF = {"mod": "modq", "lnmod": "ln", "gelu": "gelu"}  # the fused part a pending kind is counted under


def _key2d(t):
    """Identity of a (rows, width) view of a tensor: its data pointer, element count and row width."""
    return (t.data_ptr(), t.numel(), t.shape[-1])


# ------------------------------------------------------------------------------------------------------ pending inputs
class Pending:
    """An element-wise step left for the quantiser of the layer that receives ``marker`` (a tensor standing for the
    step's result): ``mod`` -- marker * (1 + scale) + shift; ``lnmod`` -- norm(marker) * (1 + scale) + shift, with
    ``norm`` an affine-free LayerNorm; ``gelu`` -- GELU(marker) (erf), looked up in a table of PyTorch's own values.
    scale / shift broadcast over groups of consecutive rows ((B, T, 1, 1, D) over a (B, T, H, W, D) marker).
    ``used`` turns True once a layer took it; the real result is computed at most once, on demand (``real()``)."""

    def __init__(self, marker, kind, scale=None, shift=None, norm=None):
        if kind not in _PRE_CODE:
            raise ValueError(f"unknown pending operation {kind!r}")
        self.key = _key2d(marker)
        self.kind = kind
        self.src = marker
        self.norm = norm
        self.used = False
        self._real = None
        self.scale, self.shift = scale, shift
        if kind != "gelu":
            width = marker.shape[-1]
            groups = scale.numel() // width
            self.s1 = (1 + scale).contiguous().view(groups, width)  # PyTorch's bf16 (1 + scale), as ComfyUI has it
            self.shift_rows = shift.contiguous().view(groups, width)
            self.rows_per_group = marker.numel() // width // groups

    def owns(self, t):
        return torch.is_tensor(t) and t.dim() >= 2 and _key2d(t.reshape(-1, t.shape[-1])) == self.key

    def real(self):
        """The step's result as a tensor (for a consumer that cannot take it pending)."""
        if self._real is None:
            if self.kind == "gelu":
                self._real = torch.nn.functional.gelu(self.src)
            else:
                from .fused_block import modulate
                base = self.norm(self.src) if self.kind == "lnmod" else self.src
                self._real = modulate(base, self.scale, self.shift)
        return self._real

    def quantise(self, x_2d, x_q, x_s, rotate):
        """x_q / x_s <- the int8 quantisation of the step's result, the step computed inside the quantiser."""
        m, k = x_2d.shape
        launch = _get_kernels()["quant_row"][(m,)]
        if self.kind == "gelu":
            launch(x_2d, _gelu_table(x_2d.device), None, x_q, x_s, 1, 0.0, K=k, PRE=PRE_GELU, ROTATE=rotate)
        else:
            eps = float(self.norm.eps) if self.kind == "lnmod" else 0.0
            launch(x_2d, self.s1, self.shift_rows, x_q, x_s, self.rows_per_group, eps, K=k, PRE=_PRE_CODE[self.kind],
                   ROTATE=rotate)


def _set_pre(marker, kind, scale=None, shift=None, norm=None):
    """Register a pending input for this thread's next int8 layer (reference :28-45); returns it."""
    pre = Pending(marker, kind, scale, shift, norm)
    _tls.pre = pre
    return pre


def _clear_pre():
    pre = getattr(_tls, "pre", None)
    _tls.pre = None
    return pre


def _materialise(pre):
    return pre.real()


def _quantise_pre(pre, x_2d, x_q, x_s, rotate=True):
    """Fill the caller's x_q [m, k] int8 and x_s [m, 1] float32 with the quantisation of the pending input's real
    value (reference :60-75)."""
    pre.quantise(x_2d, x_q, x_s, rotate)


def _pending_for(inp):
    """(this thread's pending input or None, whether ``inp`` is its marker)."""
    pre = getattr(_tls, "pre", None)
    return pre, pre is not None and pre.owns(inp)


# ------------------------------------------------------------------------------------------------------ GELU table
_gelu_by_device = {}


def _gelu_table(device):
    """PyTorch's GELU (erf form) of all 65536 bfloat16 values, indexed by their bits: the quantiser's GELU reads its
    results here, so they are PyTorch's own bits whatever erf the toolkits implement (reference :94-105)."""
    dev = torch.device(device)
    tab = _gelu_by_device.get(dev)
    if tab is None:
        # the values in signed-bit order (0x8000 .. 0xFFFF, then 0x0000 .. 0x7FFF), rolled so entry i has bits i
        values = torch.arange(-32768, 32768, dtype=torch.int32, device=dev).to(torch.int16).view(torch.bfloat16)
        tab = torch.nn.functional.gelu(values).roll(32768).contiguous()
        _gelu_by_device[dev] = tab
    return tab


def _drop_thread_state():
    """At exit, before module teardown: forget the GPU tensors held here (an allocator that shuts down first must
    not see them freed later)."""
    _gelu_by_device.clear()
    for slot in ("pre", "qkv", "res"):
        if getattr(_tls, slot, None) is not None:
            setattr(_tls, slot, None)


atexit.register(_drop_thread_state)


# ---------------------------------------------------------------------------------------------------------- GEMM
def gemm(x_q, w_q, x_s, ws, out=None, acc=None):
    """y = bf16((float(x_q @ w_q^T) * x_s) * ws) on the current stream; x_s [m] or [m, 1], ws [n] float32."""
    m, k = x_q.shape
    n = w_q.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=x_q.device)
    with _ext.on_device(x_q.device):
        rc = _ext.lib().wf_w8a8_gemm(x_q.data_ptr(), w_q.data_ptr(), x_s.data_ptr(), ws.data_ptr(), out.data_ptr(),
                                     0 if acc is None else acc.data_ptr(), m, n, k, _ext.stream_of(x_q.device))
    _ext.check(rc, "wf_w8a8_gemm")
    return out


def gemm_residual(x_q, w_q, x_s, ws, resid, gate, rows_per_group, out=None):
    """out = bf16(resid + gate[row // rows_per_group] * bf16((float(x_q @ w_q^T) * x_s) * ws)) in one launch: the
    GEMM's epilogue adds the gated residual (the bits of gemm() followed by torch.addcmul in bf16). resid / out
    [m, n] bf16, gate [groups, n] bf16, all contiguous; out may be resid."""
    m, k = x_q.shape
    n = w_q.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=x_q.device)
    with _ext.on_device(x_q.device):
        rc = _ext.lib().wf_w8a8_gemm_residual(x_q.data_ptr(), w_q.data_ptr(), x_s.data_ptr(), ws.data_ptr(),
                                              resid.data_ptr(), gate.data_ptr(), int(rows_per_group), out.data_ptr(),
                                              m, n, k, _ext.stream_of(x_q.device))
    _ext.check(rc, "wf_w8a8_gemm_residual")
    return out


Int8Weight = namedtuple("Int8Weight", "w_q ws convrot transposed")


def _int8_weight(weight):
    """The int8 operand of a weight: Int8Weight(w_q int8 [n, k] contiguous, per-channel float32 scales [n], ConvRot
    rotation, stored transposed), or None when the weight is not a TensorWiseINT8Layout tensor / pair."""
    if isinstance(weight, tuple):
        w_q, scale = weight
        convrot = transposed = False
    else:
        if getattr(weight, "_layout_cls", None) != "TensorWiseINT8Layout":
            return None
        params = getattr(weight, "_params", None)
        convrot = bool(getattr(params, "convrot", False))
        transposed = bool(getattr(params, "transposed", False))
        layout = getattr(weight, "_layout_type", None)
        split = getattr(layout, "get_plain_tensors", None) if layout is not None and not isinstance(layout, str) \
            else None
        if split is None:
            from comfy.quant_ops import TensorWiseINT8Layout
            split = TensorWiseINT8Layout.get_plain_tensors
        w_q, scale = split(weight)
        if convrot and getattr(params, "convrot_groupsize", 256) != 256:
            return None  # the quantiser's rotation is the 256-wide one
    w_q = w_q.contiguous()
    n = w_q.shape[0]
    ws = scale.reshape(-1).to(torch.float32)
    ws = (ws if ws.numel() == n else ws.expand(n)).contiguous()
    return Int8Weight(w_q, ws, convrot, transposed)


def _plain_weight(weight):
    """(w_q, ws, convrot, transposed) of an int8 weight (the tuple form of _int8_weight)."""
    w = _int8_weight(weight)
    if w is None:
        raise TypeError(f"not an int8 weight: {type(weight).__name__}")
    return tuple(w)


def _int8_proj_ok(lin):
    """The layer hands its input unchanged to ``_forward`` with an int8 weight (ComfyUI's weight-only int8 layout:
    the layer does not quantise its input itself, no AWQ pre-scale, no instance forward of its own)."""
    if not hasattr(lin, "_forward") or "forward" in lin.__dict__ or getattr(lin, "pre_quant_scale", None) is not None:
        return False
    if getattr(getattr(lin, "weight", None), "_layout_cls", None) != "TensorWiseINT8Layout":
        return False
    try:
        from comfy.quant_ops import QUANT_ALGOS
    except ImportError:
        return False
    return QUANT_ALGOS.get(getattr(lin, "quant_format", None), {}).get("quantize_input", True) is False


def int8_linear(x, w_q, w_scale, pre=PRE_NONE, s1=None, shift=None, rows_per_group=1, eps=0.0, rotate=False):
    """The W8A8 linear of BASELINE's configuration: per-token int8 quantisation of x (after the optional pending
    operation `pre`) then the int8 GEMM with the rescale epilogue. x bf16 [..., k] on CUDA; returns bf16 [..., n]."""
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    m, k = x2.shape
    w = _int8_weight((w_q, w_scale))
    x_q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    x_s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    s = _gelu_table(x.device) if pre == PRE_GELU else s1
    _get_kernels()["quant_row"][(m,)](x2, s, shift, x_q, x_s, rows_per_group, eps, K=k, PRE=pre, ROTATE=rotate)
    out = gemm(x_q, w.w_q, x_s, w.ws)
    return out.reshape(*x.shape[:-1], w.w_q.shape[0])


# ------------------------------------------------------------------------------------------------------- int8 linear
class _QuantScope:
    """The int8 copy of the last input quantised inside one ``_Overrides`` scope, reused while the same input comes
    back (q, k and v). It keeps the source tensor alive so that its address cannot be reused under the key."""

    __slots__ = ("key", "src", "x_q", "x_s")

    def __init__(self):
        self.key = self.src = self.x_q = self.x_s = None

    def get(self, key):
        return (self.x_q, self.x_s) if self.key == key else None

    def put(self, key, src, x_q, x_s):
        self.key, self.src, self.x_q, self.x_s = key, src, x_q, x_s


Quantised = namedtuple("Quantised", "x_q x_s w_q ws m n shape dtype")


def _int8_quantised(x, weight, bias):
    """The int8 operands of ``x @ weight^T`` (reference :123-188): the input quantised per token -- with a pending
    step inside when ``x`` is its marker, and shared with the other layers of the scope that read the same input --
    and the weight's int8 values and per-channel scales. None when this call is not the int8 case."""
    scope = getattr(_tls, "qkv", None)
    if scope is None or bias is not None or not torch.is_tensor(x):
        return None
    w = _int8_weight(weight)
    if w is None or w.transposed:
        return None
    if x.dtype != torch.bfloat16 or not x.is_cuda:
        return None
    x_2d = x.reshape(-1, x.shape[-1])
    if not x_2d.is_contiguous():
        x_2d = x_2d.contiguous()
    m, k = x_2d.shape
    n = w.w_q.shape[0]
    if m <= 2 or w.w_q.shape[1] != k or k % 16 or n % 8 or (w.convrot and k % 256):
        return None
    pre, pending = _pending_for(x_2d)
    if pending and pre.kind == "lnmod" and (k % 512 or k > 8192):
        # the quantiser's LayerNorm covers rows of 512 * j values up to 8192: quantise the real input instead
        _count("ln", False, f"width {k}")
        x_2d = pre.real().reshape(-1, k).contiguous()
        pending = False
    key = (x_2d.data_ptr(), tuple(x_2d.shape), tuple(x_2d.stride()), w.convrot, pending)
    hit = scope.get(key)
    if hit is None:
        x_q = torch.empty((m, k), dtype=torch.int8, device=x.device)
        x_s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
        if pending:
            pre.quantise(x_2d, x_q, x_s, w.convrot)
            _count(_PART_OF[pre.kind], True)
        else:
            _get_kernels()["quant_row"][(m,)](x_2d, None, None, x_q, x_s, 1, 0.0, K=k, PRE=PRE_NONE,
                                              ROTATE=w.convrot)
        scope.put(key, x_2d, x_q, x_s)
        hit = (x_q, x_s)
    return Quantised(hit[0], hit[1], w.w_q, w.ws, m, n, tuple(x.shape), x.dtype)


def _int8_linear_shared(x, weight, bias):
    """x @ weight^T with _int8_quantised's operands (reference :191-206); None when the layer's own path applies."""
    q = _int8_quantised(x, weight, bias)
    if q is None:
        return None
    out = gemm(q.x_q, q.w_q, q.x_s, q.ws)
    return out.view(*q.shape[:-1], q.n)


def _residual_groups(xr, gate, d):
    """(groups, rows per group) of a residual (B, T, H, W, D) with gate (B, T, 1, 1, D), or (B, N, D) with gate
    (B, 1, D); None for any other layout."""
    if xr.dim() == 5:
        b, t, h, w, _ = xr.shape
        return (b * t, h * w) if tuple(gate.shape) == (b, t, 1, 1, d) else None
    if xr.dim() == 3:
        b, n, _ = xr.shape
        return (b, n) if tuple(gate.shape) == (b, 1, d) else None
    return None


def _int8_linear_residual(x, weight, bias, res):
    """res.x + res.gate * (x @ weight^T) for the block's residual and gate (reference :212-268): one GEMM whose
    epilogue adds the gated residual for all the (batch, frame) groups at once, each row taking its group's gate row
    (the reference launches once per group). None when not possible: the caller runs the plain linear and the block
    its addcmul."""
    xr, gate = res["x"], res["gate"]
    q = _int8_quantised(x, weight, bias)
    if q is None:
        return None
    d = xr.shape[-1]
    grouping = _residual_groups(xr, gate, d)
    if (grouping is None or not xr.is_contiguous() or not xr.is_cuda or q.n != d or q.m != grouping[0] * grouping[1]
            or xr.dtype != q.dtype or gate.dtype != q.dtype):
        return None
    out = torch.empty_like(xr)
    gemm_residual(q.x_q, q.w_q, q.x_s, q.ws, xr.view(q.m, d), gate.reshape(grouping[0], d).contiguous(), grouping[1],
                  out=out.view(q.m, d))
    return out if len(q.shape) == xr.dim() else out.view(*q.shape[:-1], q.n)


def _shared_forward(input, weight, bias):
    """``_forward`` of a linear layer under _Overrides: the int8 path when it applies, else F.linear on the real
    input."""
    pre, pending = _pending_for(input)
    if pending:
        pre.used = True
    out = _int8_linear_shared(input, weight, bias)
    if out is not None:
        _count("qkv", True)
        return out
    _count("qkv", False, f"weight {type(weight).__name__}, input {getattr(input, 'dtype', None)}")
    if pending:
        input = pre.real().reshape(input.shape)
    return torch.nn.functional.linear(input, weight, bias)


def _residual_forward(input, weight, bias):
    """``_forward`` of a sub-layer's output projection while the block's residual is offered (``_tls.res``): the
    residual GEMM once, then the plain shared path."""
    res = getattr(_tls, "res", None)
    if res is not None and not res["done"]:
        pre, pending = _pending_for(input)
        out = _int8_linear_residual(input, weight, bias, res)
        if out is not None:
            if pending:
                pre.used = True
            res["done"] = True
            _count("res", True)
            return out
        _count("res", False, f"input {tuple(input.shape)} {input.dtype}")
    return _shared_forward(input, weight, bias)


class _Overrides:
    """For the duration of a ``with`` block, give some linear layers an instance ``_forward`` (``_shared_forward``
    unless a (layer, function) pair names another) and open a quantisation scope when none is open. A layer that
    already has an instance ``_forward`` (an outer override) keeps it."""

    def __init__(self, layers):
        self._plan = []
        for item in layers:
            lin, fn = item if isinstance(item, tuple) else (item, _shared_forward)
            if "_forward" not in lin.__dict__:
                self._plan.append((lin, fn))
        self._opened = False

    def __enter__(self):
        if getattr(_tls, "qkv", None) is None:
            _tls.qkv = _QuantScope()
            self._opened = True
        for lin, fn in self._plan:
            lin._forward = fn
        return self

    def __exit__(self, *exc):
        for lin, _fn in self._plan:
            lin.__dict__.pop("_forward", None)
        if self._opened:
            _tls.qkv = None
        return False


def parts():
    return _state["parts"]
