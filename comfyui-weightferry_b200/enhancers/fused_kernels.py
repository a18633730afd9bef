"""Launchers of the fused-block kernels (enhancers/fused_kernels.py of the reference): the same names, constants and
call convention, over the sm_100a kernels of csrc/fused_block.cu instead of Triton.

``_get_kernels()`` returns a dict of launchers indexed by grid, as the reference's ``NoFMA`` wrappers are
(fused_kernels.py:23-36): ``ks["quant_row"][(m,)](x, s, h, q, sc, rows_per_group, eps, K=k, PRE=PRE_LNMOD)``. The grid
and the Triton-only keywords (num_warps, BLOCK, ROWS) are accepted and ignored: each CUDA kernel has its own fixed
launch shape. Every launch goes to the current CUDA stream. (The reference's TaylorSeer kernel, ``tay``, is a
sampling-level feature outside the quantized-weight path and is not provided.)"""

import torch

from .. import _ext

# the operation the quantiser applies before the rotation (fused_kernels.py:15-18)
PRE_NONE = 0   # the input as it is
PRE_GELU = 1   # PyTorch's GELU of the bf16 input, looked up in a 65536-entry table
PRE_MOD = 2    # the scale-and-shift bf16(bf16(x * (1 + scale)) + shift)
PRE_LNMOD = 3  # LayerNorm (no affine), then the scale-and-shift

_kernels = {}


def _p(t):
    return 0 if t is None else t.data_ptr()


def _stream(t):
    return _ext.stream_of(t.device)


class _Launcher:
    """fn[grid](*args, **kw) -> fn(*args, **kw), like the reference's NoFMA.__getitem__."""

    def __init__(self, fn):
        self.fn = fn

    def __getitem__(self, grid):
        return self.fn


def _mod(a, s1, h, o, n_cols, rows_per_group, **_triton_kw):
    rows = a.numel() // n_cols
    with _ext.on_device(a.device):
        rc = _ext.lib().wf_modulate(a.data_ptr(), s1.data_ptr(), h.data_ptr(), o.data_ptr(), rows, int(n_cols),
                                    int(rows_per_group), _stream(a))
    _ext.check(rc, "wf_modulate")


def _lnmod(x, s1, h, o, rows_per_group, eps, K, **_triton_kw):
    rows = x.numel() // K
    with _ext.on_device(x.device):
        rc = _ext.lib().wf_ln_modulate(x.data_ptr(), s1.data_ptr(), h.data_ptr(), o.data_ptr(), rows, int(K),
                                       int(rows_per_group), float(eps), _stream(x))
    _ext.check(rc, "wf_ln_modulate")


def _rms128(x, w, o, n_rows, eps, RS=0, **_triton_kw):  # noqa: N803 -- the reference's keyword
    with _ext.on_device(x.device):
        rc = _ext.lib().wf_rms_norm_128(x.data_ptr(), w.data_ptr(), _ext.dtype_code(w.dtype), o.data_ptr(),
                                        int(n_rows), float(eps), _stream(x))
    _ext.check(rc, "wf_rms_norm_128")


def _quant_row(x, s, h, q, sc, rows_per_group, eps, K, PRE, ROTATE=True, **_triton_kw):  # noqa: N803
    """The quantiser with the reference's arguments: for PRE_GELU `s` is the GELU table, for PRE_MOD / PRE_LNMOD
    `s` is bf16(1 + scale) and `h` the shift; ROTATE (not in the reference, which always rotates) selects the plain
    per-token quantiser."""
    rows = x.numel() // K
    table = s if PRE == PRE_GELU else None
    s1 = s if PRE in (PRE_MOD, PRE_LNMOD) else None
    sh = h if PRE in (PRE_MOD, PRE_LNMOD) else None
    with _ext.on_device(x.device):
        rc = _ext.lib().wf_quant_rows(x.data_ptr(), _p(s1), _p(sh), _p(table), q.data_ptr(), sc.data_ptr(), rows,
                                      int(K), int(rows_per_group), float(eps), int(PRE), int(bool(ROTATE)),
                                      _stream(x))
    _ext.check(rc, "wf_quant_rows")


def _get_kernels():
    """The launchers (built once; raises ExtensionMissing when the CUDA library is not built)."""
    if _kernels:
        return _kernels
    _ext.lib()
    _kernels.update(mod=_Launcher(_mod), quant_row=_Launcher(_quant_row), rms128=_Launcher(_rms128),
                    lnmod=_Launcher(_lnmod))
    return _kernels


def quantize_rows(x2d, pre=PRE_NONE, s1=None, shift=None, gelu=None, rows_per_group=1, eps=0.0, rotate=False):
    """Per-token int8 quantisation of a contiguous bf16 [m, k]: (x_q int8 [m, k], x_s float32 [m, 1])."""
    m, k = x2d.shape
    x_q = torch.empty((m, k), dtype=torch.int8, device=x2d.device)
    x_s = torch.empty((m, 1), dtype=torch.float32, device=x2d.device)
    s = gelu if pre == PRE_GELU else s1
    _get_kernels()["quant_row"][(m,)](x2d, s, shift, x_q, x_s, rows_per_group, eps, K=k, PRE=pre, ROTATE=rotate)
    return x_q, x_s
