"""Fused element-wise work of the Cosmos-Predict2 / Anima DiT block on B200 (drop-in for enhancers/fused_block.py of
ComfyUI-WeightFerry): the same public functions, part switches and install entry point, over the sm_100a kernels.

* ``modulate(normed, scale, shift)`` (reference :103-124): ``normed * (1 + scale) + shift`` for (B, T, H, W, D) with
  (B, T, 1, 1, D) scale / shift in bf16 -- one pass, bf16 rounding after the product and after the sum exactly like
  PyTorch's two kernels. Other shapes / dtypes: PyTorch's expression, counted as a fallback.
* ``ln_modulate(norm, x, scale, shift)`` (:165-179): LayerNorm (no affine) + modulate in one pass (kernel A),
  PyTorch's vectorized Welford order reproduced; when not eligible, norm(x) then modulate().
* ``rms_norm_128(x, weight, eps, rs=0)`` (:127-139): RMSNorm over rows of 128, or None when not eligible.
* the self-attention's q / k RMSNorm + 3D RoPE is ``sage_fused.rms_rope`` (kernel B).
* ``PARTS``, ``wanted_parts()`` (WEIGHTFERRY_FUSED_BLOCK), ``stats(reset=False)``, ``install(parts=None)``.

``install`` patches ComfyUI's Cosmos ``Block.forward`` (comfy/ldm/cosmos/predict2.py) with ``_block_forward`` when
ComfyUI is present; the block body itself (adaLN chunks, the three sub-layers, the gated residuals) is
``block_forward_fused`` in streaming/cosmos_block.py, shared with the streamed / tensor-parallel stack.
"""

import torch

from .. import _ext
from ..core import env as _env
from ..utils.logging import log_info, log_warn
from .fused_kernels import _get_kernels, _kernels  # noqa: F401 -- re-exported like the reference
from .fused_state import _count, _state, _stats, _tls  # noqa: F401

PARTS = ("mod", "qkv", "nhd", "modq", "gelu", "rms", "res", "ln", "tay", "smk")
DEFAULT_PARTS = PARTS
# parts this package implements on B200 (nhd / smk are SageAttention-side, tay is TaylorSeer: outside the path)
_B200_PARTS = ("mod", "qkv", "modq", "gelu", "rms", "res", "ln")


def stats(reset=False):
    out = {k: dict(v) for k, v in _stats.items()}
    if reset:
        _stats.clear()
    return out


def wanted_parts():
    """WEIGHTFERRY_FUSED_BLOCK: 1 / unset / all = every part (default), 0 = off, or a comma separated list."""
    v = (_env.get("WEIGHTFERRY_FUSED_BLOCK") or "1").strip().lower()
    if v in ("", "0", "off", "false"):
        return ()
    if v in ("1", "on", "true"):
        return DEFAULT_PARTS
    if v == "all":
        return PARTS
    return tuple(p for p in (s.strip() for s in v.split(",")) if p in PARTS)


def modulate(normed, scale, shift):
    """normed * (1 + scale) + shift for normed (B, T, H, W, D) and scale / shift (B, T, 1, 1, D), all bfloat16; or
    normed (B, N, D) with scale / shift (B, 1, D) (the row path)."""
    if normed.dim() == 3 and scale.dim() == 3:
        B3, N3, D3 = normed.shape
        if normed.is_contiguous() and tuple(scale.shape) == (B3, 1, D3) and tuple(shift.shape) == (B3, 1, D3):
            return modulate(normed.view(B3, 1, 1, N3, D3), scale.view(B3, 1, 1, 1, D3),
                            shift.view(B3, 1, 1, 1, D3)).view(B3, N3, D3)
        _count("mod", False, "3-D input not contiguous")
        return normed * (1 + scale) + shift
    B, T, H, W, D = normed.shape
    if (normed.dtype != torch.bfloat16 or scale.dtype != torch.bfloat16 or shift.dtype != torch.bfloat16
            or not normed.is_cuda or not normed.is_contiguous() or tuple(scale.shape) != (B, T, 1, 1, D)
            or tuple(shift.shape) != (B, T, 1, 1, D) or D % 8):
        _count("mod", False, f"{normed.dtype}/{scale.dtype}/{shift.dtype} contiguous={normed.is_contiguous()}")
        return normed * (1 + scale) + shift
    _count("mod", True)
    one_plus = (1 + scale).contiguous()  # the same small bf16 tensor PyTorch makes
    out = torch.empty_like(normed)
    _get_kernels()["mod"][(B * T * H * W,)](normed, one_plus, shift.contiguous(), out, D, H * W)
    return out


def gated_residual(x, gate_rows, o, rows_per_group, out=None):
    """x + gate * o for (n, D) rows x and o, the gate row of row r being gate_rows[r // rows_per_group] -- ComfyUI's
    bf16 addcmul (the block's _add_residual, reference :527-532) in one vectorised kernel with the same bits; out may
    be x. Other dtypes / layouts take PyTorch's addcmul."""
    n, D = x.shape
    if (x.dtype == torch.bfloat16 and o.dtype == torch.bfloat16 and gate_rows.dtype == torch.bfloat16 and x.is_cuda
            and x.is_contiguous() and o.is_contiguous() and gate_rows.is_contiguous() and D % 8 == 0
            and tuple(o.shape) == (n, D) and gate_rows.shape[-1] == D and rows_per_group > 0
            and gate_rows.shape[0] * rows_per_group >= n):
        if out is None:
            out = torch.empty_like(x)
        with torch.cuda.device(x.device):
            rc = _ext.lib().wf_gated_residual(x.data_ptr(), gate_rows.data_ptr(), o.data_ptr(), out.data_ptr(), n, D,
                                              int(rows_per_group), _ext.stream_of(x.device))
        _ext.check(rc, "wf_gated_residual")
        return out
    g = gate_rows.repeat_interleave(rows_per_group, dim=0)[:n]
    res = torch.addcmul(x, g.to(x.dtype), o.to(x.dtype))
    if out is not None:
        out.copy_(res)
        return out
    return res


def rms_norm_128(x, weight, eps, rs=0):
    """torch.nn.functional.rms_norm(x, (128,), weight, eps) for bf16 x (..., 128) and a bf16 weight; None when not
    eligible (the caller runs PyTorch's)."""
    if (x.dtype != torch.bfloat16 or not x.is_cuda or x.shape[-1] != 128 or not x.is_contiguous() or weight is None
            or weight.dtype != torch.bfloat16 or tuple(weight.shape) != (128,) or weight.device != x.device
            or eps is None):
        return None
    n = x.numel() // 128
    out = torch.empty_like(x)
    _get_kernels()["rms128"][(n,)](x, weight.contiguous(), out, n, float(eps), RS=rs)
    return out


_LN_ANY_WIDTH = False  # True: kernel A for any width % 512 (not only the powers of 2 the reference fuses)


def _ln_ok(norm, x):
    """The LayerNorm can run inside kernel A: a LayerNorm without affine on a contiguous bf16 CUDA input whose rows
    PyTorch's vectorized kernel splits like the reproduction (multiples of 512; a power of 2 unless _LN_ANY_WIDTH)."""
    k = x.shape[-1]
    return ("ln" in _state["parts"] and isinstance(norm, torch.nn.LayerNorm) and "forward" not in norm.__dict__
            and norm.weight is None and norm.bias is None and len(norm.normalized_shape) == 1
            and k == norm.normalized_shape[0] and k % 512 == 0 and k <= 8192
            and (_LN_ANY_WIDTH or not k & (k - 1))
            and x.dtype == torch.bfloat16 and x.is_cuda and x.is_contiguous()
            and len(getattr(norm, "weight_function", ())) == 0 and len(getattr(norm, "bias_function", ())) == 0)


def ln_modulate_rows(x, scale, shift, eps):
    """Kernel A on (B, T, H, W, D) bf16 x with (B, T, 1, 1, D) scale / shift: LayerNorm(x) * (1 + scale) + shift."""
    B, T, H, W, D = x.shape
    out = torch.empty_like(x)
    _get_kernels()["lnmod"][(B * T * H * W,)](x, (1 + scale).contiguous(), shift.contiguous(), out, H * W,
                                               float(eps), K=D)
    return out


def ln_modulate(norm, x, scale, shift):
    """norm(x) * (1 + scale) + shift, in one pass when allowed (ln), else with the fused scale-and-shift (mod), else
    PyTorch's."""
    if _ln_ok(norm, x) and x.dim() == 5:
        B, T, H, W, D = x.shape
        if (scale.dtype == torch.bfloat16 and shift.dtype == torch.bfloat16
                and tuple(scale.shape) == (B, T, 1, 1, D) and tuple(shift.shape) == (B, T, 1, 1, D)):
            _count("ln", True)
            return ln_modulate_rows(x, scale, shift, norm.eps)
    if "mod" in _state["parts"]:
        return modulate(norm(x), scale, shift)
    return norm(x) * (1 + scale) + shift


def _block_forward(self, x_B_T_H_W_D, emb_B_T_D, crossattn_emb, rope_emb_L_1_1_D=None, adaln_lora_B_T_3D=None,
                   extra_per_block_pos_emb=None, transformer_options={}):
    """ComfyUI's Block.forward with the fused parts (reference :632-649); the body is shared with the streamed
    stack (streaming/cosmos_block.py)."""
    if "mod" not in _state["parts"]:
        return _state["orig"]["forward"](self, x_B_T_H_W_D, emb_B_T_D, crossattn_emb, rope_emb_L_1_1_D,
                                         adaln_lora_B_T_3D, extra_per_block_pos_emb, transformer_options)
    from ..streaming.cosmos_block import block_forward_fused
    return block_forward_fused(self, x_B_T_H_W_D, emb_B_T_D, crossattn_emb, rope_emb_L_1_1_D, adaln_lora_B_T_3D,
                               extra_per_block_pos_emb, transformer_options)


def install(parts=None):
    """Patch ComfyUI's Cosmos Block for the given parts (default: WEIGHTFERRY_FUSED_BLOCK). Idempotent; install(())
    restores ComfyUI's method. Returns the parts in force (() without ComfyUI)."""
    parts = tuple(wanted_parts() if parts is None else parts)
    parts = tuple(p for p in parts if p in _B200_PARTS)
    if "modq" in parts and "mod" not in parts:
        parts = tuple(p for p in parts if p != "modq")
    try:
        import comfy.ldm.cosmos.predict2 as p2
    except Exception as exc:  # noqa: BLE001
        _state["parts"] = parts  # the kernels and the streamed stack still follow the switch
        log_warn(f"Cosmos fused block: ComfyUI's Cosmos model not found ({exc}); Block.forward not patched.")
        return ()
    if parts:
        _get_kernels()  # raises when the CUDA library is missing: no silent fallback
    if _state["orig"] is None:
        _state["orig"] = {"forward": p2.Block.forward}
    _state["parts"] = parts
    p2.Block.forward = _block_forward if "mod" in parts else _state["orig"]["forward"]
    if parts:
        log_info(f"Cosmos fused block on B200: {', '.join(parts)} (WEIGHTFERRY_FUSED_BLOCK).")
    return parts
