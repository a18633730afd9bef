"""Fused element-wise work of the Cosmos-Predict2 / Anima DiT block on B200 (the role of enhancers/fused_block.py of
ComfyUI-WeightFerry): the same public functions, part switches and install entry point, over the sm_100a kernels.

* ``modulate(normed, scale, shift)`` (reference :103-124): ``normed * (1 + scale) + shift`` for (B, T, H, W, D) with
  (B, T, 1, 1, D) scale / shift in bf16 -- one pass, bf16 rounding after the product and after the sum exactly like
  PyTorch's two kernels. Other shapes / dtypes: PyTorch's expression, counted as a fallback.
* ``ln_modulate(norm, x, scale, shift)`` (:165-179): LayerNorm (no affine) + modulate in one pass (kernel A),
  PyTorch's vectorized Welford order reproduced; when not eligible, norm(x) then modulate().
* ``rms_norm_128(x, weight, eps, rs=0)`` (:127-139): RMSNorm over rows of 128, or None when not eligible.
* ``gated_residual``: the block's ``x + gate * out`` (PyTorch's bf16 addcmul) in one pass.
* ``PARTS``, ``wanted_parts()`` (WEIGHTFERRY_FUSED_BLOCK), ``stats(reset=False)``, ``install(parts=None)``.

``install`` patches ComfyUI's Cosmos classes (comfy/ldm/cosmos/predict2.py; reference :706-737):

* ``Block.forward`` -> ``_block_forward``: ComfyUI's block -- adaLN shift / scale / gate from the block's own
  modulation modules, then self-attention, cross-attention and MLP, each ``x + gate * sublayer(norm(x) * (1 + scale)
  + shift)`` -- with every sub-layer still run by the block's own modules, so that a layer's weight goes through its
  own path (ComfyUI-GGUF's dequantisation, LoRA patches, int8 QuantizedTensors). What changes is where the
  element-wise steps happen: LayerNorm + scale-and-shift in one pass (``ln`` / ``mod``) or left pending for the int8
  quantiser of the next layers (``modq``, with ``ln`` the LayerNorm too), q / k / v quantised once (``qkv``), the
  gated residual inside the output projection's int8 GEMM (``res``) or one element-wise pass;
* ``Attention.compute_qkv`` -> ``_compute_qkv``: the self-attention's q / k RMSNorm + split-half 3D RoPE in one launch
  for q and k (kernel B pair) after projections that share one quantisation; the cross-attention's q / k RMSNorm by
  the RMSNorm-128 kernel (``rms``);
* ``GPT2FeedForward.forward`` -> ``_mlp_forward``: the pending input taken by layer1's quantiser and GELU computed
  inside layer2's quantiser (``gelu``).

A part whose preconditions do not hold for a call hands that call to ComfyUI's own code; every such hand-back is
counted (``stats()``). ``transformer_options["patches"]`` turn off everything that would hide an intermediate from a
patch; ``mlp_patch`` is applied as ComfyUI applies it. The streamed / tensor-parallel stack has its own block body
(streaming/cosmos_block.py) on weights it dequantised on arrival.
"""

import torch

from .. import _ext
from ..core import env as _env
from ..utils.logging import log_info, log_warn
from . import sage_fused as _sf
from .fused_int8 import (  # noqa: F401 -- the int8 path's names stay importable from here, as in the reference
    _clear_pre, _gelu_table, _int8_linear_residual, _int8_linear_shared, _int8_proj_ok, _int8_quantised, _key2d,
    _materialise, _Overrides, _pending_for, _quantise_pre, _residual_forward, _set_pre, _shared_forward,
)
from .fused_kernels import _get_kernels, _kernels  # noqa: F401 -- re-exported like the reference
from .fused_state import COUNTERS, _count, _state, _tls  # noqa: F401

PARTS = ("mod", "qkv", "nhd", "modq", "gelu", "rms", "res", "ln", "tay", "smk")
DEFAULT_PARTS = PARTS
# parts this package implements on B200 (nhd / smk are SageAttention-side, tay is TaylorSeer: outside the path)
_B200_PARTS = ("mod", "qkv", "modq", "gelu", "rms", "res", "ln")


def stats(reset=False):
    """{part: {"used": calls fused, "fallback": calls handed to ComfyUI's code, "why": the first reason}}."""
    return COUNTERS.snapshot(reset)


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
        with _ext.on_device(x.device):
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




# ------------------------------------------------------------------------------------------------ norms of attention
def _cast_weight(mod, like):
    """(weight, release) of a ComfyUI norm module as its own forward would use it: cast to ``like``'s dtype / device
    (and through its weight patches) by comfy.ops when the module asks for that, else its parameter as it is."""
    if getattr(mod, "comfy_cast_weights", False) or getattr(mod, "weight_function", None):
        import comfy.ops
        weight, bias, stream = comfy.ops.cast_bias_weight(mod, like, offloadable=True)
        return weight, (lambda: comfy.ops.uncast_bias_weight(mod, weight, bias, stream))
    return mod.weight, (lambda: None)


def _rms_ok(norm):
    return (type(norm).__name__ == "RMSNorm" and "forward" not in norm.__dict__
            and tuple(getattr(norm, "normalized_shape", ())) == (128,) and getattr(norm, "eps", None) is not None)


def _rms_forward(mod):
    """A forward for ComfyUI's RMSNorm over rows of 128 that runs the RMSNorm-128 kernel (reference :141-162), with
    PyTorch's rms_norm for anything the kernel does not cover."""
    def forward(x):
        weight, release = _cast_weight(mod, x)
        try:
            out = rms_norm_128(x, weight, mod.eps)
            if out is None:
                _count("rms", False, f"{x.dtype} {tuple(x.shape)}")
                return torch.nn.functional.rms_norm(x, mod.normalized_shape, weight, mod.eps)
        finally:
            release()
        _count("rms", True)
        return out
    return forward


def _rope_rows(rope_emb, tokens):
    """The self-attention's rotations as the (1, tokens, 1, 64, 2, 2) float32 table kernel B reads, or None."""
    if rope_emb is None or rope_emb.dtype != torch.float32 or rope_emb.numel() != tokens * 256:
        return None
    if rope_emb.dim() == 6 and tuple(rope_emb.shape) == (1, tokens, 1, 64, 2, 2):
        return rope_emb
    return None


def _selfattn_qkv_rope(self, x, rope_emb, transformer_options):
    """ComfyUI's self-attention compute_qkv with rotary embeddings: q / k / v from their projections (one shared
    quantisation when they are int8), v's norm, then q / k RMSNorm + split-half 3D RoPE by kernel B for both in one
    launch -- or, when kernel B does not cover the case, comfy_kitchen's rms_rope_split_half as ComfyUI calls it."""
    with _Overrides((self.q_proj, self.k_proj, self.v_proj)):
        q = self.q_proj(x)
        k = self.k_proj(x)
        v = self.v_proj(x)
    q, k, v = (t.view(*t.shape[:-1], self.n_heads, self.head_dim) for t in (q, k, v))
    v = self.v_norm(v)
    q_w, q_release = _cast_weight(self.q_norm, q)
    k_w, k_release = _cast_weight(self.k_norm, k)
    try:
        f = _rope_rows(rope_emb, q.shape[1]) if q.dim() == 4 else None
        eps = self.q_norm.eps
        if f is not None and _sf.rope_ok(q, k, f, q_w, k_w, eps):
            q_out, k_out = _sf.rms_rope_pair(q, k, f, q_w, k_w, eps)
            _count("qrope", True)
            return q_out, k_out, v
        _count("qrope", False, f"q {tuple(q.shape)} {q.dtype}, rotations {tuple(rope_emb.shape)} {rope_emb.dtype}")
        import comfy.quant_ops
        q_out, k_out = comfy.quant_ops.ck.rms_rope_split_half(q, k, rope_emb, q_w, k_w, eps)
        return q_out, k_out, v
    finally:
        q_release()
        k_release()


def _compute_qkv(self, x, context=None, rope_emb=None, transformer_options={}):
    """Attention.compute_qkv with the fused parts (reference :320-346)."""
    orig = _state["orig"]["compute_qkv"]
    parts = _state["parts"]
    patches = transformer_options.get("patches", {}) if transformer_options else {}
    selfattn = getattr(self, "is_selfattn", context is None)
    if context is not None and not selfattn:
        # cross-attention: q from the (pending or modulated) block input, k / v from the text context; the q / k
        # RMSNorm-128 by the kernel
        if "rms" in parts and "attn2_patch" not in patches and _rms_ok(self.q_norm) and _rms_ok(self.k_norm):
            self.q_norm.forward = _rms_forward(self.q_norm)
            self.k_norm.forward = _rms_forward(self.k_norm)
            try:
                return orig(self, x, context, rope_emb=rope_emb, transformer_options=transformer_options)
            finally:
                self.q_norm.__dict__.pop("forward", None)
                self.k_norm.__dict__.pop("forward", None)
        return orig(self, x, context, rope_emb=rope_emb, transformer_options=transformer_options)
    if context is not None or "attn1_patch" in patches or "qkv" not in parts:
        return orig(self, x, context, rope_emb=rope_emb, transformer_options=transformer_options)
    if not all(hasattr(p, "_forward") for p in (self.q_proj, self.k_proj, self.v_proj)):
        _count("qkv", False, "projections without _forward")
        return orig(self, x, context, rope_emb=rope_emb, transformer_options=transformer_options)
    if rope_emb is not None and "rms" in parts and _rms_ok(self.q_norm) and _rms_ok(self.k_norm):
        return _selfattn_qkv_rope(self, x, rope_emb, transformer_options)
    with _Overrides((self.q_proj, self.k_proj, self.v_proj)):
        return orig(self, x, context, rope_emb=rope_emb, transformer_options=transformer_options)


# ------------------------------------------------------------------------------------------------------------ MLP
def _mlp_forward(self, x):
    """GPT2FeedForward.forward (layer1 -> GELU -> layer2) with a pending input taken by layer1's quantiser and the
    GELU computed inside layer2's quantiser (reference :424-452)."""
    orig = _state["orig"]["mlp_forward"]
    act = getattr(self, "activation", None)
    gelu_inside = ("gelu" in _state["parts"] and type(act) is torch.nn.GELU
                   and getattr(act, "approximate", "none") == "none" and _int8_proj_ok(self.layer2))
    pre = getattr(_tls, "pre", None)
    if not gelu_inside and pre is None:
        return orig(self, x)
    with _Overrides((self.layer1, self.layer2)):
        h = self.layer1(x)
        if pre is not None:
            _clear_pre()
            if not pre.used:
                # layer1 computed on the marker itself: compute it on the real input
                _count(_PART_OF_KIND[pre.kind], False, "mlp.layer1 did not take the pending input")
                h = self.layer1(pre.real().view(x.shape))
        if not (gelu_inside and h.dtype == torch.bfloat16 and h.is_cuda and h.is_contiguous()):
            return self.layer2(act(h))
        g = _set_pre(h, "gelu")
        try:
            out = self.layer2(h)
        finally:
            _clear_pre()
        if not g.used:
            _count("gelu", False, "mlp.layer2 did not take the pending input")
            out = self.layer2(act(h))
        return out


_PART_OF_KIND = {"mod": "modq", "lnmod": "ln", "gelu": "gelu"}


# ---------------------------------------------------------------------------------------------------------- block
class _BlockPass:
    """One forward of a Cosmos block with the fused parts (reference :484-532, :632-703): decides per sub-layer
    whether its input is left pending for the int8 quantisers or computed (in one pass), and whether its gated
    residual is added inside the output projection's GEMM or by one element-wise pass."""

    def __init__(self, block, transformer_options, compute_dtype, residual_dtype):
        self.block = block
        self.opts = transformer_options or {}
        self.patched = bool(self.opts.get("patches"))
        self.cd, self.rd = compute_dtype, residual_dtype
        parts = _state["parts"]
        self.parts = parts
        sa, ca, mlp = block.self_attn, block.cross_attn, block.mlp
        # the input projections that would receive a pending input all quantise it themselves (int8), and no module
        # on the way has a forward of its own that could look at the marker
        self.int8_inputs = (
            "modq" in parts and "qkv" in parts and not self.patched
            and not any("forward" in m.__dict__ or "compute_qkv" in m.__dict__ for m in (sa, ca))
            and "forward" not in mlp.__dict__
            and all(_int8_proj_ok(lin) for lin in (sa.q_proj, sa.k_proj, sa.v_proj, ca.q_proj, mlp.layer1)))

    def _pending_ok(self, t):
        return (self.int8_inputs and t.dtype == torch.bfloat16 and self.cd == torch.bfloat16 and t.is_cuda
                and t.is_contiguous())

    def _run(self, call, inp, x_res, gate, out_layer, overrides):
        """call(inp) with the residual offered to out_layer's GEMM when it can take it: (result, residual added)."""
        offer = ("res" in self.parts and out_layer is not None and not self.patched and _int8_proj_ok(out_layer)
                 and x_res.dtype == self.cd)
        slot = {"x": x_res, "gate": gate, "done": False} if offer else None
        _tls.res = slot
        try:
            layers = list(overrides) + ([(out_layer, _residual_forward)] if offer else [])
            with _Overrides(layers):
                out = call(inp)
        finally:
            _tls.res = None
        return out, bool(slot and slot["done"])

    def sub(self, norm, x, scale, shift, call, gate, out_layer, overrides=()):
        """x + gate * call(norm(x) * (1 + scale) + shift), the residual in residual_dtype."""
        if _ln_ok(norm, x) and self._pending_ok(x):
            pre = _set_pre(x, "lnmod", scale, shift, norm=norm)
            try:
                out, done = self._run(call, x, x, gate, out_layer, overrides)
            finally:
                _clear_pre()
            if pre.used:
                return self.residual(x, gate, out, done)
            _count("ln", False, "the sub-layer did not take the pending input")
        if self._pending_ok(x):
            normed = norm(x)
            pre = _set_pre(normed, "mod", scale, shift)
            try:
                out, done = self._run(call, normed, x, gate, out_layer, overrides)
            finally:
                _clear_pre()
            if pre.used:
                return self.residual(x, gate, out, done)
            _count("modq", False, "the sub-layer did not take the pending input")
            inp = pre.real()
        else:
            inp = ln_modulate(norm, x, scale, shift)
        out, done = self._run(call, inp, x, gate, out_layer, overrides)
        return self.residual(x, gate, out, done)

    def residual(self, x, gate, out, done):
        """x + gate * out (ComfyUI's addcmul in residual_dtype), or out itself when the GEMM already added it."""
        if done:
            return out
        g, o = gate.to(self.rd), out.to(self.rd)
        if "res" in self.parts and x.dim() == 5 and x.is_contiguous() and o.is_contiguous():
            B, T, H, W, D = x.shape
            if tuple(g.shape) == (B, T, 1, 1, D) and tuple(o.shape) == tuple(x.shape):
                n = B * T * H * W
                rows = gated_residual(x.view(n, D), g.reshape(B * T, D).contiguous(), o.view(n, D), H * W)
                return rows.view(x.shape)
        return torch.addcmul(x, g, o)


def _adaln(block, emb, lora):
    """(shift, scale, gate) of the three sub-layers, each (B, T, 1, 1, D), from the block's modulation modules."""
    out = []
    for mod in (block.adaln_modulation_self_attn, block.adaln_modulation_cross_attn, block.adaln_modulation_mlp):
        m = mod(emb)
        if block.use_adaln_lora:
            m = m + lora
        out.append(tuple(t.unsqueeze(2).unsqueeze(2) for t in m.chunk(3, dim=-1)))
    return out


def _block_forward(self, x_B_T_H_W_D, emb_B_T_D, crossattn_emb, rope_emb_L_1_1_D=None, adaln_lora_B_T_3D=None,
                   extra_per_block_pos_emb=None, transformer_options={}):
    """ComfyUI's Block.forward with the fused parts (reference :632-703): the same modules called with the same
    arguments in the same order."""
    if "mod" not in _state["parts"]:
        return _state["orig"]["forward"](self, x_B_T_H_W_D, emb_B_T_D, crossattn_emb, rope_emb_L_1_1_D,
                                         adaln_lora_B_T_3D, extra_per_block_pos_emb, transformer_options)
    x = x_B_T_H_W_D
    bp = _BlockPass(self, transformer_options, emb_B_T_D.dtype, x.dtype)
    if extra_per_block_pos_emb is not None:
        x = x + extra_per_block_pos_emb
    (sh_sa, sc_sa, g_sa), (sh_ca, sc_ca, g_ca), (sh_mlp, sc_mlp, g_mlp) = _adaln(self, emb_B_T_D, adaln_lora_B_T_3D)
    B, T, H, W, D = x.shape
    cd = bp.cd

    def rows(n):  # (B, T, H, W, D) -> (B, T * H * W, D)
        return n.to(cd).reshape(B, T * H * W, D)

    def attention(module, context):
        def call(n):
            out = module(rows(n), context, rope_emb=rope_emb_L_1_1_D, transformer_options=transformer_options)
            return out.reshape(B, T, H, W, D)
        return call

    x = bp.sub(self.layer_norm_self_attn, x, sc_sa, sh_sa, attention(self.self_attn, None), g_sa,
               self.self_attn.output_proj)
    x = bp.sub(self.layer_norm_cross_attn, x, sc_ca, sh_ca, attention(self.cross_attn, crossattn_emb), g_ca,
               self.cross_attn.output_proj, overrides=(self.cross_attn.q_proj,))
    patches = (transformer_options or {}).get("patches", {})
    if "mlp_patch" in patches:
        normed = ln_modulate(self.layer_norm_mlp, x, sc_mlp, sh_mlp).to(cd)
        args = {"x": normed, "transformer_options": transformer_options}
        for patch in patches["mlp_patch"]:
            args = patch(args)
        return bp.residual(x, g_mlp, self.mlp(args["x"]), False)
    return bp.sub(self.layer_norm_mlp, x, sc_mlp, sh_mlp, lambda n: self.mlp(n.to(cd)), g_mlp, self.mlp.layer2)


def install(parts=None):
    """Patch ComfyUI's Cosmos Block / Attention / GPT2FeedForward for the given parts (default:
    WEIGHTFERRY_FUSED_BLOCK). Idempotent; install(()) restores ComfyUI's methods. Returns the parts in force (()
    without ComfyUI)."""
    parts = tuple(wanted_parts() if parts is None else parts)
    parts = tuple(p for p in parts if p in _B200_PARTS)
    if "modq" in parts and "mod" not in parts:  # the pending inputs live in the fused block forward
        parts = tuple(p for p in parts if p != "modq")
    try:
        import comfy.ldm.cosmos.predict2 as p2
    except Exception as exc:  # noqa: BLE001
        _state["parts"] = parts  # the kernels and the streamed stack still follow the switch
        log_warn(f"Cosmos fused block: ComfyUI's Cosmos model not found ({exc}); nothing patched.")
        return ()
    if parts:
        _get_kernels()  # raises when the CUDA library is missing: no silent fallback
    if _state["orig"] is None:
        current = {"forward": p2.Block.forward, "compute_qkv": p2.Attention.compute_qkv,
                   "mlp_forward": p2.GPT2FeedForward.forward}
        if any(fn in (_block_forward, _compute_qkv, _mlp_forward) for fn in current.values()):
            raise RuntimeError("Cosmos fused block: ComfyUI's classes are patched but their own methods were lost")
        _state["orig"] = current
    orig = _state["orig"]
    _state["parts"] = parts
    p2.Block.forward = _block_forward if "mod" in parts else orig["forward"]
    p2.Attention.compute_qkv = _compute_qkv if ("qkv" in parts or "rms" in parts) else orig["compute_qkv"]
    p2.GPT2FeedForward.forward = _mlp_forward if ("gelu" in parts or "modq" in parts) else orig["mlp_forward"]
    if parts:
        log_info(f"Cosmos fused block on B200: {', '.join(parts)} (WEIGHTFERRY_FUSED_BLOCK).")
    return parts


def uninstall():
    """Restore ComfyUI's methods."""
    return install(())
