"""A stand-in for the parts of ComfyUI that the fused Cosmos block patch touches (ComfyUI is absent here), registered as
``comfy``, ``comfy.ops``, ``comfy.quant_ops`` and ``comfy.ldm.cosmos.predict2`` so that ``fused_block.install()``
finds and patches it the way it patches the real classes. TEST INFRASTRUCTURE: the block semantics are those the
reference restates for ComfyUI's Cosmos-Predict2 block (enhancers/fused_block.py:632-703 of ComfyUI-WeightFerry):

* ``Block``: adaLN shift / scale / gate from ``adaln_modulation_*`` (SiLU, Linear[, Linear]) plus the AdaLN-LoRA term,
  then self-attention, cross-attention and MLP, each on ``norm(x) * (1 + scale) + shift`` in compute_dtype, the
  residual added as ``addcmul(x, gate, out)`` in the residual dtype; ``transformer_options["patches"]["mlp_patch"]``
  applied to the MLP's input;
* ``Attention``: ``compute_qkv`` (projections, v_norm, and for a self-attention with rotations comfy_kitchen's
  ``rms_rope_split_half``, else the q / k RMSNorm modules), ``compute_attention`` (``attn_op`` then
  ``output_proj``), ``forward`` calling both; ``GPT2FeedForward``: layer1, GELU, layer2;
* ``comfy.ops``: a ``Linear`` whose forward hands (input, weight, bias) to ``_forward`` after applying its
  ``weight_function`` patches, an ``RMSNorm``, ``cast_bias_weight`` / ``uncast_bias_weight``;
* ``comfy.quant_ops``: a TensorWiseINT8Layout ``QuantizedTensor`` that ``F.linear`` dispatches to the stand-in of
  comfy_kitchen's int8 linear, ``QUANT_ALGOS``, and ``ck`` with that linear and ``rms_rope_split_half``.

The stand-in kitchen int8 linear quantises each token as the reference's reproduction of comfy_kitchen's ConvRot
quantiser does (on CUDA tensors this library's quantiser, which the golden vectors pin to that reproduction bit for
bit, approximate float32 division included; on CPU tensors the oracle's restatement), multiplies exactly (float64
sums of int8 products) and rescales in float32 as (acc * x_s) * w_s before the bf16 rounding -- this library's
epilogue order (comfy_kitchen's own is closed). A drop-in test thus checks the library's GEMM, its pending inputs and
its shared quantisation against an exact product, not the quantiser itself (the golden tests do that). Its ``rms_rope_split_half`` is plain PyTorch float32 arithmetic, not kitchen's exact
summation order: only paths that both use it can be compared bit for bit."""

import sys
import types

import numpy as np
import torch
import torch.nn.functional as F

NAMES = ("comfy", "comfy.ops", "comfy.quant_ops", "comfy.ldm", "comfy.ldm.cosmos", "comfy.ldm.cosmos.predict2")


# ------------------------------------------------------------------------------------------------ kitchen stand-ins
def _oracle():
    import importlib
    return importlib.import_module("oracle.oracle")


def _quantise(x2, convrot):
    """Per-token int8 quantisation as comfy_kitchen's ConvRot quantiser does it: on CUDA tensors the library's quantiser
    (pinned bit for bit to the reference's reproduction of kitchen's, whose float32 division is the GPU's
    approximate one), on CPU tensors the oracle's restatement (exact division)."""
    if x2.is_cuda:
        import importlib
        fk = importlib.import_module("comfyui-weightferry_b200.enhancers.fused_kernels")
        q, sc = fk.quantize_rows(x2.contiguous(), rotate=convrot)
        return q, sc.view(-1)
    bits = x2.contiguous().view(torch.int16).numpy().view(np.uint16)
    q, sc = _oracle().quant_rows(bits, pre=0, rotate=convrot)
    return torch.from_numpy(q), torch.from_numpy(sc)


# Set by a benchmark: on CUDA tensors the stand-in int8 linear then runs as a kernel would -- this library's
# quantiser and W8A8 GEMM, the place of comfy_kitchen's compiled one -- instead of the exact float64 product the tests
# compare against.
FAST_INT8 = False


def kitchen_int8_linear(x, qt, bias=None):
    """bf16(((float(q(x) @ w_q^T)) * x_s) * w_s) with q(x) the per-token quantisation of _quantise (ConvRot when
    the weight says so) and the product summed exactly."""
    w_q, w_s = TensorWiseINT8Layout.get_plain_tensors(qt)
    if FAST_INT8 and x.is_cuda:
        import importlib
        fi = importlib.import_module("comfyui-weightferry_b200.enhancers.fused_int8")
        y = fi.int8_linear(x, w_q, w_s, rotate=qt._params.convrot)
        return y + bias if bias is not None else y
    k = x.shape[-1]
    q, sc = _quantise(x.reshape(-1, k), qt._params.convrot)
    acc = q.double() @ w_q.double().t()           # exact: integer sums far below 2^53
    ws = w_s.reshape(-1).float()
    ws = ws if ws.numel() == w_q.shape[0] else ws.expand(w_q.shape[0])
    y = ((acc.float() * sc.view(-1, 1)) * ws.view(1, -1)).to(torch.bfloat16)
    if bias is not None:
        y = y + bias
    return y.view(*x.shape[:-1], w_q.shape[0])


def kitchen_rms_rope_split_half(q, k, freqs, q_w, k_w, eps):
    """RMSNorm over 128 then the split-half rotation (pairs d, d + 64) by the (1, L, 1, 64, 2, 2) table, in float32."""
    def one(x, w):
        xf = x.float()
        n = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(torch.bfloat16).float()
        lo, hi = n[..., :64], n[..., 64:]
        f = freqs.to(x.device)
        y0 = f[..., 0, 0] * lo + f[..., 0, 1] * hi
        y1 = f[..., 1, 0] * lo + f[..., 1, 1] * hi
        return torch.cat([y0, y1], dim=-1).to(x.dtype)
    return one(q, q_w), one(k, k_w)


# ------------------------------------------------------------------------------------------------ comfy.quant_ops
class _Int8Params:
    def __init__(self, convrot):
        self.convrot = bool(convrot)
        self.convrot_groupsize = 256
        self.transposed = False


class QuantizedTensor:
    """An int8 weight [n, k] with per-channel (or one) float32 scale; F.linear on it runs the kitchen stand-in."""

    def __init__(self, w_q, w_scale, convrot=True):
        self._qdata, self._scale = w_q, w_scale
        self._layout_cls = "TensorWiseINT8Layout"
        self._params = _Int8Params(convrot)
        self.shape = w_q.shape
        self.dtype = torch.bfloat16
        self.device = w_q.device

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func is F.linear:
            x, w = args[0], args[1]
            b = args[2] if len(args) > 2 else kwargs.get("bias")
            return kitchen_int8_linear(x, w, b)
        return NotImplemented


class TensorWiseINT8Layout:
    @staticmethod
    def get_plain_tensors(qt):
        return qt._qdata, qt._scale


QUANT_ALGOS = {"int8_tensorwise": {"quantize_input": False}}


# ------------------------------------------------------------------------------------------------ comfy.ops
def run_every_op():
    pass


def cast_bias_weight(s, input=None, dtype=None, device=None, bias_dtype=None, offloadable=False):
    """The module's weight / bias with its weight patches applied, cast to the input's dtype and device."""
    weight = s.weight
    if weight is not None and not isinstance(weight, QuantizedTensor):
        for fn in getattr(s, "weight_function", ()):
            weight = fn(weight)
        if input is not None:
            weight = weight.to(dtype=dtype or input.dtype, device=device or input.device)
    bias = getattr(s, "bias", None)
    if bias is not None and input is not None:
        bias = bias.to(dtype=bias_dtype or input.dtype, device=device or input.device)
    return (weight, bias, None) if offloadable else (weight, bias)


def uncast_bias_weight(s, weight, bias, offload_stream):
    pass


class Linear(torch.nn.Module):
    """Linear layer that prepares (input, weight, bias) and hands them to ``_forward``."""

    def __init__(self, weight, bias=None, quant_format=None):
        super().__init__()
        if isinstance(weight, QuantizedTensor):
            self.weight = weight
        else:
            self.weight = torch.nn.Parameter(weight, requires_grad=False)
        self.bias = None if bias is None else torch.nn.Parameter(bias, requires_grad=False)
        self.weight_function = []
        self.bias_function = []
        self.comfy_cast_weights = False
        self.quant_format = quant_format

    def _forward(self, input, weight, bias):
        return F.linear(input, weight, bias)

    def forward(self, input):
        run_every_op()
        if isinstance(self.weight, QuantizedTensor):
            return self._forward(input, self.weight, self.bias)
        weight, bias = cast_bias_weight(self, input)
        return self._forward(input, weight, bias)


class RMSNorm(torch.nn.Module):
    def __init__(self, dim, eps=1e-6, weight=None):
        super().__init__()
        self.normalized_shape = (dim,)
        self.eps = eps
        self.weight = torch.nn.Parameter(weight, requires_grad=False)
        self.weight_function = []
        self.bias_function = []
        self.comfy_cast_weights = False

    def forward(self, x):
        w, _b = cast_bias_weight(self, x)
        return F.rms_norm(x, self.normalized_shape, w, self.eps)


# ------------------------------------------------------------------------------------------------ predict2
def torch_attention_op(q, k, v, transformer_options={}):
    """softmax(q k^T / sqrt(d)) v for (B, S, H, D) inputs -> (B, S, H * D)."""
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
    b, h, s, d = o.shape
    return o.transpose(1, 2).reshape(b, s, h * d)


class Attention(torch.nn.Module):
    def __init__(self, linears, n_heads, head_dim, q_norm_w, k_norm_w, selfattn):
        super().__init__()
        self.is_selfattn = selfattn
        self.n_heads, self.head_dim = n_heads, head_dim
        self.q_proj, self.k_proj, self.v_proj, self.output_proj = linears
        self.q_norm = RMSNorm(head_dim, 1e-6, q_norm_w)
        self.k_norm = RMSNorm(head_dim, 1e-6, k_norm_w)
        self.v_norm = torch.nn.Identity()
        self.output_dropout = torch.nn.Identity()
        self.attn_op = torch_attention_op

    def compute_qkv(self, x, context=None, rope_emb=None, transformer_options={}):
        q = self.q_proj(x)
        src = x if context is None else context
        k = self.k_proj(src)
        v = self.v_proj(src)
        q, k, v = (t.view(*t.shape[:-1], self.n_heads, self.head_dim) for t in (q, k, v))
        v = self.v_norm(v)
        if self.is_selfattn and rope_emb is not None:
            q_w, _, _ = cast_bias_weight(self.q_norm, q, offloadable=True)
            k_w, _, _ = cast_bias_weight(self.k_norm, k, offloadable=True)
            q, k = sys.modules["comfy.quant_ops"].ck.rms_rope_split_half(q, k, rope_emb, q_w, k_w, self.q_norm.eps)
        else:
            q, k = self.q_norm(q), self.k_norm(k)
        return q, k, v

    def compute_attention(self, q, k, v, transformer_options={}):
        return self.output_dropout(self.output_proj(self.attn_op(q, k, v, transformer_options=transformer_options)))

    def forward(self, x, context=None, rope_emb=None, transformer_options={}):
        q, k, v = self.compute_qkv(x, context, rope_emb=rope_emb, transformer_options=transformer_options)
        return self.compute_attention(q, k, v, transformer_options=transformer_options)


class GPT2FeedForward(torch.nn.Module):
    def __init__(self, layer1, layer2):
        super().__init__()
        self.activation = torch.nn.GELU()
        self.layer1, self.layer2 = layer1, layer2

    def forward(self, x):
        return self.layer2(self.activation(self.layer1(x)))


class Block(torch.nn.Module):
    """The Cosmos block; ``make`` builds the linear layers (a callable (name, out, in) -> module)."""

    def __init__(self, x_dim, context_dim, num_heads, mlp_dim, use_adaln_lora, adaln_lora_dim, make, norm_w):
        super().__init__()
        # the sub-layer classes of the registered module, as a block of the real module uses its own module's classes
        # (which is what install() patches)
        p2 = sys.modules["comfy.ldm.cosmos.predict2"]
        Attention, GPT2FeedForward = p2.Attention, p2.GPT2FeedForward
        hd = x_dim // num_heads
        self.use_adaln_lora = use_adaln_lora
        for sub in ("self_attn", "cross_attn", "mlp"):
            setattr(self, f"layer_norm_{sub}", torch.nn.LayerNorm(x_dim, elementwise_affine=False, eps=1e-6))
        self.self_attn = Attention([make("self_attn.q_proj", x_dim, x_dim), make("self_attn.k_proj", x_dim, x_dim),
                                    make("self_attn.v_proj", x_dim, x_dim),
                                    make("self_attn.output_proj", x_dim, x_dim)],
                                   num_heads, hd, norm_w(), norm_w(), True)
        self.cross_attn = Attention([make("cross_attn.q_proj", x_dim, x_dim),
                                     make("cross_attn.k_proj", x_dim, context_dim),
                                     make("cross_attn.v_proj", x_dim, context_dim),
                                     make("cross_attn.output_proj", x_dim, x_dim)],
                                    num_heads, hd, norm_w(), norm_w(), False)
        self.mlp = GPT2FeedForward(make("mlp.layer1", mlp_dim, x_dim), make("mlp.layer2", x_dim, mlp_dim))
        for sub in ("self_attn", "cross_attn", "mlp"):
            if use_adaln_lora:
                seq = torch.nn.Sequential(torch.nn.SiLU(), make(f"adaln_{sub}.1", adaln_lora_dim, x_dim),
                                          make(f"adaln_{sub}.2", 3 * x_dim, adaln_lora_dim))
            else:
                seq = torch.nn.Sequential(torch.nn.SiLU(), make(f"adaln_{sub}.1", 3 * x_dim, x_dim))
            setattr(self, f"adaln_modulation_{sub}", seq)

    def forward(self, x_B_T_H_W_D, emb_B_T_D, crossattn_emb, rope_emb_L_1_1_D=None, adaln_lora_B_T_3D=None,
                extra_per_block_pos_emb=None, transformer_options={}):
        x = x_B_T_H_W_D
        residual_dtype, compute_dtype = x.dtype, emb_B_T_D.dtype
        if extra_per_block_pos_emb is not None:
            x = x + extra_per_block_pos_emb
        mods = []
        for sub in ("self_attn", "cross_attn", "mlp"):
            m = getattr(self, f"adaln_modulation_{sub}")(emb_B_T_D)
            if self.use_adaln_lora:
                m = m + adaln_lora_B_T_3D
            mods.append([c[:, :, None, None, :] for c in m.chunk(3, dim=-1)])
        B, T, H, W, D = x.shape

        def modulated(norm, x, scale, shift):
            return norm(x) * (1 + scale) + shift

        def as_rows(t):
            return t.to(compute_dtype).reshape(B, T * H * W, D)

        shift, scale, gate = mods[0]
        out = self.self_attn(as_rows(modulated(self.layer_norm_self_attn, x, scale, shift)), None,
                             rope_emb=rope_emb_L_1_1_D, transformer_options=transformer_options)
        x = torch.addcmul(x, gate.to(residual_dtype), out.reshape(B, T, H, W, D).to(residual_dtype))
        shift, scale, gate = mods[1]
        out = self.cross_attn(as_rows(modulated(self.layer_norm_cross_attn, x, scale, shift)), crossattn_emb,
                              rope_emb=rope_emb_L_1_1_D, transformer_options=transformer_options)
        x = torch.addcmul(x, gate.to(residual_dtype), out.reshape(B, T, H, W, D).to(residual_dtype))
        shift, scale, gate = mods[2]
        normed = modulated(self.layer_norm_mlp, x, scale, shift).to(compute_dtype)
        patches = (transformer_options or {}).get("patches", {})
        if "mlp_patch" in patches:
            args = {"x": normed, "transformer_options": transformer_options}
            for patch in patches["mlp_patch"]:
                args = patch(args)
            normed = args["x"]
        out = self.mlp(normed)
        return torch.addcmul(x, gate.to(residual_dtype), out.to(residual_dtype))


# ------------------------------------------------------------------------------------------------ registration
def register():
    """Put the stand-in modules into sys.modules (fresh classes each call); returns the predict2 module."""
    for name in NAMES:
        sys.modules.pop(name, None)
    mods = {name: types.ModuleType(name) for name in NAMES}
    ops, qo, p2 = mods["comfy.ops"], mods["comfy.quant_ops"], mods["comfy.ldm.cosmos.predict2"]
    for fn in (run_every_op, cast_bias_weight, uncast_bias_weight):
        setattr(ops, fn.__name__, fn)
    ops.Linear, ops.RMSNorm = Linear, RMSNorm
    qo.QuantizedTensor, qo.TensorWiseINT8Layout, qo.QUANT_ALGOS = QuantizedTensor, TensorWiseINT8Layout, QUANT_ALGOS
    qo.ck = types.SimpleNamespace(int8_linear=kitchen_int8_linear, rms_rope_split_half=kitchen_rms_rope_split_half)
    # fresh subclasses, so that patching their methods never leaks into another registration
    p2.Attention = type("Attention", (Attention,), {})
    p2.GPT2FeedForward = type("GPT2FeedForward", (GPT2FeedForward,), {})
    p2.Block = type("Block", (Block,), {})
    p2.torch_attention_op = torch_attention_op
    mods["comfy"].ops, mods["comfy"].quant_ops, mods["comfy"].ldm = ops, qo, mods["comfy.ldm"]
    mods["comfy.ldm"].cosmos = mods["comfy.ldm.cosmos"]
    mods["comfy.ldm.cosmos"].predict2 = p2
    sys.modules.update(mods)
    return p2


def unregister():
    for name in NAMES:
        sys.modules.pop(name, None)


# ------------------------------------------------------------------------------------------------ a test block
def build_block(p2, weights, x_dim=1024, ctx_dim=256, heads=8, mlp_dim=4096, lora=True, lora_dim=256, seed=0,
                device="cuda", convrot=True):
    """A Cosmos block of p2's classes with seeded weights: ``weights`` "bf16" (plain), "int8" (every projection and
    MLP layer an int8 QuantizedTensor, the adaLN layers bf16), or a callable (name, out, in, generator) -> module."""
    g = torch.Generator().manual_seed(seed)

    def make(name, n_out, n_in):
        if callable(weights):
            return weights(name, n_out, n_in, g)
        w = torch.randn((n_out, n_in), generator=g) * (0.02 if not name.startswith("adaln") else 0.01)
        if weights == "int8" and not name.startswith("adaln"):
            ws = w.abs().amax(dim=1) / 127.0
            w_q = torch.round(w / ws[:, None]).clamp(-127, 127).to(torch.int8)
            return Linear(QuantizedTensor(w_q.to(device), ws.float().to(device), convrot=convrot),
                          quant_format="int8_tensorwise")
        return Linear(w.to(torch.bfloat16).to(device))

    def norm_w():
        return (1 + torch.randn(128, generator=g) * 0.02).to(torch.bfloat16).to(device)

    blk = p2.Block(x_dim, ctx_dim, heads, mlp_dim, lora, lora_dim, make, norm_w)
    return blk.to(device)


def block_inputs(x_dim=1024, ctx_dim=256, B=2, T=1, H=16, W=16, S=64, seed=1, device="cuda", lora=True):
    """(x, emb, context, rope, adaln_lora) for build_block's block: bf16 activations, float32 rotations."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((B, T, H, W, x_dim), generator=g).to(torch.bfloat16).to(device)
    emb = (torch.randn((B, T, x_dim), generator=g) * 0.5).to(torch.bfloat16).to(device)
    ctx = torch.randn((B, S, ctx_dim), generator=g).to(torch.bfloat16).to(device)
    lora_t = (torch.randn((B, T, 3 * x_dim), generator=g) * 0.05).to(torch.bfloat16).to(device) if lora else None
    ang = torch.rand((T * H * W, 64), generator=g, dtype=torch.float64) * 6.283
    rot = torch.stack([torch.cos(ang), -torch.sin(ang), torch.sin(ang), torch.cos(ang)], dim=-1)
    rope = rot.reshape(1, T * H * W, 1, 64, 2, 2).float().contiguous().to(device)
    return x, emb, ctx, rope, lora_t
