"""CPU restatement of one Cosmos-Predict2 block as the streamed stack computes it (block_forward of
comfyui-weightferry_b200/streaming/cosmos_block.py, single rank). TEST INFRASTRUCTURE ONLY: the checker of
tests/test_block_oracle_gpu.py and of the tensor-parallel test; the product never imports it.

It follows the block the reference's fused forward runs (enhancers/fused_block.py:652-703 of ComfyUI-WeightFerry):
adaLN shift / scale / gate = (Linear(SiLU(emb)) -> Linear) + the AdaLN-LoRA term, then

    x <- x + gate_sa  * O_sa(attn(rope(rms(q)), rope(rms(k)), v))        q, k, v of LN(x) * (1 + scale) + shift
    x <- x + gate_ca  * O_ca(attn(rms(q), rms(k_ctx), v_ctx))             q of the modulated x, k / v of the context
    x <- x + gate_mlp * W2(GELU(W1(LN(x) * (1 + scale) + shift)))

built from the oracle's restatements where this library defines the arithmetic bit for bit (GGUF dequantisation,
LayerNorm + modulate, RMSNorm-128, RMSNorm-128 + split-half RoPE -- with a correctly rounded reciprocal square root
where the kernels use the hardware approximation), and float64 for what cuBLAS / SDPA / PyTorch compute (the GEMMs,
attention, SiLU, GELU, the gated residual), every intermediate rounded to bfloat16 where the GPU stores bfloat16.
"""

import numpy as np
import torch

from . import oracle


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _from_bits(b, shape):
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16).reshape(shape)


def _r16(t):
    """float64 -> bfloat16 value (kept as float64)."""
    return t.to(torch.float32).to(torch.bfloat16).to(torch.float64)


def dequant_block(flat, layout):
    """name -> float32 tensor (exact: bfloat16 values) of one block's weights from its packed host bytes (the oracle's
    dequantisation: GGUF mid float16, out bfloat16, as the stack's slots hold them) and plain parameters."""
    raw = flat.numpy() if torch.is_tensor(flat) else flat
    out = {}
    for sp, off in zip(layout.specs, layout.offsets):
        b = raw[off:off + sp.packed_bytes]
        if sp.qtype is None:
            out[sp.name] = torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(sp.dtype).reshape(
                sp.shape).to(torch.float32)
        else:
            bits = oracle.dequant_gguf(b, sp.numel, sp.qtype, 0, 1)
            out[sp.name] = _from_bits(bits, sp.shape).to(torch.float32)
    return out


def _linear(x, w):
    """bf16(x @ w^T), the product accumulated in float64."""
    return _r16(x.to(torch.float64) @ w.to(torch.float64).t())


def _attention(q, k, v):
    """softmax(q k^T / sqrt(d)) v for (B, L, H, d) float64 -> (B, L, H * d)."""
    s = torch.einsum("blhd,bshd->bhls", q, k) / np.sqrt(q.shape[-1])
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("bhls,bshd->blhd", p, v)
    return _r16(o.reshape(q.shape[0], q.shape[1], -1))


def _ln_mod(x, scale, shift, tokens, eps):
    """Kernel A's LayerNorm + modulate on (B * L, D) bf16 rows, scale / shift (B, D) (the oracle, bit for bit up to
    the reciprocal square root)."""
    s1 = _r16(1 + scale).to(torch.bfloat16)
    out = oracle.ln_modulate(_bits(x.to(torch.bfloat16)), _bits(s1), _bits(shift.to(torch.bfloat16)), tokens, eps)
    return _from_bits(out, x.shape).to(torch.float64)


def block_forward(x, emb, ctx, rope, W, heads, eps, batch, tokens, lora=None):
    """One block on the (batch * tokens, D) rows x (bf16 values as float64); emb (B, D), ctx (B, S, C), lora (B, 3 D)
    or None, rope the (1, tokens, 1, 64, 2, 2) float32 table, W the block's weights (dequant_block). Returns the new rows
    (float64 holding bfloat16 values)."""
    x = x.to(torch.float64)
    D = x.shape[1]
    hd = D // heads
    lora_t = torch.zeros((), dtype=torch.float64) if lora is None else lora.to(torch.float64)
    silu = _r16(torch.nn.functional.silu(emb.to(torch.float64)))
    f = rope.contiguous().numpy()

    def adaln(sub):
        h = _linear(silu, W[f"adaln_modulation_{sub}.1.weight"])
        m = _r16(_linear(h, W[f"adaln_modulation_{sub}.2.weight"]) + lora_t)
        return m.chunk(3, dim=-1)

    def residual(x, gate, o):
        g = gate.repeat_interleave(tokens, dim=0)
        return _r16(x + g * o)

    def rms(t, w):
        b = oracle.rms_norm_128(_bits(t.to(torch.bfloat16)), _bits(w.to(torch.bfloat16)), eps)
        return _from_bits(b, t.shape).to(torch.float64)

    def rms_rope(t, w):
        b = oracle.rms_rope128(_bits(t.to(torch.bfloat16)), f, w.to(torch.float32).numpy(), heads, tokens, eps)
        return _from_bits(b, t.shape).to(torch.float64)

    # self-attention
    shift, scale, gate = adaln("self_attn")
    n = _ln_mod(x, scale, shift, tokens, eps)
    q = _linear(n, W["self_attn.q_proj.weight"]).view(batch, tokens, heads, hd)
    k = _linear(n, W["self_attn.k_proj.weight"]).view(batch, tokens, heads, hd)
    v = _linear(n, W["self_attn.v_proj.weight"]).view(batch, tokens, heads, hd)
    q, k = rms_rope(q, W["self_attn.q_norm.weight"]), rms_rope(k, W["self_attn.k_norm.weight"])
    a = _attention(q, k, v).view(batch * tokens, D)
    x = residual(x, gate, _linear(a, W["self_attn.output_proj.weight"]))
    # cross-attention
    shift, scale, gate = adaln("cross_attn")
    n = _ln_mod(x, scale, shift, tokens, eps)
    q = rms(_linear(n, W["cross_attn.q_proj.weight"]).view(batch, tokens, heads, hd), W["cross_attn.q_norm.weight"])
    c = ctx.to(torch.float64)
    S = c.shape[1]
    kc = rms(_linear(c, W["cross_attn.k_proj.weight"]).view(batch, S, heads, hd), W["cross_attn.k_norm.weight"])
    vc = _linear(c, W["cross_attn.v_proj.weight"]).view(batch, S, heads, hd)
    a = _attention(q, kc, vc).view(batch * tokens, D)
    x = residual(x, gate, _linear(a, W["cross_attn.output_proj.weight"]))
    # MLP
    shift, scale, gate = adaln("mlp")
    n = _ln_mod(x, scale, shift, tokens, eps)
    h = _r16(torch.nn.functional.gelu(_linear(n, W["mlp.layer1.weight"])))
    return residual(x, gate, _linear(h, W["mlp.layer2.weight"]))
