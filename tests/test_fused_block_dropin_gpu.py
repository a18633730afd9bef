"""The ComfyUI block drop-in on the GPU, against the stand-in of ComfyUI's Cosmos classes (tests/fake_comfy.py),
whose int8 linear is the oracle's quantiser + an exact integer GEMM + the float32 rescale:

* parts mod, qkv, modq, gelu, res (everything but the two norm reproductions): the patched Block.forward gives the
  unpatched one's bits exactly -- for bf16 weights, int8 weights (pending scale-and-shift and GELU inside the
  quantiser, one quantisation for q / k / v, the gated residual inside the output projections' GEMM), GGUF weights
  (through ComfyUI-GGUF's own get_weight and this package's dequantisation), with and without AdaLN-LoRA, with an
  mlp_patch -- and stats() shows the int8 parts used, not handed back;
* every part (with kernel A's LayerNorm inside the quantiser and kernel B's q / k RMSNorm + RoPE): the block output
  stays within max |d| <= 0.02 * max |ref| and mean |d| <= 1e-3 * mean |ref| of the unpatched one -- the two norm
  kernels reproduce PyTorch's LayerNorm / comfy_kitchen's rms_rope bit for bit on all but a small fraction of rows
  (test_fused_gpu.py), and the stand-in's rms_rope is plain float32 PyTorch."""

import zlib

import numpy as np
import pytest

import fake_comfy
import fake_gguf_ops as fg
from conftest import wf

pytestmark = pytest.mark.gpu

NO_NORMS = ("mod", "qkv", "modq", "gelu", "res")


@pytest.fixture()
def p2(cuda):
    fb = wf("enhancers.fused_block")  # imported before the stand-in exists: no install at import
    mod = fake_comfy.register()
    saved = (fb._state["parts"], fb._state["orig"])
    fb._state["orig"] = None
    yield mod
    fb.install(())
    fb._state["parts"], fb._state["orig"] = saved
    fake_comfy.unregister()


def _both(fb, blk, inputs, parts, opts=None):
    """(patched output, unpatched output, stats of the patched run)."""
    import torch
    x, emb, ctx, rope, lora = inputs
    with torch.no_grad():
        fb.install(parts)
        fb.stats(reset=True)
        got = blk(x, emb, ctx, rope, lora, None, opts or {})
        st = fb.stats(reset=True)
        fb.install(())
        want = blk(x, emb, ctx, rope, lora, None, opts or {})
    torch.cuda.synchronize()
    return got, want, st


def _gguf_maker(device):
    import torch
    gd = wf("enhancers.gguf_dequant")
    gd.install(force=True)

    def make(name, n_out, n_in, g):
        rng = np.random.default_rng(zlib.crc32(name.encode()))
        if name.startswith("adaln"):
            w = (rng.standard_normal((n_out, n_in)) * 0.01).astype(np.float32)
            return fake_comfy.Linear(torch.from_numpy(w).to(torch.bfloat16).to(device))
        nb = n_out * n_in // 32
        raw = rng.integers(0, 256, size=(nb, 34), dtype=np.uint8)
        raw[:, 0:2] = (np.abs(rng.standard_normal(nb)) * 0.0002).astype(np.float16).view(np.uint8).reshape(nb, 2)
        return fg.Linear(fg.gguf_param(raw.reshape(-1), 8, (n_out, n_in), device))
    return make


@pytest.mark.parametrize("weights,lora", [("int8", True), ("int8", False), ("bf16", True), ("gguf", True)])
def test_dropin_bit_exact_without_the_norm_parts(p2, weights, lora):
    import torch
    fb = wf("enhancers.fused_block")
    if weights == "gguf":
        fg.register()
        w = _gguf_maker("cuda")
    else:
        w = weights
    try:
        blk = fake_comfy.build_block(p2, w, lora=lora, seed=11)
        inputs = fake_comfy.block_inputs(lora=lora, seed=12)
        got, want, st = _both(fb, blk, inputs, NO_NORMS)
    finally:
        if weights == "gguf":
            wf("enhancers.gguf_dequant").uninstall()
            fg.unregister()
    assert torch.isfinite(want.float()).all()
    assert torch.equal(got, want), f"{(got != want).sum().item()} values differ"
    if weights == "int8":
        assert st["qkv"]["used"] > 0 and st["modq"]["used"] >= 3 and st["gelu"]["used"] == 1
        assert st["res"]["used"] == 3 and st["res"]["fallback"] == 0
    else:
        assert st["mod"]["used"] == 3 and "res" not in st


def test_dropin_mlp_patch_bit_exact(p2):
    import torch
    fb = wf("enhancers.fused_block")
    blk = fake_comfy.build_block(p2, "int8", seed=21)
    inputs = fake_comfy.block_inputs(seed=22)
    seen = []

    def patch(args):
        seen.append(args["x"].dtype)
        return {"x": args["x"] * 2, "transformer_options": args["transformer_options"]}
    got, want, st = _both(fb, blk, inputs, NO_NORMS, {"patches": {"mlp_patch": [patch]}})
    assert torch.equal(got, want) and len(seen) == 2
    assert "res" not in st or st["res"]["used"] == 0  # patches: no fused residual, no pending inputs


@pytest.mark.parametrize("weights", ["int8", "bf16"])
def test_dropin_all_parts_close(p2, weights):
    import torch
    fb = wf("enhancers.fused_block")
    blk = fake_comfy.build_block(p2, weights, seed=31)
    inputs = fake_comfy.block_inputs(seed=32)
    got, want, st = _both(fb, blk, inputs, fb._B200_PARTS)
    d = (got.float() - want.float()).abs()
    ref = want.float().abs()
    assert d.max() <= 0.02 * ref.max(), (d.max().item(), ref.max().item())
    assert d.mean() <= 1e-3 * ref.mean(), (d.mean().item(), ref.mean().item())
    assert st["qrope"]["used"] == 1 and st["rms"]["used"] == 2
    if weights == "int8":
        assert st["ln"]["used"] == 3 and st["res"]["used"] == 3 and st["gelu"]["used"] == 1
    else:
        assert st["ln"]["used"] == 3
