"""The ComfyUI block drop-in on the CPU, against the stand-in of ComfyUI's Cosmos classes (tests/fake_comfy.py):
install() patches Block.forward / Attention.compute_qkv / GPT2FeedForward.forward and install(()) restores them; on
CPU tensors no kernel is eligible, so every fused part hands its call back to ComfyUI's code -- and the patched
forward, which still routes every sub-layer through the block's own modules, must give ComfyUI's bits exactly (the
same modules called with the same inputs in the same order, residual dtype and mlp_patch honoured)."""

import pytest

import fake_comfy
from conftest import wf


@pytest.fixture()
def p2():
    fb = wf("enhancers.fused_block")  # imported before the stand-in exists: no install at import
    mod = fake_comfy.register()
    saved = (fb._state["parts"], fb._state["orig"])
    fb._state["orig"] = None
    yield mod
    fb.install(())
    fb._state["parts"], fb._state["orig"] = saved
    fake_comfy.unregister()


def _run(blk, inputs, opts=None):
    x, emb, ctx, rope, lora = inputs
    return blk(x, emb, ctx, rope, lora, None, opts or {})


def test_install_patches_and_restores(p2):
    fb = wf("enhancers.fused_block")
    orig = (p2.Block.forward, p2.Attention.compute_qkv, p2.GPT2FeedForward.forward)
    parts = fb.install()
    assert set(parts) == {"mod", "qkv", "modq", "gelu", "rms", "res", "ln"}
    assert p2.Block.forward is fb._block_forward
    assert p2.Attention.compute_qkv is fb._compute_qkv
    assert p2.GPT2FeedForward.forward is fb._mlp_forward
    assert fb.install() == parts  # idempotent
    assert fb.install(()) == ()
    assert (p2.Block.forward, p2.Attention.compute_qkv, p2.GPT2FeedForward.forward) == orig
    assert fb.install(("rms",)) == ("rms",)  # only the attention norms
    assert p2.Block.forward is orig[0] and p2.Attention.compute_qkv is fb._compute_qkv


@pytest.mark.parametrize("weights", ["bf16", "int8"])
@pytest.mark.parametrize("lora", [True, False])
def test_cpu_patched_forward_is_comfyui(p2, weights, lora):
    import torch
    fb = wf("enhancers.fused_block")
    blk = fake_comfy.build_block(p2, weights, x_dim=512, ctx_dim=256, heads=4, mlp_dim=1024, lora=lora,
                                 device="cpu", seed=3)
    inputs = fake_comfy.block_inputs(x_dim=512, ctx_dim=256, H=4, W=8, S=8, device="cpu", lora=lora)
    with torch.no_grad():
        want = _run(blk, inputs)
        fb.install()
        got = _run(blk, inputs)
        patch_calls = []

        def mlp_patch(args):
            patch_calls.append(args["x"].shape)
            return {"x": args["x"] * 0.5, "transformer_options": args["transformer_options"]}
        opts = {"patches": {"mlp_patch": [mlp_patch]}}
        got_p = _run(blk, inputs, opts)
        fb.install(())
        want_p = _run(blk, inputs, opts)
    assert torch.equal(got, want)
    assert torch.equal(got_p, want_p) and len(patch_calls) == 2
    # the layers ran their own code: no _forward override or norm forward is left behind
    for lin in (blk.self_attn.q_proj, blk.mlp.layer2, blk.cross_attn.output_proj):
        assert "_forward" not in lin.__dict__
    assert "forward" not in blk.cross_attn.q_norm.__dict__


def test_cpu_residual_dtype_float32(p2):
    """A float32 residual stream with a bf16 compute dtype: ComfyUI's dtype handling is kept."""
    import torch
    fb = wf("enhancers.fused_block")
    blk = fake_comfy.build_block(p2, "bf16", x_dim=512, ctx_dim=256, heads=4, mlp_dim=1024, device="cpu", seed=5)
    x, emb, ctx, rope, lora = fake_comfy.block_inputs(x_dim=512, ctx_dim=256, H=4, W=4, S=8, device="cpu")
    x = x.float()
    with torch.no_grad():
        want = blk(x, emb, ctx, rope, lora)
        fb.install()
        got = blk(x, emb, ctx, rope, lora)
    assert got.dtype == torch.float32 and torch.equal(got, want)


def test_stats_report_fallbacks_on_cpu(p2):
    import torch
    fb = wf("enhancers.fused_block")
    blk = fake_comfy.build_block(p2, "int8", x_dim=512, ctx_dim=256, heads=4, mlp_dim=1024, device="cpu", seed=7)
    inputs = fake_comfy.block_inputs(x_dim=512, ctx_dim=256, H=4, W=4, S=8, device="cpu")
    fb.stats(reset=True)
    fb.install()
    with torch.no_grad():
        _run(blk, inputs)
    st = fb.stats(reset=True)
    assert st["qkv"]["used"] == 0 and st["qkv"]["fallback"] > 0 and st["qkv"]["why"]
    assert st["mod"]["used"] == 0 and st["mod"]["fallback"] > 0
