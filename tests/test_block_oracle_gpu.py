"""The streamed stack's block (streaming/cosmos_block.block_forward, single GPU) against the block-level oracle
(oracle/block.py: the oracle's restatements of the kernels plus float64 GEMMs, attention and activations, rounded to
bf16 where the GPU stores bf16), at a reduced configs[4] shape: Cosmos-14B widths (hidden 5120, 40 heads x 128, MLP
20480, context 1024, AdaLN-LoRA 256), 2 x 64 tokens, 2 Q8_0 blocks streamed through the slot ring.

Tolerance, stated against the oracle's y_ref, per element of the two blocks' output y and per row r of y_ref:
  |y - y_ref| <= 0.12 * rms(y_ref[r])              for every element (15 bf16 ulps of the row's scale; measured
                                                   0.082, 99.9 % of elements within 0.04),
  mean |y - y_ref| <= 0.006 * mean rms(y_ref)     over the whole output (about 1.5 bf16 ulps; measured 0.0041), and
  ||(y - x) - (y_ref - x)|| <= 1e-2 ||y_ref - x||  for the blocks' update as a whole (x the blocks' input;
                                                   measured 6.7e-3),
the last one sensitive to a wrong sub-layer. Every rounding of the two paths is a bf16 one, in different places (the
GPU's float32 accumulation and approximate reciprocal square roots against float64 and exact ones), over two blocks
whose update is about 12 times their input. The scale is the row's, not the element's: elements near zero are the
difference of large terms, whose rounding the GPU and the oracle do in different places."""

import numpy as np
import pytest

from conftest import wf

pytestmark = pytest.mark.gpu


def test_stack_blocks_match_block_oracle(cuda):
    import importlib
    import torch
    ob = importlib.import_module("oracle.block")
    cb = wf("streaming.cosmos_block")
    stk = wf("streaming.stack")
    cfg = cb.CosmosConfig()  # Cosmos-Predict2-14B widths
    batch, T, H, W, S = 2, 1, 8, 8, 32
    tokens = T * H * W
    g = torch.Generator(device="cuda").manual_seed(41)
    x = torch.randn((batch * tokens, cfg.hidden), device="cuda", generator=g).to(torch.bfloat16)
    emb = (torch.randn((batch, cfg.hidden), device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    lora = (torch.randn((batch, 3 * cfg.hidden), device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    ctx = torch.randn((batch, S, cfg.ctx_dim), device="cuda", generator=g).to(torch.bfloat16)
    rope = cb.rope3d_table(T, H, W, device="cuda")
    stack = stk.StreamedStack(cfg, 2, "cuda", seed=505, num_slots=2)
    y = stack.forward(x, emb, ctx, rope, batch, tokens, lora)
    torch.cuda.synchronize()
    ref = x.cpu().to(torch.float64)
    for b in range(2):
        Wb = ob.dequant_block(stack.host_flats[b], stack.layout)
        ref = ob.block_forward(ref, emb.cpu(), ctx.cpu(), rope.cpu(), Wb, cfg.heads, cfg.eps, batch, tokens,
                               lora.cpu())
        del Wb
    stack.close()
    y64, x64 = y.cpu().to(torch.float64), x.cpu().to(torch.float64)
    d = (y64 - ref).abs()
    row = ref.pow(2).mean(dim=1, keepdim=True).sqrt()
    rel = d / row
    upd_err = ((y64 - x64) - (ref - x64)).norm() / (ref - x64).norm()
    print(f"max |d| / row rms {rel.max().item():.4f}, p99.9 {torch.quantile(rel.flatten()[:1 << 24], 0.999).item():.4f}, "
          f"mean {(d.mean() / row.mean()).item():.2e}, exact {float((d == 0).double().mean()):.4f}, "
          f"update rel-L2 {upd_err.item():.2e}, update / x {((ref - x64).norm() / x64.norm()).item():.3f}")
    assert torch.isfinite(y64).all()
    assert rel.max() <= 0.12, f"max |d| / row rms {rel.max().item():.4f}"
    assert d.mean() <= 0.006 * row.mean()
    assert upd_err <= 1e-2, f"update rel-L2 {upd_err.item():.3e}"
