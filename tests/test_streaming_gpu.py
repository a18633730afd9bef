"""The streaming path on the GPU: slot ring + dequantisation on arrival gives the resident (not streamed) stack's
bits exactly, the slots hold the oracle's dequantised weights, slot reuse under 2 slots and many blocks is ordered,
the profiler's timeline is complete, and the forward hooks bind parameters to the slots."""

import numpy as np
import pytest

from conftest import oracle, wf

pytestmark = pytest.mark.gpu

SMALL = dict(hidden=1024, heads=8, head_dim=128, mlp=4096, ctx_dim=256, lora=64)


def _inputs(torch, cfg, batch, tokens, ctx_tokens, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((batch * tokens, cfg.hidden), device="cuda", generator=g).to(torch.bfloat16)
    emb = (torch.randn((batch, cfg.hidden), device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    lora = (torch.randn((batch, 3 * cfg.hidden), device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    ctx = torch.randn((batch, ctx_tokens, cfg.ctx_dim), device="cuda", generator=g).to(torch.bfloat16)
    return x, emb, lora, ctx


@pytest.mark.parametrize("slots", [2, 3])
def test_streamed_equals_resident(cuda, slots):
    import torch
    cb = wf("streaming.cosmos_block")
    stk = wf("streaming.stack")
    cfg = cb.CosmosConfig(**SMALL)
    batch, T, H, W = 2, 1, 16, 16
    tokens = T * H * W
    rope = cb.rope3d_table(T, H, W, device="cuda")
    x, emb, lora, ctx = _inputs(torch, cfg, batch, tokens, 64, 5)
    streamed = stk.StreamedStack(cfg, 5, "cuda", num_slots=slots, profile=True)
    resident = stk.StreamedStack(cfg, 5, "cuda", resident=True)
    a = streamed.forward(x, emb, ctx, rope, batch, tokens, lora)
    b = resident.forward(x, emb, ctx, rope, batch, tokens, lora)
    a2 = streamed.forward(x, emb, ctx, rope, batch, tokens, lora)   # a second forward reuses the slots
    torch.cuda.synchronize()
    assert torch.isfinite(a.float()).all()
    assert torch.equal(a, b) and torch.equal(a, a2)
    summ = streamed.state.profile_summary()
    assert summ["forwards_recorded"] == 2
    f = summ["per_forward"][-1]
    assert f["streamed_blocks"] == 5 and f["dma_ms"] > 0 and f["dequant_lora_ms"] >= 0
    streamed.close()
    resident.close()


def test_slot_weights_are_the_oracle_dequantisation(cuda):
    import torch
    cb = wf("streaming.cosmos_block")
    stk = wf("streaming.stack")
    cfg = cb.CosmosConfig(**SMALL)
    s = stk.StreamedStack(cfg, 3, "cuda", num_slots=2)
    st = s.state
    st.begin_forward()
    st.prefetch_first_slots()
    for b in range(3):
        W = st.acquire(b)
        torch.cuda.current_stream().synchronize()
        for sp, off in zip(s.layout.specs, s.layout.offsets):
            if sp.qtype is None or "adaln" in sp.name:
                continue
            raw = s.host_flats[b][off:off + sp.packed_bytes].numpy()
            ref = oracle().dequant_gguf(raw, sp.numel, sp.qtype, 0, 1)
            got = W[sp.name].contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
            assert np.array_equal(got, ref), (b, sp.name)
        st.release(b)
    st.end_forward()
    s.close()


def test_block_hooks_bind_slot_weights(cuda):
    """install_block_stream_hooks on plain torch blocks: each forward sees its block's dequantised weights."""
    import torch
    state_mod = wf("streaming.state")
    cb = wf("streaming.cosmos_block")
    ph = wf("core.tiers.pinned")
    n_blocks, dim = 4, 256
    specs = [state_mod.ParamSpec("lin.weight", (dim, dim), qtype=8)]
    layout = state_mod.BlockLayout(specs)
    holders, flats, dense = [], [], []
    for b in range(n_blocks):
        g = torch.Generator().manual_seed(b)
        q = torch.randint(-127, 128, (dim, dim), dtype=torch.int16, generator=g).to(torch.int8)
        d = (torch.rand((dim, dim // 32), generator=g) * 0.01).half()
        packed = cb.q8_0_pack(q, d).reshape(-1)
        h = ph.PinnedHost(layout.flat_bytes)
        h.tensor[:packed.numel()].copy_(packed)
        holders.append(h)
        flats.append(h.tensor)
        dense.append(torch.from_numpy(oracle().dequant_gguf(packed.numpy(), dim * dim, 8, 0, 1).view(np.int16))
                     .view(torch.bfloat16).reshape(dim, dim))

    class Blk(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = torch.nn.Linear(dim, dim, bias=False, device="cuda", dtype=torch.bfloat16)

        def forward(self, x):
            return self.lin(x)

    blocks = torch.nn.ModuleList([Blk() for _ in range(n_blocks)])
    st = state_mod._StreamState("cuda", flats, layout, num_slots=2)
    handles = state_mod.install_block_stream_hooks(blocks, st)
    x = torch.randn((8, dim), device="cuda").to(torch.bfloat16)
    st.begin_forward()
    y = x
    for blk in blocks:
        y = blk(y)
    ref = x
    for w in dense:
        ref = torch.nn.functional.linear(ref, w.cuda())
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    for h in handles:
        h.remove()
    ph.release_all(holders)


def test_close_right_after_forward_waits_for_transfers(cuda):
    """close() straight after a forward with no synchronisation: the transfer and dequant streams are idle when it
    returns (their copies read pinned host buffers that are unregistered next), and a new stack built on the freed
    memory gives the same bits."""
    import torch
    cb = wf("streaming.cosmos_block")
    stk = wf("streaming.stack")
    cfg = cb.CosmosConfig(**SMALL)
    batch, T, H, W = 2, 1, 8, 8
    tokens = T * H * W
    rope = cb.rope3d_table(T, H, W, device="cuda")
    x, emb, lora, ctx = _inputs(torch, cfg, batch, tokens, 16, 9)
    outs = []
    for _ in range(2):
        s = stk.StreamedStack(cfg, 6, "cuda", num_slots=2)
        y = s.forward(x, emb, ctx, rope, batch, tokens, lora)
        st = s.state
        s.close()
        assert st.copy_stream.query() and st.dequant_stream.query()
        outs.append(y)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
