"""The streaming node end to end on the GPU, in the reference's test shape (tests/test_streaming.py: the streamed
result bit for bit equal to the un-streamed one, in several modes): a small GGUF DiT -- Q8_0 and Q4_K weights, F32
norms and biases, one layer with dequant_dtype "target" -- built on a stand-in of ComfyUI-GGUF's ops module whose
dequantisation is this package's patch. Un-streamed, every layer dequantises its weight per use; streamed, the node
dequantises each block once on arrival into its slot. Both must give the same bits, across forwards, slot counts,
buffer modes and resident counts, and teardown must hand back a working resident model."""

import os

import numpy as np
import pytest

from conftest import wf
import fake_gguf_ops as fg

pytestmark = pytest.mark.gpu

DIM, HID, N_BLOCKS = 256, 1024, 5


def _packed(qt, n_values, rng):
    vpb, ts = (32, 34) if qt == 8 else (256, 144)
    nb = n_values // vpb
    raw = rng.integers(0, 256, size=(nb, ts), dtype=np.uint8)
    if qt == 8:
        raw[:, 0:2] = (np.abs(rng.standard_normal(nb)) * 0.002).astype(np.float16).view(np.uint8).reshape(nb, 2)
    else:
        for off in (0, 2):
            raw[:, off:off + 2] = rng.uniform(0, 0.01, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return raw.reshape(-1)


def _dit(torch, seed=7, plain=False, n_blocks=N_BLOCKS):
    rng = np.random.default_rng(seed)
    F = torch.nn.functional

    class Block(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.norm = torch.nn.Module()
            self.norm.weight = fg.plain_param(torch.from_numpy(1 + 0.02 * rng.standard_normal(DIM)).float(), "cuda")
            if plain:
                self.up = torch.nn.Linear(DIM, HID, device="cuda", dtype=torch.bfloat16)
                self.down = torch.nn.Linear(HID, DIM, device="cuda", dtype=torch.bfloat16)
            else:
                self.up = fg.Linear(fg.gguf_param(_packed(8, HID * DIM, rng), 8, (HID, DIM), "cuda"),
                                    fg.plain_param(torch.from_numpy(0.01 * rng.standard_normal(HID)).float(), "cuda"))
                self.down = fg.Linear(fg.gguf_param(_packed(12, DIM * HID, rng), 12, (DIM, HID), "cuda"),
                                      dequant_dtype="target")

        fail = False  # set on one block to make its forward raise once (a forward interrupted part way)

        def forward(self, x):
            if self.fail:
                self.fail = False
                raise RuntimeError("interrupted")
            h = F.layer_norm(x, (DIM,), weight=self.norm.weight.to(x.dtype))
            return x + self.down(F.gelu(self.up(h)))

    class DiT(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.blocks = torch.nn.ModuleList([Block() for _ in range(n_blocks)])

        def forward(self, x):
            for b in self.blocks:
                x = b(x)
            return x

    return DiT()


class _Patcher:
    """The ModelPatcher surface the node uses: clone(), model.diffusion_model, load_device."""

    def __init__(self, dit, torch):
        self.model = type("Model", (), {})()
        self.model.diffusion_model = dit
        self.load_device = torch.device("cuda", 0)
        self._torch = torch

    def clone(self):
        return _Patcher(self.model.diffusion_model, self._torch)


@pytest.fixture()
def gguf_patch(cuda):
    gd = wf("enhancers.gguf_dequant")
    fg.register()
    assert gd.install(force=True)
    yield gd
    gd.uninstall()
    fg.unregister()


def _x(torch):
    g = torch.Generator(device="cuda").manual_seed(3)
    return torch.randn((2, 64, DIM), device="cuda", generator=g).to(torch.bfloat16)


@pytest.mark.parametrize("opts", [dict(resident_blocks=1), dict(resident_blocks=1, prefetch_slots=2),
                                  dict(resident_blocks=2, prefetch_slots=4),
                                  dict(resident_blocks=1, buffer_mode="Single Buffer (Synchronous)"),
                                  dict(resident_blocks=1, pin_memory=False)])
def test_streamed_gguf_dit_is_bit_exact(gguf_patch, opts):
    import torch
    dn = wf("streaming.dit_node")
    dit = _dit(torch)
    x = _x(torch)
    with torch.inference_mode():
        ref = dit(x)
        gguf_patch.stats(reset=True)
        (patcher,) = dn.WeightFerryDiT().apply_streaming(_Patcher(dit, torch), **opts)
        st = dit._weightferry_stream_state
        assert st is not None and patcher.model.diffusion_model is dit
        n_res = opts["resident_blocks"]
        assert st.stream_idx == list(range(n_res, N_BLOCKS))
        # rest binding: the streamed weights wait in host memory between uses
        assert all(not p.is_cuda for i in st.stream_idx for p in dit.blocks[i].parameters())
        assert all(p.is_cuda for i in range(n_res) for p in dit.blocks[i].parameters())
        out1 = dit(x)
        out2 = dit(x)
        torch.cuda.synchronize()
        used = gguf_patch.stats()["used"]
    assert torch.equal(out1, ref) and torch.equal(out2, ref)
    # only the resident blocks dequantised per use (2 GGUF weights each, 2 forwards)
    assert used == 2 * 2 * n_res
    assert all(not p.is_cuda for i in st.stream_idx for p in dit.blocks[i].parameters())
    dn.teardown(dit)
    assert dit._weightferry_stream_state is None
    assert all(p.is_cuda for p in dit.parameters())
    with torch.inference_mode():
        assert torch.equal(dit(x), ref)


@pytest.mark.parametrize("n_res", [1, 2])
def test_self_managed_resident_blocks(gguf_patch, n_res):
    """resident_mode "Self-managed": the resident blocks' GGUF weights are dequantised once and bound for each whole
    forward -- the same bits as the layers' per-use dequantisation, no per-use dequantisation left, the packed
    weights back between forwards (also after a forward that raised), and teardown leaves a working model."""
    import torch
    dn = wf("streaming.dit_node")
    dit = _dit(torch)
    x = _x(torch)
    with torch.inference_mode():
        ref = dit(x)
    packed = {id(p): (p.data_ptr(), p.tensor_type) for i in range(n_res) for p in dit.blocks[i].parameters()
              if getattr(p, "tensor_type", None) is not None}
    (patcher,) = dn.WeightFerryDiT().apply_streaming(_Patcher(dit, torch), resident_blocks=n_res,
                                                      resident_mode=dn.RESIDENT_MODE_SELF)
    st = dit._weightferry_stream_state
    assert st.self_resident and len(st.res_entries) == 2 * n_res  # up (Q8_0, f16 mid) and down (Q4_K, "target")
    seen = []
    h = dit.blocks[0].register_forward_pre_hook(
        lambda m, a: seen.append(all(getattr(p, "tensor_type", None) is None and p.dtype == torch.bfloat16
                                     for n, p in m.named_parameters() if n.endswith("weight") and "norm" not in n)))
    gguf_patch.stats(reset=True)
    with torch.inference_mode():
        out1 = dit(x)
        out2 = dit(x)
    torch.cuda.synchronize()
    h.remove()
    assert torch.equal(out1, ref) and torch.equal(out2, ref)
    assert seen == [True, True]                       # bound during the forward
    assert gguf_patch.stats()["used"] == 0            # nothing dequantised per use
    assert all((p.data_ptr(), p.tensor_type) == packed[id(p)] for i in range(n_res)
               for p in dit.blocks[i].parameters() if id(p) in packed)  # packed again between forwards
    dit.blocks[n_res - 1].fail = True                  # a forward that raises inside a resident block
    with pytest.raises(RuntimeError):
        with torch.inference_mode():
            dit(x)
    with torch.inference_mode():
        assert torch.equal(dit(x), ref)
    dn.teardown(dit)
    assert all((p.data_ptr(), p.tensor_type) == packed[id(p)] for i in range(n_res)
               for p in dit.blocks[i].parameters() if id(p) in packed)
    with torch.inference_mode():
        assert torch.equal(dit(x), ref)


def test_streamed_slot_weights_are_the_layers_dequantisation(gguf_patch):
    """Inside a streamed block the bound weights are exactly what the layer's own dequantisation gives."""
    import torch
    dn = wf("streaming.dit_node")
    gd = gguf_patch
    dit = _dit(torch, seed=11)
    want = {}
    for i, blk in enumerate(dit.blocks):
        want[i] = (gd.dequantize(blk.up.weight.data, 8, (HID, DIM), None, torch.bfloat16),
                   gd.dequantize(blk.down.weight.data, 12, (DIM, HID), torch.bfloat16, torch.bfloat16))
    seen = {}

    def grab(i):
        def hook(module, args):
            seen[i] = (module.up.get_weight(module.up.weight, torch.bfloat16).clone(),
                       module.down.get_weight(module.down.weight, torch.bfloat16).clone())
        return hook

    dn.WeightFerryDiT().apply_streaming(_Patcher(dit, torch), resident_blocks=1, prefetch_slots=2)
    hs = [dit.blocks[i].register_forward_pre_hook(grab(i)) for i in range(N_BLOCKS)]  # after the node's hooks
    with torch.inference_mode():
        dit(_x(torch))
    torch.cuda.synchronize()
    for h in hs:
        h.remove()
    for i in range(N_BLOCKS):
        assert torch.equal(seen[i][0], want[i][0]) and torch.equal(seen[i][1], want[i][1]), i
    dn.teardown(dit)


def test_rebinding_triggers_a_new_capture(gguf_patch):
    """Weights moved by someone else (a model load) are captured again at the next forward."""
    import torch
    dn = wf("streaming.dit_node")
    dit = _dit(torch, seed=5)
    x = _x(torch)
    with torch.inference_mode():
        ref = dit(x)
        dn.WeightFerryDiT().apply_streaming(_Patcher(dit, torch), resident_blocks=1)
        st = dit._weightferry_stream_state
        for p in dit.blocks[3].parameters():
            p.data = p.data.to("cuda")
        out = dit(x)
    torch.cuda.synchronize()
    assert st.captures == 2 and torch.equal(out, ref)
    dn.teardown(dit)


def test_streamed_plain_bf16_dit(cuda):
    """A model without GGUF weights streams its bf16 parameters as they are."""
    import torch
    dn = wf("streaming.dit_node")
    dit = _dit(torch, seed=9, plain=True)
    x = _x(torch)
    with torch.inference_mode():
        ref = dit(x)
        dn.WeightFerryDiT().apply_streaming(dit, resident_blocks=2, prefetch_slots=2)
        out = dit(x)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    dn.teardown(dit)


@pytest.mark.parametrize("n_blocks,budget_blocks,slots", [(9, 6, 3), (5, 1, 2)])
def test_streamed_gguf_dit_with_ssd_tier(gguf_patch, tmp_path, monkeypatch, n_blocks, budget_blocks, slots):
    """tiering "Auto" with a RAM budget of a few blocks: the planner puts streamed blocks on the SSD (a cache file
    read back every forward through the DiskRing and the uploader thread, which dequantises them); the result equals
    the un-streamed model's bit for bit, forward after forward, and after a forward that stopped part way."""
    import torch
    dn = wf("streaming.dit_node")
    monkeypatch.setenv("WEIGHTFERRY_DISK_DIR", str(tmp_path))
    dit = _dit(torch, seed=13, n_blocks=n_blocks)
    x = _x(torch)
    specs, _ = dn.block_specs_of(dit.blocks[1])
    flat = wf("streaming.state").BlockLayout(specs).flat_bytes
    with torch.inference_mode():
        ref = dit(x)
        dn.WeightFerryDiT().apply_streaming(_Patcher(dit, torch), resident_blocks=1, prefetch_slots=slots,
                                            tiering=dn.TIERING_AUTO, ram_budget_gb=budget_blocks * flat / 1024 ** 3)
        st = dit._weightferry_stream_state
        plan = st.tier_plan
        assert plan["disk_blocks"] > 0 and st.ring.ring is not None and st.ring.uploader is not None
        assert plan["ram_blocks"] + plan["disk_blocks"] == n_blocks - 1
        assert os.path.exists(st.store.path) and len(st.disk_blocks) == plan["disk_blocks"]
        outs = [dit(x) for _ in range(3)]
        # a forward that stops part way, after the SSD tier's first blocks were queued
        dit.blocks[n_blocks - 2].fail = True
        with pytest.raises(RuntimeError, match="interrupted"):
            dit(x)
        outs += [dit(x) for _ in range(2)]
        torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, ref)
    path = st.store.path
    dn.teardown(dit)
    assert not os.path.exists(path)
    with torch.inference_mode():
        assert torch.equal(dit(x), ref)


def test_comfyui_patcher_captures_on_load(gguf_patch):
    """With a ComfyUI ModelPatcher (the stand-in of tests/fake_patcher.py) the blocks are captured in the ON_LOAD
    callback, as the reference does, not when the node runs; ON_DETACH gives the model back; a forward that comes
    without a load (ComfyUI switching back to a clone whose weights are in place) captures lazily in the wrapper.
    Every streamed forward equals the un-streamed one bit for bit."""
    import sys
    import torch
    import fake_patcher as fp
    had_comfy = "comfy" in sys.modules
    fp.register()
    try:
        dn = wf("streaming.dit_node")
        dit = _dit(torch)
        x = _x(torch)
        with torch.inference_mode():
            ref = dit(x)
            base = fp.ModelPatcher(dit, torch.device("cuda", 0), torch.bfloat16)
            (patcher,) = dn.WeightFerryDiT().apply_streaming(base, resident_blocks=1)
            assert patcher is not base and not base.callbacks
            assert getattr(dit, "_weightferry_stream_state", None) is None       # nothing captured yet
            patcher.load()                                                        # ComfyUI loads the model
            st = dit._weightferry_stream_state
            assert st is not None and all(not p.is_cuda for i in st.stream_idx for p in dit.blocks[i].parameters())
            out1 = patcher.apply_model(x)
            patcher.detach()                                                      # ComfyUI unloads it
            assert dit._weightferry_stream_state is None and all(p.is_cuda for p in dit.parameters())
            out2 = patcher.apply_model(x)                                         # no ON_LOAD: captured lazily
            assert dit._weightferry_stream_state is not None
            out3 = patcher.apply_model(x)
            torch.cuda.synchronize()
        assert torch.equal(out1, ref) and torch.equal(out2, ref) and torch.equal(out3, ref)
        dn.teardown(dit)
    finally:
        fp.unregister(drop_comfy=not had_comfy)
