"""The streaming node's host logic on the CPU: block-list discovery, the per-parameter layout (which GGUF weights
are dequantised on arrival and with which intermediate precision), auto_config's resident count, and the cases in
which apply_streaming hands the model back untouched (the reference's streaming/dit_node.py:170-230)."""

import pytest
import torch

from conftest import wf
import fake_gguf_ops as fg


def _node():
    return wf("streaming.dit_node")


def test_block_list_discovery():
    dn = _node()

    class A(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.layers = torch.nn.ModuleList([torch.nn.Linear(2, 2)])
            self.blocks = torch.nn.ModuleList([torch.nn.Linear(2, 2), torch.nn.Linear(2, 2)])

    assert len(dn._blocks(A())) == 2   # "blocks" comes first
    m = torch.nn.Module()
    m.blocks = torch.nn.ModuleList()
    m.transformer_blocks = torch.nn.ModuleList([torch.nn.Linear(2, 2)])
    assert len(dn._blocks(m)) == 1     # an empty list is skipped
    assert dn._blocks(torch.nn.Linear(2, 2)) == []


@pytest.mark.parametrize("dequant_dtype,mid", [(None, 0), ("target", 1), (torch.float32, 2), (torch.float16, 0),
                                               (torch.bfloat16, 1), ("odd", None)])
def test_param_spec_gguf(dequant_dtype, mid):
    dn = _node()
    raw = torch.zeros(64 * 64 // 32 * 34, dtype=torch.uint8)
    lin = fg.Linear(fg.gguf_param(raw, 8, (64, 64), "cpu"), dequant_dtype=dequant_dtype)
    sp, deq = dn.param_spec("weight", lin.weight, lin, torch.bfloat16)
    if mid is None:   # a precision the kernels do not take: streamed packed, dequantised by the layer per use
        assert not deq and sp.qtype is None and sp.dtype == torch.uint8 and sp.packed_bytes == raw.numel()
    else:
        assert deq and sp.qtype == 8 and sp.shape == (64, 64) and sp.mid == mid and sp.packed_bytes == raw.numel()


def test_param_spec_fallbacks():
    dn = _node()
    raw = torch.zeros(64 * 64 // 32 * 34, dtype=torch.uint8)
    lin = fg.Linear(fg.gguf_param(raw, 8, (64, 64), "cpu"))
    lin.weight.patches = [("lora", "key")]          # LoRA patches: the layer's own get_weight handles them
    sp, deq = dn.param_spec("weight", lin.weight, lin, torch.bfloat16)
    assert not deq and sp.dtype == torch.uint8
    bad = fg.gguf_param(raw[:-34], 8, (64, 64), "cpu")  # bytes that are not the logical shape's
    assert not dn.param_spec("w", bad, lin, torch.bfloat16)[1]
    odd = fg.gguf_param(raw, 99, (64, 64), "cpu")       # a type without a kernel
    assert not dn.param_spec("w", odd, lin, torch.bfloat16)[1]
    f32 = fg.plain_param(torch.ones(8), "cpu")
    sp, deq = dn.param_spec("b", f32, lin, torch.bfloat16)
    assert not deq and sp.dtype == torch.float32 and sp.shape == (8,)


def test_block_specs_layout_order():
    dn = _node()
    raw = torch.zeros(256 * 32 // 256 * 144, dtype=torch.uint8)
    blk = torch.nn.Module()
    blk.norm = torch.nn.Module()
    blk.norm.weight = fg.plain_param(torch.ones(32), "cpu")
    blk.fc = fg.Linear(fg.gguf_param(raw, 12, (32, 256), "cpu"), bias=fg.plain_param(torch.zeros(32), "cpu"))
    specs, deq = dn.block_specs_of(blk)
    assert [s.name for s in specs] == [n for n, _ in blk.named_parameters()]
    assert deq == [False, True, False]
    lay = wf("streaming.state").BlockLayout(specs)
    assert all(o % 256 == 0 for o in lay.offsets)
    assert lay.weight_bytes >= 32 * 256 * 2


def test_auto_resident():
    dn = _node()
    mb = 1024 ** 2
    # everything fits with the headroom: no streaming
    assert dn.auto_resident(10, 100 * mb, 150 * mb, 50 * mb, 2000 * mb, 500 * mb, 3, True) is None
    # 1500 usable - 500 headroom - 50 non-block - 3 slots x 150 = 500 -> 5 resident blocks of 100
    assert dn.auto_resident(10, 100 * mb, 150 * mb, 50 * mb, 1500 * mb, 500 * mb, 3, True) == 5
    # single buffer: two slots
    assert dn.auto_resident(10, 100 * mb, 150 * mb, 50 * mb, 1500 * mb, 500 * mb, 3, False) == 6
    # clamps: at least block 0, at most all but one
    assert dn.auto_resident(10, 100 * mb, 150 * mb, 50 * mb, 600 * mb, 500 * mb, 3, True) == 1
    assert dn.auto_resident(10, 1 * mb, 1, 0, 10 * mb, 1, 2, True) == 9


def test_vram_budget(monkeypatch):
    """vram_budget_gb (or WEIGHTFERRY_VRAM_BUDGET_GB; the node's value wins when > 0) bounds the usable VRAM of the
    resident-block plan to the budget minus what the process already uses; no budget leaves it at free + cached."""
    dn = _node()
    gb, mb = 1024 ** 3, 1024 ** 2
    monkeypatch.delenv("WEIGHTFERRY_VRAM_BUDGET_GB", raising=False)
    assert dn.vram_budget_bytes(0.0) is None
    assert dn.vram_budget_bytes(2.5) == int(2.5 * gb)
    monkeypatch.setenv("WEIGHTFERRY_VRAM_BUDGET_GB", "4")
    assert dn.vram_budget_bytes(0.0) == 4 * gb
    assert dn.vram_budget_bytes(1.0) == 1 * gb
    monkeypatch.setenv("WEIGHTFERRY_VRAM_BUDGET_GB", "x")
    assert dn.vram_budget_bytes(0.0) is None
    assert dn.budget_usable(3000 * mb, 500 * mb, None) == 3000 * mb
    assert dn.budget_usable(3000 * mb, 500 * mb, 2000 * mb) == 1500 * mb   # the budget binds
    assert dn.budget_usable(1000 * mb, 500 * mb, 4000 * mb) == 1000 * mb   # more budget than the device gives
    assert dn.budget_usable(1000 * mb, 5000 * mb, 4000 * mb) == 0          # already past the budget
    # the plan follows: 1500 usable -> 5 resident blocks (as test_auto_resident), 3000 -> all fit
    assert dn.auto_resident(10, 100 * mb, 150 * mb, 50 * mb, dn.budget_usable(3000 * mb, 500 * mb, 2000 * mb),
                            500 * mb, 3, True) == 5
    assert dn.auto_resident(10, 100 * mb, 150 * mb, 50 * mb, dn.budget_usable(3000 * mb, 500 * mb, None),
                            500 * mb, 3, True) is None


def test_apply_streaming_passthrough():
    dn = _node()
    node = dn.WeightFerryDiT()
    assert node.FUNCTION == "apply_streaming" and node.RETURN_TYPES == ("MODEL",)
    assert "WeightFerryDiT" in wf().NODE_CLASS_MAPPINGS

    class Patcher:
        def __init__(self, dit, device):
            self.model = type("M", (), {})()
            self.model.diffusion_model = dit
            self.load_device = torch.device(device)
            self.clones = 0

        def clone(self):
            c = Patcher(self.model.diffusion_model, self.load_device)
            self.clones += 1
            return c

    dit = torch.nn.Module()
    dit.blocks = torch.nn.ModuleList([torch.nn.Linear(4, 4) for _ in range(3)])
    p = Patcher(dit, "cpu")
    assert node.apply_streaming(p, enabled=False)[0] is p            # disabled: the same object
    out = node.apply_streaming(p, resident_blocks=1)[0]              # not CUDA: a clone, nothing installed
    assert out is not p and p.clones == 1
    assert getattr(dit, "_weightferry_stream_state", None) is None
    nob = Patcher(torch.nn.Linear(4, 4), "cuda")                     # no block list
    assert node.apply_streaming(nob)[0].model.diffusion_model is nob.model.diffusion_model
    none = type("P", (), {"model": None, "clone": lambda self: self})()
    assert node.apply_streaming(none)[0] is none                      # no diffusion model


def test_comfyui_patcher_defers_capture_to_on_load():
    """Given a ComfyUI ModelPatcher, the node registers the ON_LOAD / ON_DETACH callbacks and a DIFFUSION_MODEL
    wrapper on its clone and captures nothing yet (the capture needs ComfyUI's load); a re-application replaces the
    wrapper instead of stacking a second one; a detach before any load does nothing."""
    import sys

    import torch

    import fake_patcher as fp
    had_comfy = "comfy" in sys.modules
    fp.register()
    try:
        dn = wf("streaming.dit_node")

        class Blk(torch.nn.Module):
            def __init__(self):
                super().__init__()
                self.lin = torch.nn.Linear(8, 8)

        dit = torch.nn.Module()
        dit.blocks = torch.nn.ModuleList([Blk() for _ in range(3)])
        base = fp.ModelPatcher(dit, torch.device("cuda", 0), torch.bfloat16)
        (patcher,) = dn.WeightFerryDiT().apply_streaming(base, resident_blocks=1)
        assert patcher is not base and not base.callbacks
        assert len(patcher.callbacks[fp.CallbacksMP.ON_LOAD]) == 1
        assert len(patcher.callbacks[fp.CallbacksMP.ON_DETACH]) == 1
        wrappers = patcher.model_options["transformer_options"]["wrappers"][fp.WrappersMP.DIFFUSION_MODEL]
        assert list(wrappers) == [dn._WRAPPER_KEY] and len(wrappers[dn._WRAPPER_KEY]) == 1
        assert getattr(dit, "_weightferry_stream_state", None) is None
        (again,) = dn.WeightFerryDiT().apply_streaming(patcher, resident_blocks=1)
        w2 = again.model_options["transformer_options"]["wrappers"][fp.WrappersMP.DIFFUSION_MODEL]
        assert len(w2[dn._WRAPPER_KEY]) == 1
        again.detach()
        assert getattr(dit, "_weightferry_stream_state", None) is None
    finally:
        fp.unregister(drop_comfy=not had_comfy)
