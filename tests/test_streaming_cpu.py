"""Host-side logic of the streaming path without a GPU: flat layouts, block specs and their tensor-parallel shards
(each rank's packed Q8_0 bytes dequantise to exactly its slice of the full weight), and the pinned-buffer holder."""

import numpy as np
import pytest

from conftest import oracle, wf


def test_flat_layout_alignment():
    common = wf("streaming.common")
    offs, total = common.flat_layout([10, 300, 1, 256])
    assert offs == [0, 256, 768, 1024] and total == 1280
    assert all(o % 256 == 0 for o in offs)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_block_specs_partition_the_block(world):
    cb = wf("streaming.cosmos_block")
    full = {s.name: s for s in cb.block_specs(cb.COSMOS_14B, 1, 0)}
    shards = [cb.block_specs(cb.COSMOS_14B, world, r) for r in range(world)]
    for name, sp in full.items():
        kinds = [cb.shard_of(name, world, r) for r in range(world)]
        per = [{s.name: s for s in sh}[name] for sh in shards]
        if kinds[0] is None:
            assert all(p.shape == sp.shape for p in per)          # replicated
        else:
            assert sum(p.numel for p in per) == sp.numel          # an exact partition
            assert all(cb.full_shape(p, world) == sp.shape for p in per)
    q_bytes = sum(s.packed_bytes for s in full.values() if s.qtype is not None)
    assert q_bytes == 417_792_000  # 417,792,000 B of Q8_0 per block


@pytest.mark.parametrize("kind", ["col", "row"])
def test_q8_0_shards_dequantise_to_slices(kind):
    import torch
    cb = wf("streaming.cosmos_block")
    rows, cols, world = 64, 256, 4
    g = torch.Generator().manual_seed(3)
    q = torch.randint(-127, 128, (rows, cols), dtype=torch.int16, generator=g).to(torch.int8)
    d = (torch.rand((rows, cols // 32), generator=g) * 0.01).half()
    packed = cb.q8_0_pack(q, d)
    full = oracle().dequant_gguf(packed.numpy().reshape(-1), rows * cols, 8, 0, 2).reshape(rows, cols)
    for r in range(world):
        sh = cb.q8_0_shard(packed, (rows, cols), (kind, r, world)).numpy()
        if kind == "col":
            want = full[rows * r // world: rows * (r + 1) // world]
        else:
            want = full[:, cols * r // world: cols * (r + 1) // world]
        got = oracle().dequant_gguf(sh, want.size, 8, 0, 2).reshape(want.shape)
        assert np.array_equal(got, want)


def test_rope3d_table_is_rotations():
    import torch
    cb = wf("streaming.cosmos_block")
    f = cb.rope3d_table(1, 4, 5)
    assert tuple(f.shape) == (1, 20, 1, 64, 2, 2)
    det = f[..., 0, 0] * f[..., 1, 1] - f[..., 0, 1] * f[..., 1, 0]
    assert torch.allclose(det, torch.ones_like(det), atol=1e-5)
    assert torch.allclose(f[0, 0, 0, :, 0, 0], torch.ones(64))  # token 0: identity


def test_pinned_host_holder_exact_size():
    ph = wf("core.tiers.pinned")
    h = ph.PinnedHost(1000)
    assert h.tensor.numel() == 1000
    h.tensor.fill_(7)
    h.release()
    assert h.tensor is None


def test_gpu_numa_binding_with_a_fake_nvml(monkeypatch):
    """bind_to_gpu_numa takes the GPU's NVML CPU affinity (bitmask words) and restricts the process to the CPUs it
    may use among them; without NVML it leaves the affinity alone."""
    import os
    import types
    import torch
    pinned = wf("core.tiers.pinned")
    allowed = sorted(os.sched_getaffinity(0))
    want = allowed[: max(1, len(allowed) // 2)]
    words = [0] * 16
    for c in want:
        words[c // 64] |= 1 << (c % 64)
    seen = {}
    fake = types.SimpleNamespace(
        nvmlInit=lambda: None, nvmlShutdown=lambda: None,
        nvmlDeviceGetHandleByPciBusId=lambda bus: seen.setdefault("bus", bus),
        nvmlDeviceGetCpuAffinity=lambda h, n: words)
    props = types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x1B, pci_device_id=0)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda i: props)
    assert pinned.gpu_local_cpus(0, fake) == want and seen["bus"] == "00000000:1b:00.0"
    try:
        assert pinned.bind_to_gpu_numa(0, fake) == want
        assert sorted(os.sched_getaffinity(0)) == want
    finally:
        os.sched_setaffinity(0, allowed)
    broken = types.SimpleNamespace(nvmlInit=lambda: (_ for _ in ()).throw(RuntimeError("no driver")))
    assert pinned.bind_to_gpu_numa(0, broken) is None and sorted(os.sched_getaffinity(0)) == allowed
