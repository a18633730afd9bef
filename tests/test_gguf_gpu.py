"""GGUF dequantisation on the GPU through the C ABI, against the reference's golden vectors and the CPU oracle:
bit for bit, every format and dtype pair, odd sizes, misaligned buffers, the BASELINE shapes, the batched sweep and
the fused LoRA add."""

import ctypes
import os

import numpy as np
import pytest

from conftest import GOLDEN, oracle, wf

pytestmark = pytest.mark.gpu

G = np.load(os.path.join(GOLDEN, "gguf_dequant.npz"))
FMT = {2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34),
       10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210)}
F16_FIELDS = {2: (0,), 3: (0, 2), 6: (0,), 7: (0, 2), 8: (0,), 10: (80, 82), 11: (108,), 12: (0, 2), 13: (0, 2),
              14: (208,)}


def _np_out(t):
    import torch
    t = t.detach().cpu().reshape(-1)
    if t.dtype == torch.float32:
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def _same(a, b):
    if a.dtype == np.float32:
        an, bn = np.isnan(a), np.isnan(b)
        return bool(np.array_equal(an, bn) and np.array_equal(a.view(np.uint32)[~an], b.view(np.uint32)[~bn]))
    return bool(np.array_equal(a, b))


def _blocks(qt, n_blocks, seed):
    """Random packed blocks with finite scales in the BASELINE distributions."""
    rng = np.random.default_rng(seed)
    vpb, ts = FMT[qt]
    raw = rng.integers(0, 256, size=(n_blocks, ts), dtype=np.uint8)
    for off in F16_FIELDS[qt]:
        if vpb == 32:
            vals = (np.abs(rng.standard_normal(n_blocks)) * 0.002).astype(np.float16)
        else:
            vals = rng.uniform(0, 0.01, n_blocks).astype(np.float16)
        raw[:, off:off + 2] = vals.view(np.uint8).reshape(n_blocks, 2)
    return raw.reshape(-1)


def _dev_dequant(raw_np, n, qt, mid, out, offset=0, out_offset=0):
    """wf_dequant_gguf through the C ABI; offset / out_offset shift the buffers off their 16-byte alignment."""
    import torch
    ext = wf("_ext")
    dt = {0: torch.float16, 1: torch.bfloat16, 2: torch.float32}[out]
    src = torch.empty(raw_np.size + offset, dtype=torch.uint8, device="cuda")
    src[offset:].copy_(torch.from_numpy(raw_np))
    esz = 4 if out == 2 else 2
    dst = torch.empty(n + out_offset, dtype=dt, device="cuda")
    rc = ext.lib().wf_dequant_gguf(src.data_ptr() + offset, raw_np.size, dst.data_ptr() + out_offset * esz, n, qt,
                                   mid, out, ext.stream_of(src.device))
    ext.check(rc, "wf_dequant_gguf")
    torch.cuda.synchronize()
    return _np_out(dst[out_offset:])


@pytest.mark.parametrize("qt", sorted(FMT))
@pytest.mark.parametrize("mid", [0, 1, 2])
@pytest.mark.parametrize("out", [0, 1, 2])
def test_golden(cuda, qt, mid, out):
    raw = G[f"q{qt}_raw"]
    vpb, ts = FMT[qt]
    n = raw.size // ts * vpb
    assert _same(_dev_dequant(raw, n, qt, mid, out), G[f"q{qt}_m{mid}_o{out}"])


@pytest.mark.parametrize("qt", sorted(FMT))
@pytest.mark.parametrize("n_blocks", [1, 7, 257, 8191, 33 * 256 + 5])
def test_ragged_sizes_vs_oracle(cuda, qt, n_blocks):
    vpb, ts = FMT[qt]
    if vpb == 256:
        n_blocks = max(1, n_blocks // 8)
    raw = _blocks(qt, n_blocks, seed=qt * 1000 + n_blocks)
    n = n_blocks * vpb
    for mid, out in ((0, 1), (1, 1), (2, 2), (0, 0)):
        assert _same(_dev_dequant(raw, n, qt, mid, out), oracle().dequant_gguf(raw, n, qt, mid, out))


@pytest.mark.parametrize("qt", [8, 12, 2, 14])
@pytest.mark.parametrize("offset,out_offset", [(2, 0), (0, 1), (6, 3)])
def test_misaligned_buffers(cuda, qt, offset, out_offset):
    vpb, ts = FMT[qt]
    n_blocks = 300 if vpb == 32 else 40
    raw = _blocks(qt, n_blocks, seed=7)
    n = n_blocks * vpb
    got = _dev_dequant(raw, n, qt, 0, 1, offset=offset, out_offset=out_offset)
    assert _same(got, oracle().dequant_gguf(raw, n, qt, 0, 1))


@pytest.mark.parametrize("qt,shape", [(8, (5120, 5120)), (12, (5120, 13824))])
def test_baseline_shapes(cuda, qt, shape):
    """BASELINE configs[0] / [1] at full size, default mid float16 -> bfloat16, bit for bit against the oracle."""
    import torch
    gd = wf("enhancers.gguf_dequant")
    vpb, ts = FMT[qt]
    n = shape[0] * shape[1]
    raw = _blocks(qt, n // vpb, seed=20261201 + (0 if qt == 8 else 1))
    data = torch.from_numpy(raw).cuda()
    res = gd.dequantize(data, qt, shape, None, torch.bfloat16)
    torch.cuda.synchronize()
    assert res.shape == shape and res.dtype == torch.bfloat16
    assert _same(_np_out(res), oracle().dequant_gguf(raw, n, qt, 0, 1))


def test_batch_matches_single(cuda):
    import torch
    gd = wf("enhancers.gguf_dequant")
    shapes = [(256, 512), (1024, 256), (768, 2048), (256, 256)] * 40  # > one table of 128 tensors
    items = []
    for i, sh in enumerate(shapes):
        raw = _blocks(12, sh[0] * sh[1] // 256, seed=100 + i)
        items.append((torch.from_numpy(raw).cuda(), sh))
    outs = gd.dequantize_many(items, 12, None, torch.bfloat16)
    for (data, sh), o in zip(items, outs):
        ref = gd.dequantize(data, 12, sh, None, torch.bfloat16)
        assert torch.equal(o.view(torch.int16), ref.view(torch.int16))


def test_batch_with_misaligned_and_empty(cuda):
    import torch
    ext = wf("_ext")
    raws = [_blocks(8, nb, seed=nb) for nb in (5, 0, 700, 33)]
    srcs, dsts, tasks = [], [], (ext.DequantTask * len(raws))()
    for i, r in enumerate(raws):
        off = 2 if i == 2 else 0
        s = torch.empty(r.size + off + 1, dtype=torch.uint8, device="cuda")
        s[off:off + r.size].copy_(torch.from_numpy(r))
        d = torch.empty(r.size // 34 * 32 + 1, dtype=torch.bfloat16, device="cuda")
        srcs.append(s)
        dsts.append(d)
        tasks[i].src, tasks[i].dst, tasks[i].n_values = s.data_ptr() + off, d.data_ptr(), r.size // 34 * 32
    rc = ext.lib().wf_dequant_gguf_batch(tasks, len(raws), 8, 0, 1, ext.stream_of(torch.device("cuda")))
    ext.check(rc, "batch")
    torch.cuda.synchronize()
    for r, d in zip(raws, dsts):
        n = r.size // 34 * 32
        assert _same(_np_out(d[:n]), oracle().dequant_gguf(r, n, 8, 0, 1))


@pytest.mark.parametrize("qt", [8, 3, 12])
@pytest.mark.parametrize("mid,out", [(0, 1), (1, 0), (0, 0)])
def test_lora_golden(cuda, qt, mid, out):
    import torch
    ext = wf("_ext")
    raw = G[f"q{qt}_raw"]
    vpb, ts = FMT[qt]
    n = raw.size // ts * vpb
    sa1, sa2 = (float(x) for x in G["lora_sa"])
    dt = {0: torch.float16, 1: torch.bfloat16}[out]
    src = torch.from_numpy(raw.copy()).cuda()
    d1 = torch.from_numpy(G[f"lora_q{qt}_diff"]).cuda()
    d2 = torch.from_numpy(G[f"lora_q{qt}_diff2"]).cuda()
    w = torch.empty(n, dtype=dt, device="cuda")
    st = ext.stream_of(src.device)
    ext.check(ext.lib().wf_dequant_gguf_lora(src.data_ptr(), raw.size, d1.data_ptr(), w.data_ptr(), n, qt, mid, out,
                                             ctypes.c_float(sa1), st), "lora")
    ext.check(ext.lib().wf_lora_add(d2.data_ptr(), w.data_ptr(), n, out, ctypes.c_float(sa2), st), "lora_add")
    torch.cuda.synchronize()
    assert _same(_np_out(w), G[f"lora_q{qt}_m{mid}_o{out}"])


@pytest.mark.parametrize("qt", sorted(FMT))
@pytest.mark.parametrize("diff_offset,out", [(0, 1), (1, 1), (0, 0), (1, 0)])
def test_lora_many_chunks_vs_oracle(cuda, qt, diff_offset, out):
    """wf_dequant_gguf_lora over ~4.2 M values (more chunks than the persistent grid holds, so every CTA cycles both
    staging buffers; the last chunk ragged) against the oracle, bf16 and f16 out; diff_offset 1 moves the float32
    difference off its 16-byte alignment (the unstaged path). A few differences are huge (their products overflow
    f16 to infinity, or round to the largest finite value), infinite, or tiny (far below half an ulp of the
    weight)."""
    import torch
    ext = wf("_ext")
    vpb, ts = FMT[qt]
    n_blocks = (131_075 if vpb == 32 else 16_401)
    raw = _blocks(qt, n_blocks, seed=500 + qt)
    n = n_blocks * vpb
    rng = np.random.default_rng(600 + qt)
    diff = (rng.standard_normal(n) * 0.01).astype(np.float32)
    extreme = np.array([3.4e38, -3.4e38, np.inf, -np.inf, 1.0e5, -1.0e5, 65504 / 0.625, 1e-30, -1e-30, 3e-8],
                       dtype=np.float32)
    diff[rng.choice(n, 4096, replace=False)] = rng.choice(extreme, 4096)
    sa = 0.625
    src = torch.from_numpy(raw).cuda()
    dbuf = torch.empty(n + diff_offset, dtype=torch.float32, device="cuda")
    dbuf[diff_offset:].copy_(torch.from_numpy(diff))
    w = torch.empty(n, dtype={0: torch.float16, 1: torch.bfloat16}[out], device="cuda")
    ext.check(ext.lib().wf_dequant_gguf_lora(src.data_ptr(), raw.size, dbuf.data_ptr() + 4 * diff_offset, w.data_ptr(),
                                             n, qt, 0, out, ctypes.c_float(sa), ext.stream_of(src.device)), "lora")
    torch.cuda.synchronize()
    assert _same(_np_out(w), oracle().dequant_gguf(raw, n, qt, 0, out, diff=diff, sa=sa))


def test_dequantize_lora_entry_point(cuda):
    """gguf_dequant.dequantize_lora with two plain LoRAs (the torch.mm differences computed once here and handed to
    the oracle, so the comparison is exact)."""
    import torch
    gd = wf("enhancers.gguf_dequant")
    n_out, n_in = 512, 768
    raw = _blocks(8, n_out * n_in // 32, seed=3)
    g = torch.Generator().manual_seed(0)
    ups = [torch.randn(n_out, 16, generator=g) * 0.05 for _ in range(2)]
    downs = [torch.randn(16, n_in, generator=g) * 0.05 for _ in range(2)]
    loras = [(ups[0], downs[0], 0.8), (ups[1], downs[1], -0.3)]
    res = gd.dequantize_lora(torch.from_numpy(raw).cuda(), 8, (n_out, n_in), None, torch.bfloat16, loras)
    diffs = [torch.mm(u.cuda().float(), d.cuda().float()).cpu().numpy() for u, d in zip(ups, downs)]
    ref = oracle().dequant_gguf(raw, n_out * n_in, 8, 0, 1, diff=diffs[0], sa=0.8)
    oracle().lora_add(diffs[1], ref, 1, -0.3)
    assert _same(_np_out(res), ref)


def test_entry_point_contract(cuda):
    """dequantize(): mid defaults to float16, out to mid; None for CPU data, unknown types, wrong byte counts."""
    import torch
    gd = wf("enhancers.gguf_dequant")
    raw = _blocks(8, 64, seed=1)
    data = torch.from_numpy(raw).cuda()
    r = gd.dequantize(data, 8, (64, 32), None, None)
    assert r.dtype == torch.float16 and r.shape == (64, 32)
    assert gd.dequantize(data.cpu(), 8, (64, 32), None, None) is None
    assert gd.dequantize(data, 9, (64, 32), None, None) is None
    assert gd.dequantize(data, 8, (64, 31), None, None) is None
    assert gd.dequantize(data[:-1], 8, (64, 32), None, None) is None
    assert gd.dequantize(data, 8, (64, 32), torch.int8, None) is None


def test_c_abi_rejections(cuda):
    import torch
    ext = wf("_ext")
    L = ext.lib()
    s = torch.empty(64, dtype=torch.uint8, device="cuda")
    d = torch.empty(64, dtype=torch.bfloat16, device="cuda")
    st = ext.stream_of(s.device)
    assert L.wf_dequant_gguf(s.data_ptr(), 34, d.data_ptr(), 31, 8, 0, 1, st) == -3
    assert L.wf_dequant_gguf(s.data_ptr(), 33, d.data_ptr(), 32, 8, 0, 1, st) == -3
    assert L.wf_dequant_gguf(s.data_ptr(), 34, d.data_ptr(), 32, 9, 0, 1, st) == -2
    assert L.wf_dequant_gguf(s.data_ptr(), 34, d.data_ptr(), 32, 8, 3, 1, st) == -1
    assert L.wf_dequant_gguf(None, 34, d.data_ptr(), 32, 8, 0, 1, st) == -1
    assert L.wf_dequant_gguf(s.data_ptr(), 0, d.data_ptr(), 0, 8, 0, 1, st) == 0


def test_c_abi_rejects_unaligned_output(cuda):
    import torch
    ext = wf("_ext")
    s = torch.zeros(64, dtype=torch.uint8, device="cuda")
    d = torch.empty(64, dtype=torch.bfloat16, device="cuda")
    st = ext.stream_of(s.device)
    assert ext.lib().wf_dequant_gguf(s.data_ptr(), 34, d.data_ptr() + 1, 32, 8, 0, 1, st) == -1


def test_hbm_probe_writes_its_pattern(cuda):
    """The benchmark's mix probe (wf_hbm_probe) does the work it is timed for: out[j] = in[floor(j * r)] ^ j per
    16-byte unit with r the 32.32 fixed-point in / out ratio, every output unit written."""
    import torch
    ext = wf("_ext")
    L = ext.lib()
    n_in, n_out = 9 * 1000 + 7, 32 * 1000 + 5           # about the Q4_K sweep's 9 : 32 mix, ragged tiles
    a = torch.randint(0, 2**31 - 1, (n_in, 4), dtype=torch.int32, device="cuda")
    b = torch.zeros((n_out, 4), dtype=torch.int32, device="cuda")
    ext.check(L.wf_hbm_probe(a.data_ptr(), n_in * 16, b.data_ptr(), n_out * 16, ext.stream_of(a.device)), "probe")
    torch.cuda.synchronize()
    r = (n_in << 32) // n_out
    j = np.arange(n_out, dtype=np.uint64)
    idx = ((j * np.uint64(r)) >> np.uint64(32)).astype(np.int64)
    want = a.cpu().numpy()[idx].copy()
    want[:, 0] ^= np.arange(n_out, dtype=np.int64).astype(np.uint32).view(np.int32)
    assert np.array_equal(b.cpu().numpy(), want)
    p = a.data_ptr()
    assert L.wf_hbm_probe(p, 32, p, 16, None) == -1      # reads larger than writes
    assert L.wf_hbm_probe(p + 8, 16, p, 32, None) == -1  # alignment
    assert L.wf_hbm_probe(p, 24, p, 32, None) == -1      # not a multiple of 16
