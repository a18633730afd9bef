"""The SSD tier on the CPU (the reference's core/tiers, streaming/ssd_uploader.py): the tier planner, the safetensors
block layouts, the cache-file block store, and the DiskRing's reader threads -- cyclic order across forwards, several
readers, pieces of scattered blocks, a failed read reaching the consumer, and the restart after a forward that stopped
part way. Ring buffers are unpinned here (no GPU); the GPU path is tests/test_dit_node_gpu.py."""

import json
import os
import struct

import numpy as np
import pytest
import torch

from conftest import wf


def _tiers(mod):
    return wf("core.tiers." + mod)


def test_ssd_positions():
    plan = _tiers("plan")
    assert plan.ssd_positions(10, 0) == []
    assert plan.ssd_positions(10, 3, "tail") == [7, 8, 9]
    inter = plan.ssd_positions(10, 3, "interleave")
    assert inter == [2, 5, 9] and inter[-1] == 9          # spread out, the last block on the SSD
    assert plan.ssd_positions(4, 4) == [0, 1, 2, 3]
    assert plan.ssd_positions(35, 35) == list(range(35))


def test_plan_tiers(monkeypatch):
    plan = _tiers("plan")
    mb = 1024 ** 2
    monkeypatch.setattr(plan, "available_ram", lambda: 64 * 1024 * mb)
    probe = {"gbps": 2.0, "threads": 2, "by_threads": {1: 1.5, 2: 2.0}}
    # everything fits the budget: no SSD tier
    p = plan.plan_tiers(10, 100 * mb, ram_budget_bytes=2000 * mb, probe=probe, disk_dir="/tmp/x")
    assert p["ram_blocks"] == 10 and p["disk_blocks"] == 0 and p["ring_depth"] == 0 and not p["over_budget"]
    # 950 MB budget, 4-deep ring of 100 MB blocks: (950 - 400) // 100 = 5 in RAM, 5 on the SSD
    p = plan.plan_tiers(10, 100 * mb, ram_budget_bytes=950 * mb, probe=probe, disk_dir="/tmp/x")
    assert (p["ram_blocks"], p["disk_blocks"], p["ring_depth"]) == (5, 5, 4) and not p["over_budget"]
    assert p["disk_read_gbps"] == 2.0 and p["disk_threads"] == 2
    # ring depth from the read and compute times: 100 MB at 2 GB/s = 52 ms over 10 ms of compute -> 6 + 2 = 8 max
    p = plan.plan_tiers(10, 100 * mb, ram_budget_bytes=500 * mb, probe=probe, disk_dir="/tmp/x",
                        compute_ms_per_block=10.0, total_blocks=12)
    # (the wanted 8 buffers do not fit 500 MB: the ring shrinks to the 5 that do, no block stays in RAM)
    assert p["ring_depth"] == 5 and p["ring_depth_wanted"] == 8 and p["ram_blocks"] == 0
    assert p["disk_bound"] is True and p["disk_ms_per_forward"] > p["compute_ms_per_forward_est"]
    # a budget below even two ring buffers: reported over budget
    p = plan.plan_tiers(10, 100 * mb, ram_budget_bytes=50 * mb, probe=probe, disk_dir="/tmp/x")
    assert p["disk_blocks"] == 10 and p["ring_depth"] == 2 and p["over_budget"]
    # no read rate: all blocks stay in RAM and the error is kept
    p = plan.plan_tiers(10, 100 * mb, ram_budget_bytes=500 * mb, probe={}, disk_dir="/tmp/x")
    assert p["disk_blocks"] == 0 and p["disk_error"]
    monkeypatch.setenv("WEIGHTFERRY_DISK_THREADS", "1")
    p = plan.plan_tiers(10, 100 * mb, ram_budget_bytes=1000 * mb, probe=probe, disk_dir="/tmp/x")
    assert p["disk_threads"] == 1 and p["disk_read_gbps"] == 1.5


def _write_safetensors(path, tensors, prefix=""):
    """A safetensors file of the given (name, numpy array) in order; returns the name -> (start, end) of the data."""
    header, off, blobs = {}, 0, []
    codes = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.uint8): "U8"}
    for name, arr in tensors:
        b = arr.tobytes()
        header[prefix + name] = {"dtype": codes[arr.dtype], "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    header["__metadata__"] = {"format": "pt"}
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
    return 8 + len(h)


def _block_tensors(n_blocks, rng):
    out = []
    for i in range(n_blocks):
        out.append((f"blocks.{i}.attn.weight", rng.standard_normal((64, 48)).astype(np.float32)))
        out.append((f"blocks.{i}.attn.bias", rng.standard_normal((64,)).astype(np.float16)))
        out.append((f"blocks.{i}.q.weight", rng.integers(0, 256, (3400,), dtype=np.uint8)))
    return out


def _names(n_blocks):
    return [[f"blocks.{i}.attn.weight", f"blocks.{i}.attn.bias", f"blocks.{i}.q.weight"] for i in range(n_blocks)]


def test_file_block_layout(tmp_path):
    plan = _tiers("plan")
    rng = np.random.default_rng(0)
    tensors = _block_tensors(4, rng)
    path = str(tmp_path / "m.safetensors")
    base = _write_safetensors(path, tensors, prefix="net.")
    lay = plan.file_block_layout(path, _names(4))
    assert lay is not None and len(lay["ranges"]) == 4
    blk = 64 * 48 * 4 + 64 * 2 + 3400
    assert all(n == blk for _, n in lay["ranges"]) and lay["ranges"][0][0] == base
    assert lay["rel_offsets"] == [0, 64 * 48 * 4, 64 * 48 * 4 + 128] and lay["shapes"][0] == (64, 48)
    assert lay["dtypes"] == [torch.float32, torch.float16, torch.uint8]
    # a foreign tensor inside block 1's range: not contiguous
    t2 = tensors[:4] + [("other", np.zeros(16, np.float32))] + tensors[4:]
    _write_safetensors(path, t2)
    assert plan.file_block_layout(path, _names(4)) is None
    # a missing tensor
    assert plan.file_block_layout(path, _names(4) + [["blocks.9.x"]]) is None


def test_file_param_layout_and_piece_source(tmp_path):
    plan, src = _tiers("plan"), _tiers("sources")
    rng = np.random.default_rng(1)
    n = 3
    tensors = _block_tensors(n, rng)
    # grouped by dtype: all fp32 weights, then all fp16 biases, then all uint8 tensors
    grouped = [t for t in tensors if t[1].dtype == np.float32] + [t for t in tensors if t[1].dtype == np.float16] + \
        [t for t in tensors if t[1].dtype == np.uint8]
    path = str(tmp_path / "g.safetensors")
    _write_safetensors(path, grouped)
    assert plan.file_block_layout(path, _names(n)) is None
    lay = plan.file_param_layout(path, _names(n))
    assert lay is not None and lay["pieces_per_block"] == [3, 3, 3]
    ring = src.DiskRing(src.file_source(path, lay["ranges"]), depth=2, pin=False, threads=2)
    try:
        for cycle in range(2):
            for i in range(n):
                view, buf = ring.acquire(i)
                got = view.numpy().tobytes()
                want = bytearray(lay["block_bytes"])
                for k, (name, arr) in enumerate(tensors[3 * i:3 * i + 3]):
                    o = lay["rel_offsets"][k]
                    want[o:o + arr.nbytes] = arr.tobytes()
                assert got == bytes(want), (cycle, i)
                ring.release(buf)
    finally:
        ring.close()


@pytest.mark.parametrize("threads,depth", [(1, 2), (2, 3), (3, 3)])
def test_disk_store_and_ring_cycle(tmp_path, threads, depth):
    cf, src = _tiers("cache_files"), _tiers("sources")
    n, nbytes = 5, 10_000 + 37
    store = cf.DiskBlockStore(cf.new_cache_path(str(tmp_path)), nbytes, n)
    blocks = []
    for i in range(n):
        b = torch.randint(0, 256, (nbytes,), dtype=torch.uint8)
        st = store.staging()
        st.copy_(b)
        store.write_block(i, st)
        blocks.append(b)
    store.finalize()
    assert os.path.getsize(store.path) == n * store.stride and store.stride % 4096 == 0
    ring = src.DiskRing(store, depth=depth, pin=False, threads=threads)
    try:
        for cycle in range(3):   # reading runs on into the next forward
            for i in range(n):
                view, buf = ring.acquire(i)
                assert torch.equal(view, blocks[i]), (cycle, i)
                ring.release(buf)
            assert ring.at_cycle_start()
        with pytest.raises(RuntimeError, match="out of sync"):
            ring.acquire(3)
    finally:
        ring.close()
    store.delete()
    assert not os.path.exists(store.path)


def test_ring_restart_after_partial_forward(tmp_path):
    cf, src = _tiers("cache_files"), _tiers("sources")
    n = 4
    store = cf.DiskBlockStore(cf.new_cache_path(str(tmp_path)), 8192, n)
    for i in range(n):
        st = store.staging()
        st.fill_(i)
        store.write_block(i, st)
    store.finalize()
    ring = src.DiskRing(store, depth=2, pin=False, threads=2)
    msgs = []
    try:
        view, buf = ring.acquire(0)
        ring.release(buf)
        view, buf = ring.acquire(1)
        ring.release(buf)
        assert not ring.at_cycle_start()
        assert ring.restart_if_needed(msgs.append) and "part way" in msgs[-1]
        assert ring.at_cycle_start() and not ring.restart_if_needed(msgs.append)
        for i in range(n):
            view, buf = ring.acquire(i)
            assert int(view[0]) == i and int(view[-1]) == i
            ring.release(buf)
    finally:
        ring.close()
        store.delete()


def test_ring_reader_failure_reaches_the_consumer(tmp_path):
    cf, src = _tiers("cache_files"), _tiers("sources")
    n = 4
    store = cf.DiskBlockStore(cf.new_cache_path(str(tmp_path)), 8192, n)
    for i in range(n):
        st = store.staging()
        st.fill_(i + 1)
        store.write_block(i, st)
    store.finalize()
    with open(store.path, "r+b") as f:          # the last two blocks are lost
        f.truncate(2 * store.stride)
    ring = src.DiskRing(store, depth=4, pin=False, threads=1)
    msgs = []
    try:
        for i in range(2):                       # blocks read before the failure are still served
            view, buf = ring.acquire(i)
            assert int(view[0]) == i + 1
            ring.release(buf)
        with pytest.raises(RuntimeError, match="reader failed"):
            ring.acquire(2)
        assert ring.failed()
        # the file comes back: the restart reads the whole cycle again
        with open(store.path, "r+b") as f:
            for i in range(2, n):
                f.seek(i * store.stride)
                f.write(bytes([i + 1]) * store.stride)
        assert ring.restart_if_needed(msgs.append) and "failed" in msgs[-1]
        for i in range(n):
            view, buf = ring.acquire(i)
            assert int(view[0]) == i + 1
            ring.release(buf)
    finally:
        ring.close()
        store.delete()


def test_unbuffered_reader_end_of_file(tmp_path):
    dio = _tiers("disk_io")
    path = str(tmp_path / "f.bin")
    with open(path, "wb") as f:
        f.write(bytes(range(256)) * 20)          # 5120 bytes: one full 4 KiB page and a partial one
    buf, _ = dio.aligned_host(8192, pin=False)
    assert buf.data_ptr() % 4096 == 0
    r = dio._UnbufferedReader(path)
    try:
        r.read_into(0, 8192, buf.data_ptr(), min_bytes=5120)        # the end of the file is fine past min_bytes
        assert bytes(buf[:5120].numpy()) == bytes(range(256)) * 20
        with pytest.raises(EOFError):
            r.read_into(4096, 8192, buf.data_ptr(), min_bytes=5000)
    finally:
        r.close()


def test_probe_disk_caches_its_result(tmp_path):
    dio = _tiers("disk_io")
    p = dio.probe_disk(str(tmp_path), size_mb=8, chunk_mb=1, thread_counts=(1, 2))
    assert p["gbps"] > 0 and p["threads"] in (1, 2) and set(p["by_threads"]) == {1, 2}
    assert os.path.exists(os.path.join(str(tmp_path), dio._PROBE_FILE))
    assert not [n for n in os.listdir(str(tmp_path)) if n.endswith(".bin")]
    again = dio.probe_disk(str(tmp_path), size_mb=8, chunk_mb=1, thread_counts=(1, 2))
    assert again["by_threads"] == p["by_threads"]


def test_stale_cache_files_are_removed(tmp_path):
    cf = _tiers("cache_files")
    stale = tmp_path / "wfb200_blocks_999999999_0123456789abcdef0123456789abcdef.bin"
    stale.write_bytes(b"x" * 100)
    mine = cf.new_cache_path(str(tmp_path))
    open(mine, "wb").close()
    assert cf.cleanup_stale_cache_files(str(tmp_path)) == 100
    assert not stale.exists() and os.path.exists(mine)
