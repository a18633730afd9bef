"""The multi-rank host logic on CPU with gloo (world size 2): the TP group's all-gather / reduce-scatter of token
rows, a column / row split of a two-layer MLP combined through them equals the unsplit product (also in the
overlapped row-chunk forms mlp_rows / row_parallel_rows at 1, 2 and 4 chunks), and the sweep's
tensor bin-packing gives every rank a disjoint share whose union is the whole table."""

import os
import sys

import torch.multiprocessing as mp

from conftest import REPO


def _worker(rank, world, port, q):
    import datetime
    import importlib

    import torch
    import torch.distributed as dist
    sys.path.insert(0, REPO)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        cb = importlib.import_module("comfyui-weightferry_b200.streaming.cosmos_block")
        tp = cb.TP()
        g = torch.Generator().manual_seed(0)
        x = torch.randn(8, 16, generator=g, dtype=torch.float64)          # 8 token rows, hidden 16
        w1 = torch.randn(32, 16, generator=g, dtype=torch.float64)        # column-parallel (out rows split)
        w2 = torch.randn(16, 32, generator=g, dtype=torch.float64)        # row-parallel (in columns split)
        rows = 8 // world
        x_local = x[rank * rows:(rank + 1) * rows]
        full_x = tp.all_gather_rows(x_local)
        h = full_x @ w1[rank * 16:(rank + 1) * 16].t()                    # this rank's 16 of 32 channels
        part = h @ w2[:, rank * 16:(rank + 1) * 16].t()
        y_local = tp.reduce_scatter_rows(part)
        ref = (x @ w1.t() @ w2.t())[rank * rows:(rank + 1) * rows]
        ok = torch.allclose(y_local, ref, rtol=1e-12, atol=1e-9) and torch.equal(full_x, x)
        # the overlapped row-chunk forms (NCCL async on GPUs; the same chunk algebra here) equal the whole ones
        F = torch.nn.functional
        xx = torch.randn(16, 16, generator=g, dtype=torch.float64)
        aa = torch.randn(16, 32, generator=g, dtype=torch.float64)
        wo = torch.randn(16, 32, generator=g, dtype=torch.float64)
        r16 = 16 // world
        xl = xx[rank * r16:(rank + 1) * r16]
        w1s, w2s = w1[rank * 16:(rank + 1) * 16], w2[:, rank * 16:(rank + 1) * 16]
        ks = slice(rank * 32 // world, (rank + 1) * 32 // world)
        want_mlp = (F.gelu(xx @ w1.t()) @ w2.t())[rank * r16:(rank + 1) * r16]
        want_row = (aa @ wo.t())[rank * r16:(rank + 1) * r16]
        for chunks in ("1", "2", "4"):
            os.environ["WEIGHTFERRY_TP_CHUNKS"] = chunks
            assert tp.chunks(r16) == int(chunks)
            got_mlp = tp.mlp_rows(xl, w1s, w2s)
            got_row = tp.row_parallel_rows(aa[:, ks].contiguous(), wo[:, ks].contiguous())
            ok = ok and torch.allclose(got_mlp, want_mlp, rtol=1e-12, atol=1e-9)
            ok = ok and torch.allclose(got_row, want_row, rtol=1e-12, atol=1e-9)
        os.environ["WEIGHTFERRY_TP_CHUNKS"] = "3"
        ok = ok and tp.chunks(r16) == 1               # a count that does not divide the rows: unchunked
        os.environ.pop("WEIGHTFERRY_TP_CHUNKS")
        bench = importlib.import_module("bench")
        table = [s for _ in range(36 * world) for s in bench.cosmos14b_block_shapes()]
        sizes = [a * b for a, b in table]
        bins = bench.bin_pack(sizes, world)
        mine = set(bins[rank])
        everyone = [None] * world
        dist.all_gather_object(everyone, sorted(mine))
        union = set().union(*map(set, everyone))
        disjoint = sum(len(e) for e in everyone) == len(union)
        balanced = max(sum(sizes[i] for i in e) for e in everyone) == min(sum(sizes[i] for i in e) for e in everyone)
        q.put((rank, bool(ok), union == set(range(len(table))) and disjoint, balanced))
    finally:
        dist.destroy_process_group()


def test_tp_plumbing_and_sweep_sharding_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, 29611
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, partition, balanced in results:
        assert ok, f"rank {rank}: TP all-gather / reduce-scatter mismatch"
        assert partition, "bin-packing is not a partition of the tensor table"
        assert balanced


def _sp_worker(rank, world, port, q):
    import datetime
    import importlib

    import torch
    import torch.distributed as dist
    sys.path.insert(0, REPO)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        cb = importlib.import_module("comfyui-weightferry_b200.streaming.cosmos_block")
        ok = True
        # two samples over two ranks: one sample each, nothing exchanged
        sp = cb.SP(2, 8)
        ok = ok and sp.rows == 8 and sp.kv_ranks == 1 and sp.kv_group is None
        k = torch.full((1, 8, 2, 4), float(rank))
        ok = ok and sp.gather_kv(k, k)[0] is k
        # one sample over two ranks: keys / values gathered in token order
        sp = cb.SP(1, 8)
        ok = ok and sp.rows == 4 and sp.kv_ranks == 2
        k = torch.arange(4 * 2 * 4, dtype=torch.float32).view(1, 4, 2, 4) + 100 * rank
        v = -k
        ka, va = sp.gather_kv(k, v)
        want = torch.cat([torch.arange(32, dtype=torch.float32).view(1, 4, 2, 4) + 100 * r for r in range(world)], 1)
        ok = ok and torch.equal(ka, want) and torch.equal(va, -want)
        try:  # 6 rows per rank: neither whole samples of 4 tokens nor a divisor of one
            cb.SP(3, 4)
            ok = False
        except ValueError:
            pass
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_sp_rows_and_kv_gather_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, 29612
    procs = [ctx.Process(target=_sp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok in results:
        assert ok, f"rank {rank}: SP rows / key-value gather wrong"
