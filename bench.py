"""Benchmark of the B200 quantized-weight path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Workloads (seeded synthetic inputs with the configs' shapes and value distributions):
  sweep    (default) configs[1]: GGUF Q4_K -> bf16 dequantisation of a Cosmos-Predict2-14B checkpoint, sharded by
           tensor with no communication. Weak scaling: at N GPUs the tensor table is N x 36 blocks, bin-packed by
           bytes over the ranks, so every rank sweeps 36 blocks (14.16 G values, 7.96 GB in, 28.31 GB out) per
           step through one batched launch (wf_dequant_gguf_batch). Inputs are larger than L2, so no flush.
  q8       configs[0]: Q8_0 5120x5120 -> bf16 (one launch per step; L2 flushed between steps).
  q4k      configs[1]'s single FFN weight, Q4_K 5120x13824 -> bf16 (one launch per step; L2 flushed).
The default line also carries `stack`: configs[4], the streamed 14B block stack (the second half of BASELINE's metric,
s/step at this N, tensor-parallel over the ranks), timed after the sweep in the same run with its H2D GB/s against
the run's own pinned-copy probe, dequant-on-arrival ms per block and compute ms per forward (--stack-blocks 0: off).
Metric: GGUF dequant output GB/s (bf16 bytes written per second, all ranks). `e2e` is the same metric through the
reference-facing entry point (gguf_dequant.dequantize) with pinned host buffers: every step copies the packed
bytes host -> device, dequantises and copies the bf16 weight device -> host, for one block's 16 tensors.
--impl reference times the reference's algorithm on the host cores instead (the C restatement in oracle/, all
threads; there is no other CPU implementation of the path), on a bounded sample of the same workload.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

# dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant kernel, from one ncu capture of the same
# kernel (None until captured). Keyed by workload, scaled to the bench's launch.
NCU_TRAFFIC = {
    # one-block capture of the batched Q4_K dequantisation (221.20 MB read + 729.71 MB written) x 36 blocks
    "sweep": 34_232_680_000,
    # one configs[2] GEMM launch: 34.17 MB read + 87.15 MB written (the rest of Y still in L2 when the kernel ends)
    "w8a8": 121_317_632,
    "q8": None, "q4k": None, "prologue": None,
}

Q4K_TS, Q8_TS = 144, 34


def _pkg(mod):
    import importlib
    return importlib.import_module("comfyui-weightferry_b200." + mod)


# ----------------------------------------------------------------------------------------------------- workloads
def cosmos14b_block_shapes():
    """The 2-D weights of one Cosmos-Predict2-14B block (hidden 5120, 40 heads x 128, MLP 20480, cross-attention
    context 1024, adaLN-LoRA 256): 16 tensors, 393,216,000 values."""
    h, mlp, ctx, lora = 5120, 20480, 1024, 256
    shapes = [(h, h)] * 4                       # self-attention q, k, v, o
    shapes += [(h, h), (h, h), (h, ctx), (h, ctx)]  # cross-attention q, o, k, v
    shapes += [(mlp, h), (h, mlp)]              # MLP layer1, layer2
    for _ in range(3):                          # adaLN modulation (self-attn, cross-attn, MLP): LoRA down + up
        shapes += [(lora, h), (3 * h, lora)]
    return shapes


def bin_pack(sizes, n_bins):
    """Greedy largest-first assignment of items to the least-loaded bin; returns the item indices per bin."""
    order = sorted(range(len(sizes)), key=lambda i: -sizes[i])
    loads = [0] * n_bins
    bins = [[] for _ in range(n_bins)]
    for i in order:
        b = min(range(n_bins), key=lambda j: loads[j])
        bins[b].append(i)
        loads[b] += sizes[i]
    return bins


def fill_q4k(torch, n_blocks, device, gen):
    """Packed Q4_K super-blocks as BASELINE configs[1]: random bytes, d and dmin float16 U(0, 0.01)."""
    raw = torch.randint(0, 256, (n_blocks, Q4K_TS), dtype=torch.uint8, device=device, generator=gen)
    dd = (torch.rand((n_blocks, 2), device=device, generator=gen) * 0.01).half()
    raw[:, 0:4] = dd.view(torch.uint8)
    return raw.reshape(-1)


def fill_q8(torch, n_blocks, device, gen):
    """Packed Q8_0 blocks as BASELINE configs[0]: int8 quants uniform in [-127, 127], d = fp16(|N(0,1)| * 0.002)."""
    q = torch.randint(-127, 128, (n_blocks, 32), dtype=torch.int16, device=device, generator=gen).to(torch.int8)
    d = (torch.randn((n_blocks, 1), device=device, generator=gen).abs() * 0.002).half()
    return torch.cat([d.view(torch.uint8), q.view(torch.uint8)], dim=1).reshape(-1)


# ----------------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------------------------------- helpers
class L2Flush:
    """Evicts L2 (126 MB) between timed launches: writes a 512 MB buffer, then reads another 512 MB one. The write
    evicts the inputs; the read then replaces the lines the write left dirty with clean ones, so their write-back to
    DRAM happens here and not inside the next timed launch (where it would add up to 126 MB of writes to a kernel of
    a few tens of microseconds)."""

    def __init__(self, torch, dev):
        self.torch = torch
        self.w = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=dev)
        self.r = torch.zeros(128 * 1024 * 1024, dtype=torch.float32, device=dev)
        self.sink = torch.empty((), dtype=torch.float32, device=dev)

    def __call__(self):
        self.w.zero_()
        self.torch.sum(self.r, dim=0, dtype=self.torch.float32, out=self.sink)


L2_NOTE = "flushed before every timed launch: 512 MB written, then 512 MB read (the write-back leaves L2 first)"


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def setup_dist(torch):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        # NCCL prints its version line (and, with NCCL_DEBUG, more) on the C-level stdout when the communicator is
        # created: during that, file descriptor 1 points at stderr, so stdout carries only the JSON result line
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    return world, rank, local, dist


def max_over_ranks(torch, dist, value):
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(torch, dist, value):
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(torch, dist):
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


# ----------------------------------------------------------------------------------------------------- CPU baseline
def host_threads():
    """Host threads this process may use: the oracle's OpenMP pool is set to this explicitly, since a torchrun launch
    sets OMP_NUM_THREADS=1."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def use_all_host_threads(oracle):
    """Set the oracle's OpenMP thread count for the calling thread to host_threads(); returns it."""
    return int(oracle.set_threads(host_threads()))


def cpu_baseline_sweep(seconds=10.0):
    """The oracle port (oracle/wf_oracle.c, OpenMP, all host threads) on one BASELINE configs[1] weight, Q4_K
    5120x13824 -> bf16 (mid float16), repeated for about `seconds`. Returns (out GB/s, threads, sample text)."""
    from oracle import oracle
    rng = np.random.default_rng(20261201 + 1)
    n = 5120 * 13824
    nb = n // 256
    raw = rng.integers(0, 256, size=(nb, Q4K_TS), dtype=np.uint8)
    raw[:, 0:4] = (rng.uniform(0, 0.01, (nb, 2)).astype(np.float16)).view(np.uint8)
    threads = use_all_host_threads(oracle)
    oracle.dequant_gguf(raw, n, 12, 0, 1)  # warm-up (page faults, thread pool)
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.dequant_gguf(raw, n, 12, 0, 1)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = reps * n * 2 / el / 1e9
    return gbs, threads, f"Q4_K 5120x13824 -> bf16 (mid f16), {reps} reps in {el:.1f} s"


# ----------------------------------------------------------------------------------------------------- our arm
def run_sweep(torch, args, world, rank, dist):
    gd = _pkg("enhancers.gguf_dequant")
    ext = _pkg("_ext")
    dev = torch.device("cuda", torch.cuda.current_device())
    shapes = cosmos14b_block_shapes()
    table = [s for _ in range(args.blocks * world) for s in shapes]  # N x 36 blocks
    sizes = [a * b for a, b in table]
    mine = bin_pack(sizes, world)[rank]
    gen = torch.Generator(device=dev)
    gen.manual_seed(20261201 + 1 + rank)
    srcs, dsts = [], []
    tasks = (ext.DequantTask * len(mine))()
    n_values = 0
    for k, i in enumerate(mine):
        a, b = table[i]
        n = a * b
        src = fill_q4k(torch, n // 256, dev, gen)
        dst = torch.empty((a, b), dtype=torch.bfloat16, device=dev)
        srcs.append(src)
        dsts.append(dst)
        tasks[k].src, tasks[k].dst, tasks[k].n_values = src.data_ptr(), dst.data_ptr(), n
        n_values += n
    in_bytes = sum(s.numel() for s in srcs)
    out_bytes = n_values * 2
    lib = ext.lib()
    stream = torch.cuda.current_stream(dev)

    def step():
        rc = lib.wf_dequant_gguf_batch(tasks, len(mine), 12, 0, 1, stream.cuda_stream)
        if rc:
            ext.check(rc, "wf_dequant_gguf_batch")

    launches_per_step = -(-len(mine) // 640)
    for _ in range(args.warmup):
        step()
    barrier(torch, dist)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(torch.cuda.current_device()) as clk:
        barrier(torch, dist)
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        torch.cuda.nvtx.range_push("timed")
        for s in range(args.steps):
            ev[s][0].record(stream)
            step()
            ev[s][1].record(stream)
        torch.cuda.nvtx.range_pop()
        t_end.record(stream)
        barrier(torch, dist)
    total_ms = max_over_ranks(torch, dist, t_start.elapsed_time(t_end))
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)  # one batched launch per step (per table)
    total_out = sum_over_ranks(torch, dist, out_bytes * args.steps)
    value = total_out / (total_ms / 1e3) / 1e9
    del srcs, dsts
    torch.cuda.empty_cache()
    mix = hbm_mix_probe(torch, lib, ext, dev, in_bytes, out_bytes, stream)
    e2e = None
    if not args.no_e2e:
        e2e = e2e_block(torch, gd, dev, args)
        e2e["value"] = round(sum_over_ranks(torch, dist, e2e["value"]), 2)
    launches = int(sum_over_ranks(torch, dist, launches_per_step * args.steps))
    stack = None
    if args.stack_blocks > 0:
        torch.cuda.empty_cache()
        barrier(torch, dist)
        sr = stack_measure(torch, world, rank, dist, args.stack_blocks, args.stack_steps, args.stack_warmup,
                           parallel=args.parallel)
        stack = stack_subrecord(sr, world, args.stack_steps)
    return {
        "stack": stack,
        "value": value, "ms_per_step": total_ms / args.steps, "kern_ms": kern_ms,
        "alg_bytes_per_launch": (in_bytes + out_bytes) / launches_per_step, "clk": clk.summary(), "e2e": e2e,
        "gpu_launches": launches, "mix_gbs": mix,
        "config": {"workload": "GGUF Q4_K -> bf16 sweep of a Cosmos-Predict2-14B checkpoint (configs[1])",
                   "blocks_per_rank": args.blocks, "tensors_per_rank": len(mine), "values_per_rank": n_values,
                   "in_bytes_per_rank": in_bytes, "out_bytes_per_rank": out_bytes, "mid_dtype": "f16",
                   "sharding": "by tensor, greedy bin-pack of an N x 36-block table, no communication",
                   "l2": "inputs larger than L2 (36 GB per rank per step); no flush"},
    }


def hbm_mix_probe(torch, lib, ext, dev, in_bytes, out_bytes, stream):
    """GB/s of wf_hbm_probe -- a plain streaming kernel that reads in_bytes and writes out_bytes with coalesced
    16-byte accesses -- over buffers of the sweep's own sizes (mean of 3 launches after 1 untimed): the HBM rate this
    read : write mix reaches, beside the copy-based peak. Runs after the timed region, on its freed memory."""
    a = torch.empty(in_bytes // 16 * 16, dtype=torch.uint8, device=dev)
    b = torch.empty(out_bytes // 16 * 16, dtype=torch.uint8, device=dev)

    def go():
        ext.check(lib.wf_hbm_probe(a.data_ptr(), a.numel(), b.data_ptr(), b.numel(), stream.cuda_stream),
                  "wf_hbm_probe")

    go()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(3):
        go()
    e1.record(stream)
    torch.cuda.synchronize()
    gbs = 3 * (a.numel() + b.numel()) / (e0.elapsed_time(e1) / 1e3) / 1e9
    del a, b
    torch.cuda.empty_cache()
    return gbs


E2E_STREAMS = int(os.environ.get("WEIGHTFERRY_BENCH_E2E_STREAMS", "4"))
E2E_W8A8_CHUNKS = int(os.environ.get("WEIGHTFERRY_BENCH_E2E_CHUNKS", "8"))


def e2e_block(torch, gd, dev, args):
    """gguf_dequant.dequantize on one block's 16 Q4_K tensors with pinned host buffers: per step H2D of the packed
    bytes, the dequantisation, D2H of the bf16 weights (tensors spread over E2E_STREAMS streams, so the device-to-host
    copies -- 3.6 x the bytes of the host-to-device ones -- always have one queued while other tensors arrive and are
    dequantised)."""
    shapes = cosmos14b_block_shapes()
    gen = torch.Generator()
    gen.manual_seed(20261201 + 11)
    hosts, houts, dsrc = [], [], []
    for a, b in shapes:
        raw = torch.randint(0, 256, (a * b // 256, Q4K_TS), dtype=torch.uint8, generator=gen)
        raw[:, 0:4] = (torch.rand((a * b // 256, 2), generator=gen) * 0.01).half().view(torch.uint8)
        hosts.append(raw.reshape(-1).pin_memory())
        houts.append(torch.empty((a, b), dtype=torch.bfloat16).pin_memory())
        dsrc.append(torch.empty(raw.numel(), dtype=torch.uint8, device=dev))
    streams = [torch.cuda.Stream(dev) for _ in range(E2E_STREAMS)]
    h2d = sum(h.numel() for h in hosts)
    d2h = sum(h.numel() * 2 for h in houts)

    def step():
        for i, ((a, b), h) in enumerate(zip(shapes, hosts)):
            s = streams[i % len(streams)]
            with torch.cuda.stream(s):
                dsrc[i].copy_(h, non_blocking=True)
                w = gd.dequantize(dsrc[i], 12, (a, b), None, torch.bfloat16)
                houts[i].copy_(w, non_blocking=True)
                w.record_stream(s)
        for s in streams:
            torch.cuda.current_stream(dev).wait_stream(s)

    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize()
    steps = max(3, args.steps // 2)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / steps
    return {"value": d2h / (ms / 1e3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": round(ms, 3), "sample": "one Cosmos-14B block (16 Q4_K tensors) per step"}


def w8a8_operands(torch, dev, seed):
    """X bf16 [2 x 4096, 2048] ~ N(0, 1); W_fp ~ N(0, 0.02) [8192, 2048] -> int8 per output
    channel (symmetric, scale = amax / 127), as the int8 layout the reference consumes."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn((8192, 2048), device=dev, generator=g).to(torch.bfloat16)
    w_fp = torch.randn((8192, 2048), device=dev, generator=g) * 0.02
    ws = (w_fp.abs().amax(dim=1) / 127.0).float().contiguous()
    wq = torch.clamp(torch.round(w_fp / ws.view(-1, 1)), -127, 127).to(torch.int8).contiguous()
    return x, wq, ws


def run_w8a8(torch, args, world, rank, dist):
    """per-token quantisation (plain absmax) + tcgen05 int8 GEMM + rescale epilogue, one step = the whole
    linear; L2 flushed before every step (X and W together fit in L2)."""
    fk = _pkg("enhancers.fused_kernels")
    fi = _pkg("enhancers.fused_int8")
    ext = _pkg("_ext")
    dev = torch.device("cuda", torch.cuda.current_device())
    x, wq, ws = w8a8_operands(torch, dev, 20261201 + 2 + rank)
    M, K = x.shape
    N = wq.shape[0]
    xq = torch.empty((M, K), dtype=torch.int8, device=dev)
    xs = torch.empty((M, 1), dtype=torch.float32, device=dev)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    flush = L2Flush(torch, dev)
    lib = ext.lib()
    stream = torch.cuda.current_stream(dev)
    kq = fk._get_kernels()["quant_row"][(M,)]

    def quant():
        kq(x, None, None, xq, xs, 1, 0.0, K=K, PRE=fk.PRE_NONE, ROTATE=False)

    def gemm():
        rc = lib.wf_w8a8_gemm(xq.data_ptr(), wq.data_ptr(), xs.data_ptr(), ws.data_ptr(), y.data_ptr(), None, M, N,
                              K, stream.cuda_stream)
        if rc:
            ext.check(rc, "wf_w8a8_gemm")

    for _ in range(args.warmup):
        flush()
        quant()
        gemm()
    barrier(torch, dist)
    # the step: the whole linear, events only around it (an event between the two kernels would stop the GEMM from
    # launching as a programmatic dependent of the quantiser)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(torch.cuda.current_device()) as clk:
        barrier(torch, dist)
        for s in range(args.steps):
            flush()
            ev[s][0].record(stream)
            quant()
            gemm()
            ev[s][1].record(stream)
        barrier(torch, dist)
    step_ms = max_over_ranks(torch, dist, statistics.mean(a.elapsed_time(b) for a, b in ev))
    # the split, for the roofline of the GEMM kernel: an event between the kernels (each runs alone)
    evq = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    evg = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for s in range(args.steps):
        flush()
        evq[s][0].record(stream)
        quant()
        evq[s][1].record(stream)
        gemm()
        evg[s].record(stream)
    torch.cuda.synchronize()
    q_ms = statistics.mean(a.elapsed_time(b) for a, b in evq)
    g_ms = statistics.mean(evq[s][1].elapsed_time(evg[s]) for s in range(args.steps))
    ops = 2.0 * M * N * K
    value = sum_over_ranks(torch, dist, ops / (step_ms / 1e3) / 1e12)
    st = __import__("ctypes").c_int(0)
    lib.wf_w8a8_gemm_status(__import__("ctypes").byref(st))
    # cuBLASLt int8 through torch._int_mm on the same operands, for context (a library GEMM without the epilogue)
    lib_ms = None
    try:
        for _ in range(3):
            torch._int_mm(xq, wq.t())
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        tot = 0.0
        for _ in range(5):
            flush()
            e0.record(stream)
            torch._int_mm(xq, wq.t())
            e1.record(stream)
            torch.cuda.synchronize()
            tot += e0.elapsed_time(e1)
        lib_ms = tot / 5
    except Exception:  # noqa: BLE001 -- context only
        lib_ms = None
    sustained = w8a8_sustained(torch, lib, ext, xq, wq, xs, ws, y, stream, ops, args.sustained_seconds) \
        if args.sustained_seconds > 0 else {}
    e2e = None
    if not args.no_e2e:
        e2e = e2e_w8a8(torch, fi, x, wq, ws, dev, args)
        e2e["value"] = round(sum_over_ranks(torch, dist, e2e["value"]), 2)
    return {
        "value": value, "ms_per_step": step_ms, "kern_ms": g_ms, "alg_ops_per_launch": ops, "clk": clk.summary(),
        "sustained": sustained,
        "e2e": e2e, "gpu_launches": int(sum_over_ranks(torch, dist, 2 * args.steps)), "gemm_status": st.value,
        "config": {"workload": "W8A8 linear, X bf16 [8192, 2048] x W int8 [8192, 2048]^T -> Y bf16 [8192, 8192] "
                               "(configs[2], Cosmos-Predict2-2B MLP up-projection)",
                   "quantiser": "per-token absmax int8 (plain, no rotation)", "quant_ms": round(q_ms, 4),
                   "gemm_ms": round(g_ms, 4),
                   "cublaslt_int_mm_ms": None if lib_ms is None else round(lib_ms, 4),
                   "l2": L2_NOTE},
    }


W8A8_SUSTAINED_S = 2.0  # seconds of back-to-back launches per kernel (--sustained-seconds)


def w8a8_sustained(torch, lib, ext, xq, wq, xs, ws, y, stream, ops, seconds=W8A8_SUSTAINED_S):
    """The GEMM and cuBLASLt's `_int_mm` (int32 out, no epilogue) on the same operands, each launched back to back for
    W8A8_SUSTAINED_S seconds -- the regime of a model's forward, where the 1 kW power cap sets the clock -- with the
    clocks sampled during each run. A single launch (the step above) runs at the boost clock instead."""
    M, K = xq.shape
    N = wq.shape[0]
    yi = torch.empty((M, N), dtype=torch.int32, device=xq.device)
    wt = wq.t()

    def ours():
        rc = lib.wf_w8a8_gemm(xq.data_ptr(), wq.data_ptr(), xs.data_ptr(), ws.data_ptr(), y.data_ptr(), None, M, N,
                              K, stream.cuda_stream)
        if rc:
            ext.check(rc, "wf_w8a8_gemm")

    def cublaslt():
        torch._int_mm(xq, wt, out=yi)

    out = {}
    for name, fn in (("wf_w8a8_gemm", ours), ("cublaslt_int_mm", cublaslt)):
        try:
            for _ in range(20):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n = max(1, int(seconds / 100e-6))
            with ClockSampler(torch.cuda.current_device()) as clk:
                e0.record(stream)
                for _ in range(n):
                    fn()
                e1.record(stream)
                torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / n
            out[name] = {"us_per_launch": round(us, 2), "tops": round(ops / (us / 1e6) / 1e12, 1), "launches": n,
                         "clocks": clk.summary()}
        except Exception as e:  # noqa: BLE001 -- cuBLASLt is context only
            out[name] = {"error": str(e)[:200]}
    del yi
    return out


def e2e_w8a8(torch, fi, x, wq, ws, dev, args):
    """fused_int8.int8_linear (the package's entry point) with pinned host buffers: per step H2D of X, the linear,
    D2H of Y -- in E2E_W8A8_CHUNKS row chunks on their own streams (per-token quantisation is row by row, so the
    chunks' results are the rows of the whole linear), so one chunk's device-to-host copy overlaps the next chunk's
    host-to-device copy and linear."""
    hx = x.cpu().pin_memory()
    hy = torch.empty((x.shape[0], wq.shape[0]), dtype=torch.bfloat16).pin_memory()
    dx = torch.empty_like(x)
    n_ch = E2E_W8A8_CHUNKS
    bounds = [x.shape[0] * i // n_ch for i in range(n_ch + 1)]
    streams = [torch.cuda.Stream(dev) for _ in range(n_ch)]
    main = torch.cuda.current_stream(dev)

    def step():
        for i, s in enumerate(streams):
            s.wait_stream(main)
            with torch.cuda.stream(s):
                r0, r1 = bounds[i], bounds[i + 1]
                dx[r0:r1].copy_(hx[r0:r1], non_blocking=True)
                y = fi.int8_linear(dx[r0:r1], wq, ws)
                hy[r0:r1].copy_(y, non_blocking=True)
                y.record_stream(s)
        for s in streams:
            main.wait_stream(s)

    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize()
    steps = max(3, args.steps // 2)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / steps
    ops = 2.0 * x.shape[0] * wq.shape[0] * x.shape[1]
    return {"value": ops / (ms / 1e3) / 1e12, "unit": "TOPS", "h2d_bytes_per_step": x.numel() * 2,
            "d2h_bytes_per_step": hy.numel() * 2, "ms_per_step": round(ms, 3)}


def cpu_baseline_w8a8(seconds=10.0):
    """The reference's arithmetic on the host: per-token quantisation (oracle) + an exact int8 GEMM (torch CPU,
    int8 operands widened to float64) + the rescale, on the first 64-row slices of configs[2] until ~seconds."""
    import torch
    from oracle import oracle
    g = torch.Generator().manual_seed(20261201 + 2)
    rows = 64
    x = torch.randn((rows, 2048), generator=g).to(torch.bfloat16)
    w_fp = torch.randn((8192, 2048), generator=g) * 0.02
    ws = (w_fp.abs().amax(dim=1) / 127.0).double()
    wq = torch.clamp(torch.round(w_fp / ws.float().view(-1, 1)), -127, 127).double()
    xb = x.view(torch.int16).numpy().view(np.uint16)
    use_all_host_threads(oracle)
    torch.set_num_threads(host_threads())
    reps, t0 = 0, time.perf_counter()
    while True:
        q, sc = oracle.quant_rows(xb, pre=0, rotate=False)
        acc = torch.from_numpy(q.astype(np.float64)) @ wq.t()
        _y = (acc * torch.from_numpy(sc.astype(np.float64)).view(-1, 1) * ws.view(1, -1)).to(torch.bfloat16)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    ops = 2.0 * rows * 8192 * 2048 * reps
    return ops / el / 1e12, torch.get_num_threads(), f"{reps} x 64 rows of configs[2] in {el:.1f} s"


def h2d_probe(torch, dev, nbytes=1 << 30, reps=5, dist=None):
    """Pinned -> device cudaMemcpyAsync of 1 GiB, best of `reps` (the measured PCIe H2D bandwidth). Under several
    ranks every rank copies at the same time (a barrier before each copy), so the figure is this rank's share of
    what the host delivers to all its GPUs at once -- the bandwidth the streamed stack's ranks actually share."""
    host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    dst.copy_(host, non_blocking=True)
    torch.cuda.synchronize()
    best = 0.0
    for _ in range(reps):
        barrier(torch, dist)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dst.copy_(host, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        best = max(best, nbytes / (e0.elapsed_time(e1) / 1e3) / 1e9)
    del host, dst
    return best


_KERNEL_KINDS = (("nccl", ("nccl",)), ("attention", ("flash", "fmha", "attention", "sdpa", "softmax", "cudnn")),
                 ("gemm", ("gemm", "cutlass", "xmma", "nvjet", "sm100", "cublas")),
                 ("dequant", ("dequant_kernel",)), ("prologue", ("ln_modulate", "rms_rope", "rms128", "gated_residual")))


def kernel_breakdown(torch, step, dist):
    """GPU time of one (untimed) forward per kind of kernel on this rank, from torch.profiler's CUDA activity (names
    matched by substring: NCCL collectives, GEMMs, attention, the dequantisation on arrival, the prologue kernels,
    other) plus the host-to-device copies; each rank's figures are gathered to rank 0."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    kinds = {k: 0.0 for k, _ in _KERNEL_KINDS}
    kinds.update(other=0.0, h2d_copy=0.0)
    for ev in prof.events():
        dt = getattr(ev, "device_time_total", None)
        if dt is None:
            dt = getattr(ev, "cuda_time_total", 0.0)
        if not dt or ev.device_type is None or "cuda" not in str(ev.device_type).lower():
            continue
        name = ev.name.lower()
        if "memcpy" in name and ("htod" in name or "host to device" in name or "h2d" in name):
            kinds["h2d_copy"] += dt
            continue
        if "memcpy" in name or "memset" in name:
            continue
        for kind, keys in _KERNEL_KINDS:
            if any(k in name for k in keys):
                kinds[kind] += dt
                break
        else:
            kinds["other"] += dt
    mine = {k: round(v / 1e3, 2) for k, v in kinds.items()}  # ms
    if dist is None:
        return [mine]
    every = [None] * dist.get_world_size()
    dist.all_gather_object(every, mine)
    return every


def kernels_by_name(torch, fn, reps=5, top=14):
    """GPU time per kernel name of `reps` calls of fn (torch.profiler's CUDA activity), in ms per call, largest
    first: [(name, launches per call, ms per call), ...] for the `top` largest, plus the total."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
    agg = {}
    for ev in prof.events():
        dt = getattr(ev, "device_time_total", None)
        if dt is None:
            dt = getattr(ev, "cuda_time_total", 0.0)
        if not dt or ev.device_type is None or "cuda" not in str(ev.device_type).lower():
            continue
        name = ev.name
        if "memcpy" in name.lower() or "memset" in name.lower():
            continue
        a = agg.setdefault(name[:110], [0, 0.0])
        a[0] += 1
        a[1] += dt
    rows = sorted(agg.items(), key=lambda kv: -kv[1][1])
    out = [(name, c // reps, round(t / reps / 1e3, 4)) for name, (c, t) in rows[:top]]
    return {"kernels": out, "total_ms": round(sum(t for _, t in agg.values()) / reps / 1e3, 4)}


def stack_measure(torch, world, rank, dist, blocks, steps, warmup, slots=3, e2e=False, profile=False,
                  parallel="sp"):
    """a Cosmos-Predict2-14B-shaped stack of `blocks` blocks, Q8_0 weights in pinned host RAM streamed
    through `slots` GPU slots and dequantised on arrival, batch 2 x 4096 tokens (+ 512 context tokens), tensor-parallel
    over the ranks (column / row split, NCCL all-gather / reduce-scatter of the token rows). One step = one forward;
    `steps` forwards timed with CUDA events on the compute stream, max over ranks; then one more forward with the
    streaming profiler's event timeline on (not timed)."""
    cb = _pkg("streaming.cosmos_block")
    stk = _pkg("streaming.stack")
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = cb.COSMOS_14B
    tp = cb.TP()
    batch, T, H, W, S = 2, 1, 64, 64, 512
    tokens = T * H * W
    # each rank's pinned weights on its GPU's NUMA node (first touch after binding): no cross-socket DMA
    numa_cpus = _pkg("core.tiers.pinned").bind_to_gpu_numa(dev.index) if world > 1 else None
    probe = h2d_probe(torch, dev, dist=dist)
    t_build = time.perf_counter()
    sp = cb.SP(batch, tokens) if parallel == "sp" else None
    stack = stk.StreamedStack(cfg, blocks, dev, tp, seed=20261201 + 4, num_slots=slots, parallel=parallel, sp=sp)
    build_s = time.perf_counter() - t_build
    g = torch.Generator(device=dev)
    g.manual_seed(20261201 + 4)
    rows = batch * tokens // tp.world
    x_full = torch.randn((batch * tokens, cfg.hidden), device=dev, generator=g).to(torch.bfloat16)
    x = x_full[tp.rank * rows:(tp.rank + 1) * rows].contiguous()
    del x_full
    emb = (torch.randn((batch, cfg.hidden), device=dev, generator=g) * 0.5).to(torch.bfloat16)
    lora = (torch.randn((batch, 3 * cfg.hidden), device=dev, generator=g) * 0.05).to(torch.bfloat16)
    ctx = torch.randn((batch, S, cfg.ctx_dim), device=dev, generator=g).to(torch.bfloat16)
    rope = cb.rope3d_table(T, H, W, device=dev)

    def step():
        return stack.forward(x, emb, ctx, rope, batch, tokens, lora)

    for _ in range(warmup):
        out = step()
    barrier(torch, dist)
    stream = torch.cuda.current_stream(dev)
    with ClockSampler(torch.cuda.current_device()) as clk:
        barrier(torch, dist)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            out = step()
        e1.record(stream)
        barrier(torch, dist)
    ms = max_over_ranks(torch, dist, e0.elapsed_time(e1) / steps)
    finite = bool(torch.isfinite(out.float()).all().item())
    h2d_rank = blocks * stack.bytes_per_block
    h2d_rate = h2d_rank / (ms / 1e3) / 1e9
    prof_mod = _pkg("streaming.profiler")
    stack.state.profiler = prof_mod._StreamProfiler(stack.state.num_stream, stack.bytes_per_block)
    step()
    summ = stack.state.profile_summary()["per_forward"][-1]
    stack.state.profiler = None
    breakdown = kernel_breakdown(torch, step, dist) if profile else None
    flops = cb.flops_per_block(cfg, batch, tokens, S) * blocks
    e2e_rec = None
    if e2e:
        hx = x.cpu().pin_memory()
        hy = torch.empty_like(hx).pin_memory()
        dx = torch.empty_like(x)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(max(1, steps // 2)):
            dx.copy_(hx, non_blocking=True)
            y = stack.forward(dx, emb, ctx, rope, batch, tokens, lora)
            hy.copy_(y, non_blocking=True)
        t1.record()
        torch.cuda.synchronize()
        e_ms = max_over_ranks(torch, dist, t0.elapsed_time(t1) / max(1, steps // 2))
        e2e_rec = {"value": round(e_ms / 1e3, 4), "unit": "s/step", "h2d_bytes_per_step": hx.numel() * 2 + h2d_rank,
                   "d2h_bytes_per_step": hy.numel() * 2,
                   "note": "activation rows H2D + D2H per step around the streamed forward; weights stream H2D inside"}
    stack.close()
    del stack
    torch.cuda.empty_cache()
    return {"ms": ms, "clk": clk.summary(), "e2e": e2e_rec, "finite": finite, "probe": probe, "h2d_rate": h2d_rate,
            "h2d_rank": h2d_rank, "flops": flops, "summary": summ, "build_s": build_s, "blocks": blocks,
            "breakdown": breakdown, "parallel": parallel,
            "slots": slots, "numa_cpus": None if numa_cpus is None else len(numa_cpus)}


def _parallel_text(parallel, world):
    if parallel == "sp":
        return (f"sp{world} (each rank streams 1/{world} of every block's bytes, all-gathered over NVLink into "
                "whole blocks; token rows split over the ranks; keys / values gathered within a sample)")
    return f"tp{world} (column/row split, sequence-sharded residual)"


def stack_subrecord(r, world, steps):
    """The stack's half of BASELINE's metric as a sub-record of the default line."""
    summ = r["summary"]
    return {
        "metric": "streamed 14B DiT block-stack s/step", "value": round(r["ms"] / 1e3, 5), "unit": "s/step",
        "higher_is_better": False, "scaling": "strong", "steps": steps, "n_gpus": world,
        "parallelism": _parallel_text(r["parallel"], world), "blocks": r["blocks"],
        "h2d_gbs_per_rank": round(r["h2d_rate"], 2), "h2d_probe_gbs_per_rank": round(r["probe"], 2),
        "h2d_probe_note": "1 GiB pinned copies on every rank at once: this rank's share of the host's bandwidth",
        "h2d_frac_of_probe": round(r["h2d_rate"] / r["probe"], 4),
        "h2d_bytes_per_block_per_rank": r["h2d_rank"] // r["blocks"],
        "dequant_on_arrival_ms_per_block_per_rank": round(summ["dequant_lora_ms"] / max(1, summ["streamed_blocks"]),
                                                           4),
        "compute_ms_per_forward": summ["streamed_compute_ms"], "dma_ms_per_forward": summ["dma_ms"],
        "stall_ms_per_forward": summ["stall_ms"], "forward_ms_profiled": summ["forward_ms"],
        "tflops_per_gpu": round(r["flops"] / world / (r["ms"] / 1e3) / 1e12, 1), "finite_output": r["finite"],
        "build_s": round(r["build_s"], 1), "clocks": r["clk"],
        "note": "timed after the sweep in the same run; profiled timeline from one extra (untimed) forward"}


def run_stack(torch, args, world, rank, dist):
    return stack_measure(torch, world, rank, dist, args.blocks, args.steps, args.warmup, slots=args.slots,
                         e2e=not args.no_e2e, profile=args.profile, parallel=args.parallel)


def cpu_baseline_stack(seconds=10.0):
    """The block's work on the host: the oracle's Q8_0 dequantisation of one Cosmos-14B block (all tensors) and a
    torch CPU forward of its projections on 64 token rows, extrapolated by FLOPs to 8192 rows and 36 blocks."""
    import torch
    from oracle import oracle
    rng = np.random.default_rng(4)
    sizes = [(a, b) for a, b in cosmos14b_block_shapes()]
    t0 = time.perf_counter()
    deq_s = 0.0
    gemm_s = 0.0
    reps = 0
    while time.perf_counter() - t0 < seconds:
        for a, b in sizes[:4] + sizes[8:10]:
            nb = a * b // 32
            raw = np.empty((nb, 34), dtype=np.uint8)
            raw[:, 2:] = rng.integers(0, 256, size=(nb, 32), dtype=np.uint8)
            raw[:, 0:2] = (np.abs(rng.standard_normal((nb, 1))) * 0.002).astype(np.float16).view(np.uint8)
            t = time.perf_counter()
            w = oracle.dequant_gguf(raw, a * b, 8, 0, 1)
            deq_s += time.perf_counter() - t
            wt = torch.from_numpy(w.view(np.int16)).view(torch.bfloat16).reshape(a, b).float()
            x = torch.randn((64, b))
            t = time.perf_counter()
            _y = x @ wt.t()
            gemm_s += time.perf_counter() - t
        reps += 1
    # the sample covered q/k/v/o and the MLP (the block's dominant bytes and FLOPs): scale GEMMs to 8192 rows
    per_block = deq_s / reps * (417_792_000 / (34 / 32 * sum(a * b for a, b in sizes[:4] + sizes[8:10])))
    per_block += gemm_s / reps * (8192 / 64)
    return per_block * 36, torch.get_num_threads(), (f"{reps} reps of the oracle dequant + CPU GEMMs of one block's "
                                                     "q/k/v/o/MLP weights on 64 rows, extrapolated to 8192 rows, "
                                                     "all weights and 36 blocks")


def finish_stack(torch, args, world, rank, dist, r):
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, threads, sample = cpu_baseline_stack(args.cpu_seconds)
        cpu = {"value": round(v, 2), "unit": "s/step", "cores": threads, "kind": "port", "sample": sample}
    if dist is not None:
        dist.barrier()
    if rank == 0:
        frac = r["h2d_rate"] / r["probe"]
        print(json.dumps({
            "metric": "streamed 14B DiT block-stack s/step", "value": round(r["ms"] / 1e3, 5), "unit": "s/step",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms"], 3),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "Q8_0 -> bf16",
            "data": "synthetic (seeded)",
            "config": {"workload": "Cosmos-Predict2-14B-shaped stack (configs[4]): 36 blocks, hidden 5120, 40 x 128 "
                                   "heads, MLP 20480, Q8_0 weights in pinned host RAM, batch 2 x 4096 tokens + 512 "
                                   "context tokens", "blocks": args.blocks, "slots": r["slots"],
                       "parallelism": _parallel_text(r["parallel"], world),
                       "h2d_bytes_per_block_per_rank": r["h2d_rank"] // args.blocks,
                       "h2d_probe_gbs_per_rank": round(r["probe"], 2), "finite_output": r["finite"],
                       "numa_local_cpus_per_rank": r.get("numa_cpus"),
                       "build_s": round(r["build_s"], 1),
                       "timeline_one_forward": r["summary"],
                       "kernel_ms_per_rank_one_forward": r.get("breakdown")},
            "roofline": {"bound": "pcie_h2d", "achieved": round(r["h2d_rate"], 2), "peak": round(r["probe"], 2),
                         "unit": "GB/s per rank", "frac": round(frac, 4), "traffic": None,
                         "peak_source": "pinned 1 GiB cudaMemcpyAsync H2D measured in this run, every rank copying "
                                        "at once",
                         "tflops_per_gpu": round(r["flops"] / world / (r["ms"] / 1e3) / 1e12, 1)},
            "cpu_baseline": cpu, "e2e": r["e2e"], "gpu_launches": None, "clocks": r["clk"]}), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_prologue(torch, args, world, rank, dist):
    """the fused Cosmos-Predict2-2B block prologue. Kernel A (LayerNorm + adaLN modulate) on x
    [2, 4096, 2048]; kernel B (RMSNorm-128 + 3D RoPE) on q and k [2, 4096, 16, 128], one launch for both. One step =
    A + B. Timed as a sequence of launches, the way the block runs them, over 8 rotating sets of tensors (1.6 GB, 13x
    L2), so each launch reads inputs that are not in L2 and no flush is needed: per kernel, a run of 8 * steps
    launches of it between two events, and the step as A + B alternating."""
    fb = _pkg("enhancers.fused_block")
    sf = _pkg("enhancers.sage_fused")
    cb = _pkg("streaming.cosmos_block")
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(20261201 + 3 + rank)
    n_sets = 8
    sets = []
    for _ in range(n_sets):
        x = torch.randn((2, 1, 64, 64, 2048), device=dev, generator=g).to(torch.bfloat16)
        q = torch.randn((2, 4096, 16, 128), device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn((2, 4096, 16, 128), device=dev, generator=g).to(torch.bfloat16)
        sets.append((x, q, k, torch.empty_like(x)))
    sc = (torch.randn((2, 1, 1, 1, 2048), device=dev, generator=g) * 0.1).to(torch.bfloat16)
    sh = (torch.randn((2, 1, 1, 1, 2048), device=dev, generator=g) * 0.1).to(torch.bfloat16).contiguous()
    wq = (1 + torch.randn(128, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    wk = (1 + torch.randn(128, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    rope = cb.rope3d_table(1, 64, 64, device=dev)
    stream = torch.cuda.current_stream(dev)
    s1 = (1 + sc).contiguous()
    ln = fb._get_kernels()["lnmod"][(8192,)]
    fk = _pkg("enhancers.fused_kernels")
    kq = fk._get_kernels()["quant_row"][(8192,)]
    xq = torch.empty((8192, 2048), dtype=torch.int8, device=dev)
    xs = torch.empty((8192, 1), dtype=torch.float32, device=dev)

    def kernel_a(i):
        x, _q, _k, out = sets[i % n_sets]
        ln(x, s1, sh, out, 4096, 1e-6, K=2048)

    def kernel_b(i):
        _x, q, k, _o = sets[i % n_sets]
        return sf.rms_rope_pair(q, k, rope, wq, wk, 1e-6)

    # the int8 quantisers the W8A8 block runs on the same x (context, not part of the step): plain per-token, and
    # with the LayerNorm + modulate pending (kernel A's arithmetic with a quantising epilogue)
    def quant_plain(i):
        kq(sets[i % n_sets][0], None, None, xq, xs, 1, 0.0, K=2048, PRE=fk.PRE_NONE, ROTATE=False)

    def quant_lnmod(i):
        kq(sets[i % n_sets][0], s1, sh, xq, xs, 4096, 1e-6, K=2048, PRE=fk.PRE_LNMOD, ROTATE=False)

    def timed(fn, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(n):
            fn(i)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    n = n_sets * args.steps
    for i in range(max(args.warmup, 1) * n_sets):
        kernel_a(i)
        kernel_b(i)
    barrier(torch, dist)
    with ClockSampler(torch.cuda.current_device()) as clk:
        barrier(torch, dist)
        a_ms = timed(kernel_a, n)
        b_ms = timed(kernel_b, n)
        step_run_ms = timed(lambda i: (kernel_a(i), kernel_b(i)), n)
        barrier(torch, dist)
    # context: PyTorch's copy of the same bytes over the same rotation
    dst_a, dst_b = [torch.empty_like(s_[0]) for s_ in sets], [torch.empty_like(s_[1]) for s_ in sets]
    copy_a = timed(lambda i: dst_a[i % n_sets].copy_(sets[i % n_sets][0]), n)
    copy_b = timed(lambda i: (dst_b[i % n_sets].copy_(sets[i % n_sets][1]),
                              dst_b[(i + 1) % n_sets].copy_(sets[i % n_sets][2])), n)
    del dst_a, dst_b
    for i in range(n_sets):
        quant_plain(i)
        quant_lnmod(i)
    qp_ms = timed(quant_plain, n)
    ql_ms = timed(quant_lnmod, n)
    x, q, k, _o = sets[0]
    bytes_a = 2 * x.numel() * 2                          # read x + write out (+16 KB parameters)
    bytes_b = 2 * (q.numel() + k.numel()) * 2 + rope.numel() * 4  # q, k in + out; the table (one launch for both)
    step_ms = max_over_ranks(torch, dist, step_run_ms)
    value = sum_over_ranks(torch, dist, (bytes_a + bytes_b) / (step_ms / 1e3) / 1e9)
    return {"value": value, "ms": step_ms, "a_ms": a_ms, "b_ms": b_ms, "bytes_a": bytes_a, "bytes_b": bytes_b,
            "clk": clk.summary(), "launches": int(sum_over_ranks(torch, dist, 2 * n)),
            "copy_a_us": copy_a * 1e3, "copy_b_us": copy_b * 1e3, "quant_plain_us": qp_ms * 1e3,
            "quant_lnmod_us": ql_ms * 1e3, "quant_bytes": x.numel() * 3 + 8192 * 4}


def run_block(torch, args, world, rank, dist):
    """The fused Cosmos block drop-in against the unpatched block forward, on a Cosmos-Predict2-2B block at configs[3]'s
    shape (x [2, 1, 64, 64, 2048], 16 heads of 128, MLP 8192, AdaLN-LoRA 256, 512 context tokens of 1024). ComfyUI is
    absent, so the block is the stand-in of its Cosmos classes the drop-in tests use (tests/fake_comfy.py): the
    unpatched forward is PyTorch's LayerNorm, modulation, RMSNorm, float32 RoPE and addcmul around the Linear modules
    and SDPA; the patched one is install()'s. bf16 weights time both; int8 (ConvRot) weights time the patched forward,
    its GEMMs this library's W8A8 path -- the two layers it leaves to ComfyUI (the cross-attention's k / v
    projections of the context) run on the same kernels in place of comfy_kitchen's. The reference's figure for this
    comparison: fused Anima block 22.1 vs 30.3 ms (RTX 4060)."""
    sys.path.insert(0, os.path.join(REPO, "tests"))
    fb = _pkg("enhancers.fused_block")  # imported before the stand-in exists: nothing installed at import
    import fake_comfy
    fake_comfy.FAST_INT8 = True  # the layers the drop-in leaves to ComfyUI run on kernels, as comfy_kitchen's would
    p2 = fake_comfy.register()
    dims = dict(x_dim=2048, ctx_dim=1024, heads=16, mlp_dim=8192, lora=True, lora_dim=256)
    inputs = fake_comfy.block_inputs(x_dim=2048, ctx_dim=1024, B=2, T=1, H=64, W=64, S=512, lora=True,
                                     device=f"cuda:{torch.cuda.current_device()}")
    x, emb, ctx, rope, lora_t = inputs
    stream = torch.cuda.current_stream()
    n = max(args.steps, 5)

    def timed(blk, parts):
        fb.install(parts)
        with torch.no_grad():
            for _ in range(args.warmup):
                blk(x, emb, ctx, rope, lora_t, None, {})
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(n):
                out = blk(x, emb, ctx, rope, lora_t, None, {})
            e1.record(stream)
            torch.cuda.synchronize()
        fb.install(())
        return e0.elapsed_time(e1) / n, out

    parts = ("mod", "qkv", "modq", "gelu", "rms", "res", "ln")
    with ClockSampler(torch.cuda.current_device()) as clk:
        blk = fake_comfy.build_block(p2, "bf16", device=x.device, **dims)
        un_ms, ref = timed(blk, ())
        fu_ms, got = timed(blk, parts)
        fb.stats(reset=True)
        del blk
        blk8 = fake_comfy.build_block(p2, "int8", device=x.device, convrot=True, **dims)
        fb.install(parts)
        with torch.no_grad():
            blk8(x, emb, ctx, rope, lora_t, None, {})
        st8 = fb.stats(reset=True)
        fb.install(())
        i8_ms, _ = timed(blk8, parts)
    breakdown = None
    if args.profile:  # (outside the timed runs and the clock record)
        breakdown = {}
        for name, w in (("bf16", "bf16"), ("int8_convrot", "int8")):
            b = blk8 if w == "int8" else fake_comfy.build_block(p2, "bf16", device=x.device, **dims)
            fb.install(parts)
            with torch.no_grad():
                breakdown[name] = kernels_by_name(torch, lambda: b(x, emb, ctx, rope, lora_t, None, {}))
            fb.install(())
            del b
    del blk8
    d = (got.float() - ref.float()).abs()
    fake_comfy.unregister()
    return {"unpatched_ms": max_over_ranks(torch, dist, un_ms), "fused_ms": max_over_ranks(torch, dist, fu_ms),
            "int8_fused_ms": max_over_ranks(torch, dist, i8_ms), "int8_stats": st8, "breakdown": breakdown,
            "rel_max_diff": float(d.max() / ref.float().abs().max()), "clk": clk.summary(), "n": n}


def finish_block(torch, args, world, rank, dist, r):
    if dist is not None:
        dist.barrier()
    if rank == 0:
        tokens = 2 * 64 * 64
        print(json.dumps({
            "metric": "fused Cosmos block forward ms (drop-in vs unpatched)", "value": round(r["fused_ms"], 4),
            "unit": "ms/block", "n_gpus": world, "steps": r["n"], "warmup": args.warmup,
            "ms_per_step": round(r["fused_ms"], 4), "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 (int8 line: int8 x int8 GEMMs)", "data": "synthetic (seeded)",
            "config": {"workload": "Cosmos-Predict2-2B block (configs[3] shape): x [2, 1, 64, 64, 2048], 16 heads, MLP "
                                   "8192, AdaLN-LoRA 256, 512 context tokens of 1024; ComfyUI's Cosmos classes as the "
                                   "drop-in tests' stand-in",
                       "tokens": tokens, "unpatched_bf16_ms": round(r["unpatched_ms"], 4),
                       "fused_bf16_ms": round(r["fused_ms"], 4),
                       "speedup_bf16": round(r["unpatched_ms"] / r["fused_ms"], 3),
                       "fused_int8_ms": round(r["int8_fused_ms"], 4),
                       "speedup_int8_vs_unpatched_bf16": round(r["unpatched_ms"] / r["int8_fused_ms"], 3),
                       "int8_parts_used": r["int8_stats"],
                       "bf16_fused_vs_unpatched_rel_max_diff": round(r["rel_max_diff"], 5),
                       "reference_figure": "fused Anima block 22.1 vs 30.3 ms per block (x1.37), RTX 4060",
                       "kernel_ms_per_forward": r["breakdown"]},
            "roofline": None, "cpu_baseline": None, "e2e": None, "gpu_launches": None, "clocks": r["clk"]}),
              flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


QUANT_WIDTHS = (2048, 4096, 5120, 6144, 8192)
QUANT_MODES = (("plain", 0, 0), ("gelu", 1, 0), ("convrot", 0, 1), ("convrot_gelu", 1, 1), ("lnmod", 3, 0),
               ("lnmod_convrot", 3, 1))


def run_quant(torch, args, world, rank, dist):
    """The int8 per-token quantiser (wf_quant_rows) on 8192 rows of each width in QUANT_WIDTHS, in each mode of
    QUANT_MODES (pre none / GELU table / pending LayerNorm + modulate, with and without the ConvRot rotation), timed
    as a run of 8 * steps launches over 8 rotating inputs (larger than L2 from K = 2048 on) between two events."""
    ext = _pkg("_ext")
    fi = _pkg("enhancers.fused_int8")
    lib = ext.lib()
    dev = torch.device("cuda", torch.cuda.current_device())
    st = ext.stream_of(dev)
    gelu = fi._gelu_table(dev)
    rows, n_sets = 8192, 8
    res = {}
    with ClockSampler(torch.cuda.current_device()) as clk:
        for K in QUANT_WIDTHS:
            g = torch.Generator(device=dev)
            g.manual_seed(20261201 + K + rank)
            xs = [(torch.randn((rows, K), device=dev, generator=g) * 2).to(torch.bfloat16) for _ in range(n_sets)]
            s1 = (1 + 0.1 * torch.randn((2, K), device=dev, generator=g)).to(torch.bfloat16)
            sh = (0.1 * torch.randn((2, K), device=dev, generator=g)).to(torch.bfloat16)
            q = torch.empty((rows, K), dtype=torch.int8, device=dev)
            sc = torch.empty((rows,), dtype=torch.float32, device=dev)
            for name, pre, rot in QUANT_MODES:
                def launch(i, pre=pre, rot=rot):
                    ext.check(lib.wf_quant_rows(xs[i % n_sets].data_ptr(), s1.data_ptr() if pre == 3 else None,
                                                sh.data_ptr() if pre == 3 else None,
                                                gelu.data_ptr() if pre == 1 else None, q.data_ptr(), sc.data_ptr(),
                                                rows, K, 4096, 1e-6, pre, rot, st), "wf_quant_rows")
                for i in range(2 * n_sets):
                    launch(i)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                n = n_sets * max(args.steps, 3)
                e0.record()
                for i in range(n):
                    launch(i)
                e1.record()
                torch.cuda.synchronize()
                res[f"{K}_{name}"] = max_over_ranks(torch, dist, e0.elapsed_time(e1) * 1e3 / n)
            del xs
    return {"us": res, "clk": clk.summary(), "rows": rows, "launches": int(sum_over_ranks(
        torch, dist, len(res) * (n + 2 * n_sets)))}


def finish_quant(torch, args, world, rank, dist, r):
    if dist is not None:
        dist.barrier()
    if rank == 0:
        peak, kind = measured_peaks()
        us = r["us"]
        base = us["2048_plain"]
        nbytes = r["rows"] * 2048 * 3 + r["rows"] * 4  # x read, int8 written, scales
        table = {K: {name: round(us[f"{K}_{name}"], 2) for name, _, _ in QUANT_MODES} for K in QUANT_WIDTHS}
        print(json.dumps({
            "metric": "int8 per-token quantiser us per launch (8192 x 2048, plain)", "value": round(base, 2),
            "unit": "us", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(base / 1e3, 5),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 in, int8 out",
            "data": "synthetic (seeded)",
            "config": {"workload": "wf_quant_rows on 8192 rows, every width and mode (us per launch)",
                       "us_per_launch": table, "rows_per_modulation_group": 4096,
                       "l2": "8 rotating inputs (128 MB to 1 GB together); no flush"},
            "roofline": {"bound": "hbm", "achieved": round(nbytes / base / 1e3, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(nbytes / base / 1e3 / peak, 4), "traffic": None,
                         "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({kind})",
                         "kernel": "quant_rows_plain_kernel<0, 8> (8192 x 2048)"},
            "cpu_baseline": None, "e2e": None, "gpu_launches": r["launches"], "clocks": r["clk"]}), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def cpu_baseline_prologue(seconds=10.0):
    """The oracle's kernel A and kernel B on the first 512 rows / tokens of configs[3], repeated for ~seconds."""
    import torch
    from oracle import oracle
    cb = _pkg("streaming.cosmos_block")
    g = torch.Generator().manual_seed(3)
    x = torch.randn((512, 2048), generator=g).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    s1 = (1 + torch.randn((1, 2048), generator=g) * 0.1).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    sh = (torch.randn((1, 2048), generator=g) * 0.1).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    q = torch.randn((1, 32, 16, 128), generator=g).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    f = cb.rope3d_table(1, 64, 64).numpy()[:, :32]
    w = np.ones(128, dtype=np.float32)
    threads = use_all_host_threads(oracle)
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        oracle.ln_modulate(x, s1, sh, 512, 1e-6)
        oracle.rms_rope128(q, f, w, 16, 32, 1e-6)
        oracle.rms_rope128(q, f, w, 16, 32, 1e-6)
        reps += 1
    el = time.perf_counter() - t0
    nbytes = reps * (2 * 512 * 2048 * 2 + 2 * 2 * 32 * 16 * 128 * 2)
    return nbytes / el / 1e9, threads, f"{reps} x (512 rows of kernel A + 32 tokens of kernel B on q, k)"


def finish_prologue(torch, args, world, rank, dist, r):
    peak, kind = measured_peaks()
    a_rate = r["bytes_a"] / (r["a_ms"] / 1e3) / 1e9
    b_rate = r["bytes_b"] / (r["b_ms"] / 1e3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, threads, sample = cpu_baseline_prologue(args.cpu_seconds)
        cpu = {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample}
    if dist is not None:
        dist.barrier()
    if rank == 0:
        dominant = "B" if r["b_ms"] >= r["a_ms"] else "A"
        ach = b_rate if dominant == "B" else a_rate
        print(json.dumps({
            "metric": "fused block prologue GB/s (LN+modulate, QK RMSNorm+RoPE)", "value": round(r["value"], 1),
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(r["ms"], 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 (f32 math)", "data": "synthetic (seeded)",
            "config": {"workload": "Cosmos-Predict2-2B block prologue (configs[3]): x [2, 4096, 2048], q / k "
                                   "[2, 4096, 16, 128], 3D RoPE of 1 x 64 x 64 patches",
                       "kernel_a_us": round(r["a_ms"] * 1e3, 2), "kernel_a_gbs": round(a_rate, 1),
                       "kernel_a_bytes": r["bytes_a"], "kernel_b_us_q_and_k": round(r["b_ms"] * 1e3, 2),
                       "kernel_b_gbs": round(b_rate, 1), "kernel_b_bytes": r["bytes_b"],
                       "torch_copy_same_bytes_us": {"a": round(r["copy_a_us"], 2), "b_q_and_k": round(r["copy_b_us"], 2)},
                       "int8_quantiser_us": {"plain": round(r["quant_plain_us"], 2),
                                             "lnmod_pending": round(r["quant_lnmod_us"], 2),
                                             "bytes": r["quant_bytes"],
                                             "frac_plain": round(r["quant_bytes"] / r["quant_plain_us"] / 1e3 / peak, 4),
                                             "frac_lnmod": round(r["quant_bytes"] / r["quant_lnmod_us"] / 1e3 / peak, 4)},
                       "l2": "inputs larger than L2: each launch of a run reads one of 8 rotating tensor sets "
                             "(1.6 GB); no flush"},
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(ach / peak, 4), "traffic": NCU_TRAFFIC.get("prologue"),
                         "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({kind})",
                         "kernel": "rms_rope_v2_kernel" if dominant == "B" else "ln_modulate_kernel<4>",
                         "kernel_a_frac": round(a_rate / peak, 4), "kernel_b_frac": round(b_rate / peak, 4)},
            "cpu_baseline": cpu, "e2e": None, "gpu_launches": r["launches"], "clocks": r["clk"]}), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_single_weight(torch, args, world, rank, dist, which):
    """configs[0] (Q8_0 5120x5120) or configs[1]'s weight (Q4_K 5120x13824): one launch per weight, as a GGUF layer
    dequantises its weight on every use. Timed as a run of launches over rotating sets of weights whose bytes exceed
    L2 five times over (so each launch reads from HBM and no flush is needed), between two CUDA events."""
    ext = _pkg("_ext")
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev)
    if which == "q8":
        shape, qt = (5120, 5120), 8
        gen.manual_seed(20261201 + 0 + rank)
        fill = lambda: fill_q8(torch, shape[0] * shape[1] // 32, dev, gen)  # noqa: E731
    else:
        shape, qt = (5120, 13824), 12
        gen.manual_seed(20261201 + 1 + rank)
        fill = lambda: fill_q4k(torch, shape[0] * shape[1] // 256, dev, gen)  # noqa: E731
    n = shape[0] * shape[1]
    per_set = fill().numel() + 2 * n
    n_sets = max(2, -(-640 * 1024 * 1024 // per_set))
    sets = [(fill(), torch.empty(shape, dtype=torch.bfloat16, device=dev)) for _ in range(n_sets)]
    lib = ext.lib()
    stream = torch.cuda.current_stream(dev)

    def launch(i):
        src, dst = sets[i % n_sets]
        rc = lib.wf_dequant_gguf(src.data_ptr(), src.numel(), dst.data_ptr(), n, qt, 0, 1, stream.cuda_stream)
        if rc:
            ext.check(rc, "wf_dequant_gguf")

    def probe(i):  # the same byte counts through a no-arithmetic streaming kernel
        src, dst = sets[i % n_sets]
        ext.check(lib.wf_hbm_probe(src.data_ptr(), src.numel() // 16 * 16, dst.data_ptr(), 2 * n // 16 * 16,
                                   stream.cuda_stream), "wf_hbm_probe")

    def timed(fn, count):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(count):
            fn(i)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / count

    count = n_sets * max(1, args.steps // 2)
    for i in range(max(args.warmup, 1) * n_sets):
        launch(i)
    barrier(torch, dist)
    with ClockSampler(torch.cuda.current_device()) as clk:
        barrier(torch, dist)
        kern_ms = timed(launch, count)
        barrier(torch, dist)
    probe_ms = timed(probe, count)
    ms = max_over_ranks(torch, dist, kern_ms)
    src0 = sets[0][0]
    out_bytes = n * 2
    value = sum_over_ranks(torch, dist, out_bytes / (ms / 1e3) / 1e9)
    mix = (src0.numel() // 16 * 16 + out_bytes // 16 * 16) / (probe_ms / 1e3) / 1e9
    return {
        "value": value, "ms_per_step": ms, "kern_ms": kern_ms, "alg_bytes_per_launch": src0.numel() + out_bytes,
        "clk": clk.summary(), "e2e": None, "gpu_launches": int(sum_over_ranks(torch, dist, count)),
        "mix_gbs": mix,
        "config": {"workload": f"GGUF {'Q8_0' if qt == 8 else 'Q4_K'} {shape[0]}x{shape[1]} -> bf16 (one weight)",
                   "mid_dtype": "f16",
                   "l2": f"inputs larger than L2: a run of {count} launches over {n_sets} rotating weights "
                         f"({n_sets * per_set / 1e9:.2f} GB); no flush",
                   "timing": "CUDA events around the run / launches (a step = one launch)"},
    }


# ------------------------------------------------------------------------------------ §8(f) rows: formats, LoRA, SSD
GGUF_GEOMETRY = {2: ("Q4_0", 32, 18, (0,)), 3: ("Q4_1", 32, 20, (0, 2)), 6: ("Q5_0", 32, 22, (0,)),
                 7: ("Q5_1", 32, 24, (0, 2)), 8: ("Q8_0", 32, 34, (0,)), 10: ("Q2_K", 256, 84, (80, 82)),
                 11: ("Q3_K", 256, 110, (108,)), 12: ("Q4_K", 256, 144, (0, 2)), 13: ("Q5_K", 256, 176, (0, 2)),
                 14: ("Q6_K", 256, 210, (208,))}


def fill_gguf(torch, qt, n_values, device, gen):
    """Random packed blocks of GGML type qt with every float16 field (d, dmin) finite: U(0, 0.01)."""
    _name, vpb, ts, f16 = GGUF_GEOMETRY[qt]
    nb = n_values // vpb
    raw = torch.randint(0, 256, (nb, ts), dtype=torch.uint8, device=device, generator=gen)
    for off in f16:
        raw[:, off:off + 2] = (torch.rand((nb, 1), device=device, generator=gen) * 0.01).half().view(torch.uint8)
    return raw.reshape(-1)


def time_launches(torch, flush, stream, fn, steps):
    """Mean CUDA-event time (ms) of fn over `steps` launches, L2 flushed before each."""
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        flush()
        ev[i][0].record(stream)
        fn()
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    return statistics.mean(a.elapsed_time(b) for a, b in ev)


def run_formats(torch, args, world, rank, dist):
    """§8(f) 2: every GGML type of the kernel family on one 5120 x 13824 weight (bf16 out, mid f16), L2 flushed per
    launch; each against the copy peak and against wf_hbm_probe over its own in / out bytes after the same flush."""
    ext = _pkg("_ext")
    lib = ext.lib()
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev)
    flush = L2Flush(torch, dev)
    n = 5120 * 13824
    dst = torch.empty(n, dtype=torch.bfloat16, device=dev)
    peak, _kind = measured_peaks()
    per, gbs_all = {}, []
    with ClockSampler(torch.cuda.current_device()) as clk:
        for qt, (name, _vpb, _ts, _f16) in GGUF_GEOMETRY.items():
            gen = torch.Generator(device=dev)
            gen.manual_seed(20261201 + 100 + qt)
            src = fill_gguf(torch, qt, n, dev, gen)

            def launch():
                ext.check(lib.wf_dequant_gguf(src.data_ptr(), src.numel(), dst.data_ptr(), n, qt, 0, 1,
                                              stream.cuda_stream), "wf_dequant_gguf")

            for _ in range(args.warmup):
                launch()
            ms = time_launches(torch, flush, stream, launch, args.steps)
            pin, pout = src.numel() // 16 * 16, n * 2
            pms = time_launches(torch, flush, stream, lambda: ext.check(lib.wf_hbm_probe(
                src.data_ptr(), pin, dst.data_ptr(), pout, stream.cuda_stream), "probe"), args.steps)
            alg = (src.numel() + 2 * n) / (ms / 1e3) / 1e9
            mix = (pin + pout) / (pms / 1e3) / 1e9
            per[name] = {"us": round(ms * 1e3, 2), "alg_gbs": round(alg, 1), "frac_of_copy_peak": round(alg / peak, 4),
                         "mix_ceiling_gbs": round(mix, 1), "frac_of_mix_ceiling": round(alg / mix, 4),
                         "in_bytes": src.numel(), "out_bytes": 2 * n}
            gbs_all.append(2 * n / (ms / 1e3) / 1e9)
            del src
    geo = float(np.exp(np.mean(np.log(gbs_all))))
    fr = [v["frac_of_mix_ceiling"] for v in per.values()]
    return {"value": geo, "per": per, "clk": clk.summary(), "peak": peak, "min_frac_mix": min(fr),
            "mean_frac_copy": float(np.mean([v["frac_of_copy_peak"] for v in per.values()]))}


def finish_formats(torch, args, world, rank, dist, r):
    if rank == 0:
        print(json.dumps({
            "metric": "GGUF dequant out GB/s, all 10 GGML types (geometric mean)", "value": round(r["value"], 2),
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8->bf16 (mid f16)",
            "data": "synthetic (seeded random blocks, float16 fields U(0, 0.01))",
            "config": {"workload": "one 5120 x 13824 weight per GGML type -> bf16", "l2": L2_NOTE,
                       "per_format": r["per"]},
            "roofline": {"bound": "hbm", "peak": r["peak"], "unit": "GB/s",
                         "mean_frac_of_copy_peak": round(r["mean_frac_copy"], 4),
                         "min_frac_of_mix_ceiling": round(r["min_frac_mix"], 4),
                         "kernel": "dequant_kernel (single weight)"},
            "clocks": r["clk"]}), flush=True)


def run_lora(torch, args, world, rank, dist):
    """§8(f) 1: LoRA-in-dequant (wf_dequant_gguf_lora: w = R_out(dequant + R_out(diff * sa))) on configs[1]'s Q4_K
    weight with a float32 LoRA difference of the same shape, against the plain dequantisation of the same weight."""
    ext = _pkg("_ext")
    lib = ext.lib()
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev)
    flush = L2Flush(torch, dev)
    n = 5120 * 13824
    gen = torch.Generator(device=dev)
    gen.manual_seed(20261201 + 1)
    src = fill_q4k(torch, n // 256, dev, gen)
    diff = torch.randn(n, device=dev, generator=gen) * 0.01
    dst = torch.empty(n, dtype=torch.bfloat16, device=dev)

    def lora():
        ext.check(lib.wf_dequant_gguf_lora(src.data_ptr(), src.numel(), diff.data_ptr(), dst.data_ptr(), n, 12, 0, 1,
                                           0.75, stream.cuda_stream), "lora")

    def plain():
        ext.check(lib.wf_dequant_gguf(src.data_ptr(), src.numel(), dst.data_ptr(), n, 12, 0, 1, stream.cuda_stream),
                  "plain")

    for _ in range(args.warmup):
        lora()
        plain()
    with ClockSampler(torch.cuda.current_device()) as clk:
        ms = time_launches(torch, flush, stream, lora, args.steps)
        ms_plain = time_launches(torch, flush, stream, plain, args.steps)
    alg = src.numel() + 4 * n + 2 * n
    return {"ms": ms, "ms_plain": ms_plain, "alg": alg, "clk": clk.summary(), "n": n}


def finish_lora(torch, args, world, rank, dist, r):
    if rank == 0:
        peak, kind = measured_peaks()
        achieved = r["alg"] / (r["ms"] / 1e3) / 1e9
        print(json.dumps({
            "metric": "GGUF dequant + LoRA out GB/s", "value": round(2 * r["n"] / (r["ms"] / 1e3) / 1e9, 2),
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms"], 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8 + f32 diff -> bf16",
            "data": "synthetic (seeded)",
            "config": {"workload": "Q4_K 5120 x 13824 + float32 LoRA difference (sa 0.75) -> bf16 (configs[1] weight)",
                       "plain_dequant_ms": round(r["ms_plain"], 4), "l2": L2_NOTE,
                       "alg_bytes": r["alg"], "bytes": "packed + 4 B of difference + 2 B of output per value"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({kind})",
                         "kernel": "dequant_kernel<LORA> (single weight)"},
            "clocks": r["clk"]}), flush=True)


def mount_of(path):
    """(mount point, filesystem type, device) of the longest /proc/mounts entry holding path."""
    best = ("", "?", "?")
    try:
        with open("/proc/mounts") as f:
            for ln in f:
                dev, mnt, fstype = ln.split()[:3]
                if (path == mnt or path.startswith(mnt.rstrip("/") + "/")) and len(mnt) >= len(best[0]):
                    best = (mnt, fstype, dev)
    except OSError:
        pass
    return {"mount": best[0], "type": best[1], "device": best[2]}


def run_ssd(torch, args, world, rank, dist):
    """§8(f) 4: the SSD tier's read path -- blocks of configs[4]'s size (417,793,024 B) written once to a cache file
    (O_DIRECT) in a fresh folder under the streaming tier's default cache folder (WEIGHTFERRY_DISK_DIR, else the
    temp folder), then read back cyclically by a DiskRing (pinned 4 KiB aligned buffers, the probe's best
    reader-thread count) and copied to a GPU slot on a side stream, as the uploader does; against the drive's own
    probed read rate over the same folder. Reports the folder's filesystem; deletes its files."""
    import shutil
    tiers = "core.tiers."
    dio, cf, src_mod = _pkg(tiers + "disk_io"), _pkg(tiers + "cache_files"), _pkg(tiers + "sources")
    dev = torch.device("cuda", torch.cuda.current_device())
    folder = os.path.join(cf.default_cache_dir(), f"bench_{os.getpid()}")
    os.makedirs(folder, exist_ok=True)
    fs = mount_of(folder)
    n_blocks, block = args.ssd_blocks, 417_793_024
    try:
        probe = dio.probe_disk(folder, size_mb=1024, chunk_mb=64, thread_counts=(1, 2, 4))
        store = cf.DiskBlockStore(cf.new_cache_path(folder), block, n_blocks)
        st = store.staging()
        g = torch.Generator()
        g.manual_seed(20261201 + 4)
        t0 = time.perf_counter()
        for i in range(n_blocks):
            st.copy_(torch.randint(0, 256, (block,), dtype=torch.uint8, generator=g))
            store.write_block(i, st)
        store.finalize()
        write_s = time.perf_counter() - t0
        ring = src_mod.DiskRing(store, depth=4, pin=True, threads=probe["threads"])
        slot = torch.empty(block, dtype=torch.uint8, device=dev)
        cs = torch.cuda.Stream(device=dev)
        try:
            for i in range(n_blocks):  # one warm-up cycle
                view, b = ring.acquire(i)
                with torch.cuda.stream(cs):
                    slot.copy_(view, non_blocking=True)
                    ring.release(b, cs)
            cs.synchronize()
            t0 = time.perf_counter()
            cycles = max(1, args.steps // n_blocks)
            for _ in range(cycles):
                for i in range(n_blocks):
                    view, b = ring.acquire(i)
                    with torch.cuda.stream(cs):
                        slot.copy_(view, non_blocking=True)
                        ring.release(b, cs)
            cs.synchronize()
            el = time.perf_counter() - t0
        finally:
            ring.close()
            store.delete()
    finally:
        shutil.rmtree(folder, ignore_errors=True)
    gbs = cycles * n_blocks * block / el / 1e9
    return {"gbs": gbs, "probe": probe, "cycles": cycles, "fs": fs, "folder": folder, "threads": ring.threads, "n_blocks": n_blocks, "write_gbs": n_blocks * block / write_s
            / 1e9, "el": el}


def finish_ssd(torch, args, world, rank, dist, r):
    if rank == 0:
        peak = r["probe"]["gbps"]
        print(json.dumps({
            "metric": "SSD tier block read to GPU GB/s", "value": round(r["gbs"], 3), "unit": "GB/s", "n_gpus": world,
            "steps": r["cycles"] * r["n_blocks"], "warmup": r["n_blocks"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bytes", "data": "synthetic (seeded random bytes)",
            "config": {"workload": f"{r['n_blocks']} Cosmos-14B Q8_0 blocks of 417,793,024 B in a cache file on the "
                                   "box's drive, DiskRing depth 4 -> one GPU slot",
                       "drive_probe": r["probe"], "cache_write_gbs": round(r["write_gbs"], 3),
                       "folder": r["folder"], "filesystem": r["fs"], "ring_threads": r["threads"],
                       "timed_s": round(r["el"], 3), "timing": "host wall clock around whole cycles (the copies "
                                                            "are synchronised at the end)"},
            "roofline": {"bound": "disk", "achieved": round(r["gbs"], 3), "peak": peak, "unit": "GB/s",
                         "frac": round(r["gbs"] / peak, 4), "peak_source": "probe_disk of the same folder (O_DIRECT "
                                                                          "reads, best thread count)"}}),
              flush=True)


# ----------------------------------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="sweep",
                    choices=["sweep", "q8", "q4k", "w8a8", "stack", "prologue", "formats", "lora", "ssd", "block",
                             "quant"])
    ap.add_argument("--ssd-blocks", type=int, default=8, help="ssd: blocks in the cache file")
    ap.add_argument("--slots", type=int, default=3, help="stack: GPU slots of the streaming ring")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--parallel", default="sp", choices=["sp", "tp"],
                    help="stack over N GPUs: sp = whole blocks per rank on its token rows, weights gathered; tp = "
                         "tensor parallel")
    ap.add_argument("--profile", action="store_true",
                    help="stack: GPU time per kind of kernel of one extra forward (torch.profiler), every rank; "
                         "block: GPU time per kernel of five extra forwards")
    ap.add_argument("--blocks", type=int, default=36, help="sweep: checkpoint blocks per rank (36 = Cosmos-14B)")
    ap.add_argument("--sustained-seconds", type=float, default=W8A8_SUSTAINED_S,
                    help="w8a8: seconds of back-to-back launches of the GEMM and of cuBLASLt (0: skip)")
    ap.add_argument("--stack-blocks", type=int, default=36,
                    help="sweep: blocks of the streamed-stack sub-record timed after the sweep (0: none)")
    ap.add_argument("--stack-steps", type=int, default=3, help="sweep: timed forwards of the stack sub-record")
    ap.add_argument("--stack-warmup", type=int, default=2, help="sweep: untimed forwards before them")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        return run_reference(args)

    import torch
    world, rank, local, dist = setup_dist(torch)
    if args.workload == "sweep":
        r = run_sweep(torch, args, world, rank, dist)
    elif args.workload == "formats":
        return finish_formats(torch, args, world, rank, dist, run_formats(torch, args, world, rank, dist))
    elif args.workload == "lora":
        return finish_lora(torch, args, world, rank, dist, run_lora(torch, args, world, rank, dist))
    elif args.workload == "ssd":
        return finish_ssd(torch, args, world, rank, dist, run_ssd(torch, args, world, rank, dist))
    elif args.workload == "prologue":
        return finish_prologue(torch, args, world, rank, dist, run_prologue(torch, args, world, rank, dist))
    elif args.workload == "stack":
        return finish_stack(torch, args, world, rank, dist, run_stack(torch, args, world, rank, dist))
    elif args.workload == "w8a8":
        return finish_w8a8(torch, args, world, rank, dist, run_w8a8(torch, args, world, rank, dist))
    elif args.workload == "block":
        return finish_block(torch, args, world, rank, dist, run_block(torch, args, world, rank, dist))
    elif args.workload == "quant":
        return finish_quant(torch, args, world, rank, dist, run_quant(torch, args, world, rank, dist))
    else:
        r = run_single_weight(torch, args, world, rank, dist, args.workload)
    peak, peak_kind = measured_peaks()
    achieved = r["alg_bytes_per_launch"] / (r["kern_ms"] / 1e3) / 1e9
    traffic = NCU_TRAFFIC.get(args.workload)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload in ("sweep", "q4k"):
        gbs, threads, sample = cpu_baseline_sweep(args.cpu_seconds)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample}
    if dist is not None:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": "GGUF dequant out GB/s", "value": round(r["value"], 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms_per_step"], 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8->bf16 (f32 math)",
            "data": "synthetic (seeded, BASELINE configs distributions)", "config": r["config"],
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                         "kernel": "dequant_kernel<12,f16,bf16> (batched)" if args.workload == "sweep"
                         else "dequant_kernel (single weight)"},
            "cpu_baseline": cpu, "e2e": r["e2e"], "gpu_launches": r["gpu_launches"], "clocks": r["clk"],
        }
        if r.get("stack") is not None:
            line["stack"] = r["stack"]
        if r.get("mix_gbs"):
            # the copy-based peak assumes read = write; this traffic is write-heavy (in : out about 1 : 3.6), and a
            # plain streaming kernel with the same byte counts (wf_hbm_probe) is the ceiling it is measured against too
            line["roofline"]["mix_ceiling"] = {"gbs": round(r["mix_gbs"], 1), "frac": round(achieved / r["mix_gbs"], 4),
                                               "probe": "wf_hbm_probe over the same in / out byte counts"
                                                        + (" over the same rotation" if args.workload != "sweep"
                                                           else "")}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def measured_int8_peak(sustained=False):
    """Dense int8 tensor peak: twice the measured dense bf16 GEMM rate (B200's int8 dense rate is twice bf16's), as a
    burst (a kernel timed alone) or sustained (back to back for seconds, under the power cap)."""
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    try:
        with open(path) as f:
            p = json.load(f)
        return 2.0 * float(p[key]), f"2 x MEASURED_PEAKS.json {key} (measured, {'sustained' if sustained else 'burst'})"
    except (OSError, KeyError, ValueError):
        return (2.0 * 1400.0, "2 x fallback sustained bf16 1400 TFLOP/s") if sustained else \
            (2.0 * 1590.0, "2 x fallback bf16 1590 TFLOP/s")


def sustained_record(sus):
    """The back-to-back GEMM runs, with the GEMM's fraction of the sustained int8 peak."""
    peak, src = measured_int8_peak(sustained=True)
    rec = dict(sus)
    ours = sus.get("wf_w8a8_gemm", {})
    if "tops" in ours:
        rec["roofline"] = {"bound": "tensor", "achieved": ours["tops"], "peak": round(peak, 1), "unit": "TOPS",
                           "frac": round(ours["tops"] / peak, 4), "peak_source": src}
    if not sus:
        return None
    rec["note"] = ("each kernel launched back to back for --sustained-seconds on the same operands (L2-warm), "
                   "clocks sampled meanwhile; cuBLASLt writes int32 without the rescale")
    return rec


def finish_w8a8(torch, args, world, rank, dist, r):
    peak, src = measured_int8_peak()
    achieved = r["alg_ops_per_launch"] / (r["kern_ms"] / 1e3) / 1e12
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, threads, sample = cpu_baseline_w8a8(args.cpu_seconds)
        cpu = {"value": round(v, 4), "unit": "TOPS", "cores": threads, "kind": "port", "sample": sample}
    if dist is not None:
        dist.barrier()
    if rank == 0:
        print(json.dumps({
            "metric": "W8A8 linear int8 TOPS (quantise + GEMM + rescale)", "value": round(r["value"], 2),
            "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(r["ms_per_step"], 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 x int8 -> int32, bf16 out", "data": "synthetic (seeded)",
            "config": r["config"],
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS",
                         "frac": round(achieved / peak, 4), "traffic": NCU_TRAFFIC.get("w8a8"), "peak_source": src,
                         "kernel": ("w8a8_gemm_kernel" if os.environ.get("WEIGHTFERRY_W8A8_1SM") == "1"
                                    else "w8a8_gemm_2sm_kernel")},
            "sustained": sustained_record(r["sustained"]),
            "cpu_baseline": cpu, "e2e": r["e2e"], "gpu_launches": r["gpu_launches"], "clocks": r["clk"],
            "gemm_status": r["gemm_status"]}), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args):
    """The reference arm: the reference's dequantisation arithmetic on the host cores (oracle port, OpenMP, all
    threads) on the same metric / config; rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle
    shapes = cosmos14b_block_shapes()
    # bounded sample: 4 of the block's tensors (one of each kind) per step
    sample = [shapes[0], shapes[6], shapes[8], shapes[11]]
    rng = np.random.default_rng(20261201 + 1)
    raws = []
    for a, b in sample:
        nb = a * b // 256
        raw = rng.integers(0, 256, size=(nb, Q4K_TS), dtype=np.uint8)
        raw[:, 0:4] = (rng.uniform(0, 0.01, (nb, 2)).astype(np.float16)).view(np.uint8)
        raws.append((raw, a * b))
    threads = use_all_host_threads(oracle)

    def step():
        for raw, n in raws:
            oracle.dequant_gguf(raw, n, 12, 0, 1)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    out_bytes = sum(n for _r, n in raws) * 2 * args.steps
    v = out_bytes / el / 1e9
    desc = "Q4_K -> bf16 (mid f16) of 4 Cosmos-14B block tensors (5120x5120, 5120x1024, 20480x5120, 15360x256)"
    print(json.dumps({
        "impl": "reference", "metric": "GGUF dequant out GB/s", "value": round(v, 3), "unit": "GB/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8->bf16 (f32 math)", "data": "synthetic (seeded)",
        "config": {"workload": "GGUF Q4_K -> bf16 sweep (configs[1]), bounded CPU sample per step"},
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


if __name__ == "__main__":
    main()
