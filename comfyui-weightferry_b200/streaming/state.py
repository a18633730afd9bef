"""Block-streaming state with dequantisation on arrival (the reference's streaming/state.py _StreamState, :21-323).

The reference keeps every streamed block in one flat pinned host buffer, copies it on a side stream into one of N
GPU slots when the slot's previous block has finished computing (``computed_events[slot]``), and binds the block's
parameters to the slot before its forward (``transferred_events[s]``). A GGUF block travels as its packed bytes and is
dequantised later, per layer and per use, on the compute stream (enhancers/gguf_dequant.py:464-492).

Here the same protocol carries one change the B200 build is for: the block is dequantised on arrival. Per issue:

  copy stream     wait computed[slot] -> H2D of the block's packed bytes into the slot -> record transferred[s]
  dequant stream  wait transferred[s] -> one batched GGUF launch per quantisation type for all the block's
                  tensors (wf_dequant_gguf_batch) into the slot's bf16 weights -> record ready[s]
  compute stream  wait ready[s] -> the block's forward on bf16 weights -> record computed[slot]

so the copy of block s+1 overlaps the dequantisation of block s, and both overlap the compute of the blocks before.
Slot reuse is ordered through the events exactly as in the reference (a slot's bytes and weights are overwritten only
after the compute of the block that last used them). Parameters that are not GGUF-quantised (norm weights, biases)
are used straight from the slot's packed bytes.

Switches: WEIGHTFERRY_SLOTS (slot count, default 3 as the node's prefetch_slots), WEIGHTFERRY_PREFETCH_PRIORITY
(stream priority of the transfer streams), WEIGHTFERRY_PROFILE (the event timeline of streaming/profiler.py).
"""

import ctypes
import time

import torch

from .. import _ext
from ..core import env as _env
from .common import flat_layout, views
from .profiler import _StreamProfiler

_GGUF_GEOMETRY = {2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34),
                  10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210)}
_DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


class ParamSpec:
    """One parameter of a streamed block: GGUF-quantised (qtype, logical shape) or plain (dtype, shape). ``mid`` is
    the intermediate precision of the dequantisation (0 f16 -- ComfyUI-GGUF's default --, 1 bf16, 2 f32), the one
    the layer's own dequantisation would use, so that the slot holds the same bits."""

    def __init__(self, name, shape, qtype=None, dtype=None, mid=0):
        self.name = name
        self.shape = tuple(int(s) for s in shape)
        self.qtype = None if qtype is None else int(qtype)
        self.dtype = dtype
        self.mid = int(mid)
        n = 1
        for s in self.shape:
            n *= s
        self.numel = n
        if self.qtype is not None:
            vpb, ts = _GGUF_GEOMETRY[self.qtype]
            if n % vpb:
                raise ValueError(f"{name}: {n} values is not a whole number of GGML type {self.qtype} blocks")
            self.packed_bytes = n // vpb * ts
        else:
            self.packed_bytes = n * dtype.itemsize


class BlockLayout:
    """Where each parameter of a block lives: in the flat packed buffer (host and slot, 256-byte aligned) and, for
    GGUF parameters, in the slot's dequantised weight buffer (compute dtype, 256-byte aligned)."""

    def __init__(self, specs, compute_dtype=torch.bfloat16, pad_to=1):
        self.specs = list(specs)
        self.compute_dtype = compute_dtype
        self.offsets, self.flat_bytes = flat_layout([p.packed_bytes for p in self.specs])
        # a flat size that splits into `pad_to` equal, 256-byte aligned ranges (the gathered transfer's shards)
        unit = 256 * max(1, int(pad_to))
        self.flat_bytes = (self.flat_bytes + unit - 1) // unit * unit
        q = [p for p in self.specs if p.qtype is not None]
        self.q_specs = q
        self.w_offsets, self.weight_bytes = flat_layout([p.numel * compute_dtype.itemsize for p in q])

    @property
    def quantised_bytes(self):
        return sum(p.packed_bytes for p in self.q_specs)


class _StreamState:
    """GPU slots, transfer / dequant streams and events of one streamed block list (one owner, one device)."""

    def __init__(self, device, host_flats, layout, num_slots=None, profile=None, ring=None, gather=None):
        self.device = torch.device(device)
        self.host_flats = host_flats          # per block: flat pinned uint8 tensor (DMA source), None: SSD tier
        self.layout = layout
        # gather = (process group, rank, world): each host flat holds only this rank's equal byte range of the block;
        # the ranks' ranges are all-gathered into the slot after the copy (streaming/stack.py's "sp" mode)
        self.gather = gather if gather is not None and gather[2] > 1 else None
        if self.gather is not None:
            _g, grank, gworld = self.gather
            if layout.flat_bytes % gworld or ring is not None:
                raise ValueError("a gathered transfer needs a flat size divisible by the ranks and no SSD tier")
            self.shard_bytes = layout.flat_bytes // gworld
            self.shard_lo = grank * self.shard_bytes
        self.num_stream = len(host_flats)
        # SSD tier: the blocks without a host flat are read by `ring` (core/tiers/sources.DiskRing) in block order
        disk = [s for s, f in enumerate(host_flats) if f is None]
        self.disk_index = {s: k for k, s in enumerate(disk)}
        if disk and (ring is None or ring.n != len(disk)):
            raise ValueError(f"{len(disk)} blocks have no host flat; the SSD ring must serve exactly those")
        self.ring = ring if disk else None
        if num_slots is None:
            env_slots = _env.get("WEIGHTFERRY_SLOTS")
            num_slots = int(env_slots) if env_slots else 3
        self.num_slots = max(2, min(int(num_slots), max(2, self.num_stream)))
        self.is_double = True
        lib = _ext.lib()
        self._lib = lib
        with torch.cuda.device(self.device):
            self.slot_flats = [torch.empty(layout.flat_bytes, dtype=torch.uint8, device=self.device)
                               for _ in range(self.num_slots)]
            self.slot_weights = [torch.empty(max(layout.weight_bytes, 1), dtype=torch.uint8, device=self.device)
                                 for _ in range(self.num_slots)]
            prio = _env.get("WEIGHTFERRY_PREFETCH_PRIORITY")
            kw = {"priority": int(prio)} if prio else {}
            self.copy_stream = torch.cuda.Stream(device=self.device, **kw)
            self.dequant_stream = torch.cuda.Stream(device=self.device, **kw)
            self.prefetch_stream = self.copy_stream  # the reference's name for the transfer stream
            self.transferred_events = [torch.cuda.Event() for _ in range(self.num_stream)]
            self.ready_events = [torch.cuda.Event() for _ in range(self.num_stream)]
            self.computed_events = [torch.cuda.Event() for _ in range(self.num_slots)]
            # the slots were allocated on the current stream: the first transfer into each waits for it
            cur = torch.cuda.current_stream(self.device)
            for ev in self.computed_events:
                ev.record(cur)
        self.slot_views = [self._bind_views(i) for i in range(self.num_slots)]
        self._tasks = [self._build_tasks(i) for i in range(self.num_slots)]
        self.issued = [False] * self.num_stream
        self.lookahead = True  # False: a block's transfer is issued when it starts (single buffer), not ahead
        want_prof = profile if profile is not None else _env.get("WEIGHTFERRY_PROFILE") == "1"
        self.profiler = _StreamProfiler(self.num_stream, layout.flat_bytes) if want_prof else None
        self.uploader = None
        if self.gather is not None:
            import torch.distributed as dist
            self._dist = dist
            with torch.cuda.device(self.device):
                self.gather_stream = torch.cuda.Stream(device=self.device)
        if self.ring is not None:
            from .ssd_uploader import _SsdUploader
            self.uploader = _SsdUploader(self)

    # ------------------------------------------------------------------------------------------------ layout
    def _bind_views(self, slot):
        """name -> tensor of the slot: dequantised weights (compute dtype, logical shape) or plain parameters."""
        lay = self.layout
        out = {}
        packed = views(self.slot_flats[slot], [p.packed_bytes for p in lay.specs], lay.offsets)
        qi = 0
        for p, raw in zip(lay.specs, packed):
            if p.qtype is not None:
                o = lay.w_offsets[qi]
                nb = p.numel * lay.compute_dtype.itemsize
                out[p.name] = self.slot_weights[slot][o:o + nb].view(lay.compute_dtype).view(p.shape)
                qi += 1
            else:
                out[p.name] = raw.view(p.dtype).view(p.shape)
        return out

    def _build_tasks(self, slot):
        """Per (GGML type, intermediate precision): the prebuilt wf_dequant_task table of this slot (packed bytes ->
        weights)."""
        lay = self.layout
        groups = {}
        flat_ptr = self.slot_flats[slot].data_ptr()
        w_ptr = self.slot_weights[slot].data_ptr()
        qi = 0
        for p, off in zip(lay.specs, lay.offsets):
            if p.qtype is None:
                continue
            groups.setdefault((p.qtype, p.mid), []).append((flat_ptr + off, w_ptr + lay.w_offsets[qi], p.numel))
            qi += 1
        tables = []
        for (qt, mid), items in groups.items():
            arr = (_ext.DequantTask * len(items))()
            for i, (s, d, n) in enumerate(items):
                arr[i].src, arr[i].dst, arr[i].n_values = s, d, n
            tables.append((qt, mid, arr, len(items)))
        return tables

    def slot_of(self, s_idx):
        return s_idx % self.num_slots

    # ------------------------------------------------------------------------------------------------ pipeline
    def materialize(self, s_idx, slot_idx):
        """H2D of block s_idx's packed bytes into slot slot_idx on the copy stream, then its dequantisation on the
        dequant stream; records transferred / ready events."""
        prof = self.profiler
        cs, ds = self.copy_stream, self.dequant_stream
        with torch.cuda.stream(cs):
            cs.wait_event(self.computed_events[slot_idx])
            if prof is not None:
                prof.record(s_idx, "dma0", cs)
            if self.gather is None:
                self.slot_flats[slot_idx].copy_(self.host_flats[s_idx], non_blocking=True)
            else:
                mine = self.slot_flats[slot_idx][self.shard_lo:self.shard_lo + self.shard_bytes]
                mine.copy_(self.host_flats[s_idx], non_blocking=True)
            if prof is not None:
                prof.record(s_idx, "dma1", cs)
            self.transferred_events[s_idx].record(cs)
        if self.gather is not None:
            # the other ranks' ranges over NVLink, in place, on a stream of its own so that the copy stream goes on
            # with the next block's bytes; NCCL runs it after this block's copy, the wait puts the gather stream
            # behind it without blocking the host, and the dequantisation waits for the gather stream
            gs = self.gather_stream
            with torch.cuda.stream(gs):
                gs.wait_event(self.transferred_events[s_idx])
                work = self._dist.all_gather_into_tensor(self.slot_flats[slot_idx], mine, group=self.gather[0],
                                                         async_op=True)
                work.wait()
                self.transferred_events[s_idx].record(gs)
        ds.wait_event(self.transferred_events[s_idx])
        self.dequant_slot(slot_idx, ds)
        if prof is not None:
            prof.record(s_idx, "ready", ds)
        self.ready_events[s_idx].record(ds)

    def dequant_slot(self, slot_idx, stream):
        """The slot's GGUF weights from its packed bytes: one batched launch per (type, precision) on ``stream``."""
        code = _DTYPE_CODE[self.layout.compute_dtype]
        for qt, mid, arr, n in self._tasks[slot_idx]:
            rc = self._lib.wf_dequant_gguf_batch(arr, n, qt, mid, code, stream.cuda_stream)
            if rc:
                _ext.check(rc, "wf_dequant_gguf_batch")

    def issue_prefetch(self, s_idx):
        """Transfer + dequantisation of block s_idx into its slot, after that slot's last reader finished."""
        if self.profiler is not None:
            self.profiler.mark(s_idx, "cpu_issue")
        with torch.cuda.device(self.device):
            if self.host_flats[s_idx] is None:
                self.uploader.submit(s_idx, self.slot_of(s_idx))  # SSD tier: the uploader thread copies
            else:
                self.materialize(s_idx, self.slot_of(s_idx))
        self.issued[s_idx] = True

    def begin_forward(self):
        if self.uploader is not None and (self.uploader.outstanding() or self.uploader.error is not None
                                          or not self.ring.at_cycle_start() or self.ring.failed()):
            # the previous forward stopped part way: finish the uploads it queued, then restart the SSD read cycle
            self.uploader.drain()
            self.ring.restart_if_needed(lambda msg: print(f"[streaming] {msg}", flush=True))
            self.uploader.error = None
        self.issued = [False] * self.num_stream
        if self.profiler is not None:
            self.profiler.begin_forward(torch.cuda.current_stream(self.device))

    def end_forward(self):
        if self.profiler is not None:
            self.profiler.end_forward(torch.cuda.current_stream(self.device))

    def prefetch_first_slots(self):
        for s_idx in range(min(self.num_slots, self.num_stream)):
            if not self.issued[s_idx]:
                self.issue_prefetch(s_idx)

    def acquire(self, s_idx):
        """Before block s_idx runs: make the compute stream wait for its weights; returns the slot's views."""
        t0 = time.perf_counter()
        compute = torch.cuda.current_stream(self.device)
        if not self.issued[s_idx]:
            self.issue_prefetch(s_idx)  # the prefetch chain was broken (a skipped block): issue now
        prof = self.profiler
        if prof is not None:
            prof.record(s_idx, "wait0", compute)
        if self.host_flats[s_idx] is None:
            self.uploader.wait(s_idx)  # ready[s] is recorded by the uploader thread
        compute.wait_event(self.ready_events[s_idx])
        if prof is not None:
            prof.record(s_idx, "start", compute)
            prof.add_cpu(time.perf_counter() - t0)
        return self.slot_views[self.slot_of(s_idx)]

    def release(self, s_idx):
        """After block s_idx's forward was issued: free its slot for the block that takes it next."""
        t0 = time.perf_counter()
        compute = torch.cuda.current_stream(self.device)
        if self.profiler is not None:
            self.profiler.record(s_idx, "end", compute)
        slot = self.slot_of(s_idx)
        self.computed_events[slot].record(compute)
        nxt = s_idx + self.num_slots
        if self.lookahead and nxt < self.num_stream and not self.issued[nxt]:
            self.issue_prefetch(nxt)
        if self.profiler is not None:
            self.profiler.add_cpu(time.perf_counter() - t0)

    def close(self):
        """Stop the SSD tier's threads (uploader, ring readers), release its buffers, and wait for the transfer and
        dequant streams: their H2D copies read the pinned host flats, which the owner unregisters right after close
        (a copy still running from unregistered memory would read freed pages)."""
        if self.uploader is not None:
            self.uploader.drain()
            self.uploader.close()
            self.uploader = None
        if self.gather is not None:
            import torch.distributed as dist
            self._dist = dist
            with torch.cuda.device(self.device):
                self.gather_stream = torch.cuda.Stream(device=self.device)
        if self.ring is not None:
            self.ring.close()
            self.ring = None
        self.copy_stream.synchronize()
        if self.gather is not None:
            self.gather_stream.synchronize()
        self.dequant_stream.synchronize()

    def profile_summary(self):
        return None if self.profiler is None else self.profiler.summary()

    def slot_bytes(self):
        return self.num_slots * (self.layout.flat_bytes + self.layout.weight_bytes)


def install_block_stream_hooks(blocks, state):
    """Forward pre / post hooks on a list of torch blocks (the reference's _install_block_stream_hooks,
    streaming/load_steps.py:451-522): before block s runs its parameters are bound to the slot's tensors (the
    dequantised weights), after it the slot is released and the block num_slots ahead is prefetched. Returns the
    hook handles. Parameter names must match the layout's ParamSpec names (module.named_parameters())."""
    handles = []

    def make_pre(s_idx):
        def pre(module, args):
            if s_idx == 0:
                state.prefetch_first_slots()
            tensors = state.acquire(s_idx)
            for name, p in module.named_parameters():
                t = tensors.get(name)
                if t is not None:
                    p.data = t
        return pre

    def make_post(s_idx):
        def post(module, args, output):
            state.release(s_idx)
        return post

    for s_idx, blk in enumerate(blocks):
        handles.append(blk.register_forward_pre_hook(make_pre(s_idx)))
        handles.append(blk.register_forward_hook(make_post(s_idx)))
    return handles


def capture_block(params, specs, holder_cls=None):
    """One block's packed host bytes in a flat pinned buffer (the reference's _capture_streamed_blocks,
    load_steps.py:1152-1274, for one block): params maps name -> CPU tensor (packed uint8 for GGUF specs, the value
    otherwise). Returns (PinnedHost, layout)."""
    from ..core.tiers.pinned import PinnedHost
    layout = BlockLayout(specs)
    holder = (holder_cls or PinnedHost)(layout.flat_bytes)
    flat = holder.tensor
    for p, off in zip(layout.specs, layout.offsets):
        src = params[p.name].contiguous().reshape(-1).view(torch.uint8)
        if src.numel() != p.packed_bytes:
            raise ValueError(f"{p.name}: {src.numel()} bytes, the layout expects {p.packed_bytes}")
        flat[off:off + p.packed_bytes].copy_(src)
    return holder, layout


def as_task_array(items):
    arr = (_ext.DequantTask * len(items))()
    for i, (s, d, n) in enumerate(items):
        arr[i].src, arr[i].dst, arr[i].n_values = s, d, n
    return arr


_ = ctypes  # the task tables are ctypes arrays built once per slot
