"""CUDA-event timeline of the block-streaming pipeline (WEIGHTFERRY_PROFILE=1; the role of streaming/profiler.py in
the reference, whose event names and summary fields are kept so that the same tools read both).

Per streamed block, events on the GPU timeline (so that events of different streams compare):

    dma0 -> dma1    host -> GPU copy of the block's packed bytes (copy stream)
    dma1 -> ready   dequantisation on arrival, the batched GGUF kernel (dequant stream)
    wait0 -> start  the compute stream waiting for the block's weights: the transfer time left exposed
    start -> end    the block's compute
    cpu_issue       recorded on an idle stream, so it completes when the host reaches it: when the transfer was issued

summary() folds each complete forward into the reference's fields (forward_ms, dma_ms, dequant_lora_ms, stall_ms,
streamed_compute_ms, compute_idle_ms, overlap_ratio, dma_gbps, cpu_hook_ms) and averages them over the forwards
after the first (which pays one-time costs).
"""

import torch

# per-block spans summed over a forward: (summary field, first event, second event)
_SPANS = (("dma_ms", "dma0", "dma1"), ("dequant_lora_ms", "dma1", "ready"), ("stall_ms", "wait0", "start"),
          ("streamed_compute_ms", "start", "end"))
_AVERAGED = ("forward_ms", "streamed_compute_ms", "compute_idle_ms", "dma_ms", "dequant_lora_ms", "stall_ms",
             "overlap_ratio", "dma_gbps", "cpu_hook_ms")


def _timed_event(stream):
    ev = torch.cuda.Event(enable_timing=True)
    ev.record(stream)
    return ev


class _ForwardTimeline:
    """The events of one forward: its bracket, each streamed block's named events, and host time in the hooks."""

    __slots__ = ("begin", "finish", "blocks", "host_seconds")

    def __init__(self, begin):
        self.begin, self.finish = begin, None
        self.blocks = {}
        self.host_seconds = 0.0

    def put(self, s_idx, name, event):
        self.blocks.setdefault(s_idx, {})[name] = event

    def fold(self, bytes_per_block):
        """This forward's summary row (its events must have completed)."""
        spans = dict.fromkeys((f for f, _a, _b in _SPANS), 0.0)
        for events in self.blocks.values():
            for field, first, second in _SPANS:
                if first in events and second in events:
                    spans[field] += events[first].elapsed_time(events[second])
        total = self.begin.elapsed_time(self.finish)
        moved = spans["dma_ms"] + spans["dequant_lora_ms"]
        n = len(self.blocks)
        row = {"forward_ms": round(total, 3), "streamed_blocks": n}
        row.update({k: round(v, 3) for k, v in spans.items()})
        row["compute_idle_ms"] = round(total - spans["streamed_compute_ms"], 3)
        row["overlap_ratio"] = (round(min(1.0, max(0.0, 1.0 - spans["stall_ms"] / moved)), 3) if moved > 0
                                else None)
        row["dma_gbps"] = (round(bytes_per_block * n / (spans["dma_ms"] * 1e-3) / 1e9, 2) if spans["dma_ms"] > 0
                           else None)
        row["cpu_hook_ms"] = round(self.host_seconds * 1e3, 3)
        return row


class _StreamProfiler:
    """Records the pipeline's events per forward (at most MAX_FORWARDS forwards) and summarises them."""

    MAX_FORWARDS = 64

    def __init__(self, num_stream, host_bytes, is_double=True, no_staging=False):
        self.num_stream = num_stream
        self.host_bytes = host_bytes
        self.is_double = is_double
        self.no_staging = no_staging
        self.forwards = []
        self.cur = None
        self.marker_stream = torch.cuda.Stream()  # idle: an event on it marks when the host got there

    def begin_forward(self, stream):
        if len(self.forwards) >= self.MAX_FORWARDS:
            self.cur = None
            return
        self.cur = _ForwardTimeline(_timed_event(stream))
        self.forwards.append(self.cur)

    def end_forward(self, stream):
        if self.cur is not None:
            self.cur.finish = _timed_event(stream)
            self.cur = None

    def record(self, s_idx, name, stream):
        if self.cur is not None:
            self.cur.put(s_idx, name, _timed_event(stream))

    def mark(self, s_idx, name):
        self.record(s_idx, name, self.marker_stream)

    def add_cpu(self, seconds):
        if self.cur is not None:
            self.cur.host_seconds += seconds

    def summary(self):
        torch.cuda.synchronize()
        rows = [f.fold(self.host_bytes) for f in self.forwards if f.finish is not None]
        steady = rows[1:] or rows
        mean = {}
        for field in _AVERAGED:
            vals = [r[field] for r in steady if r[field] is not None]
            mean[field] = round(sum(vals) / len(vals), 3) if vals else None
        return {"forwards_recorded": len(rows), "host_mb_per_block": round(self.host_bytes / 1024 ** 2, 1),
                "double_buffer": self.is_double, "storage_dtype_path": not self.no_staging,
                "mean_excluding_first_forward": mean, "per_forward": rows}
