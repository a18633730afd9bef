"""CUDA-event timeline of the block-streaming pipeline (streaming/profiler.py of the reference, :9-134;
WEIGHTFERRY_PROFILE=1). Per streamed block, on the GPU timeline:
  dma0 -> dma1   host -> GPU copy of the block's packed bytes
  dma1 -> ready  dequantisation on arrival (the batched GGUF kernel)
  wait0 -> start compute stream stalled on this block's transfer (exposed transfer time)
  start -> end   block compute
summary() reports per forward the same fields as the reference (forward_ms, dma_ms, dequant_lora_ms, stall_ms,
overlap_ratio, dma_gbps, ...)."""

import torch


class _StreamProfiler:
    MAX_FORWARDS = 64

    def __init__(self, num_stream, host_bytes, is_double=True, no_staging=False):
        self.num_stream = num_stream
        self.host_bytes = host_bytes
        self.is_double = is_double
        self.no_staging = no_staging
        self.forwards = []
        self.cur = None
        self.marker_stream = torch.cuda.Stream()

    @staticmethod
    def _event(stream):
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        return e

    def mark(self, s_idx, name):
        if self.cur is not None:
            self.cur["blocks"].setdefault(s_idx, {})[name] = self._event(self.marker_stream)

    def begin_forward(self, stream):
        if len(self.forwards) >= self.MAX_FORWARDS:
            self.cur = None
            return
        self.cur = {"start": self._event(stream), "blocks": {}, "cpu_hook_s": 0.0}
        self.forwards.append(self.cur)

    def end_forward(self, stream):
        if self.cur is not None:
            self.cur["end"] = self._event(stream)
            self.cur = None

    def record(self, s_idx, name, stream):
        if self.cur is not None:
            self.cur["blocks"].setdefault(s_idx, {})[name] = self._event(stream)

    def add_cpu(self, seconds):
        if self.cur is not None:
            self.cur["cpu_hook_s"] += seconds

    def summary(self):
        torch.cuda.synchronize()
        per_forward = []
        for f in self.forwards:
            if "end" not in f:
                continue
            dma = conv = stall = comp = 0.0
            for b in f["blocks"].values():
                if "dma0" in b and "dma1" in b:
                    dma += b["dma0"].elapsed_time(b["dma1"])
                if "dma1" in b and "ready" in b:
                    conv += b["dma1"].elapsed_time(b["ready"])
                if "wait0" in b and "start" in b:
                    stall += b["wait0"].elapsed_time(b["start"])
                if "start" in b and "end" in b:
                    comp += b["start"].elapsed_time(b["end"])
            transfer = dma + conv
            n_blocks = len(f["blocks"])
            forward_ms = f["start"].elapsed_time(f["end"])
            per_forward.append({
                "forward_ms": round(forward_ms, 3),
                "streamed_blocks": n_blocks,
                "streamed_compute_ms": round(comp, 3),
                "compute_idle_ms": round(forward_ms - comp, 3),
                "dma_ms": round(dma, 3),
                "dequant_lora_ms": round(conv, 3),
                "stall_ms": round(stall, 3),
                "overlap_ratio": round(max(0.0, min(1.0, 1.0 - stall / transfer)), 3) if transfer > 0 else None,
                "dma_gbps": round(self.host_bytes * n_blocks / (dma / 1000) / 1e9, 2) if dma > 0 else None,
                "cpu_hook_ms": round(f["cpu_hook_s"] * 1000, 3),
            })
        later = per_forward[1:] or per_forward
        mean = {}
        for k in ("forward_ms", "streamed_compute_ms", "compute_idle_ms", "dma_ms", "dequant_lora_ms", "stall_ms",
                  "overlap_ratio", "dma_gbps", "cpu_hook_ms"):
            vals = [x[k] for x in later if x[k] is not None]
            mean[k] = round(sum(vals) / len(vals), 3) if vals else None
        return {"forwards_recorded": len(per_forward), "host_mb_per_block": round(self.host_bytes / 1024 ** 2, 1),
                "double_buffer": self.is_double, "storage_dtype_path": not self.no_staging,
                "mean_excluding_first_forward": mean, "per_forward": per_forward}
