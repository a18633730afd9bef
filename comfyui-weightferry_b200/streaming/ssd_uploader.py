"""The background thread that moves SSD-tier blocks into their GPU slots (streaming/ssd_uploader.py of the
reference, :17-120), with this build's dequantisation on arrival.

Jobs (block, slot, slot-free event) are submitted in block order when the compute thread would issue the prefetch.
Per job the thread takes the block's bytes from the DiskRing (waiting for its reader threads when needed) and, on
its own two CUDA streams:

  copy stream     wait slot-free -> H2D of the packed bytes out of the pinned ring buffer -> give the buffer back to
                  the ring (its reader waits for this copy before reusing it) -> record transferred[s]
  dequant stream  wait transferred[s] -> the slot's batched GGUF launches -> record ready[s]

then marks the job done. ``wait(s)`` (before block s computes) returns once ready[s] has been recorded; the compute
stream then waits on it like for a RAM-tier block. A failure inside the thread is raised by ``wait``."""

import queue
import sys
import threading
import time

import torch


class _SsdUploader:
    def __init__(self, state):
        self.state = state
        self.device = state.device
        with torch.cuda.device(self.device):
            self.copy_stream = torch.cuda.Stream(device=self.device)
            self.dequant_stream = torch.cuda.Stream(device=self.device)
        self.done = [threading.Event() for _ in range(state.num_stream)]
        self.main_wait_s = 0.0
        self.error = None
        self.submitted = 0
        self.waited = 0
        self._q = queue.Queue()
        # the slots may be inference tensors (created under torch.inference_mode); threads do not inherit the mode
        self.inference = torch.is_inference_mode_enabled()
        self._thread = threading.Thread(target=self._run, daemon=True, name="wfb200-ssd-upload")
        self._thread.start()

    def submit(self, s_idx, slot_idx):
        # a fresh event for "the slot's last reader has finished": computed_events[slot] is recorded again by later
        # blocks, and a wait on a later recording would make this copy wait for compute that needs it
        free = torch.cuda.Event()
        free.record(torch.cuda.current_stream(self.device))
        self.done[s_idx].clear()
        self.submitted += 1
        self._q.put((s_idx, slot_idx, free))

    def _run(self):
        with torch.inference_mode(self.inference):
            torch.cuda.set_device(self.device)
            while True:
                job = self._q.get()
                if job is None:
                    self._q.task_done()
                    return
                s_idx, slot_idx, free = job
                try:
                    if self.error is None:
                        self._upload(s_idx, slot_idx, free)
                except Exception as exc:  # noqa: BLE001 -- raised on the compute thread by wait()
                    self.error = exc
                finally:
                    self.done[s_idx].set()
                    self._q.task_done()

    def _upload(self, s_idx, slot_idx, free):
        st = self.state
        src, buf = st.ring.acquire(st.disk_index[s_idx])
        prof = st.profiler
        cs, ds = self.copy_stream, self.dequant_stream
        with torch.cuda.stream(cs):
            cs.wait_event(free)
            if prof is not None:
                prof.record(s_idx, "dma0", cs)
            st.slot_flats[slot_idx].copy_(src, non_blocking=True)
            st.ring.release(buf, cs)
            if prof is not None:
                prof.record(s_idx, "dma1", cs)
            st.transferred_events[s_idx].record(cs)
        ds.wait_event(st.transferred_events[s_idx])
        st.dequant_slot(slot_idx, ds)
        if prof is not None:
            prof.record(s_idx, "ready", ds)
        st.ready_events[s_idx].record(ds)

    def wait(self, s_idx):
        if not self.done[s_idx].is_set():
            t0 = time.perf_counter()
            self.done[s_idx].wait()
            self.main_wait_s += time.perf_counter() - t0
        self.waited += 1
        if self.error is not None:
            raise RuntimeError(f"DiT Layer Streaming: SSD upload failed: {self.error}") from self.error

    def outstanding(self):
        """Jobs submitted whose block was not waited for (a forward stopped part way)."""
        return self.submitted - self.waited

    def drain(self):
        """Finish every submitted job and the GPU work it enqueued; forget the jobs nobody waited for."""
        if sys.is_finalizing():
            return
        self._q.join()
        self.copy_stream.synchronize()
        self.dequant_stream.synchronize()
        self.submitted = self.waited = 0

    def close(self):
        self._q.put(None)
        if sys.is_finalizing():
            return
        self._thread.join(timeout=60)
