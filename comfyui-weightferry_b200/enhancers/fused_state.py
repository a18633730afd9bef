"""State the fused-block modules share (the role of enhancers/fused_state.py in the reference, :1-22).

* ``_state``: the parts switched on by ``fused_block.install`` and ComfyUI's original methods it replaced.
* ``_tls``: per-thread hand-offs between a block and its layers for the duration of one call: ``pre`` (a pending
  input), ``qkv`` (the shared quantisation scope), ``res`` (the residual the output projection may absorb).
* ``COUNTERS`` / ``_count``: how often each part ran fused and how often it handed the call back to ComfyUI's code,
  with the first reason given; ``fused_block.stats()`` reports them as {part: {"used", "fallback", "why"}}.
"""

import threading

_state = {"parts": (), "orig": None}
_tls = threading.local()


class PartCounters:
    """Thread-safe per-part tallies (the uploader thread and the sampler thread may both count)."""

    def __init__(self):
        self._lock = threading.Lock()
        self._rows = {}

    def tally(self, part, used, why=None):
        with self._lock:
            row = self._rows.get(part)
            if row is None:
                row = self._rows[part] = [0, 0, None]
            if used:
                row[0] += 1
            else:
                row[1] += 1
                if row[2] is None:
                    row[2] = why

    def snapshot(self, reset=False):
        with self._lock:
            out = {p: {"used": u, "fallback": f, "why": w} for p, (u, f, w) in self._rows.items()}
            if reset:
                self._rows.clear()
        return out

    def get(self, part):
        with self._lock:
            return part in self._rows and self._rows[part][0] + self._rows[part][1] > 0


COUNTERS = PartCounters()


def _count(part, used, why=None):
    COUNTERS.tally(part, used, why)
