"""Shared state of the fused block (enhancers/fused_state.py of the reference, :1-22): the installed parts, the
per-thread pending input / shared quantisation / pending residual, and the per-part used / fallback counters."""

import threading

_state = {"parts": (), "orig": None}
# calls per part: used / fell back to the host's code, with the first reason seen (stats())
_stats = {}
_tls = threading.local()


def _count(part, used, why=None):
    st = _stats.setdefault(part, {"used": 0, "fallback": 0, "why": None})
    if used:
        st["used"] += 1
    else:
        st["fallback"] += 1
        if st["why"] is None:
            st["why"] = why
