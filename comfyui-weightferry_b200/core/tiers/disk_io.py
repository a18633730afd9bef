"""File I/O of the SSD tier (core/tiers/disk_io.py of the reference, :1-203): reads and writes of 4 KiB aligned ranges
that bypass the page cache, 4 KiB aligned host buffers, and the drive's read-speed probe.

Linux is the platform here: the unbuffered path is ``O_DIRECT`` (the reference's Windows path is
FILE_FLAG_NO_BUFFERING; on Linux it reads through the page cache). ``O_DIRECT`` keeps a 15 GB checkpoint from filling
the page cache with pages that are read once per forward, and lets the reader threads stream at the drive's rate. A
file system that refuses ``O_DIRECT`` (tmpfs, some network mounts) falls back to ordinary reads. ``os.preadv`` and
``os.pwritev`` release the GIL for the system call, so several reader threads overlap their reads."""

import json
import os
import threading
import time
import weakref

import torch

from .pinned import MB, PinnedHost

ALIGN_IO = 4096  # offsets, sizes and buffer addresses of unbuffered I/O are multiples of this

_OPEN_READERS = weakref.WeakSet()


def align_up(n, a=ALIGN_IO):
    return (int(n) + a - 1) // a * a


def aligned_host(nbytes, pin=True):
    """A 4 KiB aligned uint8 host buffer of ``nbytes``: (tensor, PinnedHost holder or None). Pinned buffers are the
    DMA source of the host-to-device copies; unpinned ones serve as scratch."""
    if pin:
        h = PinnedHost(nbytes, align=ALIGN_IO)
        return h.tensor, h
    raw = torch.empty(int(nbytes) + ALIGN_IO, dtype=torch.uint8, device="cpu")
    off = (-raw.data_ptr()) % ALIGN_IO
    return raw[off:off + int(nbytes)], None


def _open_direct(path, flags):
    """(fd, direct?) -- O_DIRECT when the file system takes it, else an ordinary descriptor."""
    direct = getattr(os, "O_DIRECT", 0)
    if direct:
        try:
            return os.open(path, flags | direct), True
        except OSError:
            pass
    return os.open(path, flags), False


def _view(ptr, nbytes):
    import ctypes
    return memoryview((ctypes.c_char * int(nbytes)).from_address(int(ptr))).cast("B")


class _UnbufferedReader:
    """Reads 4 KiB aligned ranges of a file into 4 KiB aligned host memory (O_DIRECT where possible)."""

    _CHUNK = 64 * MB

    def __init__(self, path):
        self.path = path
        self.fd, self.direct = _open_direct(path, os.O_RDONLY)
        _OPEN_READERS.add(self)

    def read_into(self, offset, nbytes, dst_ptr, min_bytes=None):
        """Read ``nbytes`` (a multiple of 4 KiB) at ``offset`` (a multiple of 4 KiB) to address ``dst_ptr``. Reaching
        the end of the file is fine once ``min_bytes`` (default: all) have been read."""
        if self.fd is None:
            raise OSError(f"reader of {self.path} is closed")
        need = nbytes if min_bytes is None else min_bytes
        done = 0
        while done < nbytes:
            n = min(self._CHUNK, nbytes - done)
            got = os.preadv(self.fd, [_view(dst_ptr + done, n)], offset + done)
            done += max(got, 0)
            if got < n:  # a regular file reads short only at its end (and O_DIRECT could not continue unaligned)
                if done >= need:
                    return
                raise EOFError(f"unexpected end of {self.path} at byte {offset + done}")

    def close(self):
        if self.fd is not None:
            os.close(self.fd)
            self.fd = None


class _UnbufferedWriter:
    """Writes 4 KiB aligned ranges from 4 KiB aligned host memory (O_DIRECT where possible: no dirty pages to flush;
    else ordinary writes and an fsync in close())."""

    _CHUNK = 64 * MB

    def __init__(self, path):
        self.path = path
        self.fd, self.direct = _open_direct(path, os.O_WRONLY)

    def write_from(self, offset, nbytes, src_ptr):
        done = 0
        while done < nbytes:
            n = min(self._CHUNK, nbytes - done)
            done += os.pwritev(self.fd, [_view(src_ptr + done, n)], offset + done)

    def close(self):
        if self.fd is not None:
            if not self.direct:
                os.fsync(self.fd)
            os.close(self.fd)
            self.fd = None


_PROBE_FILE = "weightferry_b200_disk_probe.json"
_PROBE_VERSION = 1


def _timed_parallel_read(path, nbytes, chunk_bytes, threads):
    """GB/s of reading ``nbytes`` of ``path`` in ``chunk_bytes`` pieces with ``threads`` readers (chunk i -> thread
    i % threads)."""
    errors = []

    def work(t):
        reader = None
        try:
            buf, _ = aligned_host(chunk_bytes, pin=False)
            reader = _UnbufferedReader(path)
            for i, off in enumerate(range(0, nbytes, chunk_bytes)):
                if i % threads == t:
                    reader.read_into(off, chunk_bytes, buf.data_ptr())
        except Exception as exc:  # noqa: BLE001 -- re-raised below once every thread ended
            errors.append(exc)
        finally:
            if reader is not None:
                reader.close()

    workers = [threading.Thread(target=work, args=(t,), daemon=True) for t in range(threads)]
    t0 = time.perf_counter()
    for w in workers:
        w.start()
    for w in workers:
        w.join()
    dt = time.perf_counter() - t0
    if errors:
        raise errors[0]
    return nbytes / dt / 1e9


def probe_disk(directory, size_mb=512, chunk_mb=32, thread_counts=(1, 2, 4), max_age_s=7 * 24 * 3600):
    """Unbuffered read rate of the drive holding ``directory`` with 1 / 2 / 4 reader threads (the reference's
    probe_disk), cached in the directory for a week: {"gbps": best GB/s, "threads": its thread count,
    "by_threads": {threads: GB/s}, "direct": O_DIRECT used}."""
    os.makedirs(directory, exist_ok=True)
    cache_path = os.path.join(directory, _PROBE_FILE)
    try:
        with open(cache_path, encoding="utf-8") as f:
            cached = json.load(f)
        if (time.time() - cached.get("time", 0) < max_age_s and cached.get("version") == _PROBE_VERSION
                and cached.get("size_mb") == size_mb and cached.get("chunk_mb") == chunk_mb
                and sorted(int(k) for k in cached.get("by_threads", {})) == sorted(thread_counts)):
            by = {int(k): v for k, v in cached["by_threads"].items()}
            best = max(by, key=by.get)
            return {"gbps": by[best], "threads": best, "by_threads": by, "direct": cached.get("direct")}
    except (OSError, ValueError, KeyError, TypeError):  # no, old or damaged cache: measure again
        pass
    path = os.path.join(directory, f"weightferry_b200_disk_probe_{os.getpid()}.bin")
    nbytes = size_mb * MB
    block = os.urandom(MB)
    with open(path, "wb") as f:
        for _ in range(size_mb):
            f.write(block)
        f.flush()
        os.fsync(f.fileno())
    try:
        probe_reader = _UnbufferedReader(path)
        direct = probe_reader.direct
        probe_reader.close()
        by = {n: round(_timed_parallel_read(path, nbytes, chunk_mb * MB, n), 2) for n in thread_counts}
    finally:
        try:
            os.remove(path)
        except OSError:
            pass
    best = max(by, key=by.get)
    try:
        with open(cache_path, "w", encoding="utf-8") as f:
            json.dump({"version": _PROBE_VERSION, "by_threads": by, "size_mb": size_mb, "chunk_mb": chunk_mb,
                       "time": time.time(), "direct": direct}, f)
    except OSError:  # the result is cached only to skip the probe next time
        pass
    return {"gbps": by[best], "threads": best, "by_threads": by, "direct": direct}
