"""File I/O of the SSD tier (core/tiers/disk_io.py of the reference, :1-203): reads and writes of 4 KiB aligned ranges
that bypass the page cache, 4 KiB aligned host buffers, and the drive's read-speed probe.

Linux is the platform here: the unbuffered path is ``O_DIRECT`` (the reference's Windows path is
FILE_FLAG_NO_BUFFERING; on Linux it reads through the page cache). ``O_DIRECT`` keeps a 15 GB checkpoint from filling
the page cache with pages that are read once per forward, and lets the reader threads stream at the drive's rate. A
file system that refuses ``O_DIRECT`` (tmpfs, some network mounts) falls back to ordinary reads. ``os.preadv`` and
``os.pwritev`` release the GIL for the system call, so several reader threads overlap their reads."""

import json
from concurrent.futures import ThreadPoolExecutor
import os
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
    """GB/s of an unbuffered read of the first ``nbytes`` of ``path`` by ``threads`` readers at once, each reading
    its own contiguous share in ``chunk_bytes`` pieces into its own aligned buffer."""
    pieces = list(range(0, nbytes, chunk_bytes))
    shares = [pieces[len(pieces) * t // threads:len(pieces) * (t + 1) // threads] for t in range(threads)]

    def read_share(offsets):
        buf, _holder = aligned_host(chunk_bytes, pin=False)
        reader = _UnbufferedReader(path)
        try:
            for off in offsets:
                reader.read_into(off, min(chunk_bytes, nbytes - off), buf.data_ptr())
        finally:
            reader.close()

    with ThreadPoolExecutor(max_workers=threads) as pool:
        start = time.perf_counter()
        for fut in [pool.submit(read_share, share) for share in shares]:
            fut.result()  # re-raises a reader's error
        elapsed = time.perf_counter() - start
    return nbytes / elapsed / 1e9


def _cached_probe(cache_path, size_mb, chunk_mb, thread_counts, max_age_s):
    """{threads: GB/s} from an earlier probe of the same sizes younger than max_age_s, or None."""
    try:
        with open(cache_path, encoding="utf-8") as f:
            rec = json.load(f)
        fresh = time.time() - float(rec["time"]) < max_age_s
        same = (rec["version"], rec["size_mb"], rec["chunk_mb"]) == (_PROBE_VERSION, size_mb, chunk_mb)
        by = {int(k): float(v) for k, v in rec["by_threads"].items()}
        if fresh and same and sorted(by) == sorted(thread_counts):
            return by, rec.get("direct")
    except (OSError, ValueError, KeyError, TypeError):  # none, old or damaged: measure again
        pass
    return None


def probe_disk(directory, size_mb=512, chunk_mb=32, thread_counts=(1, 2, 4), max_age_s=7 * 24 * 3600):
    """Unbuffered read rate of the drive holding ``directory`` with 1 / 2 / 4 reader threads (the role of the
    reference's probe_disk, core/tiers/disk_io.py:165-203), kept in the directory for a week: {"gbps": best GB/s,
    "threads": its thread count, "by_threads": {threads: GB/s}, "direct": O_DIRECT used}."""
    os.makedirs(directory, exist_ok=True)
    cache_path = os.path.join(directory, _PROBE_FILE)
    hit = _cached_probe(cache_path, size_mb, chunk_mb, thread_counts, max_age_s)
    if hit is None:
        path = os.path.join(directory, f"weightferry_b200_disk_probe_{os.getpid()}.bin")
        nbytes = size_mb * MB
        try:
            with open(path, "wb") as f:  # incompressible bytes, on the drive before the timed reads
                pattern = os.urandom(MB)
                for _ in range(size_mb):
                    f.write(pattern)
                f.flush()
                os.fsync(f.fileno())
            check = _UnbufferedReader(path)
            direct = check.direct
            check.close()
            by = {n: round(_timed_parallel_read(path, nbytes, chunk_mb * MB, n), 2) for n in thread_counts}
        finally:
            try:
                os.remove(path)
            except OSError:
                pass
        try:
            with open(cache_path, "w", encoding="utf-8") as f:
                json.dump({"version": _PROBE_VERSION, "time": time.time(), "size_mb": size_mb, "chunk_mb": chunk_mb,
                           "by_threads": by, "direct": direct}, f)
        except OSError:  # kept only to skip the probe next time
            pass
    else:
        by, direct = hit
    best = max(by, key=by.get)
    return {"gbps": by[best], "threads": best, "by_threads": by, "direct": direct}
