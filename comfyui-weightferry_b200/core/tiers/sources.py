"""Block sources of the SSD tier and the reader ring that feeds them to the GPU (core/tiers/sources.py of the
reference, :1-355).

A source is either a DiskBlockStore (cache_files.py) or the model file itself: FileBlockSource (every block one
contiguous byte range of the file) or PieceFileSource (a block scattered over several ranges, packed in file order).
All expose ``n_blocks``, ``block_bytes``, ``buf_bytes`` and either ``read_spec(i)`` (one aligned read) or
``read_block(reader, i, dst_ptr, scratch_ptr)`` (several).

DiskRing keeps ``depth`` pinned 4 KiB aligned buffers filled by reader threads with the SSD-tier blocks in cyclic
order 0, 1, ..., n-1, 0, 1, ... -- a forward pass consumes them in that order, so reading simply runs on into the
next forward. ``acquire(d)`` waits for block d; ``release(buf, stream)`` records when the host-to-device copy out of
the buffer has finished (a CUDA event on the copy stream) and frees the buffer for the read ``depth`` positions
ahead; the reader waits for that event before it overwrites the buffer. A forward that stopped part way (an
exception) or a failed read is repaired by ``restart_if_needed()`` at the end of the forward, which restarts the
cycle at block 0."""

import ctypes
import sys
import threading
import time

from .disk_io import ALIGN_IO, _UnbufferedReader, align_up, aligned_host
from .pinned import release_all

_JOIN_TIMEOUT_S = 60  # how long close / resync wait for a reader thread inside a read


class FileBlockSource:
    """Blocks read straight from the model file: block i is the byte range ranges[i] = (absolute offset, size); a
    read covers its 4 KiB aligned superset and the block starts ``voff`` bytes into the buffer. Never deletes the
    file."""

    is_model_file = True

    def __init__(self, path, ranges):
        self.path = path
        self.ranges = [(int(o), int(n)) for o, n in ranges]
        self.n_blocks = len(self.ranges)
        self.block_bytes = max(n for _, n in self.ranges)
        self.buf_bytes = max(align_up(o + n) - o // ALIGN_IO * ALIGN_IO for o, n in self.ranges)

    def read_spec(self, i):
        o, n = self.ranges[i]
        start = o // ALIGN_IO * ALIGN_IO
        return start, align_up(o + n) - start, o - start, n

    def delete(self):
        pass  # the model file is not ours


class PieceFileSource:
    """Blocks read straight from the model file when each is several ranges (plan.file_param_layout): ``pieces[i]``
    is a list of (absolute offset, bytes, offset in the packed block). Each piece is read as its aligned superset
    into an unpinned scratch buffer and copied to its place. Never deletes the file."""

    is_model_file = True

    def __init__(self, path, pieces):
        self.path = path
        self.pieces = [[(int(o), int(n), int(d)) for o, n, d in blk] for blk in pieces]
        self.n_blocks = len(self.pieces)
        self.block_bytes = max(max(d + n for _, n, d in blk) for blk in self.pieces)
        self.buf_bytes = align_up(self.block_bytes)
        self.scratch_bytes = max(align_up(o + n) - o // ALIGN_IO * ALIGN_IO for blk in self.pieces for o, n, _ in blk)

    def read_block(self, reader, i, dst_ptr, scratch_ptr):
        for o, n, d in self.pieces[i]:
            start = o // ALIGN_IO * ALIGN_IO
            reader.read_into(start, align_up(o + n) - start, scratch_ptr, min_bytes=o - start + n)
            ctypes.memmove(dst_ptr + d, scratch_ptr + (o - start), n)
        return max(d + n for _, n, d in self.pieces[i])

    def delete(self):
        pass


def file_source(path, ranges):
    """FileBlockSource for one range per block, PieceFileSource for lists of pieces."""
    if ranges and isinstance(ranges[0], list):
        return PieceFileSource(path, ranges)
    return FileBlockSource(path, ranges)


class DiskRing:
    """Reader threads filling ``depth`` pinned buffers with a source's blocks in cyclic order (see the module text).

    Bookkeeping, all under one condition variable: position p of the cycle (block p % n) goes to buffer p % depth;
    readers claim positions in order and may read position p once p < consumed + depth (the buffer's previous
    position was released) -- then wait for that release's copy event before overwriting; a buffer publishes the
    position it holds when its read is complete, and acquire() waits for that. ``threads`` readers (at most
    ``depth``) each read one whole block at a time through their own file handle."""

    def __init__(self, store, depth, pin=True, threads=1):
        self.store = store
        self.n = store.n_blocks
        self.depth = max(1, int(depth))
        got = [aligned_host(store.buf_bytes, pin=pin) for _ in range(self.depth)]
        self.bufs = [t for t, _ in got]
        self._holders = [h for _, h in got]
        self.threads = max(1, min(int(threads), self.depth))
        self.wait_s = 0.0
        self._cv = threading.Condition()
        self._workers, self._handles = [], []
        self._start()

    # ------------------------------------------------------------------------------------------------ readers
    def _start(self):
        self._held = [-1] * self.depth             # cyclic position whose bytes the buffer holds (-1: none yet)
        self._view = [(0, 0)] * self.depth         # (offset in the buffer, bytes) of that block
        self._copy_done = [None] * self.depth      # CUDA event of the last copy out of the buffer
        self._claimed = 0                          # next position a reader takes
        self._consumed = 0                         # positions handed out and released
        self._error = None
        self._stopping = False
        self._handles = [_UnbufferedReader(self.store.path) for _ in range(self.threads)]
        self._workers = [threading.Thread(target=self._reader, args=(h,), daemon=True, name=f"wfb200-ssd-ring-{i}")
                         for i, h in enumerate(self._handles)]
        for w in self._workers:
            w.start()

    def _stop(self):
        with self._cv:
            self._stopping = True
            self._cv.notify_all()
        if not sys.is_finalizing():
            for w in self._workers:
                w.join(timeout=_JOIN_TIMEOUT_S)
            alive = [w.name for w in self._workers if w.is_alive()]
            if alive:
                # a reader still inside a read keeps its handle and the buffer it writes into
                raise TimeoutError(f"SSD ring: reader threads still running after {_JOIN_TIMEOUT_S} s: {alive}")
        for h in self._handles:
            h.close()
        self._workers, self._handles = [], []

    def _reader(self, handle):
        scratch, s_holder = (None, None)
        if hasattr(self.store, "read_block"):
            scratch, s_holder = aligned_host(self.store.scratch_bytes, pin=False)
        try:
            while True:
                with self._cv:
                    while not self._stopping and self._claimed >= self._consumed + self.depth:
                        self._cv.wait()
                    if self._stopping:
                        return
                    pos = self._claimed
                    self._claimed += 1
                    buf = pos % self.depth
                    done = self._copy_done[buf]
                if done is not None:
                    done.synchronize()  # the copy out of this buffer has finished
                view = self._read(handle, pos % self.n, buf, scratch)
                with self._cv:
                    self._view[buf] = view
                    self._held[buf] = pos
                    self._cv.notify_all()
        except BaseException as exc:  # noqa: BLE001 -- handed to the consumer by acquire()
            with self._cv:
                if self._error is None:
                    self._error = exc
                self._cv.notify_all()
            print(f"[tiers] SSD ring reader failed: {exc!r}", flush=True)
        finally:
            if s_holder is not None:
                s_holder.release()

    def _read(self, handle, d, buf, scratch):
        t0 = time.perf_counter()
        if scratch is not None:
            view = (0, self.store.read_block(handle, d, self.bufs[buf].data_ptr(), scratch.data_ptr()))
        else:
            off, length, voff, n = self.store.read_spec(d)
            handle.read_into(off, length, self.bufs[buf].data_ptr(), min_bytes=voff + n)
            view = (voff, n)
        dt = time.perf_counter() - t0
        if dt > 1.0:
            print(f"[tiers] slow SSD read: block {d} ({view[1] / 2 ** 20:.0f} MB) took {dt:.1f} s", flush=True)
        return view

    # ------------------------------------------------------------------------------------------------ consumer
    def acquire(self, d):
        """(pinned uint8 view holding SSD-tier block d, buffer index); waits for the reader."""
        with self._cv:
            pos = self._consumed
            if pos % self.n != d:
                raise RuntimeError(f"SSD ring out of sync: expected block {pos % self.n}, got {d}")
            buf = pos % self.depth
            t0 = time.perf_counter()
            while self._held[buf] != pos and self._error is None:
                if not self._cv.wait(60):
                    print(f"[tiers] still waiting for SSD block {d} after {time.perf_counter() - t0:.0f} s (claimed "
                          f"{self._claimed}, consumed {self._consumed}, buffers hold {self._held})", flush=True)
            self.wait_s += time.perf_counter() - t0
            if self._held[buf] != pos:
                raise RuntimeError(f"SSD ring: a reader failed ({self._error!r})") from self._error
            voff, n = self._view[buf]
        return self.bufs[buf][voff:voff + n], buf

    def release(self, buf, stream=None):
        """The copy out of buffer ``buf`` is enqueued on ``stream`` (None: already finished); the buffer may be
        refilled with the block ``depth`` positions ahead once that copy is done."""
        ev = None
        if stream is not None:
            import torch
            ev = torch.cuda.Event()
            ev.record(stream)
        with self._cv:
            self._copy_done[buf] = ev
            self._consumed += 1
            self._cv.notify_all()

    def at_cycle_start(self):
        return self._consumed % self.n == 0

    def failed(self):
        return self._error is not None

    def restart_if_needed(self, warn=print):
        """At the end of a forward: restart the cycle when the forward stopped part way through the SSD tier or a
        reader failed (also while reading ahead for the next forward). Returns True when restarted; a restart that
        times out leaves the ring marked failed, so the next forward reports it."""
        if self.at_cycle_start() and not self.failed():
            return False
        warn("SSD read-ahead: " + ("a reader failed; " if self.failed() else
                                   "the forward pass stopped part way through the SSD tier; ") + "restarting it.")
        try:
            self.resync()
        except TimeoutError as exc:
            self._error = self._error or exc
            warn(f"SSD read-ahead: could not restart ({exc}); the next forward will report it.")
            return False
        return True

    def resync(self):
        """Stop the readers, let the copies in flight finish, and restart the cycle at block 0."""
        self._stop()
        for ev in self._copy_done:
            if ev is not None:
                ev.synchronize()
        self._start()

    def close(self, release_buffers=True):
        self._stop()
        if release_buffers:
            for ev in self._copy_done:
                if ev is not None:
                    ev.synchronize()
            release_all(self._holders)
            self._holders = []
