"""SSD cache files of the streaming tier (core/tiers/cache_files.py of the reference, :1-190): their directory and
names, clean-up of files left by processes that ended, and DiskBlockStore, the fixed-stride file that holds the
SSD-tier blocks when they are not read straight from the model file."""

import atexit
import os
import re
import tempfile

from .. import env as _env
from .disk_io import _OPEN_READERS, _UnbufferedWriter, align_up, aligned_host

_LIVE_CACHE_FILES = set()
_CLEANED_DIRS = set()
_CACHE_FILE_RE = re.compile(r"^wfb200_blocks_(\d+)_[0-9a-f]{32}\.bin$")


def default_cache_dir():
    """WEIGHTFERRY_DISK_DIR, else ComfyUI's temp folder, else the system temp folder (a ``weightferry_cache`` folder
    in either)."""
    d = _env.get("WEIGHTFERRY_DISK_DIR")
    if d:
        return d
    try:
        import folder_paths  # ComfyUI
        return os.path.join(folder_paths.get_temp_directory(), "weightferry_cache")
    except (ImportError, AttributeError):
        return os.path.join(tempfile.gettempdir(), "weightferry_cache")


def _delete_live_cache_files():
    for reader in list(_OPEN_READERS):
        try:
            reader.close()
        except Exception:  # noqa: BLE001 -- at exit: close what can be closed, then delete
            pass
    for path in list(_LIVE_CACHE_FILES):
        try:
            os.remove(path)
        except OSError:
            pass
        _LIVE_CACHE_FILES.discard(path)


atexit.register(_delete_live_cache_files)


def new_cache_path(directory):
    """A new cache file name ``wfb200_blocks_<pid>_<uuid>.bin`` in ``directory`` (the pid lets a later process tell
    files of ended processes apart)."""
    import uuid
    return os.path.join(directory, f"wfb200_blocks_{os.getpid()}_{uuid.uuid4().hex}.bin")


def cleanup_stale_cache_files(directory):
    """Delete the cache files of processes that no longer run; returns the bytes freed."""
    try:
        import psutil
    except ImportError:  # without psutil no clean-up
        return 0
    freed = 0
    try:
        names = os.listdir(directory)
    except OSError:
        return 0
    for name in names:
        m = _CACHE_FILE_RE.match(name)
        if m is None:
            continue
        pid = int(m.group(1))
        if pid == os.getpid() or psutil.pid_exists(pid):
            continue
        path = os.path.join(directory, name)
        try:
            size = os.path.getsize(path)
            os.remove(path)
            freed += size
        except OSError:
            pass
    return freed


class DiskBlockStore:
    """Fixed-stride block file: block i at offset i * stride (stride = block bytes rounded up to 4 KiB), written
    through O_DIRECT from a 4 KiB aligned staging buffer. Shares the block-source read interface: ``n_blocks``,
    ``block_bytes``, ``buf_bytes`` (aligned read buffer size) and ``read_spec(i)`` -> (aligned file offset, aligned
    length, offset of the block in the buffer, block bytes). Deleted by ``delete()`` or at process exit."""

    is_model_file = False

    def __init__(self, path, block_bytes, n_blocks):
        self.path = path
        self.block_bytes = int(block_bytes)
        self.stride = align_up(self.block_bytes)
        self.buf_bytes = self.stride
        self.n_blocks = int(n_blocks)
        directory = os.path.dirname(path) or "."
        os.makedirs(directory, exist_ok=True)
        self.cleanup_report = None
        if directory not in _CLEANED_DIRS:
            _CLEANED_DIRS.add(directory)
            self.cleanup_report = {"freed_bytes": cleanup_stale_cache_files(directory)}
        _LIVE_CACHE_FILES.add(path)
        with open(path, "wb"):
            pass
        self._stage, self._writer = None, None

    def staging(self):
        """The block_bytes host buffer to fill and pass to write_block (the head of the aligned stride buffer, so
        the write needs no copy)."""
        if self._stage is None:
            self._stage, _ = aligned_host(self.stride, pin=False)
        return self._stage[:self.block_bytes]

    def write_block(self, i, cpu_uint8):
        """Write one block (a uint8 CPU tensor of block_bytes) to its place."""
        if cpu_uint8.numel() != self.block_bytes:
            raise ValueError(f"block of {cpu_uint8.numel()} bytes, the store holds {self.block_bytes}")
        if not 0 <= i < self.n_blocks:
            raise IndexError(f"block {i} of {self.n_blocks}")
        stage = self.staging()
        if cpu_uint8.data_ptr() != stage.data_ptr():
            stage.copy_(cpu_uint8)
        if self.stride > self.block_bytes:
            self._stage[self.block_bytes:].zero_()
        if self._writer is None:
            self._writer = _UnbufferedWriter(self.path)
        self._writer.write_from(i * self.stride, self.stride, self._stage.data_ptr())

    def finalize(self):
        """All blocks written: close the writer (fsync when it was buffered) and drop the staging buffer."""
        if self._writer is not None:
            self._writer.close()
            self._writer = None
        self._stage = None

    def read_spec(self, i):
        return i * self.stride, self.stride, 0, self.block_bytes

    def delete(self):
        self.finalize()
        try:
            os.remove(self.path)
        except OSError:
            pass
        _LIVE_CACHE_FILES.discard(self.path)

