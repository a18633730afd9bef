"""Page-locked host memory of exactly the requested size (core/tiers/pinned.py of the reference, :74-192).

PyTorch's pinned allocator rounds every allocation up to a power of two and caches freed blocks; registering an
ordinary allocation with cudaHostRegister pins exactly what is needed and release() returns it at once. When
registration fails the buffer falls back to PyTorch's pinned allocator (still page-locked)."""

import threading

import torch

MB = 1024 * 1024
_REGISTERED = {"bytes": 0, "count": 0}
_LOCK = threading.RLock()


class PinnedHost:
    """Page-locked host buffer of exactly ``nbytes`` (plus optional alignment); ``.tensor`` is the uint8 view.
    Without a CUDA driver (nothing can be page-locked) the buffer stays pageable."""

    def __init__(self, nbytes, align=0):
        self.nbytes = int(nbytes)
        self._base = torch.empty(self.nbytes + align, dtype=torch.uint8, device="cpu")
        self._ptr = self._base.data_ptr()
        self.registered = False
        if self._base.numel() > 0:
            try:
                err = torch.cuda.cudart().cudaHostRegister(self._ptr, self._base.numel(), 0)
                self.registered = int(err) == 0
            except Exception:  # noqa: BLE001 -- not registered: use PyTorch's pinned allocator below
                self.registered = False
        if self.registered:
            with _LOCK:
                _REGISTERED["bytes"] += self._base.numel()
                _REGISTERED["count"] += 1
        elif self._base.numel() > 0:
            try:
                self._base = torch.empty(self.nbytes + align, dtype=torch.uint8, device="cpu", pin_memory=True)
                self._ptr = self._base.data_ptr()
            except RuntimeError:  # no CUDA driver: an ordinary (pageable) buffer, still correct for copies
                pass
        off = (-self._ptr) % align if align else 0
        self.tensor = self._base[off:off + self.nbytes]

    def release(self):
        if self._base is None:
            return
        if self.registered:
            try:
                torch.cuda.cudart().cudaHostUnregister(self._ptr)
            except Exception:  # noqa: BLE001 -- releasing during shutdown
                pass
            with _LOCK:
                _REGISTERED["bytes"] -= self._base.numel()
                _REGISTERED["count"] -= 1
            self.registered = False
        self.tensor = None
        self._base = None

    def __del__(self):
        try:
            self.release()
        except Exception:  # noqa: BLE001 -- __del__ must not raise
            pass


def gpu_local_cpus(device_index, nvml=None):
    """The CPUs on the NUMA node of CUDA device ``device_index`` (NVML's CPU affinity of the GPU found by its PCI bus
    id, so CUDA_VISIBLE_DEVICES renumbering does not matter), or None when NVML cannot tell."""
    try:
        if nvml is None:
            import pynvml as nvml
        props = torch.cuda.get_device_properties(device_index)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        nvml.nvmlInit()
        try:
            h = nvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = nvml.nvmlDeviceGetCpuAffinity(h, 16)   # 16 x 64 CPUs
        finally:
            nvml.nvmlShutdown()
    except Exception:  # noqa: BLE001 -- no NVML, no such device: leave the affinity alone
        return None
    cpus = [64 * i + b for i, w in enumerate(words) for b in range(64) if (int(w) >> b) & 1]
    return cpus or None


def bind_to_gpu_numa(device_index, nvml=None):
    """Restrict this process to the CPUs local to the GPU, so that pinned host buffers allocated (first touched) from
    now on live on the GPU's NUMA node and its host-to-device copies do not cross sockets. Returns the CPUs bound,
    or None (left unchanged)."""
    import os
    cpus = gpu_local_cpus(device_index, nvml)
    if not cpus:
        return None
    try:
        allowed = os.sched_getaffinity(0)
        mine = sorted(set(cpus) & allowed)
        if not mine:
            return None
        os.sched_setaffinity(0, mine)
        return mine
    except (AttributeError, OSError):
        return None


def release_all(holders):
    for h in holders or ():
        if h is not None:
            h.release()


def empty_host_cache():
    """Return memory cached by PyTorch's pinned allocator to the OS, when this PyTorch exposes it."""
    fn = getattr(torch._C, "_host_emptyCache", None)
    if fn is not None:
        try:
            fn()
        except Exception:  # noqa: BLE001 -- best effort
            pass


def registered_bytes():
    with _LOCK:
        return _REGISTERED["bytes"], _REGISTERED["count"]


def mem_snapshot():
    """Process RSS, system available RAM and pinned host memory, in MB (logging)."""
    snap = {}
    try:
        import psutil
        snap["rss_mb"] = round(psutil.Process().memory_info().rss / MB, 1)
        snap["sys_available_mb"] = round(psutil.virtual_memory().available / MB, 1)
    except Exception:  # noqa: BLE001 -- logging only
        pass
    snap["weightferry_registered_pinned_mb"] = round(_REGISTERED["bytes"] / MB, 1)
    return snap
