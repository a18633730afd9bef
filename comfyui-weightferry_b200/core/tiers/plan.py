"""Tier planning of the streamed blocks (core/tiers/plan.py of the reference, :1-255): how many stay in pinned RAM
and which are served from the SSD (plan_tiers, ssd_positions), and the safetensors byte layouts that let the SSD tier
read whole blocks straight from a model file (file_block_layout, file_param_layout)."""

import json
import math
import struct

import torch

from .. import env as _env
from .disk_io import probe_disk
from .pinned import MB


def ssd_positions(num_stream, n_disk, layout=None):
    """Streamed-block indices served from the SSD (ascending), ``n_disk`` of ``num_stream``. "interleave" (default,
    WEIGHTFERRY_SSD_LAYOUT): spread evenly with the last block on the SSD, so the reader keeps reading while the GPU
    computes the RAM-tier blocks between two SSD blocks; "tail": the last n_disk blocks."""
    layout = layout or _env.get("WEIGHTFERRY_SSD_LAYOUT")
    if n_disk <= 0:
        return []
    if layout == "tail" or n_disk >= num_stream:
        return list(range(num_stream - n_disk, num_stream))
    return [int((k + 1) * num_stream / n_disk) - 1 for k in range(n_disk)]


def available_ram():
    """Available system RAM in bytes (psutil)."""
    import psutil
    return psutil.virtual_memory().available


def plan_tiers(num_stream, block_bytes, ram_budget_bytes=None, ram_margin_bytes=None, disk_dir=None,
               compute_ms_per_block=None, total_blocks=None, probe=None):
    """Split the streamed blocks between pinned RAM and the SSD (the reference's plan_tiers, :60-151).

    * RAM budget: ``ram_budget_bytes``, else available RAM minus a margin (WEIGHTFERRY_RAM_MARGIN_GB, default 6).
    * Ring depth: enough read-ahead to cover one block's SSD read with block compute (+2), 2..8 (4 without a compute
      time); the ring is pinned RAM and counts against the budget, shrinking to what fits (at least 2).
    * The SSD tier is predicted to bind when reading the SSD blocks takes longer than a forward's compute.
    ``probe``: the drive's read rate ({"gbps", "threads", "by_threads"}); measured with probe_disk when None.
    Without a read rate (the probe failed) every block stays in RAM and the plan carries the error."""
    avail = available_ram()
    if ram_margin_bytes is None:
        ram_margin_bytes = int(float(_env.get("WEIGHTFERRY_RAM_MARGIN_GB")) * 1024 ** 3)
    budget = ram_budget_bytes if ram_budget_bytes is not None else max(0, avail - ram_margin_bytes)
    if disk_dir is None:
        from .cache_files import default_cache_dir
        disk_dir = default_cache_dir()

    disk_threads, disk_gbps, by_threads, disk_error = 1, None, None, None
    try:
        p = probe if probe is not None else probe_disk(disk_dir)
        disk_gbps, disk_threads, by_threads = p["gbps"], p["threads"], p.get("by_threads")
        env_threads = _env.get("WEIGHTFERRY_DISK_THREADS")
        if env_threads and by_threads:
            disk_threads = max(1, int(env_threads))
            disk_gbps = by_threads.get(disk_threads, disk_gbps)
    except Exception as exc:  # noqa: BLE001 -- plan without an SSD tier; the error stays in the plan
        disk_error = str(exc)

    t_disk_ms = None if not disk_gbps else block_bytes / (disk_gbps * 1e9) * 1000
    if t_disk_ms is not None and compute_ms_per_block:
        depth = max(2, min(8, math.ceil(t_disk_ms / compute_ms_per_block) + 2))
    else:
        depth = 4
    depth_wanted = depth
    if disk_gbps is None or budget >= num_stream * block_bytes:
        ram_blocks = num_stream
    else:
        ram_blocks = int(max(0, min(num_stream, (budget - depth * block_bytes) // block_bytes)))
        if ram_blocks == 0 and depth * block_bytes > budget:
            depth = max(2, min(depth, int(budget // block_bytes)))
    n_disk = num_stream - ram_blocks
    if n_disk == 0:
        depth = 0
    host_planned = (ram_blocks + depth) * block_bytes
    plan = {
        "ram_blocks": ram_blocks,
        "disk_blocks": n_disk,
        "ring_depth": depth,
        "ring_depth_wanted": depth_wanted if n_disk else 0,
        "block_mb": round(block_bytes / MB, 1),
        "ram_budget_mb": round(budget / MB, 1),
        "available_ram_mb": round(avail / MB, 1),
        "host_ram_planned_mb": round(host_planned / MB, 1),
        "over_budget": host_planned > budget,
        "disk_dir": disk_dir,
        "disk_read_gbps": disk_gbps,
        "disk_threads": disk_threads,
        "disk_read_gbps_by_threads": by_threads,
        "disk_error": disk_error,
        "disk_ms_per_block": None if t_disk_ms is None else round(t_disk_ms, 2),
        "compute_ms_per_block": None if compute_ms_per_block is None else round(compute_ms_per_block, 2),
    }
    if t_disk_ms is not None and compute_ms_per_block and total_blocks:
        plan["disk_ms_per_forward"] = round(n_disk * t_disk_ms, 1)
        plan["compute_ms_per_forward_est"] = round(total_blocks * compute_ms_per_block, 1)
        plan["disk_bound"] = n_disk * t_disk_ms > total_blocks * compute_ms_per_block
    return plan


# ------------------------------------------------------------------------------------------- safetensors layouts
def safetensors_header(path):
    """(header dict without __metadata__, absolute offset of the data section) of a safetensors file: an 8-byte
    little-endian header length, the JSON header, then the data."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    header.pop("__metadata__", None)
    return header, 8 + n


_PREFIXES = ("", "net.", "model.diffusion_model.", "diffusion_model.", "model.")

_ST_DTYPES = {"F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
              "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2, "I64": torch.int64, "I32": torch.int32,
              "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8, "BOOL": torch.bool}


def _find(header, name):
    """The header entry of ``name`` under any of the usual file prefixes, or None."""
    for pre in _PREFIXES:
        info = header.get(pre + name)
        if info is not None:
            return info
    return None


def _entries(header, base, names):
    """Per name (absolute start, bytes, torch dtype, shape) of its tensor in the file, or None when one is missing or
    of a dtype without a torch counterpart."""
    out = []
    for name in names:
        info = _find(header, name)
        if info is None or info.get("dtype") not in _ST_DTYPES:
            return None
        a, b = info["data_offsets"]
        out.append((base + a, b - a, _ST_DTYPES[info["dtype"]], tuple(info["shape"])))
    return out


def file_block_layout(path, block_names):
    """Byte layout of whole blocks in a safetensors file, or None. ``block_names``: per block, its parameter names
    relative to the diffusion model (any usual file prefix is matched). Every block must be one contiguous byte range
    holding exactly its tensors, laid out like the first block. Returns {"ranges": [(absolute offset, bytes)],
    "rel_offsets" (per parameter, block_names order), "dtypes", "shapes"}."""
    header, base = safetensors_header(path)
    blocks = [_entries(header, base, names) for names in block_names]
    if not blocks or any(b is None for b in blocks):
        return None
    ref = None
    ranges = []
    for ents in blocks:
        lo = min(e[0] for e in ents)
        span = max(e[0] + e[1] for e in ents) - lo
        if span != sum(e[1] for e in ents):
            return None  # a gap or a foreign tensor inside the block's range
        shape_rel = ([e[0] - lo for e in ents], [e[3] for e in ents])
        if ref is None:
            ref = shape_rel
        elif shape_rel != ref:
            return None
        ranges.append((lo, span))
    return {"ranges": ranges, "rel_offsets": ref[0], "dtypes": [e[2] for e in blocks[0]], "shapes": ref[1]}


def file_param_layout(path, block_names):
    """Byte layout of blocks whose tensors are scattered in a safetensors file (for example grouped by dtype), or
    None. A block is packed densely in its file order, which must be the same for every block. Returns {"ranges":
    per block its pieces (absolute offset, bytes, offset in the packed block) with neighbouring tensors merged,
    "rel_offsets" (per parameter, block_names order), "param_abs", "block_bytes", "dtypes", "shapes",
    "pieces_per_block"}."""
    header, base = safetensors_header(path)
    blocks = [_entries(header, base, names) for names in block_names]
    if not blocks or any(b is None for b in blocks):
        return None
    first = blocks[0]
    order = sorted(range(len(first)), key=lambda k: first[k][0])
    packed = [0] * len(first)
    cursor = 0
    for k in order:
        packed[k] = cursor
        cursor += first[k][1]
    shapes = [e[3] for e in first]
    all_pieces, param_abs = [], []
    for ents in blocks:
        if sorted(range(len(ents)), key=lambda k: ents[k][0]) != order or [e[3] for e in ents] != shapes:
            return None
        pieces = []
        for k in order:
            start, nbytes = ents[k][0], ents[k][1]
            if pieces:
                p_start, p_len, p_dst = pieces[-1]
                if p_start + p_len == start and p_dst + p_len == packed[k]:
                    pieces[-1] = (p_start, p_len + nbytes, p_dst)
                    continue
            pieces.append((start, nbytes, packed[k]))
        all_pieces.append(pieces)
        param_abs.append([e[0] for e in ents])
    return {"ranges": all_pieces, "rel_offsets": packed, "param_abs": param_abs, "block_bytes": cursor,
            "dtypes": [e[2] for e in first], "shapes": shapes, "pieces_per_block": [len(p) for p in all_pieces]}
