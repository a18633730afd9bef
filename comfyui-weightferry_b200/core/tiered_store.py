"""Tiered weight store of the streaming path (the reference's core/tiered_store.py, a re-export of its tiers/
package): exact-size pinned RAM for the RAM tier; for the SSD tier the O_DIRECT reader / writer and probe, the tier
planner and safetensors layouts, the fixed-stride cache file and the pinned read-ahead ring (DiskRing) with its
model-file sources. The implementation lives in core/tiers/, split by concern. The reference's persistent cross-run
cache (PersistentBlockStore, persist_dir, persist_enforce_cap) is not part of this path."""

from .tiers.pinned import PinnedHost, empty_host_cache, mem_snapshot, registered_bytes, release_all  # noqa: F401
from .tiers.disk_io import ALIGN_IO, _UnbufferedReader, align_up, aligned_host, probe_disk  # noqa: F401
from .tiers.plan import (  # noqa: F401
    available_ram, file_block_layout, file_param_layout, plan_tiers, safetensors_header, ssd_positions,
)
from .tiers.cache_files import (  # noqa: F401
    DiskBlockStore, cleanup_stale_cache_files, default_cache_dir, new_cache_path,
)
from .tiers.sources import DiskRing, FileBlockSource, PieceFileSource, file_source  # noqa: F401
