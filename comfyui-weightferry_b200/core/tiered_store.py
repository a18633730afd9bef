"""Host tiers of the streaming path: exact-size pinned RAM (the reference's core/tiered_store.py re-export; the SSD
ring and tier planner of the reference are not part of this path)."""

from .tiers.pinned import PinnedHost, empty_host_cache, mem_snapshot, registered_bytes, release_all  # noqa: F401
