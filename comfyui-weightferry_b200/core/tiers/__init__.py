"""Host-memory tiers of the streaming path (pinned RAM)."""
