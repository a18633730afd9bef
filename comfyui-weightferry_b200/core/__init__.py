"""Configuration and host-memory tiers of the streaming path."""
