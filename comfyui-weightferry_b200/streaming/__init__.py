"""Block streaming: pinned host blocks, GPU slot ring with dequantisation on arrival, profiler, TP block stack."""
