"""WeightFerry-B200: the quantized-weight hot path of ComfyUI-WeightFerry's DiT layer streaming, rebuilt for B200.

Loaded by ComfyUI as a custom-node package (by folder path, like the reference's __init__.py:84-97): at import it
installs the GGUF dequantisation patch and the fused Cosmos / Anima block when ComfyUI-GGUF / ComfyUI's Cosmos
classes are present. Outside ComfyUI (tests, benchmarks) importing it installs nothing.

Modules: ``enhancers`` (gguf_dequant, fused_kernels, fused_int8, fused_block, sage_fused -- the reference's
entry points over the CUDA kernels), ``streaming`` (the ⚡ DiT Layer Streaming node ``WeightFerryDiT``, slot ring
with dequant-on-arrival, profiler, tensor-parallel block stack), ``core`` (switches, pinned host buffers), ``_ext`` (the C-ABI binding)."""

from .streaming.dit_node import NODE_CLASS_MAPPINGS, NODE_DISPLAY_NAME_MAPPINGS  # noqa: E402,F401


def _install_at_import():
    import sys
    if "comfy" not in sys.modules:
        return
    from .enhancers import gguf_dequant
    try:
        from .enhancers import fused_block
        fused_block.install()
    except ImportError:
        pass
    gguf_dequant.install()


_install_at_import()
