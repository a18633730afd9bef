"""The reference's kernel-layer entry points (enhancers/*.py of ComfyUI-WeightFerry) over the B200 kernels."""
