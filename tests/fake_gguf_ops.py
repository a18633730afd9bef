"""A stand-in for ComfyUI-GGUF's ``ops`` module (absent here), registered as ``ComfyUI-GGUF.ops`` so that
``gguf_dequant.install()`` finds and patches it the way it patches the real one. It keeps what the streaming node and
the dequantisation patch touch: ``dequantize_tensor(tensor, dtype, dequant_dtype)`` looked up at call time, weights
that carry ``tensor_type`` / ``tensor_shape``, and ``GGMLLayer.get_weight`` calling it per use (ComfyUI-GGUF's
ops.py semantics: plain types are cast with ``.to(dtype)``, quantised ones dequantised). Its own dequantisation of
quantised types is deliberately absent: a test that reaches it has lost the B200 patch."""

import sys
import types

import torch
import torch.nn.functional as F

NAME = "ComfyUI-GGUF.ops"
F32, F16, BF16 = 0, 1, 30   # GGML type ids of the plain types (TORCH_COMPATIBLE_QTYPES with None)


def _dequantize_tensor(tensor, dtype=None, dequant_dtype=None):
    qtype = getattr(tensor, "tensor_type", None)
    if qtype in (None, F32, F16, BF16):
        return tensor.to(dtype) if dtype is not None else tensor
    raise NotImplementedError(f"the stand-in does not dequantise GGML type {qtype}")


class GGMLLayer(torch.nn.Module):
    dequant_dtype = None
    patch_dtype = None

    def get_weight(self, tensor, dtype):
        if tensor is None:
            return None
        mod = sys.modules[NAME]
        w = mod.dequantize_tensor(tensor, dtype, self.dequant_dtype)
        return w.as_subclass(torch.Tensor) if type(w) is not torch.Tensor else w


class Linear(GGMLLayer):
    def __init__(self, weight, bias=None, dequant_dtype=None):
        super().__init__()
        self.weight = weight
        self.bias = bias
        self.dequant_dtype = dequant_dtype

    def forward(self, x):
        return F.linear(x, self.get_weight(self.weight, x.dtype), self.get_weight(self.bias, x.dtype))


def gguf_param(raw_u8, qtype, shape, device):
    """A parameter holding packed GGUF bytes with ComfyUI-GGUF's tensor_type / tensor_shape."""
    p = torch.nn.Parameter(torch.as_tensor(raw_u8).to(device), requires_grad=False)
    p.tensor_type = int(qtype)
    p.tensor_shape = torch.Size(shape)
    return p


def plain_param(t, device):
    p = torch.nn.Parameter(t.to(device), requires_grad=False)
    p.tensor_type = F32 if t.dtype == torch.float32 else (BF16 if t.dtype == torch.bfloat16 else F16)
    p.tensor_shape = t.shape
    return p


def register():
    """Put the stand-in into sys.modules (fresh each call); returns it."""
    mod = types.ModuleType(NAME)
    mod.dequantize_tensor = _dequantize_tensor
    mod.GGMLLayer = GGMLLayer
    mod.Linear = Linear
    sys.modules[NAME] = mod
    return mod


def unregister():
    sys.modules.pop(NAME, None)
