"""A stand-in for ComfyUI's ModelPatcher and its comfy.patcher_extension (absent here): what the streaming node's
ComfyUI integration touches -- ``add_callback`` with the ON_LOAD / ON_DETACH callbacks (called with ComfyUI's
arguments when the model is loaded to / detached from the GPU), ``model_options`` wrappers of the DIFFUSION_MODEL kind
(each called as wrapper(executor, *args) around the diffusion model's forward), ``clone()`` that copies the options
and callbacks, ``model.diffusion_model``, ``load_device``. TEST INFRASTRUCTURE: the calling order follows the
reference's use of these hooks (streaming/dit_node.py:298-490 of ComfyUI-WeightFerry); a test drives load / forward /
detach by hand to reproduce ComfyUI's sequences, including a forward without a load."""

import sys
import types

NAME = "comfy.patcher_extension"


class CallbacksMP:
    ON_LOAD = "on_load"
    ON_DETACH = "on_detach"


class WrappersMP:
    DIFFUSION_MODEL = "diffusion_model"


def add_wrapper_with_key(wrapper_type, key, fn, obj, is_model_options=False):
    options = obj if is_model_options else obj.model_options
    table = options.setdefault("transformer_options", {}).setdefault("wrappers", {}).setdefault(wrapper_type, {})
    table.setdefault(key, []).append(fn)


class ModelPatcher:
    def __init__(self, dit, load_device, compute_dtype=None):
        self.model = types.SimpleNamespace(diffusion_model=dit, manual_cast_dtype=compute_dtype)
        self.load_device = load_device
        self.model_options = {"transformer_options": {}}
        self.callbacks = {}

    def clone(self):
        other = ModelPatcher.__new__(ModelPatcher)
        other.model, other.load_device = self.model, self.load_device
        other.model_options = _copy_options(self.model_options)
        other.callbacks = {k: list(v) for k, v in self.callbacks.items()}
        return other

    def add_callback(self, kind, fn):
        self.callbacks.setdefault(kind, []).append(fn)

    def load(self, device_to=None):
        for fn in self.callbacks.get(CallbacksMP.ON_LOAD, []):
            fn(self, device_to if device_to is not None else self.load_device, 0, False, True)

    def detach(self):
        for fn in self.callbacks.get(CallbacksMP.ON_DETACH, []):
            fn(self, True)

    def apply_model(self, *args, **kwargs):
        """The diffusion model's forward through this patcher's DIFFUSION_MODEL wrappers, outermost first."""
        wrappers = self.model_options.get("transformer_options", {}).get("wrappers", {})
        fns = [f for group in wrappers.get(WrappersMP.DIFFUSION_MODEL, {}).values() for f in group]

        def run(i, *a, **k):
            if i == len(fns):
                return self.model.diffusion_model(*a, **k)
            return fns[i](lambda *aa, **kk: run(i + 1, *aa, **kk), *a, **k)
        return run(0, *args, **kwargs)


def _copy_options(d):
    return {k: _copy_options(v) if isinstance(v, dict) else (list(v) if isinstance(v, list) else v)
            for k, v in d.items()}


def register():
    """Put comfy.patcher_extension into sys.modules (a bare ``comfy`` package too when there is none)."""
    comfy = sys.modules.get("comfy")
    if comfy is None:
        comfy = types.ModuleType("comfy")
        sys.modules["comfy"] = comfy
    mod = types.ModuleType(NAME)
    mod.CallbacksMP, mod.WrappersMP, mod.add_wrapper_with_key = CallbacksMP, WrappersMP, add_wrapper_with_key
    sys.modules[NAME] = mod
    comfy.patcher_extension = mod
    return mod


def unregister(drop_comfy=False):
    sys.modules.pop(NAME, None)
    if drop_comfy:
        sys.modules.pop("comfy", None)
