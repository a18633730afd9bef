"""The ⚡ DiT Layer Streaming node over this package's slot ring with dequantisation on arrival (the reference's
streaming/dit_node.py:38-455, WeightFerryDiT.apply_streaming).

``WeightFerryDiT().apply_streaming(model, ...)`` keeps the reference's signature, option strings and return value
``(MODEL,)``. ``model`` is a ComfyUI ModelPatcher (``clone()``, ``model.diffusion_model``, ``load_device``) or, outside
ComfyUI, the diffusion model itself (an ``nn.Module``). On a CUDA model whose diffusion model has a block list
(``blocks`` / ``transformer_blocks`` / ``layers`` / ``block``, the reference's streaming/common.py:125-144) it

1. keeps blocks 0 .. resident_blocks-1 where they are and streams the others; ``auto_config`` picks the resident count
   from the usable VRAM the way streaming/auto_config.py:15-85 does, and streams nothing when the model fits;
2. captures every streamed block into one exact-size pinned host buffer (core/tiers/pinned.py) with the 256-byte
   aligned flat layout of streaming/common.py:87-120. A GGUF weight (ComfyUI-GGUF's GGMLTensor: ``tensor_type``,
   ``tensor_shape``) travels as its packed bytes and is dequantised on arrival, with the intermediate precision its
   layer would use (``dequant_dtype``: None -> f16, "target" -> the compute dtype), so the slot holds the bits the
   layer's own dequantisation gives; a GGUF weight carrying LoRA patches, or of a type or precision the kernels do not
   take, travels packed and its layer dequantises it per use as before. The parameters are then bound to the host
   bytes (the reference's rest binding, dit_node.py:331-339), which frees their GPU memory;
3. builds the slot ring (streaming/state.py: ``prefetch_slots`` GPU slots, copy and dequant streams, events) and hooks
   every streamed block: before it runs, its parameters are bound to its slot (a dequantised GGUF weight is marked as
   a plain tensor for the block's duration: ComfyUI-GGUF's ``dequantize_tensor`` then returns it as it is); after it,
   the slot is released, the block ``prefetch_slots`` ahead is prefetched and the rest binding comes back;
4. brackets every forward of the diffusion model (the reference's streaming_diffusion_model_wrapper,
   dit_node.py:414-455) with begin_forward / end_forward, starting the first transfers before the resident blocks
   run, and captures again when something else rebound the streamed parameters (a ComfyUI model load).

With ``tiering`` "Auto (GPU / RAM / SSD)" (or WEIGHTFERRY_TIERING=auto) and a RAM budget (``ram_budget_gb`` or
WEIGHTFERRY_RAM_BUDGET_GB; else the available RAM minus WEIGHTFERRY_RAM_MARGIN_GB), core/tiers/plan.plan_tiers splits
the streamed blocks between pinned RAM and the SSD (the reference's tier planner, core/tiers/plan.py:60-151): the SSD
blocks, interleaved among the others, are written to a cache file (O_DIRECT) and read back every forward by a
DiskRing of pinned buffers and the uploader thread (streaming/ssd_uploader.py), which also dequantises them; their
parameters rest on a mapping of the cache file.

Options of the reference that select parts outside the quantized-weight path -- chunk streaming, SageAttention,
the fp8 storage host format -- are accepted and logged as not used here. resident_mode "Self-managed" dequantises the
resident blocks' GGUF weights once and binds them for each whole forward. "Single Buffer (Synchronous)" issues each block's transfer when the block starts (no look-ahead). A VRAM budget
(vram_budget_gb or WEIGHTFERRY_VRAM_BUDGET_GB) bounds what the automatic resident-block choice counts as usable."""

import weakref

import torch

from ..core import env as _env
from ..core.tiers.cache_files import DiskBlockStore, default_cache_dir, new_cache_path
from ..core.tiers.pinned import PinnedHost, release_all
from ..core.tiers.plan import plan_tiers, ssd_positions
from ..core.tiers.sources import DiskRing
from ..utils.logging import log_info, log_warn
from .state import _GGUF_GEOMETRY, BlockLayout, ParamSpec, _StreamState

# option values of the node (the reference's streaming/common.py:89-96 and dit_node.py:61-65): kept as they are,
# since saved workflows carry them
BUFFER_DOUBLE = "Double Buffer (Async Prefetch, Recommended)"
BUFFER_SINGLE = "Single Buffer (Synchronous)"
TIERING_RAM = "RAM (all streamed blocks pinned in RAM)"
TIERING_AUTO = "Auto (GPU / RAM / SSD)"
RESIDENT_MODE_COMFY = "ComfyUI (Dynamic VRAM)"
RESIDENT_MODE_SELF = "Self-managed (fixed on GPU)"
HOST_FORMAT_BAKED = "Compute dtype, LoRA baked (fast with LoRA)"
HOST_FORMAT_STORAGE = "Storage dtype (fp8), LoRA on GPU (half transfer)"

_BLOCK_LIST_ATTRS = ("blocks", "transformer_blocks", "layers", "block")
_STATE_ATTR = "_weightferry_stream_state"
_MID_CODE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}
_MID_DTYPE = {v: k for k, v in _MID_CODE.items()}


def _blocks(dit):
    """The first non-empty ModuleList among the block-list attribute names, else []."""
    for name in _BLOCK_LIST_ATTRS:
        lst = getattr(dit, name, None)
        if isinstance(lst, torch.nn.ModuleList) and len(lst) > 0:
            return lst
    return []


def _param_owner(blk, name):
    mod_name, _, _ = name.rpartition(".")
    return blk.get_submodule(mod_name) if mod_name else blk


def _raw(t):
    """The plain tensor under a parameter (a GGMLTensor or Parameter subclass becomes a torch.Tensor view)."""
    t = t.detach()
    return t if type(t) is torch.Tensor else t.as_subclass(torch.Tensor)


def _nbytes(t):
    return t.numel() * t.element_size()


def _gguf_mid(module, compute_dtype):
    """The dequantisation's intermediate precision code for a layer's ``dequant_dtype``, or None when the kernels do
    not take it (ComfyUI-GGUF: None -> f16, "target" -> the requested dtype, else a torch dtype)."""
    dd = getattr(module, "dequant_dtype", None)
    if dd == "target":
        dd = compute_dtype
    if dd is None:
        return 0
    return _MID_CODE.get(dd) if isinstance(dd, torch.dtype) else None


def param_spec(name, p, module, compute_dtype):
    """(ParamSpec, dequantised-on-arrival?) for one parameter of a streamed block."""
    raw = _raw(p)
    qtype = getattr(p, "tensor_type", None)
    try:
        qtype = None if qtype is None else int(qtype)
    except (TypeError, ValueError):
        qtype = None
    if qtype in _GGUF_GEOMETRY and raw.dtype == torch.uint8 and not getattr(p, "patches", None):
        mid = _gguf_mid(module, compute_dtype)
        shape = tuple(int(s) for s in getattr(p, "tensor_shape", raw.shape))
        if mid is not None:
            try:
                spec = ParamSpec(name, shape, qtype=qtype, mid=mid)
            except ValueError:
                spec = None
            if spec is not None and spec.packed_bytes == _nbytes(raw):
                return spec, True
    return ParamSpec(name, tuple(raw.shape), dtype=raw.dtype), False


def block_specs_of(blk, compute_dtype=torch.bfloat16):
    """The streamed layout of one block: a ParamSpec per parameter (named_parameters order) and which of them are
    dequantised on arrival."""
    specs, deq = [], []
    for name, p in blk.named_parameters():
        sp, d = param_spec(name, p, _param_owner(blk, name), compute_dtype)
        specs.append(sp)
        deq.append(d)
    return specs, deq


def _same_layout(a, b):
    return [(s.name, s.shape, s.qtype, s.dtype, s.mid) for s in a] == [(s.name, s.shape, s.qtype, s.dtype, s.mid)
                                                                       for s in b]


def auto_resident(num_blocks, block_bytes, slot_bytes, nonblock_bytes, usable, headroom, prefetch_slots, is_double):
    """Resident block count for the usable VRAM (the reference's _auto_config, streaming/auto_config.py:56-77): None
    when the whole model fits with the headroom (no streaming), else the blocks that fit beside the non-block weights,
    the slots and the headroom, at least 1 and at most num_blocks - 1."""
    fit_all = num_blocks * block_bytes + nonblock_bytes + headroom
    if fit_all <= usable:
        return None
    slots = (max(2, int(prefetch_slots)) if is_double else 2) * slot_bytes
    resident = int((usable - headroom - nonblock_bytes - slots) // max(1, block_bytes))
    return max(1, min(num_blocks - 1, resident))


def vram_budget_bytes(node_gb):
    """The VRAM budget in bytes (core/vram_budget.py:35-43 of the reference): the node's vram_budget_gb when > 0,
    else WEIGHTFERRY_VRAM_BUDGET_GB, else None (no budget: every free byte is used)."""
    gb = float(node_gb or 0.0)
    if gb <= 0:
        try:
            gb = float(_env.get("WEIGHTFERRY_VRAM_BUDGET_GB") or 0)
        except ValueError:
            gb = 0.0
    return int(gb * 1024 ** 3) if gb > 0 else None


def budget_usable(free_plus_cached, process_in_use, budget):
    """The VRAM the resident-block plan may count on: free + PyTorch's cached bytes, and with a budget at most what the
    budget leaves beside what this process already uses (the reference keeps that much free by raising ComfyUI's
    reserve, streaming/auto_config.py:52-54; here the plan itself stays inside it). The budget only moves which
    blocks stream, never the output."""
    if budget is None:
        return int(free_plus_cached)
    return max(0, min(int(free_plus_cached), int(budget) - int(process_in_use)))


class _PageableHost:
    """A plain (pageable) host buffer with PinnedHost's interface, for pin_memory=False."""

    def __init__(self, nbytes):
        self.nbytes = int(nbytes)
        self.tensor = torch.empty(self.nbytes, dtype=torch.uint8)

    def release(self):
        self.tensor = None


class _NodeState:
    """One streaming configuration of a diffusion model: the captured blocks, their rest binding and the slot ring."""

    def __init__(self, owner, dit, stream_idx, device, pin_memory, num_slots, lookahead, compute_dtype,
                 tiering_auto=False, ram_budget_bytes=None, self_resident=False):
        self.owner = owner
        self.self_resident = self_resident
        self.res_entries = []  # self-managed resident GGUF weights: (param, packed data, dequantised weight, tensor_type)
        self.res_bound = False
        self.tiering_auto = tiering_auto
        self.ram_budget_bytes = ram_budget_bytes
        self.tier_plan = None
        self.store = None
        self.disk_blocks = []
        self.dit = dit
        self.stream_idx = list(stream_idx)
        self.device = torch.device(device)
        self.pin_memory = pin_memory
        self.num_slots = num_slots
        self.lookahead = lookahead
        self.compute_dtype = compute_dtype
        self.handles = []
        self.holders = []
        self.entries = []   # per streamed block: [(param, name, dequantised?, rest tensor, tensor_type)]
        self.ring = None
        self.captures = 0
        self.bound = set()  # streamed blocks whose parameters are bound to their slot (between pre and post hook)

    def start(self):
        """Capture the streamed blocks, build the resident ones and hook the model (any earlier configuration of the
        model is torn down first)."""
        teardown(self.dit)
        self.capture()
        self.build_resident()
        self.install_hooks()
        setattr(self.dit, _STATE_ATTR, self)
        n_deq = sum(1 for _p, _n, d, _r, _t in self.entries[0] if d)
        log_info(f"DiT Layer Streaming: {len(self.stream_idx)} streaming blocks, pin_memory={self.pin_memory}, "
                 f"double_buffer={self.lookahead}, slots={self.ring.num_slots}; per block "
                 f"{self.layout.flat_bytes / 1024 ** 2:.1f} MB host, {n_deq} GGUF weights dequantised on arrival"
                 + (f"; self-managed resident blocks: {len(self.res_entries)} GGUF weights dequantised once."
                    if self.self_resident else "."))

    # ------------------------------------------------------------------------------------------------ capture
    def capture(self):
        """Every streamed block into its host buffer, parameters bound to it, and a new slot ring."""
        self.drop_ring()
        blocks = _blocks(self.dit)
        streamed = [blocks[i] for i in self.stream_idx]
        specs, deq = block_specs_of(streamed[0], self.compute_dtype)
        for i, blk in zip(self.stream_idx[1:], streamed[1:]):
            other, _ = block_specs_of(blk, self.compute_dtype)
            if not _same_layout(specs, other):
                raise ValueError(f"streamed block {i} has another parameter layout than block {self.stream_idx[0]}")
        layout = BlockLayout(specs, compute_dtype=self.compute_dtype)
        self._plan_tiers(len(streamed), layout.flat_bytes)
        disk_set = set(self.disk_blocks)
        holder_cls = PinnedHost if self.pin_memory else _PageableHost
        flats, pending = [], []
        for b, blk in enumerate(streamed):
            if b in disk_set:  # SSD tier: the block's flat bytes go to the cache file
                flat = self.store.staging()
                flats.append(None)
            else:
                holder = holder_cls(layout.flat_bytes)
                self.holders.append(holder)
                flat = holder.tensor
                flats.append(flat)
            params = dict(blk.named_parameters())  # (the alignment gaps between parameters are never read)
            block_params = []
            for sp, d, off in zip(specs, deq, layout.offsets):
                p = params[sp.name]
                raw = _raw(p)
                flat[off:off + sp.packed_bytes].copy_(raw.reshape(-1).view(torch.uint8))
                block_params.append((p, sp, d, off, raw.dtype, raw.shape))
            if b in disk_set:
                self.store.write_block(self.disk_blocks.index(b), flat)
            pending.append(block_params)
        ring = None
        if self.store is not None:
            self.store.finalize()
            # the SSD-tier parameters rest on a mapping of the cache file (no RAM held for them)
            mapped = torch.from_file(self.store.path, shared=True, size=self.store.stride * self.store.n_blocks,
                                     dtype=torch.uint8)
            for k, b in enumerate(self.disk_blocks):
                flats_b = mapped[k * self.store.stride:k * self.store.stride + layout.flat_bytes]
                pending[b] = [(p, sp, d, off, dt, sh, flats_b) for p, sp, d, off, dt, sh in pending[b]]
            plan = self.tier_plan
            ring = DiskRing(self.store, depth=max(2, plan["ring_depth"]), pin=self.pin_memory,
                            threads=plan["disk_threads"])
        for b, block_params in enumerate(pending):
            entries = []
            for item in block_params:
                p, sp, d, off, dt, sh = item[:6]
                src = item[6] if len(item) > 6 else flats[b]
                rest = src[off:off + sp.packed_bytes].view(dt).view(sh)
                entries.append((p, sp.name, d, rest, getattr(p, "tensor_type", None)))
            self.entries.append(entries)
        # the rest binding: between uses the streamed parameters are the host bytes (their GPU copies are freed)
        for entries in self.entries:
            for p, _name, _d, rest, _tt in entries:
                p.data = rest
        self.ring = _StreamState(self.device, flats, layout, num_slots=self.num_slots, ring=ring)
        self.ring.lookahead = self.lookahead
        self.layout = layout
        self.captures += 1
        if self.device.type == "cuda":
            torch.cuda.empty_cache()

    def bindings_intact(self):
        for entries in self.entries:
            for p, _name, _d, rest, _tt in entries:
                if p.data_ptr() != rest.data_ptr():
                    return False
        return bool(self.entries)

    # ------------------------------------------------------------------------------------------------ resident blocks
    def build_resident(self):
        """Self-managed resident blocks (the reference's RESIDENT_MODE_SELF, streaming/state.py:80-95): the GGUF
        weights of the blocks that do not stream are dequantised once, in one batched launch per (type, intermediate
        precision), into GPU tensors of the compute dtype -- the bits their layers' per-use dequantisation gives --
        and bound for each whole forward instead of being dequantised at every use. Weights the streamed path would
        keep packed (LoRA patches, other intermediate precisions) stay packed here too. Their VRAM stays occupied
        for the whole generation."""
        self.unbind_resident()
        self.res_entries = []
        if not self.self_resident:
            return
        from ..enhancers import gguf_dequant as _gd
        stream = set(self.stream_idx)
        groups = {}
        for i, blk in enumerate(_blocks(self.dit)):
            if i in stream:
                continue
            for name, p in blk.named_parameters():
                sp, d = param_spec(name, p, _param_owner(blk, name), self.compute_dtype)
                if d:
                    groups.setdefault((sp.qtype, sp.mid), []).append((p, sp))
        for (qt, mid), items in groups.items():
            packed = [(_raw(p).reshape(-1).to(self.device), sp.shape) for p, sp in items]
            outs = _gd.dequantize_many(packed, qt, _MID_DTYPE[mid], self.compute_dtype)
            for (p, _sp), w in zip(items, outs):
                self.res_entries.append((p, p.data, w, getattr(p, "tensor_type", None)))

    def resident_intact(self):
        return all(p.data_ptr() == packed.data_ptr() for p, packed, _w, _tt in self.res_entries)

    def bind_resident(self):
        for p, _packed, w, _tt in self.res_entries:
            p.data = w
            p.tensor_type = None  # a plain tensor for the whole forward: used as it is
        self.res_bound = bool(self.res_entries)

    def unbind_resident(self):
        if not self.res_bound:
            return
        for p, packed, _w, tt in self.res_entries:
            p.data = packed
            p.tensor_type = tt
        self.res_bound = False

    def _plan_tiers(self, num_stream, block_bytes):
        """With tiering "Auto": how many streamed blocks go to the SSD (core/tiers/plan.plan_tiers), their positions
        (interleaved) and the cache file that holds them."""
        self.disk_blocks, self.tier_plan = [], None
        if not self.tiering_auto:
            return
        plan = plan_tiers(num_stream, block_bytes, ram_budget_bytes=self.ram_budget_bytes, disk_dir=default_cache_dir())
        self.tier_plan = plan
        if plan["disk_error"] is not None:
            log_warn(f"DiT Layer Streaming [tiers]: no SSD tier ({plan['disk_error']}); every block in RAM.")
        if plan["disk_blocks"] <= 0:
            return
        self.disk_blocks = ssd_positions(num_stream, plan["disk_blocks"])
        self.store = DiskBlockStore(new_cache_path(plan["disk_dir"]), block_bytes, len(self.disk_blocks))
        log_info(f"DiT Layer Streaming [tiers]: {plan['ram_blocks']} streamed blocks in pinned RAM, "
                 f"{plan['disk_blocks']} on the SSD ({self.store.path}), ring depth {plan['ring_depth']}, "
                 f"{plan['disk_threads']} reader thread(s), drive {plan['disk_read_gbps']} GB/s.")

    def drop_ring(self):
        if self.ring is not None:
            self.ring.close()
        self.ring = None
        self.entries = []
        release_all(self.holders)
        self.holders = []
        if self.store is not None:
            self.store.delete()
            self.store = None

    # ------------------------------------------------------------------------------------------------ hooks
    def install_hooks(self):
        blocks = _blocks(self.dit)
        for k, i in enumerate(self.stream_idx):
            self.handles.append(blocks[i].register_forward_pre_hook(self._make_pre(k)))
            self.handles.append(blocks[i].register_forward_hook(self._make_post(k)))
        self.handles.append(self.dit.register_forward_pre_hook(self._dit_pre))
        self.handles.append(self.dit.register_forward_hook(self._dit_post))

    def _make_pre(self, k):
        def pre(module, args):
            if self.ring is None:
                return
            views = self.ring.acquire(k)
            self.bound.add(k)
            for p, name, d, _rest, _tt in self.entries[k]:
                p.data = views[name]
                if d:
                    p.tensor_type = None  # a plain tensor while the block runs: used as it is
        return pre

    def _restore(self, k):
        for p, _name, d, rest, tt in self.entries[k]:
            p.data = rest
            if d:
                p.tensor_type = tt
        self.bound.discard(k)

    def _make_post(self, k):
        def post(module, args, output):
            if self.ring is None:
                return
            self.ring.release(k)
            self._restore(k)
        return post

    def _dit_pre(self, module, args):
        if getattr(self.dit, _STATE_ATTR, None) is not self:
            return
        if self.bound:
            # the last forward stopped inside a streamed block (an exception skipped its post hook): its parameters
            # go back to the host bytes (the reference restores the rest binding in a finally), and the GPU work it
            # queued finishes before any slot is written again
            for k in list(self.bound):
                self._restore(k)
            torch.cuda.synchronize(self.device)
        self.unbind_resident()  # (still bound when the last forward raised)
        if self.ring is None or not self.bindings_intact():
            log_info("DiT Layer Streaming: the streamed weights were rebound; capturing them again.")
            self.capture()
            self.build_resident()
        elif not self.resident_intact():
            self.build_resident()
        self.bind_resident()
        self.ring.begin_forward()
        if self.lookahead:
            self.ring.prefetch_first_slots()

    def _dit_post(self, module, args, output):
        self.unbind_resident()
        if self.ring is not None:
            self.ring.end_forward()

    # ------------------------------------------------------------------------------------------------ teardown
    def teardown(self):
        """Hooks off; the streamed parameters back on the GPU as plain copies of their host bytes."""
        for h in self.handles:
            h.remove()
        self.handles = []
        self.unbind_resident()
        self.res_entries = []
        for entries in self.entries:
            for p, _name, d, rest, tt in entries:
                p.data = rest.to(self.device)
                if d:
                    p.tensor_type = tt
        self.drop_ring()
        if getattr(self.dit, _STATE_ATTR, None) is self:
            setattr(self.dit, _STATE_ATTR, None)


_WRAPPER_KEY = "weightferry_b200_streaming"


def _patcher_extension(patcher):
    """ComfyUI's patcher_extension module when ``patcher`` is a ComfyUI ModelPatcher that takes callbacks (the
    capture then waits for ComfyUI's model load), else None (the capture happens now)."""
    if not (hasattr(patcher, "add_callback") and isinstance(getattr(patcher, "model_options", None), dict)):
        return None
    try:
        import comfy.patcher_extension as ext
    except ImportError:
        return None
    return ext


def _hook_patcher(patcher, dit, st, ext):
    """The reference's ModelPatcher integration (streaming/dit_node.py:298-490): the capture runs in ComfyUI's ON_LOAD
    callback, when the model's weights are on the GPU with their LoRA / quantisation patches applied; ON_DETACH
    tears it down; a DIFFUSION_MODEL wrapper captures lazily when ComfyUI ran a forward without an ON_LOAD for this
    configuration (a switch back to a clone whose weights were already in place skips the load). The per-forward
    bracket itself is the diffusion model's forward hooks (install_hooks)."""
    def on_load(mp, device_to=None, lowvram_model_memory=0, force_patch_weights=False, full_load=False):
        target = torch.device(device_to if device_to is not None else getattr(mp, "load_device", st.device))
        if target.type != "cuda":
            return
        st.start()

    def on_detach(mp, unpatch_all=True, *args, **kwargs):
        if getattr(dit, _STATE_ATTR, None) is st:
            teardown(dit)

    # the wrapper lives in the patcher's model_options: a weak reference avoids a patcher -> options -> patcher cycle
    patcher_ref = weakref.ref(patcher)

    def wrapper(executor, *args, **kwargs):
        if getattr(dit, _STATE_ATTR, None) is not st:
            mp = patcher_ref()
            if mp is not None:
                on_load(mp, getattr(mp, "load_device", None))
                if getattr(dit, _STATE_ATTR, None) is st:
                    log_info("DiT Layer Streaming: ON_LOAD was skipped by ComfyUI; captured at the forward.")
        return executor(*args, **kwargs)

    patcher.add_callback(ext.CallbacksMP.ON_LOAD, on_load)
    patcher.add_callback(ext.CallbacksMP.ON_DETACH, on_detach)
    wrappers = patcher.model_options.setdefault("transformer_options", {}).setdefault("wrappers", {})
    wrappers.setdefault(ext.WrappersMP.DIFFUSION_MODEL, {}).pop(_WRAPPER_KEY, None)
    ext.add_wrapper_with_key(ext.WrappersMP.DIFFUSION_MODEL, _WRAPPER_KEY, wrapper, patcher.model_options,
                             is_model_options=True)


def teardown(dit):
    """Undo apply_streaming on a diffusion model (the reference's streaming/teardown.py for one model)."""
    st = getattr(dit, _STATE_ATTR, None)
    if st is not None:
        st.teardown()


class WeightFerryDiT:
    """⚡ DiT Layer Streaming (low VRAM)."""

    @classmethod
    def INPUT_TYPES(cls):
        return {
            "required": {
                "model": ("MODEL",),
                "enabled": ("BOOLEAN", {"default": True}),
                "pin_memory": ("BOOLEAN", {"default": True}),
                "buffer_mode": ([BUFFER_DOUBLE, BUFFER_SINGLE], {"default": BUFFER_DOUBLE}),
                "resident_blocks": ("INT", {"default": 8, "min": 0, "max": 256, "step": 1}),
                "sage_attention": ("BOOLEAN", {"default": False}),
                "host_format": ([HOST_FORMAT_BAKED, HOST_FORMAT_STORAGE], {"default": HOST_FORMAT_BAKED}),
                "tiering": ([TIERING_RAM, TIERING_AUTO], {"default": TIERING_RAM}),
                "ram_budget_gb": ("FLOAT", {"default": 0.0, "min": 0.0, "max": 512.0, "step": 0.5}),
                "resident_mode": ([RESIDENT_MODE_COMFY, RESIDENT_MODE_SELF], {"default": RESIDENT_MODE_COMFY}),
                "sage_pv_fp16": ("BOOLEAN", {"default": False}),
                "auto_config": ("BOOLEAN", {"default": True}),
                "prefetch_slots": ("INT", {"default": 3, "min": 2, "max": 6, "step": 1}),
                "vram_budget_gb": ("FLOAT", {"default": 0.0, "min": 0.0, "max": 512.0, "step": 0.5}),
            }
        }

    RETURN_TYPES = ("MODEL",)
    RETURN_NAMES = ("model",)
    FUNCTION = "apply_streaming"
    CATEGORY = "WeightFerry/streaming"
    TITLE = "⚡ DiT Layer Streaming (low VRAM)"

    def apply_streaming(self, model, enabled: bool = True, pin_memory: bool = True, buffer_mode: str = BUFFER_DOUBLE,
                        resident_blocks: int = 8, sage_attention: bool = False, host_format: str = HOST_FORMAT_BAKED,
                        prefetch_slots: int = 3, resident_mode: str = RESIDENT_MODE_COMFY, tiering: str = TIERING_RAM,
                        ram_budget_gb: float = 0.0, auto_config: bool = False, sage_pv_fp16: bool = False,
                        vram_budget_gb: float = 0.0):
        if not enabled:
            log_info("DiT Layer Streaming: Disabled, passing original model.")
            return (model,)
        unused = [n for n, on in (("sage_attention", sage_attention), ("sage_pv_fp16", sage_pv_fp16),
                                  ("host_format=storage", host_format == HOST_FORMAT_STORAGE)) if on]
        if unused:
            log_info(f"DiT Layer Streaming: not used by this build: {', '.join(unused)}.")

        if isinstance(model, torch.nn.Module) and not hasattr(model, "model"):
            patcher, dit = model, model
        else:
            patcher = model.clone() if hasattr(model, "clone") else model
            dit = getattr(getattr(patcher, "model", None), "diffusion_model", None)
        if dit is None:
            log_warn("DiT Layer Streaming: Model has no 'diffusion_model', skipping.")
            return (model,)
        device = getattr(patcher, "load_device", None)
        if device is None:
            first = next(dit.parameters(), None)
            device = first.device if first is not None else torch.device("cpu")
        device = torch.device(device)
        if device.type != "cuda":
            log_warn("DiT Layer Streaming: Device is not CUDA, skipping.")
            return (patcher,)
        blocks = _blocks(dit)
        if len(blocks) == 0:
            log_warn(f"DiT Layer Streaming: no transformer block list ({', '.join(_BLOCK_LIST_ATTRS)}) on "
                     f"{type(dit).__name__}, skipping.")
            return (patcher,)
        num_blocks = len(blocks)
        is_double = "Double Buffer" in buffer_mode
        compute_dtype = getattr(getattr(patcher, "model", None), "manual_cast_dtype", None) or torch.bfloat16

        if auto_config or _env.get("WEIGHTFERRY_AUTO") == "1":
            auto = self._auto(dit, blocks, device, prefetch_slots, is_double, compute_dtype,
                              vram_budget_bytes(vram_budget_gb))
            if auto is None:
                log_info("DiT Layer Streaming [auto]: the whole model fits in VRAM; streaming not used.")
                return (patcher,)
            resident_blocks = auto
        resident_k = max(1, min(num_blocks, int(resident_blocks)))
        stream_idx = list(range(resident_k, num_blocks))
        if not stream_idx:
            log_info("DiT Layer Streaming: All blocks resident, no streaming offload registered.")
            return (patcher,)

        teardown(dit)  # an earlier configuration of this model (the reference's _teardown(dit, "re-load"))
        num_slots = max(2, int(prefetch_slots)) if is_double else 2
        env_tiering = _env.get("WEIGHTFERRY_TIERING")
        tiering_auto = (env_tiering == "auto") if env_tiering else tiering == TIERING_AUTO
        env_budget = _env.get("WEIGHTFERRY_RAM_BUDGET_GB")
        ram_budget_bytes = int(float(env_budget if env_budget else ram_budget_gb) * 1024 ** 3) or None
        st = _NodeState(object(), dit, stream_idx, device, pin_memory, num_slots, is_double, compute_dtype,
                        tiering_auto=tiering_auto, ram_budget_bytes=ram_budget_bytes,
                        self_resident=resident_mode == RESIDENT_MODE_SELF)
        ext = _patcher_extension(patcher)
        if ext is not None:
            _hook_patcher(patcher, dit, st, ext)
            log_info(f"DiT Layer Streaming: {resident_k}/{num_blocks} resident, {len(stream_idx)} streaming blocks; "
                     "hooked to the ModelPatcher, the blocks are captured when ComfyUI loads the model.")
            return (patcher,)
        st.start()
        return (patcher,)

    @staticmethod
    def _auto(dit, blocks, device, prefetch_slots, is_double, compute_dtype, budget=None):
        block_ids = {id(p) for blk in blocks for p in blk.parameters()}
        block_bytes = max(sum(_nbytes(_raw(p)) for p in blk.parameters()) for blk in blocks)
        nonblock = sum(_nbytes(_raw(p)) for p in dit.parameters() if id(p) not in block_ids)
        specs, _ = block_specs_of(blocks[-1], compute_dtype)
        lay = BlockLayout(specs, compute_dtype=compute_dtype)
        free, _total = torch.cuda.mem_get_info(device)
        stats = torch.cuda.memory_stats(device)
        cached = stats.get("reserved_bytes.all.current", 0) - stats.get("active_bytes.all.current", 0)
        in_use = stats.get("active_bytes.all.current", 0)
        headroom = int(_env.get("WEIGHTFERRY_AUTO_HEADROOM_MB")) * 1024 ** 2
        usable = budget_usable(free + cached, in_use, budget)
        if budget is not None:
            log_info(f"DiT Layer Streaming [auto]: VRAM budget {budget / 1024 ** 3:.2f} GB -> "
                     f"{usable / 1024 ** 2:.0f} MB usable (free + cached {(free + cached) / 1024 ** 2:.0f} MB).")
        return auto_resident(len(blocks), block_bytes, lay.flat_bytes + lay.weight_bytes, nonblock, usable,
                             headroom, prefetch_slots, is_double)


NODE_CLASS_MAPPINGS = {"WeightFerryDiT": WeightFerryDiT}
NODE_DISPLAY_NAME_MAPPINGS = {"WeightFerryDiT": WeightFerryDiT.TITLE}
