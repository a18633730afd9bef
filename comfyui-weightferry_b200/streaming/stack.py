"""A streamed DiT block stack: every block's GGUF weights in pinned host RAM, streamed through the GPU slot ring and
dequantised on arrival (streaming/state.py), the blocks run by cosmos_block.block_forward, single-GPU or
tensor-parallel. This is the ⚡ DiT Layer Streaming node's forward (streaming/dit_node.py:414-455 and the block hooks
of load_steps.py:451-522 of the reference) for a Cosmos-Predict2 model whose blocks are all streamed.

``resident=True`` keeps every block's dequantised weights on the GPU instead (the no-streaming configuration the
reference's test compares against); both modes run the same kernels on the same bits, so their outputs are equal."""

import torch

from .. import _ext
from ..core.tiers.pinned import PinnedHost, release_all
from . import cosmos_block as cb
from .state import BlockLayout, _StreamState


class StreamedStack:
    def __init__(self, cfg, n_blocks, device, tp=None, qtype=cb.Q8_0, seed=20261201, num_slots=None, profile=None,
                 resident=False):
        self.cfg = cfg
        self.n_blocks = n_blocks
        self.device = torch.device(device)
        self.tp = tp or cb.TP()
        self.specs = cb.block_specs(cfg, self.tp.world, self.tp.rank, qtype)
        self.layout = BlockLayout(self.specs)
        self.holders = []
        self.host_flats = []
        for b in range(n_blocks):
            params = cb.make_block_params(cfg, self.specs, self.tp.world, self.tp.rank, seed + b, self.device)
            holder = PinnedHost(self.layout.flat_bytes)
            flat = holder.tensor
            for sp, off in zip(self.layout.specs, self.layout.offsets):
                flat[off:off + sp.packed_bytes].copy_(params[sp.name].reshape(-1).view(torch.uint8))
            self.holders.append(holder)
            self.host_flats.append(flat)
        self.resident = resident
        self.state = None
        self.resident_weights = None
        if resident:
            self.resident_weights = [self._dequant_resident(f) for f in self.host_flats]
        else:
            self.state = _StreamState(self.device, self.host_flats, self.layout, num_slots=num_slots,
                                      profile=profile)

    def _dequant_resident(self, host_flat):
        """A block's weights dequantised once and kept (the non-streamed reference configuration)."""
        lay = self.layout
        flat = host_flat.to(self.device)
        wbuf = torch.empty(max(lay.weight_bytes, 1), dtype=torch.uint8, device=self.device)
        out = {}
        groups = {}
        qi = 0
        for sp, off in zip(lay.specs, lay.offsets):
            raw = flat[off:off + sp.packed_bytes]
            if sp.qtype is None:
                out[sp.name] = raw.view(sp.dtype).view(sp.shape)
                continue
            o = lay.w_offsets[qi]
            qi += 1
            w = wbuf[o:o + sp.numel * 2].view(torch.bfloat16).view(sp.shape)
            groups.setdefault(sp.qtype, []).append((raw.data_ptr(), w.data_ptr(), sp.numel))
            out[sp.name] = w
        stream = _ext.stream_of(self.device)
        for qt, items in groups.items():
            arr = (_ext.DequantTask * len(items))()
            for i, (s, d, n) in enumerate(items):
                arr[i].src, arr[i].dst, arr[i].n_values = s, d, n
            _ext.check(_ext.lib().wf_dequant_gguf_batch(arr, len(items), qt, 0, 1, stream), "dequant")
        out["_keep"] = (flat, wbuf)
        return out

    @property
    def bytes_per_block(self):
        return self.layout.flat_bytes

    def forward(self, x_rows, emb, ctx, rope, batch, tokens, lora_term=None):
        """All blocks on this rank's token rows; returns the new rows."""
        if self.resident:
            for W in self.resident_weights:
                x_rows = cb.block_forward(x_rows, emb, ctx, rope, W, self.cfg, self.tp, batch, tokens, lora_term)
            return x_rows
        st = self.state
        st.begin_forward()
        st.prefetch_first_slots()
        for s in range(self.n_blocks):
            W = st.acquire(s)
            x_rows = cb.block_forward(x_rows, emb, ctx, rope, W, self.cfg, self.tp, batch, tokens, lora_term)
            st.release(s)
        st.end_forward()
        return x_rows

    def close(self):
        if self.state is not None:
            self.state.close()
        release_all(self.holders)
        self.holders = []
        self.host_flats = []
