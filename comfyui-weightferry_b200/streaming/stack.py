"""A streamed DiT block stack: every block's GGUF weights in pinned host RAM, streamed through the GPU slot ring and
dequantised on arrival (streaming/state.py), the blocks run by cosmos_block.block_forward, single-GPU or
tensor-parallel. This is the ⚡ DiT Layer Streaming node's forward (streaming/dit_node.py:414-455 and the block hooks
of load_steps.py:451-522 of the reference) for a Cosmos-Predict2 model whose blocks are all streamed.

``resident=True`` keeps every block's dequantised weights on the GPU instead (the no-streaming configuration the
reference's test compares against); both modes run the same kernels on the same bits, so their outputs are equal.

Over several GPUs (one process each) the stack runs in one of two ways:

* ``parallel="sp"`` (the default): each rank keeps in pinned host memory only its equal byte range of every block's
  packed bytes and copies that range into its slot; an all-gather over NVLink on the transfer stream completes the
  block in every rank's slot before it is dequantised (each byte crosses PCIe once, on one rank). Every rank then
  runs whole blocks on its own token rows (cosmos_block.block_forward_sp): the ranks of one sample gather their
  keys and values for the self-attention, and nothing else of the activations moves. The weight gather depends on
  no activation, so it overlaps the compute of the blocks before;
* ``parallel="tp"``: tensor parallel (column / row split of the projections, NCCL all-gather / reduce-scatter of the
  token rows around every sub-layer, cosmos_block.block_forward); each rank streams its shards of the weights."""

import torch

from .. import _ext
from ..core.tiers.pinned import PinnedHost, release_all
from . import cosmos_block as cb
from .state import BlockLayout, _StreamState


class StreamedStack:
    def __init__(self, cfg, n_blocks, device, tp=None, qtype=cb.Q8_0, seed=20261201, num_slots=None, profile=None,
                 resident=False, parallel="tp", sp=None):
        self.cfg = cfg
        self.n_blocks = n_blocks
        self.device = torch.device(device)
        self.parallel = parallel
        self.tp = tp or cb.TP()
        self.sp = sp
        gather = None
        if parallel == "sp":
            if self.sp is None:
                raise ValueError("parallel='sp' needs the SP ranks (cosmos_block.SP)")
            world, rank = self.sp.world, self.sp.rank
            self.specs = cb.block_specs(cfg, 1, 0, qtype)          # whole blocks on every rank
            self.layout = BlockLayout(self.specs, pad_to=world)
            shard = self.layout.flat_bytes // world
            lo, hi = rank * shard, (rank + 1) * shard                # this rank's byte range of each block
            gather = (self.sp.world_group, rank, world) if world > 1 else None
            gen_world, gen_rank = 1, 0
        elif parallel == "tp":
            self.specs = cb.block_specs(cfg, self.tp.world, self.tp.rank, qtype)
            self.layout = BlockLayout(self.specs)
            lo, hi = 0, self.layout.flat_bytes
            gen_world, gen_rank = self.tp.world, self.tp.rank
        else:
            raise ValueError(f"parallel must be 'sp' or 'tp', not {parallel!r}")
        self.holders = []
        self.host_flats = []
        full = torch.empty(self.layout.flat_bytes, dtype=torch.uint8) if lo or hi != self.layout.flat_bytes else None
        for b in range(n_blocks):
            params = cb.make_block_params(cfg, self.specs, gen_world, gen_rank, seed + b, self.device)
            holder = PinnedHost(hi - lo)
            flat = holder.tensor if full is None else full
            if full is not None:
                full.zero_()
            for sp_, off in zip(self.layout.specs, self.layout.offsets):
                flat[off:off + sp_.packed_bytes].copy_(params[sp_.name].reshape(-1).view(torch.uint8))
            if full is not None:
                holder.tensor.copy_(full[lo:hi])
            self.holders.append(holder)
            self.host_flats.append(holder.tensor)
        self.resident = resident
        self.state = None
        self.resident_weights = None
        if resident:
            if gather is not None:
                raise ValueError("resident blocks are not gathered: use parallel='sp' streamed, or one rank")
            self.resident_weights = [self._dequant_resident(f) for f in self.host_flats]
        else:
            self.state = _StreamState(self.device, self.host_flats, self.layout, num_slots=num_slots,
                                      profile=profile, gather=gather)

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
        """Bytes this rank copies host-to-device per block."""
        return self.host_flats[0].numel() if self.host_flats else self.layout.flat_bytes

    def _block(self, x_rows, emb, ctx, rope, W, batch, tokens, lora_term):
        if self.parallel == "sp":
            return cb.block_forward_sp(x_rows, emb, ctx, rope, W, self.cfg, self.sp, batch, tokens, lora_term)
        return cb.block_forward(x_rows, emb, ctx, rope, W, self.cfg, self.tp, batch, tokens, lora_term)

    def forward(self, x_rows, emb, ctx, rope, batch, tokens, lora_term=None):
        """All blocks on this rank's token rows; returns the new rows."""
        if self.resident:
            for W in self.resident_weights:
                x_rows = self._block(x_rows, emb, ctx, rope, W, batch, tokens, lora_term)
            return x_rows
        st = self.state
        st.begin_forward()
        st.prefetch_first_slots()
        for s in range(self.n_blocks):
            W = st.acquire(s)
            x_rows = self._block(x_rows, emb, ctx, rope, W, batch, tokens, lora_term)
            st.release(s)
        st.end_forward()
        return x_rows

    def close(self):
        if self.state is not None:
            self.state.close()
        release_all(self.holders)
        self.holders = []
        self.host_flats = []
