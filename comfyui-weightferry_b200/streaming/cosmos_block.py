"""The Cosmos-Predict2 DiT block on B200, single-GPU or tensor-parallel, on streamed (dequantised) weights.

The block is ComfyUI's comfy/ldm/cosmos/predict2.py Block as the reference's fused forward runs it
(enhancers/fused_block.py:652-703): adaLN shift / scale / gate from the timestep embedding (+ the AdaLN-LoRA term),
then three sub-layers, each ``x = x + gate * sublayer(LayerNorm(x) * (1 + scale) + shift)``:

* self-attention: q / k / v projections, per-head RMSNorm-128 + 3D RoPE on q and k (kernel B), attention
  (PyTorch SDPA), output projection;
* cross-attention: q projection + RMSNorm-128 of q, k / v from the text context + RMSNorm-128 of k, attention,
  output projection;
* MLP: layer1, GELU, layer2.

LayerNorm + modulate is kernel A (one pass), the projections are cuBLAS bf16 GEMMs on the weights the streaming
state dequantised on arrival.

Tensor parallel over N GPUs (one process per GPU, NCCL over NVLink): the residual stream is sharded by token rows
(each rank holds rows [r * R, (r + 1) * R) of the B * L rows); before each sub-layer the modulated rows are
all-gathered, q / k / v / layer1 (and the cross-attention's q, k, v) are column-parallel (each rank owns
heads / N heads and 20480 / N MLP channels), the output projections are row-parallel and their partial sums are
reduce-scattered back to the token shards. Each rank streams only its shards of the block's weights (the adaLN
weights, 4 % of the bytes, are replicated). Parameter names follow ComfyUI's module paths.
"""

import torch
import torch.nn.functional as F

from ..core import env as _env

from ..enhancers import fused_block as _fb
from ..enhancers import sage_fused as _sf
from .state import ParamSpec

Q8_0 = 8


class CosmosConfig:
    def __init__(self, hidden=5120, heads=40, head_dim=128, mlp=20480, ctx_dim=1024, lora=256, eps=1e-6):
        self.hidden, self.heads, self.head_dim, self.mlp = hidden, heads, head_dim, mlp
        self.ctx_dim, self.lora, self.eps = ctx_dim, lora, eps


COSMOS_14B = CosmosConfig()
COSMOS_2B = CosmosConfig(hidden=2048, heads=16, mlp=8192)


def block_specs(cfg, world=1, rank=0, qtype=Q8_0):
    """ParamSpecs of this rank's share of one block: column-parallel projections split their output rows,
    row-parallel ones their input columns, the adaLN output layers (3 D outputs) their output rows too (each rank
    computes its slice of shift / scale / gate and the (B, 3 D) result is gathered: a few KB instead of streaming the
    whole layer to every rank); the adaLN input layers and the norm weights are replicated."""
    if cfg.heads % world or cfg.mlp % world or cfg.hidden % world:
        raise ValueError(f"{world} ranks do not divide heads {cfg.heads} / mlp {cfg.mlp}")
    D, Dw, Mw = cfg.hidden, cfg.hidden // world, cfg.mlp // world
    s = []
    for name in ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight"):
        s.append(ParamSpec(name, (Dw, D), qtype=qtype))
    s.append(ParamSpec("self_attn.output_proj.weight", (D, Dw), qtype=qtype))
    s.append(ParamSpec("cross_attn.q_proj.weight", (Dw, D), qtype=qtype))
    s.append(ParamSpec("cross_attn.k_proj.weight", (Dw, cfg.ctx_dim), qtype=qtype))
    s.append(ParamSpec("cross_attn.v_proj.weight", (Dw, cfg.ctx_dim), qtype=qtype))
    s.append(ParamSpec("cross_attn.output_proj.weight", (D, Dw), qtype=qtype))
    s.append(ParamSpec("mlp.layer1.weight", (Mw, D), qtype=qtype))
    s.append(ParamSpec("mlp.layer2.weight", (D, Mw), qtype=qtype))
    for sub in ("self_attn", "cross_attn", "mlp"):
        s.append(ParamSpec(f"adaln_modulation_{sub}.1.weight", (cfg.lora, D), qtype=qtype))
        s.append(ParamSpec(f"adaln_modulation_{sub}.2.weight", (3 * D // world, cfg.lora), qtype=qtype))
    for sub in ("self_attn", "cross_attn"):
        s.append(ParamSpec(f"{sub}.q_norm.weight", (cfg.head_dim,), dtype=torch.bfloat16))
        s.append(ParamSpec(f"{sub}.k_norm.weight", (cfg.head_dim,), dtype=torch.bfloat16))
    return s


def shard_of(name, world, rank):
    """How parameter `name` is split across ranks: ("col", lo, hi) on rows, ("row", lo, hi) on columns (fractions
    of the full dimension as rank / world), or None (replicated)."""
    if world == 1:
        return None
    if name.endswith(("q_proj.weight", "k_proj.weight", "v_proj.weight", "mlp.layer1.weight", ".2.weight")):
        return ("col", rank, world)
    if name.endswith(("output_proj.weight", "mlp.layer2.weight")):
        return ("row", rank, world)
    return None


def full_shape(spec, world):
    kind = shard_of(spec.name, world, 0)
    if kind is None:
        return spec.shape
    if kind[0] == "col":
        return (spec.shape[0] * world, spec.shape[1])
    return (spec.shape[0], spec.shape[1] * world)


def q8_0_pack(q_int8, d_f16):
    """Q8_0 blocks from int8 quants [rows, cols] and float16 scales [rows, cols / 32]: (rows, cols / 32 * 34) bytes."""
    rows, cols = q_int8.shape
    nb = cols // 32
    q = q_int8.view(torch.uint8).reshape(rows, nb, 32)
    d = d_f16.contiguous().view(torch.uint8).reshape(rows, nb, 2)
    return torch.cat([d, q], dim=2).reshape(rows, nb * 34)


def q8_0_shard(packed_full, shape, kind):
    """The packed bytes of one rank's shard of a Q8_0 weight [rows, cols] (kind from shard_of)."""
    rows, cols = shape
    nb = cols // 32
    p = packed_full.view(rows, nb, 34)
    if kind is None:
        return p.reshape(-1)
    _, r, w = kind
    if kind[0] == "col":
        lo, hi = rows * r // w, rows * (r + 1) // w
        return p[lo:hi].reshape(-1)
    lo, hi = nb * r // w, nb * (r + 1) // w
    return p[:, lo:hi].contiguous().reshape(-1)


def make_block_params(cfg, specs, world, rank, seed, device, d_scale=0.002):
    """Seeded synthetic weights of one block as BASELINE configs[4] describes them (Q8_0 as configs[0]: quants
    uniform in [-127, 127], d = fp16(|N(0,1)| * 0.002); the adaLN weights scaled down so the gates stay small;
    norm weights 1 + N(0, 0.02)), generated in full on `device` and cut to this rank's shard. Returns name -> CPU
    tensor (packed uint8 for quantised parameters)."""
    out = {}
    g = torch.Generator(device=device)
    for i, sp in enumerate(specs):
        g.manual_seed(seed * 1000 + i)
        if sp.qtype is None:
            w = (1 + torch.randn(sp.shape, device=device, generator=g) * 0.02).to(sp.dtype)
            out[sp.name] = w.cpu()
            continue
        rows, cols = full_shape(sp, world)
        q = torch.randint(-127, 128, (rows, cols), dtype=torch.int16, device=device, generator=g).to(torch.int8)
        scale = d_scale * (0.05 if "adaln" in sp.name else 1.0)
        d = (torch.randn((rows, cols // 32), device=device, generator=g).abs() * scale).half()
        packed = q8_0_pack(q, d)
        out[sp.name] = q8_0_shard(packed, (rows, cols), shard_of(sp.name, world, rank)).cpu()
    return out


# ---------------------------------------------------------------------------------------------- RoPE
def rope3d_table(T, H, W, head_dim=128, theta=10000.0, h_extra=4.0, w_extra=4.0, t_extra=1.0, device=None):
    """Cosmos-Predict2's 3D RoPE rotations as a (1, T*H*W, 1, head_dim/2, 2, 2) float32 table (VideoRopePosition3DEmb's
    layout as the reference's rope_scale.py:29-60 restates it): head dim split into h / w / t channel groups
    (128 -> 42 / 42 / 44), NTK factors from the extrapolation ratios, tokens in (t h w) order, t then h then w."""
    dim_h = head_dim // 6 * 2
    dim_t = head_dim - 2 * dim_h
    rng_hw = torch.arange(0, dim_h, 2, dtype=torch.float64) / dim_h
    rng_t = torch.arange(0, dim_t, 2, dtype=torch.float64) / dim_t
    h_ntk = h_extra ** (dim_h / (dim_h - 2))
    w_ntk = w_extra ** (dim_h / (dim_h - 2))
    t_ntk = t_extra ** (dim_t / (dim_t - 2))
    hf = 1.0 / ((theta * h_ntk) ** rng_hw)
    wf = 1.0 / ((theta * w_ntk) ** rng_hw)
    tf = 1.0 / ((theta * t_ntk) ** rng_t)
    ht = torch.outer(torch.arange(H, dtype=torch.float64), hf)
    wt = torch.outer(torch.arange(W, dtype=torch.float64), wf)
    tt = torch.outer(torch.arange(T, dtype=torch.float64), tf)

    def rot(e):
        return torch.stack([torch.cos(e), -torch.sin(e), torch.sin(e), torch.cos(e)], dim=-1)
    ht, wt, tt = rot(ht), rot(wt), rot(tt)
    nt, nh = tt.shape[1], ht.shape[1]
    em = torch.cat([tt[:, None, None].expand(T, H, W, nt, 4), ht[None, :, None].expand(T, H, W, nh, 4),
                    wt[None, None, :].expand(T, H, W, nh, 4)], dim=-2)
    return em.reshape(1, T * H * W, 1, head_dim // 2, 2, 2).float().contiguous().to(device)


# ---------------------------------------------------------------------------------------------- TP plumbing
class TP:
    """The tensor-parallel group of the stack: the initialised torch.distributed group (NCCL over NVLink for CUDA
    tensors), or a single rank when there is none / ``single=True``."""

    def __init__(self, group=None, single=False):
        import torch.distributed as dist
        on = dist.is_available() and dist.is_initialized() and not single
        self.dist = dist if on else None
        self.group = group
        self.world = self.dist.get_world_size(group) if self.dist else 1
        self.rank = self.dist.get_rank(group) if self.dist else 0
        self.gloo = bool(self.dist) and self.dist.get_backend(group) == "gloo"

    def all_gather_rows(self, x_local):
        """(R, ...) rows of every rank -> (world * R, ...) in rank order."""
        if self.world == 1:
            return x_local
        x_local = x_local.contiguous()
        if self.gloo:  # gloo has no all_gather_into_tensor
            parts = [torch.empty_like(x_local) for _ in range(self.world)]
            self.dist.all_gather(parts, x_local, group=self.group)
            return torch.cat(parts, dim=0)
        out = torch.empty((x_local.shape[0] * self.world,) + tuple(x_local.shape[1:]), dtype=x_local.dtype,
                          device=x_local.device)
        self.dist.all_gather_into_tensor(out, x_local, group=self.group)
        return out

    # -------------------------------------------------------------------- overlapped row chunks (NCCL's own stream)
    def chunks(self, n):
        """Row chunks of the overlapped sub-layers: WEIGHTFERRY_TP_CHUNKS when it divides n, else 1. Off (1) by
        default: at 2 GPUs the overlap made a block slower (3.61 against 3.47 ms), NCCL's ring kernels taking SMs from
        the concurrent GEMMs, and the chunked GEMMs being smaller."""
        c = int(_env.get("WEIGHTFERRY_TP_CHUNKS"))
        return c if self.world > 1 and c > 1 and n % c == 0 else 1

    def _gather_async(self, x_local):
        """(buffer of every rank's rows in rank order, work or None); NCCL runs it on its own stream."""
        x_local = x_local.contiguous()
        if self.gloo:
            return self.all_gather_rows(x_local), None
        out = torch.empty((x_local.shape[0] * self.world,) + tuple(x_local.shape[1:]), dtype=x_local.dtype,
                          device=x_local.device)
        return out, self.dist.all_gather_into_tensor(out, x_local, group=self.group, async_op=True)

    def _scatter_async(self, out_rows, x_full):
        """out_rows <- this rank's rows of the sum over ranks of x_full; returns the work (None when done)."""
        if self.gloo:
            out_rows.copy_(self.reduce_scatter_rows(x_full))
            return None
        return self.dist.reduce_scatter_tensor(out_rows, x_full.contiguous(), group=self.group, async_op=True)

    def mlp_rows(self, normed_rows, w1, w2):
        """reduce_scatter_rows(layer2(gelu(layer1(all_gather_rows(normed_rows))))) in row chunks: chunk c takes rows
        [c * m, (c + 1) * m) of every rank (rank-major, so the chunked all-gather / reduce-scatter compose as the
        whole ones do); the all-gather of chunk c + 1 and the reduce-scatter of chunk c run on NCCL's stream while
        the compute stream does chunk c's and c + 1's GEMMs."""
        n = normed_rows.shape[0]
        C = self.chunks(n)
        if C == 1:
            return self.reduce_scatter_rows(F.linear(F.gelu(F.linear(self.all_gather_rows(normed_rows), w1)), w2))
        m = n // C
        out = torch.empty((n, w2.shape[0]), dtype=normed_rows.dtype, device=normed_rows.device)
        gathered = [self._gather_async(normed_rows[0:m])]
        pending = []
        for c in range(C):
            if c + 1 < C:
                gathered.append(self._gather_async(normed_rows[(c + 1) * m:(c + 2) * m]))
            buf, work = gathered[c]
            if work is not None:
                work.wait()
            y = F.linear(F.gelu(F.linear(buf, w1)), w2)
            gathered[c] = None
            pending.append((self._scatter_async(out[c * m:(c + 1) * m], y), y))
        for work, _y in pending:
            if work is not None:
                work.wait()
        return out

    def row_parallel_rows(self, a_full, w):
        """reduce_scatter_rows(linear(a_full, w)) for a_full in natural row order (world * n rows), in row chunks:
        chunk c is rows [c * m, (c + 1) * m) of every rank's share; its reduce-scatter runs on NCCL's stream while
        the next chunk's GEMM runs."""
        n = a_full.shape[0] // self.world
        C = self.chunks(n)
        if C == 1:
            return self.reduce_scatter_rows(F.linear(a_full, w))
        m = n // C
        K = a_full.shape[1]
        parts = a_full.view(self.world, C, m, K)
        out = torch.empty((n, w.shape[0]), dtype=a_full.dtype, device=a_full.device)
        pending = []
        for c in range(C):
            y = F.linear(parts[:, c], w).reshape(self.world * m, w.shape[0])
            pending.append((self._scatter_async(out[c * m:(c + 1) * m], y), y))
        for work, _y in pending:
            if work is not None:
                work.wait()
        return out

    def reduce_scatter_rows(self, x_full):
        """Sum over ranks of (world * R, ...) -> this rank's (R, ...) rows."""
        if self.world == 1:
            return x_full
        rows = x_full.shape[0] // self.world
        x_full = x_full.contiguous()
        if self.gloo:  # gloo has no reduce_scatter_tensor
            t = x_full.clone()
            self.dist.all_reduce(t, group=self.group)
            return t[self.rank * rows:(self.rank + 1) * rows].contiguous()
        out = torch.empty((rows,) + tuple(x_full.shape[1:]), dtype=x_full.dtype, device=x_full.device)
        self.dist.reduce_scatter_tensor(out, x_full, group=self.group)
        return out


def _ln_mod_rows(x_rows, scale_b, shift_b, row0, rows_per_batch, eps):
    """Kernel A over this rank's token rows [row0, row0 + n) of a (B * L, D) stream whose batch b has rows
    [b * L, (b + 1) * L): scale / shift are (B, D). The shard either holds whole batches or lies inside one."""
    n, D = x_rows.shape
    if n >= rows_per_batch:
        b0, nb = row0 // rows_per_batch, n // rows_per_batch
        sc, sh, rpg = scale_b[b0:b0 + nb], shift_b[b0:b0 + nb], rows_per_batch
    else:
        b0 = row0 // rows_per_batch
        sc, sh, rpg = scale_b[b0:b0 + 1], shift_b[b0:b0 + 1], n
    g = sc.shape[0]
    out = _fb.ln_modulate_rows(x_rows.view(g, 1, 1, rpg, D), sc.view(g, 1, 1, 1, D), sh.view(g, 1, 1, 1, D), eps)
    return out.view(n, D)


def _residual(x_rows, gate_b, o, row0, rows_per_batch):
    """x + gate * o on the shard's rows (ComfyUI's addcmul, the bits of enhancers/fused_block.gated_residual), gate_b
    (B, D) broadcast over each batch's rows."""
    n, D = x_rows.shape
    b0 = row0 // rows_per_batch
    if n >= rows_per_batch:
        nb = n // rows_per_batch
        return _fb.gated_residual(x_rows, gate_b[b0:b0 + nb].contiguous(), o.contiguous(), rows_per_batch)
    return _fb.gated_residual(x_rows, gate_b[b0:b0 + 1].contiguous(), o.contiguous(), n)


def _attention(q, k, v):
    """softmax(q k^T / sqrt(d)) v for (B, L, H, d) tensors -> (B, L, H * d)."""
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
    B, H, L, d = o.shape
    return o.transpose(1, 2).reshape(B, L, H * d)


def adaln(W, sub, emb, lora_term, tp=None):
    """(shift, scale, gate), each (B, D), of one sub-layer: Linear(Linear(SiLU(emb))) + AdaLN-LoRA term. Under
    tensor parallelism the output layer holds this rank's 3 D / world outputs: the (B, 3 D) result is gathered."""
    h = F.linear(F.silu(emb), W[f"adaln_modulation_{sub}.1.weight"])
    m = F.linear(h, W[f"adaln_modulation_{sub}.2.weight"])
    if tp is not None and tp.world > 1:
        m = tp.all_gather_rows(m.t().contiguous()).t()
    return (m + lora_term).chunk(3, dim=-1)


def block_forward(x_rows, emb, ctx, rope, W, cfg, tp, batch, tokens, lora_term=None):
    """One block on this rank's token rows x_rows (n, D) of the (batch * tokens, D) stream; emb (B, D) timestep
    embedding, ctx (B, S, ctx_dim) text context, rope (1, tokens, 1, 64, 2, 2), lora_term (B, 3D) the AdaLN-LoRA
    term (or None). W: name -> this rank's tensors. Returns the new (n, D) rows."""
    n, D = x_rows.shape
    row0 = tp.rank * n
    hd = cfg.head_dim
    Hw = cfg.heads // tp.world
    if lora_term is None:
        lora_term = emb.new_zeros(())
    eps = cfg.eps

    # --- self-attention
    shift, scale, gate = adaln(W, "self_attn", emb, lora_term, tp)
    normed = tp.all_gather_rows(_ln_mod_rows(x_rows, scale, shift, row0, tokens, eps))       # (B*L, D)
    q = F.linear(normed, W["self_attn.q_proj.weight"]).view(batch, tokens, Hw, hd)
    k = F.linear(normed, W["self_attn.k_proj.weight"]).view(batch, tokens, Hw, hd)
    v = F.linear(normed, W["self_attn.v_proj.weight"]).view(batch, tokens, Hw, hd)
    q, k = _sf.rms_rope_pair(q, k, rope, W["self_attn.q_norm.weight"], W["self_attn.k_norm.weight"], eps)
    a = _attention(q, k, v).view(batch * tokens, Hw * hd)
    o = tp.row_parallel_rows(a, W["self_attn.output_proj.weight"])                          # (n, D)
    x_rows = _residual(x_rows, gate, o, row0, tokens)

    # --- cross-attention
    shift, scale, gate = adaln(W, "cross_attn", emb, lora_term, tp)
    normed = tp.all_gather_rows(_ln_mod_rows(x_rows, scale, shift, row0, tokens, eps))
    q = F.linear(normed, W["cross_attn.q_proj.weight"]).view(batch, tokens, Hw, hd)
    q = _fb.rms_norm_128(q.contiguous(), W["cross_attn.q_norm.weight"], eps)
    S = ctx.shape[1]
    kc = F.linear(ctx, W["cross_attn.k_proj.weight"]).view(batch, S, Hw, hd)
    kc = _fb.rms_norm_128(kc.contiguous(), W["cross_attn.k_norm.weight"], eps)
    vc = F.linear(ctx, W["cross_attn.v_proj.weight"]).view(batch, S, Hw, hd)
    a = _attention(q, kc, vc).view(batch * tokens, Hw * hd)
    o = tp.row_parallel_rows(a, W["cross_attn.output_proj.weight"])
    x_rows = _residual(x_rows, gate, o, row0, tokens)

    # --- MLP
    shift, scale, gate = adaln(W, "mlp", emb, lora_term, tp)
    o = tp.mlp_rows(_ln_mod_rows(x_rows, scale, shift, row0, tokens, eps), W["mlp.layer1.weight"],
                    W["mlp.layer2.weight"])
    return _residual(x_rows, gate, o, row0, tokens)


class SP:
    """The sequence-parallel ranks of the streamed stack (streaming/stack.py, parallel="sp"): the (batch * tokens, D)
    token rows split into equal ranges in rank order, each rank running whole blocks on its range. A range either
    holds whole samples or lies inside one sample; the ranks that share a sample (``kv_ranks`` of them) gather
    their keys and values for the self-attention, within a process group of their own."""

    def __init__(self, batch, tokens, group=None):
        import torch.distributed as dist
        self.dist = dist if dist.is_available() and dist.is_initialized() else None
        self.world_group = group
        self.world = self.dist.get_world_size(group) if self.dist else 1
        self.rank = self.dist.get_rank(group) if self.dist else 0
        self.gloo = bool(self.dist) and self.dist.get_backend(group) == "gloo"
        rows = batch * tokens
        if rows % self.world:
            raise ValueError(f"{self.world} ranks do not divide {rows} token rows")
        self.rows = rows // self.world
        if self.rows >= tokens:
            if self.rows % tokens:
                raise ValueError(f"a rank's {self.rows} rows are not whole samples of {tokens} tokens")
            self.kv_ranks = 1
        else:
            if tokens % self.rows:
                raise ValueError(f"{self.rows} rows per rank do not divide a sample of {tokens} tokens")
            self.kv_ranks = tokens // self.rows
        self.kv_group = None
        if self.kv_ranks > 1:
            members = None
            for g in range(self.world // self.kv_ranks):  # every rank creates every group, in one order
                ranks = list(range(g * self.kv_ranks, (g + 1) * self.kv_ranks))
                pg = self.dist.new_group(ranks)
                if self.rank in ranks:
                    members = pg
            self.kv_group = members

    def gather_kv(self, k, v):
        """This sample's keys and values of every rank that holds part of it, in token order: (1, L_local, H, d)
        each -> (1, L, H, d) each."""
        if self.kv_ranks == 1:
            return k, v
        out = []
        for t in (k, v):
            t = t.contiguous()
            shape = (t.shape[0], t.shape[1] * self.kv_ranks) + tuple(t.shape[2:])
            if self.gloo:
                parts = [torch.empty_like(t) for _ in range(self.kv_ranks)]
                self.dist.all_gather(parts, t, group=self.kv_group)
                out.append(torch.cat(parts, dim=1))
            else:
                full = torch.empty(shape, dtype=t.dtype, device=t.device)
                self.dist.all_gather_into_tensor(full, t, group=self.kv_group)
                out.append(full)
        return out[0], out[1]


def block_forward_sp(x_rows, emb, ctx, rope, W, cfg, sp, batch, tokens, lora_term=None):
    """One block with whole weights on this rank's token rows x_rows (n, D) -- rows [rank * n, (rank + 1) * n) of
    the (batch * tokens, D) stream; emb (B, D), ctx (B, S, ctx_dim), rope (1, tokens, 1, 64, 2, 2), lora_term
    (B, 3D) or None as in block_forward. Only the self-attention's keys and values cross ranks (SP.gather_kv)."""
    n, D = x_rows.shape
    row0 = sp.rank * n
    hd, H, eps = cfg.head_dim, cfg.heads, cfg.eps
    b0 = row0 // tokens
    if n >= tokens:
        nb, L, t0 = n // tokens, tokens, 0
    else:
        nb, L, t0 = 1, n, row0 % tokens
    emb_b, ctx_b = emb[b0:b0 + nb], ctx[b0:b0 + nb]
    lora_b = emb.new_zeros(()) if lora_term is None else lora_term[b0:b0 + nb]
    rope_b = rope[:, t0:t0 + L]

    # --- self-attention: local q; keys and values of the whole sample
    shift, scale, gate = adaln(W, "self_attn", emb_b, lora_b)
    normed = _ln_mod_rows(x_rows, scale, shift, 0, L, eps)
    q = F.linear(normed, W["self_attn.q_proj.weight"]).view(nb, L, H, hd)
    k = F.linear(normed, W["self_attn.k_proj.weight"]).view(nb, L, H, hd)
    v = F.linear(normed, W["self_attn.v_proj.weight"]).view(nb, L, H, hd)
    q, k = _sf.rms_rope_pair(q, k, rope_b, W["self_attn.q_norm.weight"], W["self_attn.k_norm.weight"], eps)
    k, v = sp.gather_kv(k, v)
    a = _attention(q, k, v).view(n, D)
    x_rows = _residual(x_rows, gate, F.linear(a, W["self_attn.output_proj.weight"]), 0, L)

    # --- cross-attention
    shift, scale, gate = adaln(W, "cross_attn", emb_b, lora_b)
    normed = _ln_mod_rows(x_rows, scale, shift, 0, L, eps)
    q = _fb.rms_norm_128(F.linear(normed, W["cross_attn.q_proj.weight"]).view(nb, L, H, hd).contiguous(),
                         W["cross_attn.q_norm.weight"], eps)
    S = ctx_b.shape[1]
    kc = _fb.rms_norm_128(F.linear(ctx_b, W["cross_attn.k_proj.weight"]).view(nb, S, H, hd).contiguous(),
                          W["cross_attn.k_norm.weight"], eps)
    vc = F.linear(ctx_b, W["cross_attn.v_proj.weight"]).view(nb, S, H, hd)
    a = _attention(q, kc, vc).view(n, D)
    x_rows = _residual(x_rows, gate, F.linear(a, W["cross_attn.output_proj.weight"]), 0, L)

    # --- MLP
    shift, scale, gate = adaln(W, "mlp", emb_b, lora_b)
    h = F.gelu(F.linear(_ln_mod_rows(x_rows, scale, shift, 0, L, eps), W["mlp.layer1.weight"]))
    return _residual(x_rows, gate, F.linear(h, W["mlp.layer2.weight"]), 0, L)


def flops_per_block(cfg, batch, tokens, ctx_tokens):
    """Dense GEMM + attention FLOPs of one block (all ranks together)."""
    M, D, Mh = batch * tokens, cfg.hidden, cfg.mlp
    gemm = 2 * M * D * D * 4 + 2 * M * D * D * 2 + 2 * batch * ctx_tokens * cfg.ctx_dim * D * 2 + 2 * M * D * Mh * 2
    attn = 4 * batch * tokens * tokens * D + 4 * batch * tokens * ctx_tokens * D
    return gemm + attn

