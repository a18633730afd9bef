"""torchrun worker of the tensor-parallel GPU test (tests/test_tp_gpu.py): each rank streams its shards of a small
Cosmos stack and runs it tensor-parallel over NCCL; rank 0 also runs the same stack on one GPU with the full weights
(same seeds) and broadcasts the result, and every rank checks its own token rows (its shard) against it:

  |y - y_ref| <= 0.2 * rms(y_ref row)              per element (the three reduce-scatters of a block each add one
                                                   bf16 rounding of two partial sums to the row-parallel outputs,
                                                   which the following sub-layers carry on, over three blocks whose
                                                   update is about 12 times their input: measured 0.125), and
  ||(y - x) - (y_ref - x)|| <= 1e-2 ||y_ref - x||  for the shard's update (x its input rows): a head group or MLP
                                                   slice taken from the wrong shard changes about 1 / world of a
                                                   sub-layer's output, far above this bound.

The overlapped row-chunk form (WEIGHTFERRY_TP_CHUNKS=4) must agree with the unchunked one within 1e-2 relative L2.
Exit code 0 = every rank within tolerance."""

import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    import importlib
    cb = importlib.import_module("comfyui-weightferry_b200.streaming.cosmos_block")
    stk = importlib.import_module("comfyui-weightferry_b200.streaming.stack")
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    cfg = cb.CosmosConfig(hidden=1024, heads=8, head_dim=128, mlp=4096, ctx_dim=256, lora=64)
    batch, T, H, W = 2, 1, 16, 16
    tokens = T * H * W
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn((batch * tokens, cfg.hidden), device="cuda", generator=g).to(torch.bfloat16)
    emb = (torch.randn((batch, cfg.hidden), device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    lora = (torch.randn((batch, 3 * cfg.hidden), device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    ctx = torch.randn((batch, 64, cfg.ctx_dim), device="cuda", generator=g).to(torch.bfloat16)
    rope = cb.rope3d_table(T, H, W, device="cuda")
    tp = cb.TP()
    rows = batch * tokens // world
    stack = stk.StreamedStack(cfg, 3, "cuda", tp, seed=77, num_slots=2)
    out = stack.forward(x[rank * rows:(rank + 1) * rows].contiguous(), emb, ctx, rope, batch, tokens, lora)
    # the same forward with the overlapped row chunks (WEIGHTFERRY_TP_CHUNKS=4): only GEMM shapes differ
    os.environ["WEIGHTFERRY_TP_CHUNKS"] = "4"
    chunked = stack.forward(x[rank * rows:(rank + 1) * rows].contiguous(), emb, ctx, rope, batch, tokens, lora)
    os.environ.pop("WEIGHTFERRY_TP_CHUNKS")
    chunk_err = ((chunked.float() - out.float()).norm() / out.float().norm()).item()
    ref = torch.empty((batch * tokens, cfg.hidden), dtype=torch.bfloat16, device="cuda")
    if rank == 0:
        single = stk.StreamedStack(cfg, 3, "cuda", cb.TP(single=True), seed=77, num_slots=2)
        ref.copy_(single.forward(x, emb, ctx, rope, batch, tokens, lora))
        single.close()
    dist.broadcast(ref, 0)
    mine = slice(rank * rows, (rank + 1) * rows)
    y, yr, x0 = out.double(), ref[mine].double(), x[mine].double()
    rel = ((y - yr).abs() / yr.pow(2).mean(dim=1, keepdim=True).sqrt()).max().item()
    upd = (((y - x0) - (yr - x0)).norm() / (yr - x0).norm()).item()
    print(f"rank {rank}: tp{world} vs single GPU: max |d| / row rms {rel:.4f}, update rel-L2 {upd:.3e}; "
          f"row chunks vs none {chunk_err:.3e}", flush=True)
    ok = torch.ones(1, device="cuda")
    if not (rel <= 0.2 and upd <= 1e-2 and chunk_err < 1e-2 and torch.isfinite(y).all()):
        ok.zero_()
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    stack.close()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok.item() == 1 else 1)


if __name__ == "__main__":
    main()
