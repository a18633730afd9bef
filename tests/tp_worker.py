"""torchrun worker of the tensor-parallel GPU test (tests/test_tp_gpu.py): each rank streams its shards of a small
Cosmos stack and runs it tensor-parallel over NCCL; rank 0 gathers the token rows and compares them with the same
stack run on one GPU with the full weights (same seeds). Exit code 0 = within tolerance."""

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
    full = tp.all_gather_rows(out)
    ok = torch.ones(1, device="cuda")
    if rank == 0:
        single = stk.StreamedStack(cfg, 3, "cuda", cb.TP(single=True), seed=77, num_slots=2)
        ref = single.forward(x, emb, ctx, rope, batch, tokens, lora)
        err = ((full.float() - ref.float()).norm() / ref.float().norm()).item()
        print(f"tp{world} vs single-GPU relative L2 error {err:.3e}; row chunks vs none {chunk_err:.3e}", flush=True)
        if not (err < 2e-2 and chunk_err < 1e-2 and torch.isfinite(full.float()).all()):
            ok.zero_()
        single.close()
    dist.broadcast(ok, 0)
    stack.close()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok.item() == 1 else 1)


if __name__ == "__main__":
    main()
