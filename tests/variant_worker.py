"""Runs the prologue kernels (LayerNorm + modulate, RMSNorm-128 + RoPE) on seeded inputs and saves their outputs, so
that a test can compare the kernel variants the environment selects (WEIGHTFERRY_ROPE_V1, WEIGHTFERRY_ROPE_ROWS,
WEIGHTFERRY_ROPE_PREFETCH, WEIGHTFERRY_LN_PREFETCH, WEIGHTFERRY_QUANT_PREFETCH) bit for bit, and the int8
quantisers (plain and with the LayerNorm + modulate pending) besides. Usage: python variant_worker.py OUT.pt"""

import importlib
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
ext = importlib.import_module("comfyui-weightferry_b200._ext")
fk = importlib.import_module("comfyui-weightferry_b200.enhancers.fused_kernels")
sf = importlib.import_module("comfyui-weightferry_b200.enhancers.sage_fused")
cb = importlib.import_module("comfyui-weightferry_b200.streaming.cosmos_block")

LN_CASES = [  # (rows, K, rows per modulation group): odd row counts, pairs that straddle a group boundary
    (1, 2048, 1), (2, 1024, 1), (3, 512, 2), (301, 1536, 7), (300, 2048, 100), (8192, 2048, 4096), (257, 5120, 5),
    (4099, 1024, 4099),
]
ROPE_CASES = [(16, 4096), (40, 1024), (3, 256), (20, 64)]  # (heads, tokens), batch 2
QUANT_CASES = [(8192, 2048, 4096), (301, 1024, 7), (2000, 5120, 1000), (33, 512, 33)]  # (rows, K, rows per group)


def main(path):
    lib = ext.lib()
    out = {}
    g = torch.Generator(device="cuda").manual_seed(11)
    for rows, K, rpg in LN_CASES:
        groups = (rows + rpg - 1) // rpg
        x = (torch.randn((rows, K), device="cuda", generator=g) * 2 - 0.5).to(torch.bfloat16)
        s1 = (1 + torch.randn((groups, K), device="cuda", generator=g) * 0.1).to(torch.bfloat16)
        sh = (torch.randn((groups, K), device="cuda", generator=g) * 0.1).to(torch.bfloat16)
        o = torch.empty_like(x)
        ext.check(lib.wf_ln_modulate(x.data_ptr(), s1.data_ptr(), sh.data_ptr(), o.data_ptr(), rows, K, rpg, 1e-6,
                                     ext.stream_of(x.device)), "ln_modulate")
        out[("ln", rows, K, rpg)] = o.cpu()
    for rows, K, rpg in QUANT_CASES:
        groups = (rows + rpg - 1) // rpg
        x = (torch.randn((rows, K), device="cuda", generator=g) * 2).to(torch.bfloat16)
        s1 = (1 + torch.randn((groups, K), device="cuda", generator=g) * 0.1).to(torch.bfloat16)
        sh = (torch.randn((groups, K), device="cuda", generator=g) * 0.1).to(torch.bfloat16)
        for pre in (fk.PRE_NONE, fk.PRE_LNMOD):
            xq, xs = fk.quantize_rows(x, pre=pre, s1=s1, shift=sh, rows_per_group=rpg, eps=1e-6)
            out[("quant", rows, K, rpg, pre)] = (xq.cpu().to(torch.int16), xs.cpu().view(torch.int32))
    for heads, L in ROPE_CASES:
        q = torch.randn((2, L, heads, 128), device="cuda", generator=g).to(torch.bfloat16) * 3
        k = torch.randn((2, L, heads, 128), device="cuda", generator=g).to(torch.bfloat16)
        f = cb.rope3d_table(1, L // 64 if L >= 64 else 1, 64 if L >= 64 else L, device="cuda")
        for wdt in (torch.bfloat16, torch.float16, torch.float32):
            wq = (1 + torch.randn(128, device="cuda", generator=g) * 0.02).to(wdt)
            wk = (1 + torch.randn(128, device="cuda", generator=g) * 0.02).to(wdt)
            qo, ko = sf.rms_rope_pair(q, k, f, wq, wk, 1e-6)
            q1 = sf.rms_rope(q, f, wq, 1e-6)
            out[("rope", heads, L, str(wdt))] = (qo.cpu(), ko.cpu(), q1.cpu())
    torch.cuda.synchronize()
    torch.save(out, path)
    print("cases", len(out))


if __name__ == "__main__":
    main(sys.argv[1])
