"""Worker of tests/test_concurrent_launch_gpu.py, run in a fresh process so that its first launches are the first of
the process: two host threads -- the compute thread and the SSD uploader's, in the streaming node -- start their
batched GGUF dequantisations at the same moment on their own streams (the launchers' per-device caches are filled by
whichever comes first), many times; every output must equal the same launch made alone. Prints OK on success."""

import importlib
import os
import sys
import threading

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    gd = importlib.import_module("comfyui-weightferry_b200.enhancers.gguf_dequant")
    fk = importlib.import_module("comfyui-weightferry_b200.enhancers.fused_kernels")
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(3)
    jobs = []
    for qt, ts, vpb in ((8, 34, 32), (12, 144, 256)):
        items = []
        for rows in (256, 512, 768):
            n = rows * 1024
            raw = torch.randint(0, 256, (n // vpb * ts,), dtype=torch.uint8, device=dev, generator=g)
            raw.view(-1, ts)[:, 0:2] = (torch.rand((n // vpb, 1), device=dev, generator=g) * 0.01).half().view(
                torch.uint8)
            items.append((raw, (rows, 1024)))
        jobs.append((qt, items))
    torch.cuda.synchronize()
    start = threading.Barrier(3)
    results = [None, None]
    errors = []

    def run(i):
        try:
            qt, items = jobs[i]
            s = torch.cuda.Stream(device=dev)
            outs = []
            start.wait()
            with torch.cuda.stream(s):
                for _ in range(20):
                    outs.append(gd.dequantize_many(items, qt, None, torch.bfloat16))
                    x = torch.randn((300, 1024), device=dev, generator=None).to(torch.bfloat16)
                    fk.quantize_rows(x)  # the quantiser's launcher cache too
            s.synchronize()
            results[i] = outs
        except Exception as exc:  # noqa: BLE001 -- reported below
            errors.append(exc)

    threads = [threading.Thread(target=run, args=(i,)) for i in range(2)]
    for t in threads:
        t.start()
    start.wait()
    for t in threads:
        t.join()
    if errors:
        raise errors[0]
    for i, (qt, items) in enumerate(jobs):
        alone = gd.dequantize_many(items, qt, None, torch.bfloat16)
        torch.cuda.synchronize()
        for outs in results[i]:
            for a, b in zip(outs, alone):
                if not torch.equal(a.view(torch.int16), b.view(torch.int16)):
                    print(f"type {qt}: a concurrent launch differs from the launch alone")
                    sys.exit(1)
    print("OK")


if __name__ == "__main__":
    main()
