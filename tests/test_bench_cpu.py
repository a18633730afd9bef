"""bench.py's host-side pieces without a GPU: its command line accepts every workload, its GGML geometry table agrees
with the library's own table and the oracle's, its synthetic GGUF blocks carry finite float16 scales, the SSD
workload can name the filesystem it measures, and the reference arm keeps the launch contract under torchrun."""

import ctypes
import importlib
import json
import os
import socket
import subprocess
import sys

import numpy as np
import torch

from conftest import REPO, wf


def _bench():
    sys.path.insert(0, REPO)
    try:
        return importlib.import_module("bench")
    finally:
        sys.path.remove(REPO)


def test_command_line_lists_every_workload():
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--help"], capture_output=True, text=True,
                         timeout=120, cwd=REPO)
    assert out.returncode == 0, out.stderr
    for w in ("sweep", "q8", "q4k", "w8a8", "stack", "prologue", "formats", "lora", "ssd", "block", "quant"):
        assert w in out.stdout
    assert "--impl" in out.stdout and "--ssd-blocks" in out.stdout


def test_quant_workload_covers_every_mode_once():
    b = _bench()
    assert [m for m, _, _ in b.QUANT_MODES] == ["plain", "gelu", "convrot", "convrot_gelu", "lnmod", "lnmod_convrot"]
    assert {(pre, rot) for _, pre, rot in b.QUANT_MODES} == {(0, 0), (1, 0), (0, 1), (1, 1), (3, 0), (3, 1)}
    assert all(k % 512 == 0 and k <= 8192 for k in b.QUANT_WIDTHS)  # every mode takes every width


def test_gguf_geometry_matches_the_library_and_the_oracle():
    bench = _bench()
    lib = wf("_ext").lib()
    from oracle import oracle
    for qt, (_name, vpb, ts, f16) in bench.GGUF_GEOMETRY.items():
        a, b = ctypes.c_int(0), ctypes.c_int(0)
        assert lib.wf_gguf_block_info(qt, ctypes.byref(a), ctypes.byref(b)) == 0
        assert (a.value, b.value) == (vpb, ts)
        assert all(0 <= off <= ts - 2 for off in f16)
        raw = np.zeros(2 * ts, dtype=np.uint8)  # two all-zero blocks: a valid input of this type
        assert oracle.dequant_gguf(raw, 2 * vpb, qt, 0, 1).size == 2 * vpb


def test_fill_gguf_scales_are_finite():
    bench = _bench()
    gen = torch.Generator().manual_seed(5)
    for qt, (_name, vpb, ts, f16) in bench.GGUF_GEOMETRY.items():
        raw = bench.fill_gguf(torch, qt, 4 * vpb, torch.device("cpu"), gen).numpy().reshape(4, ts)
        for off in f16:
            d = raw[:, off:off + 2].copy().view(np.float16).astype(np.float32)
            assert np.all(np.isfinite(d)) and np.all(d >= 0) and np.all(d <= 0.01)


def test_mount_of_names_a_filesystem():
    bench = _bench()
    m = bench.mount_of(REPO)
    assert set(m) == {"mount", "type", "device"}
    assert REPO.startswith(m["mount"].rstrip("/") or "/")


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def test_reference_arm_prints_one_line_from_rank_0_under_torchrun():
    """`bench.py --impl reference` launched as the driver launches it for N > 1 (torchrun, one process per rank): rank
    0 alone times the reference's algorithm on the host and prints one JSON line; every rank exits 0."""
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(_free_port()), os.path.join(REPO, "bench.py"), "--impl", "reference",
           "--gpus", "2", "--steps", "1", "--warmup", "3"]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, out.stdout
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and rec["n_gpus"] == 2 and rec["value"] > 0
    assert rec["e2e"]["h2d_bytes_per_step"] == 0 and rec["cpu_baseline"]["kind"] in ("port", "reference")
