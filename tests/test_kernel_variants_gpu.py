"""The prologue kernels' variants give the same bits: RMSNorm-128 + RoPE's warp-per-token kernel at 2, 4 and 8 rows
in flight and with its L2 prefetch off or far ahead, against the earlier staged kernel; LayerNorm + modulate and the
int8 quantisers with their L2 prefetch on, off and far ahead. Each variant is chosen by an environment variable that
is read once per process, so every variant runs in its own process (tests/variant_worker.py) on the same seeded
inputs: odd row counts, row pairs across a modulation-group boundary, every weight dtype, q and k in one launch and
one tensor alone."""

import os
import subprocess
import sys

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

VARIANTS = {
    "reference": {"WEIGHTFERRY_ROPE_V1": "1", "WEIGHTFERRY_LN_PREFETCH": "0", "WEIGHTFERRY_QUANT_PREFETCH": "0"},
    "default": {},
    "rope_rows_2": {"WEIGHTFERRY_ROPE_ROWS": "2"},
    "rope_rows_8": {"WEIGHTFERRY_ROPE_ROWS": "8"},
    "no_prefetch": {"WEIGHTFERRY_ROPE_PREFETCH": "0"},
    "far_prefetch": {"WEIGHTFERRY_ROPE_PREFETCH": "9", "WEIGHTFERRY_LN_PREFETCH": "9",
                     "WEIGHTFERRY_QUANT_PREFETCH": "9"},
}


def _run(tmp_path, name):
    env = {k: v for k, v in os.environ.items() if k not in ("WEIGHTFERRY_ROPE_V1", "WEIGHTFERRY_ROPE_ROWS",
                                                             "WEIGHTFERRY_ROPE_PREFETCH", "WEIGHTFERRY_LN_PREFETCH",
                                                             "WEIGHTFERRY_QUANT_PREFETCH")}
    env.update(VARIANTS[name])
    path = str(tmp_path / f"{name}.pt")
    res = subprocess.run(["timeout", "-k", "10", "300", sys.executable, os.path.join(REPO, "tests", "variant_worker.py"),
                          path], cwd=REPO, capture_output=True, text=True, env=env)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    import torch
    return torch.load(path)


def _same(a, b):
    import torch
    if isinstance(a, tuple):
        return all(_same(x, y) for x, y in zip(a, b))
    return torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_prologue_variants_bit_identical(cuda, tmp_path):
    ref = _run(tmp_path, "reference")
    for name in ("default", "rope_rows_2", "rope_rows_8", "no_prefetch", "far_prefetch"):
        got = _run(tmp_path, name)
        assert got.keys() == ref.keys()
        bad = [k for k in ref if not _same(ref[k], got[k])]
        assert not bad, f"{name}: {bad}"
