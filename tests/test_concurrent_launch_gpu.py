"""Batched dequantisation launched from two host threads at once (the streaming node's compute thread and its SSD
uploader thread do this), as the first launches of a fresh process: the per-device launch caches are filled by
whichever thread comes first, and every output equals the same launch made alone."""

import os
import subprocess
import sys

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu


def test_two_threads_launch_batched_dequant_concurrently(cuda):
    res = subprocess.run(["timeout", "-k", "10", "240", sys.executable,
                          os.path.join(REPO, "tests", "concurrent_worker.py")], cwd=REPO, capture_output=True,
                         text=True)
    assert res.returncode == 0 and "OK" in res.stdout, res.stdout[-2000:] + res.stderr[-2000:]
