"""Shared test setup: the `gpu` marker, the repository on sys.path, and import helpers for the package (its folder
name, comfyui-weightferry_b200, is loaded by path the way ComfyUI loads custom nodes) and the CPU oracle."""

import importlib
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

PKG = "comfyui-weightferry_b200"
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100) and the built CUDA library")


def wf(mod=""):
    """Import a module of the package, e.g. wf("enhancers.gguf_dequant")."""
    return importlib.import_module(PKG + ("." + mod if mod else ""))


def oracle():
    return importlib.import_module("oracle.oracle")


@pytest.fixture(scope="session")
def cuda():
    """The torch module with a usable sm_100 device, or skip."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _minor = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.skip(f"not an sm_100 device (capability {major})")
    return torch
