"""The C-ABI library without a GPU: it loads, exports every entry point include/*.h declares (and the ctypes
binding declares the same set), answers its table queries, and the pure host-side logic of the package behaves."""

import ctypes
import glob
import os
import re

import pytest

from conftest import REPO, wf


def _declared():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        for m in re.finditer(r"WF_API\s+[\w\s\*]+?\b(wf_\w+)\s*\(", open(h).read()):
            names.add(m.group(1))
    return names


def test_header_declares_entry_points():
    names = _declared()
    assert {"wf_dequant_gguf", "wf_dequant_gguf_batch", "wf_version"} <= names


def test_library_exports_every_declared_symbol():
    ext = wf("_ext")
    lib = ext.lib()
    for name in _declared():
        assert hasattr(lib, name), name
    assert set(ext.SIGNATURES) == _declared()


def test_version_and_status_strings():
    ext = wf("_ext")
    assert ext.lib().wf_version() >= 10000
    assert "disagree" in ext.status_string(-3)
    assert "unsupported" in ext.status_string(-2)


@pytest.mark.parametrize("qt,vpb,ts", [(2, 32, 18), (3, 32, 20), (6, 32, 22), (7, 32, 24), (8, 32, 34),
                                       (10, 256, 84), (11, 256, 110), (12, 256, 144), (13, 256, 176),
                                       (14, 256, 210)])
def test_block_info_matches_reference_tables(qt, vpb, ts):
    ext = wf("_ext")
    gd = wf("enhancers.gguf_dequant")
    a, b = ctypes.c_int(), ctypes.c_int()
    assert ext.lib().wf_gguf_block_info(qt, ctypes.byref(a), ctypes.byref(b)) == 0
    assert (a.value, b.value) == (vpb, ts)
    table_ts = gd._FORMATS[qt][1] if qt in gd._FORMATS else gd._KFORMATS[qt][1]
    assert table_ts == ts


def test_block_info_rejects_unknown_type():
    ext = wf("_ext")
    a, b = ctypes.c_int(), ctypes.c_int()
    assert ext.lib().wf_gguf_block_info(9, ctypes.byref(a), ctypes.byref(b)) == -2


def test_no_device_is_reported_not_crashed():
    """Without a GPU the entry points refuse with WF_ERR_DEVICE (or a CUDA status) instead of launching."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    ext = wf("_ext")
    rc = ext.lib().wf_dequant_gguf(ctypes.c_void_p(16), 34, ctypes.c_void_p(16), 32, 8, 0, 1, None)
    assert rc != 0


def test_dequantize_cpu_tensor_is_not_this_case():
    """The reference leaves CPU tensors to ComfyUI-GGUF's code (None); so does the drop-in."""
    import torch
    gd = wf("enhancers.gguf_dequant")
    assert gd.dequantize(torch.zeros(34, dtype=torch.uint8), 8, (1, 32), None, None) is None
    assert gd.dequantize(torch.zeros(144, dtype=torch.uint8), 12, (1, 256), None, None) is None
    assert gd._supported(8) and gd._supported(12) and not gd._supported(9)


def test_kquants_switch(monkeypatch):
    gd = wf("enhancers.gguf_dequant")
    env = wf("core.env")
    monkeypatch.setenv("WEIGHTFERRY_GGUF_KQUANTS", "0")
    assert not gd._supported(12) and gd._supported(8)
    monkeypatch.setenv("WEIGHTFERRY_GGUF_KQUANTS", "1")
    assert gd._supported(12)
    with pytest.raises(KeyError):
        env.get("WEIGHTFERRY_NO_SUCH_SWITCH")


def test_settings_file(monkeypatch, tmp_path):
    env = wf("core.env")
    f = tmp_path / "weightferry.env"
    f.write_text("# comment\nWEIGHTFERRY_SLOTS=4\nWEIGHTFERRY_UNKNOWN=1\n")
    monkeypatch.setenv("WEIGHTFERRY_SETTINGS_FILE", str(f))
    monkeypatch.delenv("WEIGHTFERRY_SLOTS", raising=False)
    env.reset_file_cache()
    try:
        assert env.get("WEIGHTFERRY_SLOTS") == "4"
        monkeypatch.setenv("WEIGHTFERRY_SLOTS", "2")
        assert env.get("WEIGHTFERRY_SLOTS") == "2"
    finally:
        env.reset_file_cache()


def test_lora_factors_rules():
    import torch
    gd = wf("enhancers.gguf_dequant")

    class LoRAAdapter:
        def __init__(self, w):
            self.weights = w

    up, down = torch.zeros(8, 2), torch.zeros(2, 16)
    ok = [(1.0, LoRAAdapter((up, down, 4.0, None, None, None)), 1.0, None, None)]
    assert gd.lora_factors(ok, 8, 16) == [(up, down, 2.0)]
    assert gd.lora_factors([(1.0, LoRAAdapter((up, down, None, None, None, None)), 1.0, None, None)], 8, 16)[0][2] == 1.0
    bad_dora = [(1.0, LoRAAdapter((up, down, 4.0, None, torch.zeros(1), None)), 1.0, None, None)]
    assert gd.lora_factors(bad_dora, 8, 16) is None
    assert gd.lora_factors([(1.0, LoRAAdapter((up, down, 4.0, None, None, None)), 0.5, None, None)], 8, 16) is None
    assert gd.lora_factors(ok, 9, 16) is None
