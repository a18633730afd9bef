"""The CPU oracle (oracle/wf_oracle.c) against the golden vectors made by running the reference's own Triton kernels
(tests/golden/make_golden.py): bit for bit, every format, every (mid, out) dtype pair, LoRA adds included."""

import os

import numpy as np
import pytest

from conftest import GOLDEN, oracle

G = np.load(os.path.join(GOLDEN, "gguf_dequant.npz"))
FMT = {2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34),
       10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210)}


def _same_bits(a, b):
    a = np.asarray(a)
    b = np.asarray(b)
    if a.dtype == np.float32:
        # NaN payloads are not part of the contract; every other value bit for bit
        an, bn = np.isnan(a), np.isnan(b)
        return bool(np.array_equal(an, bn) and np.array_equal(a.view(np.uint32)[~an], b.view(np.uint32)[~bn]))
    return bool(np.array_equal(a, b))


@pytest.mark.parametrize("qt", sorted(FMT))
@pytest.mark.parametrize("mid", [0, 1, 2])
@pytest.mark.parametrize("out", [0, 1, 2])
def test_dequant_matches_reference_kernel(qt, mid, out):
    raw = G[f"q{qt}_raw"]
    vpb, ts = FMT[qt]
    n = raw.size // ts * vpb
    got = oracle().dequant_gguf(raw, n, qt, mid, out)
    assert _same_bits(got, G[f"q{qt}_m{mid}_o{out}"])


@pytest.mark.parametrize("qt", [8, 3, 12])
@pytest.mark.parametrize("mid", [0, 1])
@pytest.mark.parametrize("out", [1, 0])
def test_lora_matches_reference_kernel(qt, mid, out):
    raw = G[f"q{qt}_raw"]
    vpb, ts = FMT[qt]
    n = raw.size // ts * vpb
    sa1, sa2 = (float(x) for x in G["lora_sa"])
    w = oracle().dequant_gguf(raw, n, qt, mid, out, diff=G[f"lora_q{qt}_diff"], sa=sa1)
    oracle().lora_add(G[f"lora_q{qt}_diff2"], w, out, sa2)
    assert _same_bits(w, G[f"lora_q{qt}_m{mid}_o{out}"])


def test_oracle_rejects_bad_shapes():
    with pytest.raises(ValueError):
        oracle().dequant_gguf(np.zeros(33, np.uint8), 32, 8, 0, 1)
    with pytest.raises(ValueError):
        oracle().dequant_gguf(np.zeros(34, np.uint8), 32, 9, 0, 1)


@pytest.mark.parametrize("qt", sorted(FMT))
def test_oracle_f32_matches_gguf_py(qt):
    """An independent pin: with float32 intermediates the chain is gguf-py's numpy dequantize (gguf 0.19)."""
    gguf = pytest.importorskip("gguf")
    raw = G[f"q{qt}_raw"]
    vpb, ts = FMT[qt]
    n = raw.size // ts * vpb
    ref = gguf.quants.dequantize(raw.reshape(-1, ts), gguf.GGMLQuantizationType(qt)).reshape(-1).astype(np.float32)
    got = oracle().dequant_gguf(raw, n, qt, 2, 2)
    assert _same_bits(got, ref)


# ---------------------------------------------------------------------------------------------- fused block
F = np.load(os.path.join(GOLDEN, "fused_block.npz"))


def test_modulate_matches_reference_kernel():
    got = oracle().modulate(F["mod_x"], F["mod_s1"], F["mod_shift"], int(F["mod_rpg"][0]))
    assert np.array_equal(got, F["mod_out"])


@pytest.mark.parametrize("K", [1024, 2048])
def test_ln_modulate_matches_reference_kernel(K):
    got = oracle().ln_modulate(F[f"lnmod{K}_x"], F[f"lnmod{K}_s1"], F[f"lnmod{K}_shift"], 4, 1e-6)
    assert np.array_equal(got, F[f"lnmod{K}_out"])


def test_rms_norm_128_matches_reference_kernel():
    got = oracle().rms_norm_128(F["rms_x"], F["rms_w"], 1e-6)
    assert np.array_equal(got, F["rms_out"])


def test_rms_rope128_matches_reference_kernel():
    B, L, H = (int(v) for v in F["rope_shape"])
    w = (F["rope_w"].astype(np.uint32) << 16).view(np.float32)
    got = oracle().rms_rope128(F["rope_x"], F["rope_f"], w, H, L, 1e-6)
    assert np.array_equal(got, F["rope_out"])


@pytest.mark.parametrize("pre", [0, 1, 2, 3])
def test_quant_rows_matches_reference_kernel(pre):
    kw = dict(pre=pre, rotate=True)
    if pre == 1:
        kw.update(gelu=F["q_gelu"])
    if pre in (2, 3):
        kw.update(s1=F["q_s1"], shift=F["q_shift"], rows_per_group=4, eps=1e-6)
    q, sc = oracle().quant_rows(F["q_x"], **kw)
    assert np.array_equal(sc.view(np.uint32), F[f"q_pre{pre}_scale"].view(np.uint32))
    assert np.array_equal(q, F[f"q_pre{pre}_q"])
