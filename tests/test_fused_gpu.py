"""Fused-block prologue kernels on the GPU through the C ABI / the drop-in functions, against the reference's golden
vectors and the CPU oracle.

Tolerances: modulate is exact (no approximation on either side). The kernels that go through the hardware
rsqrt.approx (LayerNorm + modulate, RMSNorm-128, RMSNorm + RoPE) compute one reciprocal square root per row; the
goldens and the oracle use the correctly rounded one. Each row must therefore equal, bit for bit, the oracle's row
computed with a reciprocal square root within 2 float32 ulps of the correctly rounded one (the approximation's
bound) -- a tighter check than "2 bf16 ulps" of the outputs, which a cancellation in x * (1 + scale) + shift would
make meaningless. The quantiser divides with the hardware's approximate division like the reference on the GPU, so
its scales are within 2 float32 ulps of the exact-division goldens and its int8 values within 1 of them, on a
handful of values at most."""

import os

import numpy as np
import pytest

from conftest import GOLDEN, oracle, wf

pytestmark = pytest.mark.gpu

F = np.load(os.path.join(GOLDEN, "fused_block.npz"))


def _t(bits, shape=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()
    return t.reshape(shape) if shape is not None else t


def _bits(t):
    import torch
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16).reshape(-1)


def _ord(b):
    b = b.astype(np.int32)
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


def ulp16(a, b):
    return np.abs(_ord(np.asarray(a).reshape(-1)) - _ord(np.asarray(b).reshape(-1)))


def test_modulate_golden(cuda):
    fk = wf("enhancers.fused_kernels")
    import torch
    x = _t(F["mod_x"])
    o = torch.empty_like(x)
    fk._get_kernels()["mod"][(12,)](x, _t(F["mod_s1"]), _t(F["mod_shift"]), o, 1024, int(F["mod_rpg"][0]))
    assert np.array_equal(_bits(o), F["mod_out"].reshape(-1))


def test_modulate_entry_point_baseline_shape(cuda):
    """modulate() on BASELINE configs[3]: x (2, 1, 64, 64, 2048), scale / shift (2, 1, 1, 1, 2048)."""
    import torch
    fb = wf("enhancers.fused_block")
    g = torch.Generator(device="cuda").manual_seed(20261201 + 3)
    x = torch.randn((2, 1, 64, 64, 2048), device="cuda", generator=g).to(torch.bfloat16)
    sc = (torch.randn((2, 1, 1, 1, 2048), device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    sh = (torch.randn((2, 1, 1, 1, 2048), device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    out = fb.modulate(x, sc, sh)
    ref = oracle().modulate(_bits(x).reshape(-1, 2048), _bits((1 + sc).contiguous()).reshape(2, 2048),
                            _bits(sh).reshape(2, 2048), 64 * 64)
    assert np.array_equal(_bits(out), ref.reshape(-1))
    # and PyTorch's own two bf16 kernels give the same bits
    assert torch.equal(out, x * (1 + sc) + sh)


@pytest.mark.parametrize("K", [1024, 2048])
def test_ln_modulate_golden(cuda, K):
    import torch
    fk = wf("enhancers.fused_kernels")
    x = _t(F[f"lnmod{K}_x"])
    o = torch.empty_like(x)
    fk._get_kernels()["lnmod"][(12,)](x, _t(F[f"lnmod{K}_s1"]), _t(F[f"lnmod{K}_shift"]), o, 4, 1e-6, K=K)
    got = _bits(o)
    exact = np.all(got.reshape(12, K) == F[f"lnmod{K}_out"].reshape(12, K), axis=1)
    ok = oracle().rows_match_some_rstd(got, lambda k: oracle().ln_modulate(
        F[f"lnmod{K}_x"].reshape(12, K), F[f"lnmod{K}_s1"], F[f"lnmod{K}_shift"], 4, 1e-6, rstd_ulps=k), K)
    assert (exact | ok).all()


def test_ln_modulate_baseline_vs_oracle_and_torch(cuda):
    """Kernel A at BASELINE configs[3] (8192 rows of 2048) against the oracle (2 ulp) and against PyTorch's own
    LayerNorm + two bf16 kernels (2 ulp)."""
    import torch
    fb = wf("enhancers.fused_block")
    g = torch.Generator(device="cuda").manual_seed(20261201 + 3)
    x = torch.randn((2, 1, 64, 64, 2048), device="cuda", generator=g).to(torch.bfloat16)
    sc = (torch.randn((2, 1, 1, 1, 2048), device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    sh = (torch.randn((2, 1, 1, 1, 2048), device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    out = fb.ln_modulate_rows(x, sc, sh, 1e-6)
    xb, s1b, shb = _bits(x).reshape(-1, 2048), _bits((1 + sc).contiguous()).reshape(2, 2048), _bits(sh).reshape(2, 2048)
    ok = oracle().rows_match_some_rstd(_bits(out), lambda k: oracle().ln_modulate(xb, s1b, shb, 4096, 1e-6,
                                                                                  rstd_ulps=k), 2048)
    assert ok.all(), f"{(~ok).sum()} rows"
    # PyTorch's own LayerNorm (the same vectorized Welford order and hardware rsqrt) then its two bf16 kernels
    norm = torch.nn.LayerNorm(2048, elementwise_affine=False, eps=1e-6)
    pt = norm(x) * (1 + sc) + sh
    same = torch.eq(out.view(torch.int16), pt.view(torch.int16)).all(dim=-1).float().mean().item()
    assert same > 0.999, f"rows bit-identical with PyTorch: {same}"


@pytest.mark.parametrize("K", [512, 1536, 5120])
def test_ln_modulate_other_widths_vs_oracle(cuda, K):
    import torch
    lib, ext = wf("_ext").lib(), wf("_ext")
    g = torch.Generator(device="cuda").manual_seed(K)
    rows = 300
    x = (torch.randn((rows, K), device="cuda", generator=g) * 3 - 1).to(torch.bfloat16)
    s1 = (1 + torch.randn((3, K), device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    sh = (torch.randn((3, K), device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    o = torch.empty_like(x)
    ext.check(lib.wf_ln_modulate(x.data_ptr(), s1.data_ptr(), sh.data_ptr(), o.data_ptr(), rows, K, 100, 1e-5,
                                 ext.stream_of(x.device)), "ln")
    xb, s1b, shb = _bits(x).reshape(rows, K), _bits(s1).reshape(3, K), _bits(sh).reshape(3, K)
    ok = oracle().rows_match_some_rstd(_bits(o), lambda k: oracle().ln_modulate(xb, s1b, shb, 100, 1e-5,
                                                                                rstd_ulps=k), K)
    assert ok.all()


def test_rms_norm_128_golden_and_torch(cuda):
    import torch
    fb = wf("enhancers.fused_block")
    x = _t(F["rms_x"], (40, 128))
    w = _t(F["rms_w"])
    out = fb.rms_norm_128(x, w, 1e-6)
    ok = oracle().rows_match_some_rstd(_bits(out), lambda k: oracle().rms_norm_128(F["rms_x"], F["rms_w"], 1e-6,
                                                                                   rstd_ulps=k), 128)
    assert ok.all()
    big = torch.randn((2, 4096, 16, 128), device="cuda").to(torch.bfloat16)
    o2 = fb.rms_norm_128(big, w, 1e-6)
    bb, wb = _bits(big).reshape(-1, 128), _bits(w)
    ok = oracle().rows_match_some_rstd(_bits(o2), lambda k: oracle().rms_norm_128(bb, wb, 1e-6, rstd_ulps=k), 128)
    assert ok.all()
    pt = torch.nn.functional.rms_norm(big, (128,), w, 1e-6)
    same = torch.eq(o2.view(torch.int16), pt.view(torch.int16)).all(dim=-1).float().mean().item()
    assert same > 0.99, f"rows bit-identical with PyTorch's rms_norm: {same}"
    assert fb.rms_norm_128(big.float(), w, 1e-6) is None


def test_rms_rope_golden(cuda):
    import torch
    sf = wf("enhancers.sage_fused")
    B, L, H = (int(v) for v in F["rope_shape"])
    x = _t(F["rope_x"], (B, L, H, 128))
    f = torch.from_numpy(F["rope_f"]).cuda()
    w = _t(F["rope_w"])
    out = sf.rms_rope(x, f, w, 1e-6)
    wf32 = (F["rope_w"].astype(np.uint32) << 16).view(np.float32)
    ok = oracle().rows_match_some_rstd(_bits(out), lambda k: oracle().rms_rope128(
        F["rope_x"], F["rope_f"], wf32, H, L, 1e-6, rstd_ulps=k), 128)
    assert ok.all()


def rope3d_table(T, H, W, theta=10000.0, h_extra=4.0, w_extra=4.0, t_extra=1.0):
    """Cosmos-Predict2's 3D RoPE rotations (1, T*H*W, 1, 64, 2, 2): head dim 128 -> 42 h / 42 w / 44 t channels,
    NTK factors from the extrapolation ratios, tokens in (t h w) order, t then h then w frequencies."""
    import torch
    dim_h, dim_t = 42, 44
    rng_hw = torch.arange(0, dim_h, 2, dtype=torch.float64) / dim_h
    rng_t = torch.arange(0, dim_t, 2, dtype=torch.float64) / dim_t
    h_ntk = h_extra ** (dim_h / (dim_h - 2))
    w_ntk = w_extra ** (dim_h / (dim_h - 2))
    t_ntk = t_extra ** (dim_t / (dim_t - 2))
    hf = 1.0 / ((theta * h_ntk) ** rng_hw)
    wf_ = 1.0 / ((theta * w_ntk) ** rng_hw)
    tf = 1.0 / ((theta * t_ntk) ** rng_t)
    ht, wt, tt = torch.outer(torch.arange(H).double(), hf), torch.outer(torch.arange(W).double(), wf_), \
        torch.outer(torch.arange(T).double(), tf)

    def rot(e):
        return torch.stack([torch.cos(e), -torch.sin(e), torch.sin(e), torch.cos(e)], dim=-1)
    ht, wt, tt = rot(ht), rot(wt), rot(tt)
    em = torch.cat([tt[:, None, None].expand(T, H, W, 22, 4), ht[None, :, None].expand(T, H, W, 21, 4),
                    wt[None, None, :].expand(T, H, W, 21, 4)], dim=-2)
    return em.reshape(1, T * H * W, 1, 64, 2, 2).float().contiguous()


def test_rms_rope_baseline_vs_oracle(cuda):
    """Kernel B at BASELINE configs[3]: q, k (2, 4096, 16, 128) with the 3D RoPE of 1 x 64 x 64 latent patches."""
    import torch
    sf = wf("enhancers.sage_fused")
    g = torch.Generator(device="cuda").manual_seed(20261201 + 3)
    q = torch.randn((2, 4096, 16, 128), device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn((2, 4096, 16, 128), device="cuda", generator=g).to(torch.bfloat16)
    wq = (1 + torch.randn(128, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    wk = (1 + torch.randn(128, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    f = rope3d_table(1, 64, 64).cuda()
    assert sf.rope_ok(q, k, f, wq, wk, 1e-6)
    qo, ko = sf.rms_rope_pair(q, k, f, wq, wk, 1e-6)
    fn = f.cpu().numpy()
    for src, w, o in ((q, wq, qo), (k, wk, ko)):
        wf32 = w.float().cpu().numpy()
        sb = _bits(src).reshape(2, 4096, 16, 128)
        ok = oracle().rows_match_some_rstd(_bits(o), lambda kk: oracle().rms_rope128(sb, fn, wf32, 16, 4096, 1e-6,
                                                                                    rstd_ulps=kk), 128)
        assert ok.all()


@pytest.mark.parametrize("heads", [3, 20, 40])
@pytest.mark.parametrize("strided", [False, True])
def test_rms_rope_heads_vs_oracle(cuda, heads, strided):
    """Head counts that are not 16: fewer than one 4-row group (3), more than one 16-head group per token (20, 40 as
    Cosmos-Predict2-14B), over enough tokens that every warp cycles both staging buffers; strided: a rotation table
    whose last axis is a slice (the scalar-load path)."""
    import torch
    sf = wf("enhancers.sage_fused")
    g = torch.Generator(device="cuda").manual_seed(77 + heads)
    B, L = 2, 1031
    x = torch.randn((B, L, heads, 128), device="cuda", generator=g).to(torch.bfloat16)
    w = (1 + torch.randn(128, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    fb = torch.randn((1, L, 1, 64, 2, 3 if strided else 2), device="cuda", generator=g)
    f = fb[..., :2]
    out = sf.rms_rope(x, f, w, 1e-6)
    fn = np.ascontiguousarray(f.cpu().numpy())
    wf32 = w.float().cpu().numpy()
    ok = oracle().rows_match_some_rstd(_bits(out), lambda kk: oracle().rms_rope128(_bits(x), fn, wf32, heads, L, 1e-6,
                                                                                  rstd_ulps=kk), 128)
    assert ok.all()


@pytest.mark.parametrize("heads,strided,wdt", [(16, False, "bf16"), (40, True, "f32"), (5, False, "f16")])
def test_rms_rope_pair_matches_single_launches(cuda, heads, strided, wdt):
    """wf_rms_rope128_pair (q and k in one launch) gives the bits of two wf_rms_rope128 launches; q / k scales of
    different dtypes fall back to two launches."""
    import torch
    sf = wf("enhancers.sage_fused")
    dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[wdt]
    g = torch.Generator(device="cuda").manual_seed(91 + heads)
    B, L = 2, 515
    q = torch.randn((B, L, heads, 128), device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn((B, L, heads, 128), device="cuda", generator=g).to(torch.bfloat16) * 3
    wq = (1 + torch.randn(128, device="cuda", generator=g) * 0.02).to(dt)
    wk = (1 + torch.randn(128, device="cuda", generator=g) * 0.02).to(dt)
    fb = torch.randn((1, L, 1, 64, 2, 3 if strided else 2), device="cuda", generator=g)
    f = fb[..., :2]
    qo, ko = sf.rms_rope_pair(q, k, f, wq, wk, 1e-6)
    assert torch.equal(qo.view(torch.int16), sf.rms_rope(q, f, wq, 1e-6).view(torch.int16))
    assert torch.equal(ko.view(torch.int16), sf.rms_rope(k, f, wk, 1e-6).view(torch.int16))
    q2, k2 = sf.rms_rope_pair(q, k, f, wq, wk.float() if dt != torch.float32 else wk.half(), 1e-6)
    assert torch.equal(q2.view(torch.int16), qo.view(torch.int16))


@pytest.mark.parametrize("pre", [0, 1, 2, 3])
def test_quant_rows_golden(cuda, pre):
    import torch
    fk = wf("enhancers.fused_kernels")
    x = _t(F["q_x"], (12, 1024))
    s = _t(F["q_gelu"]) if pre == 1 else _t(F["q_s1"], (3, 1024))
    h = _t(F["q_shift"], (3, 1024))
    q = torch.empty((12, 1024), dtype=torch.int8, device="cuda")
    sc = torch.empty((12, 1), dtype=torch.float32, device="cuda")
    rpg, eps = (4, 1e-6) if pre in (2, 3) else (1, 0.0)
    fk._get_kernels()["quant_row"][(12,)](x, s, h, q, sc, rpg, eps, K=1024, PRE=pre)
    torch.cuda.synchronize()
    gs = F[f"q_pre{pre}_scale"]
    got_s = sc.cpu().numpy().reshape(-1)
    assert np.max(np.abs(got_s.view(np.int32).astype(np.int64) - gs.view(np.int32).astype(np.int64))) <= 2
    dq = np.abs(q.cpu().numpy().astype(np.int32) - F[f"q_pre{pre}_q"].astype(np.int32))
    assert dq.max() <= 1 and (dq > 0).sum() <= 8


def test_quant_rows_plain_baseline_vs_oracle(cuda):
    """The plain per-token absmax quantiser at BASELINE configs[2] (X [8192, 2048] ~ N(0, 1))."""
    import torch
    fk = wf("enhancers.fused_kernels")
    g = torch.Generator(device="cuda").manual_seed(20261201 + 2)
    x = torch.randn((8192, 2048), device="cuda", generator=g).to(torch.bfloat16)
    x_q, x_s = fk.quantize_rows(x, rotate=False)
    torch.cuda.synchronize()
    rq, rs = oracle().quant_rows(_bits(x).reshape(8192, 2048), pre=0, rotate=False)
    ds = np.abs(x_s.cpu().numpy().reshape(-1).view(np.int32).astype(np.int64) - rs.view(np.int32).astype(np.int64))
    assert ds.max() <= 2
    dq = np.abs(x_q.cpu().numpy().astype(np.int32) - rq.astype(np.int32))
    assert dq.max() <= 1 and (dq > 0).mean() < 1e-4


def test_quant_rows_rotated_ragged_rows(cuda):
    import torch
    fk = wf("enhancers.fused_kernels")
    g = torch.Generator(device="cuda").manual_seed(5)
    for k in (256, 768, 5120):
        x = (torch.randn((33, k), device="cuda", generator=g) * 4).to(torch.bfloat16)
        x[7] = 0
        x_q, x_s = fk.quantize_rows(x, rotate=True)
        torch.cuda.synchronize()
        rq, rs = oracle().quant_rows(_bits(x).reshape(33, k), pre=0, rotate=True)
        assert float(x_s[7, 0]) == 1e-30 or abs(float(x_s[7, 0]) - 1e-30) < 1e-36
        dq = np.abs(x_q.cpu().numpy().astype(np.int32) - rq.astype(np.int32))
        assert dq.max() <= 1 and (dq > 0).sum() <= 4


def test_fused_c_abi_rejections(cuda):
    import torch
    ext = wf("_ext")
    L = ext.lib()
    x = torch.zeros((4, 1000), dtype=torch.bfloat16, device="cuda")
    st = ext.stream_of(x.device)
    p = x.data_ptr()
    assert L.wf_ln_modulate(p, p, p, p, 4, 1000, 1, 1e-6, st) == -1     # K not a multiple of 512
    assert L.wf_modulate(p, p, p, p, 4, 1001, 1, st) == -1              # d not a multiple of 8
    assert L.wf_quant_rows(p, None, None, None, p, p, 4, 1000, 1, 0.0, 0, 1, st) == -1  # rotate needs K % 256
    assert L.wf_quant_rows(p, None, None, None, p, p, 4, 1024, 1, 0.0, 2, 0, st) == -1  # modulate needs s1 / shift


@pytest.mark.parametrize("rotate", [0, 1])
@pytest.mark.parametrize("pre", [0, 1, 2])
@pytest.mark.parametrize("k", [256, 768, 1280, 2048, 4096, 5120, 6144, 8192, 20480, 1000])
def test_quant_rows_register_kernel_matches_shared_kernel(cuda, pre, k, rotate):
    """The register-resident quantiser (16-byte aligned operands, K = 256 * n for the sizes it takes: one warp per row
    up to K = 3072, four for 4096 - 6144, eight from 8192, with or without the ConvRot Hadamard) and the shared-memory
    one (any K % 4 == 0; reached here through an x that is only 8-byte aligned) give the same bits."""
    import torch
    if rotate and k % 256:
        pytest.skip("the rotation needs K % 256 == 0")
    ext = wf("_ext")
    L = ext.lib()
    g = torch.Generator(device="cuda").manual_seed(k + pre)
    rows, rpg = 37, 5
    groups = (rows + rpg - 1) // rpg
    base = (torch.randn((rows * k + 8,), device="cuda", generator=g) * 3).to(torch.bfloat16)
    x_al = base[:rows * k].clone()                                    # 16-byte aligned
    x_al[3 * k:4 * k] = 0                                             # an all-zero row
    x_mis = base[4:4 + rows * k]                                      # 8-byte aligned only
    x_mis.copy_(x_al)
    s1 = (1 + 0.1 * torch.randn((groups * k,), device="cuda", generator=g)).to(torch.bfloat16)
    sh = (0.1 * torch.randn((groups * k,), device="cuda", generator=g)).to(torch.bfloat16)
    gelu = wf("enhancers.fused_int8")._gelu_table(torch.device("cuda")) if pre == 1 else None
    outs = []
    for x in (x_al, x_mis):
        q = torch.empty((rows, k), dtype=torch.int8, device="cuda")
        sc = torch.empty((rows,), dtype=torch.float32, device="cuda")
        rc = L.wf_quant_rows(x.data_ptr(), s1.data_ptr() if pre == 2 else None, sh.data_ptr() if pre == 2 else None,
                             gelu.data_ptr() if pre == 1 else None, q.data_ptr(), sc.data_ptr(), rows, k, rpg, 0.0,
                             pre, rotate, ext.stream_of(x.device))
        ext.check(rc, "wf_quant_rows")
        outs.append((q, sc))
    torch.cuda.synchronize()
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1].view(torch.int32), outs[1][1].view(torch.int32))
    if pre != 2:                                                      # (with modulate the row becomes the shift)
        assert float(outs[0][1][3]) == pytest.approx(1e-30)


@pytest.mark.parametrize("n,D,rpg", [(4096, 5120, 4096), (300, 1024, 7), (8192, 2048, 4096), (8, 8, 1)])
def test_gated_residual_equals_addcmul(cuda, n, D, rpg):
    """wf_gated_residual (the block's residual update) gives PyTorch's bf16 addcmul bit for bit, also in place."""
    import torch
    fb = wf("enhancers.fused_block")
    g = torch.Generator(device="cuda").manual_seed(n + D)
    x = torch.randn((n, D), device="cuda", generator=g).to(torch.bfloat16)
    o = (torch.randn((n, D), device="cuda", generator=g) * 3).to(torch.bfloat16)
    groups = (n + rpg - 1) // rpg
    gate = (torch.randn((groups, D), device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    want = torch.addcmul(x, gate.repeat_interleave(rpg, dim=0)[:n], o)
    got = fb.gated_residual(x, gate, o, rpg)
    inplace = x.clone()
    fb.gated_residual(inplace, gate, o, rpg, out=inplace)
    torch.cuda.synchronize()
    assert torch.equal(got, want) and torch.equal(inplace, want)
    if n % rpg == 0:   # the block's broadcast form
        b = n // rpg
        assert torch.equal(torch.addcmul(x.view(b, rpg, D), gate.view(b, 1, D), o.view(b, rpg, D)).view(n, D), want)


@pytest.mark.parametrize("k,rpg", [(2048, 4096), (512, 3), (5120, 100), (8192, 7)])
def test_quant_rows_lnmod_equals_lnmod_then_quant(cuda, k, rpg):
    """The quantiser with the pending LayerNorm + modulate (pre 3, the fused kernel) gives exactly kernel A's bf16
    rows (wf_ln_modulate) quantised by the plain quantiser (pre 0): the same values, rounded the same way."""
    import torch
    ext = wf("_ext")
    L = ext.lib()
    g = torch.Generator(device="cuda").manual_seed(k + rpg)
    rows = 300
    groups = (rows + rpg - 1) // rpg
    x = (torch.randn((rows, k), device="cuda", generator=g) * 2 + 0.5).to(torch.bfloat16)
    x[5] = 1.0                                                      # a constant row: variance 0
    s1 = (1 + 0.1 * torch.randn((groups, k), device="cuda", generator=g)).to(torch.bfloat16)
    sh = (0.1 * torch.randn((groups, k), device="cuda", generator=g)).to(torch.bfloat16)
    st = ext.stream_of(x.device)
    q3 = torch.empty((rows, k), dtype=torch.int8, device="cuda")
    s3 = torch.empty((rows,), dtype=torch.float32, device="cuda")
    ext.check(L.wf_quant_rows(x.data_ptr(), s1.data_ptr(), sh.data_ptr(), None, q3.data_ptr(), s3.data_ptr(), rows, k,
                              rpg, 1e-6, 3, 0, st), "quant pre 3")
    y = torch.empty_like(x)
    ext.check(L.wf_ln_modulate(x.data_ptr(), s1.data_ptr(), sh.data_ptr(), y.data_ptr(), rows, k, rpg, 1e-6, st), "ln")
    q0 = torch.empty_like(q3)
    s0 = torch.empty_like(s3)
    ext.check(L.wf_quant_rows(y.data_ptr(), None, None, None, q0.data_ptr(), s0.data_ptr(), rows, k, 1, 0.0, 0, 0, st),
              "quant pre 0")
    torch.cuda.synchronize()
    assert torch.equal(q3, q0)
    assert torch.equal(s3.view(torch.int32), s0.view(torch.int32))


@pytest.mark.parametrize("k,rpg", [(2048, 4096), (512, 3), (1536, 7), (5120, 100), (8192, 7)])
def test_quant_rows_lnmod_rotated_register_equals_shared(cuda, k, rpg):
    """The pending LayerNorm + modulate with the ConvRot rotation (pre 3, rotate): the register kernel (8-byte aligned
    q) gives the bits of the shared-memory kernel (reached here through a q that is only 4-byte aligned) and of kernel
    A's rows rotated and quantised by the plain rotated quantiser."""
    import torch
    ext = wf("_ext")
    L = ext.lib()
    g = torch.Generator(device="cuda").manual_seed(3 * k + rpg)
    rows = 301
    groups = (rows + rpg - 1) // rpg
    x = (torch.randn((rows, k), device="cuda", generator=g) * 2 + 0.5).to(torch.bfloat16)
    x[5] = 1.0                                                      # a constant row: variance 0
    s1 = (1 + 0.1 * torch.randn((groups, k), device="cuda", generator=g)).to(torch.bfloat16)
    sh = (0.1 * torch.randn((groups, k), device="cuda", generator=g)).to(torch.bfloat16)
    st = ext.stream_of(x.device)
    outs = []
    for off in (0, 4):                                              # q 8-byte aligned, then only 4-byte aligned
        buf = torch.empty((rows * k + 8,), dtype=torch.int8, device="cuda")
        sc = torch.empty((rows,), dtype=torch.float32, device="cuda")
        ext.check(L.wf_quant_rows(x.data_ptr(), s1.data_ptr(), sh.data_ptr(), None, buf.data_ptr() + off,
                                  sc.data_ptr(), rows, k, rpg, 1e-6, 3, 1, st), "quant pre 3 rotate")
        outs.append((buf[off:off + rows * k].clone(), sc))
    y = torch.empty_like(x)
    ext.check(L.wf_ln_modulate(x.data_ptr(), s1.data_ptr(), sh.data_ptr(), y.data_ptr(), rows, k, rpg, 1e-6, st), "ln")
    q0 = torch.empty((rows * k,), dtype=torch.int8, device="cuda")
    s0 = torch.empty((rows,), dtype=torch.float32, device="cuda")
    ext.check(L.wf_quant_rows(y.data_ptr(), None, None, None, q0.data_ptr(), s0.data_ptr(), rows, k, 1, 0.0, 0, 1, st),
              "quant pre 0 rotate")
    torch.cuda.synchronize()
    for q, sc in outs[1:] + [(q0, s0)]:
        assert torch.equal(outs[0][0], q)
        assert torch.equal(outs[0][1].view(torch.int32), sc.view(torch.int32))
