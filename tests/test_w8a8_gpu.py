"""W8A8 linear on the GPU: the tcgen05 int8 GEMM's int32 accumulators bit for bit against an exact (float64) matrix
product of the same int8 operands, its bf16 outputs within 1 bf16 ulp of the float64 restatement
bf16(acc * x_s[m] * w_s[n]), for one tile, ragged edges, many tiles and the BASELINE shape; the kernel's status word
must read 0 (no pipeline wait ran out of time)."""

import pytest

from conftest import wf

pytestmark = pytest.mark.gpu


def _gemm(xq, wq, xs, ws, with_acc=True):
    import torch
    ext = wf("_ext")
    m, k = xq.shape
    n = wq.shape[0]
    y = torch.empty((m, n), dtype=torch.bfloat16, device=xq.device)
    acc = torch.empty((m, n), dtype=torch.int32, device=xq.device) if with_acc else None
    rc = ext.lib().wf_w8a8_gemm(xq.data_ptr(), wq.data_ptr(), xs.data_ptr(), ws.data_ptr(), y.data_ptr(),
                                acc.data_ptr() if acc is not None else None, m, n, k, ext.stream_of(xq.device))
    ext.check(rc, "wf_w8a8_gemm")
    torch.cuda.synchronize()
    st = __import__("ctypes").c_int(-1)
    ext.check(ext.lib().wf_w8a8_gemm_status(__import__("ctypes").byref(st)), "status")
    assert st.value == 0, f"GEMM pipeline wait expired (code {st.value})"
    return y, acc


def _ord16(t):
    import torch
    b = t.contiguous().view(torch.int16).to(torch.int32)
    return torch.where(b < 0, -(b & 0x7FFF), b)


def _check(xq, wq, xs, ws, y, acc):
    import torch
    exact = xq.double() @ wq.double().t()
    if acc is not None:
        assert torch.equal(acc.double(), exact), "int32 accumulators differ"
    ref = (exact * xs.double().view(-1, 1) * ws.double().view(1, -1)).to(torch.bfloat16)
    d = (_ord16(y) - _ord16(ref)).abs()
    assert int(d.max()) <= 1, f"bf16 outputs differ by {int(d.max())} ulp"


def _operands(m, n, k, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    xq = torch.randint(-128, 128, (m, k), dtype=torch.int16, device="cuda", generator=g).to(torch.int8)
    wq = torch.randint(-127, 128, (n, k), dtype=torch.int16, device="cuda", generator=g).to(torch.int8)
    xs = torch.rand((m,), device="cuda", generator=g) * 0.02 + 1e-4
    ws = torch.rand((n,), device="cuda", generator=g) * 0.001 + 1e-5
    return xq, wq, xs, ws


@pytest.mark.parametrize("m,n,k", [(128, 256, 128), (128, 256, 2048), (300, 520, 272), (1, 8, 16),
                                   (1024, 2048, 2048), (2048, 512, 4096)])
def test_gemm_exact_accumulators(cuda, m, n, k):
    xq, wq, xs, ws = _operands(m, n, k, seed=m * 7 + n * 3 + k)
    y, acc = _gemm(xq, wq, xs, ws)
    _check(xq, wq, xs, ws, y, acc)
    y2, _ = _gemm(xq, wq, xs, ws, with_acc=False)
    assert torch_equal(y, y2)


def torch_equal(a, b):
    import torch
    return torch.equal(a, b)


@pytest.mark.parametrize("m,n", [(300, 520), (129, 264), (1, 8), (255, 2056)])
def test_gemm_output_bounds(cuda, m, n):
    """The tile stores are clipped at row m and column n: a y that ends inside a larger buffer leaves the bytes
    after it untouched."""
    import torch
    ext = wf("_ext")
    k = 64
    xq, wq, xs, ws = _operands(m, n, k, seed=m + n)
    buf = torch.full((m * n + 4096,), 7.0, dtype=torch.bfloat16, device="cuda")
    y = buf[:m * n].view(m, n)
    rc = ext.lib().wf_w8a8_gemm(xq.data_ptr(), wq.data_ptr(), xs.data_ptr(), ws.data_ptr(), y.data_ptr(), None,
                                m, n, k, ext.stream_of(xq.device))
    ext.check(rc, "wf_w8a8_gemm")
    torch.cuda.synchronize()
    assert bool((buf[m * n:] == 7.0).all()), "the GEMM wrote past the end of y"
    _check(xq, wq, xs, ws, y, None)


def test_gemm_extreme_values(cuda):
    """All operands at -128 / 127: accumulators at their largest magnitude (k * 128 * 128 fits int32)."""
    import torch
    m, n, k = 256, 256, 4096
    xq = torch.full((m, k), -128, dtype=torch.int8, device="cuda")
    wq = torch.full((n, k), 127, dtype=torch.int8, device="cuda")
    wq[::2] = -128
    xs = torch.ones(m, device="cuda")
    ws = torch.full((n,), 1e-6, device="cuda")
    y, acc = _gemm(xq, wq, xs, ws)
    _check(xq, wq, xs, ws, y, acc)


def test_gemm_baseline_shape(cuda):
    """X [8192, 2048] per-token quantised, W [8192, 2048] per-channel -> Y [8192, 8192]."""
    import torch
    fk = wf("enhancers.fused_kernels")
    g = torch.Generator(device="cuda").manual_seed(20261201 + 2)
    x = torch.randn((8192, 2048), device="cuda", generator=g).to(torch.bfloat16)
    w_fp = torch.randn((8192, 2048), device="cuda", generator=g) * 0.02
    ws = (w_fp.abs().amax(dim=1) / 127.0).float().contiguous()
    wq = torch.clamp(torch.round(w_fp / ws.view(-1, 1)), -127, 127).to(torch.int8).contiguous()
    xq, xs = fk.quantize_rows(x, rotate=False)
    y, acc = _gemm(xq, wq, xs.view(-1), ws)
    _check(xq, wq, xs.view(-1), ws, y, acc)
    y2, _ = _gemm(xq, wq, xs.view(-1), ws, with_acc=False)
    assert torch.equal(y, y2)


def test_gemm_rejections(cuda):
    import torch
    ext = wf("_ext")
    t = torch.zeros(4096, dtype=torch.int8, device="cuda")
    p = t.data_ptr()
    st = ext.stream_of(t.device)
    assert ext.lib().wf_w8a8_gemm(p, p, p, p, p, None, 16, 16, 24, st) == -1   # k % 16
    assert ext.lib().wf_w8a8_gemm(p, p, p, p, p, None, 16, 12, 32, st) == -1   # n % 8
    assert ext.lib().wf_w8a8_gemm(p + 1, p, p, p, p, None, 16, 16, 32, st) == -1  # alignment


def test_int8_linear_entry_points(cuda):
    """int8_linear (plain) equals quantise + GEMM; the reference-named _int8_linear_shared shares one quantisation
    between q / k / v under _Overrides' cache and handles a pending modulate inside the quantiser."""
    import torch
    fi = wf("enhancers.fused_int8")
    fk = wf("enhancers.fused_kernels")
    fs = wf("enhancers.fused_state")
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn((2, 300, 1024), device="cuda", generator=g).to(torch.bfloat16)
    wq = torch.randint(-127, 128, (768, 1024), dtype=torch.int16, device="cuda", generator=g).to(torch.int8)
    ws = torch.rand(768, device="cuda", generator=g) * 1e-3
    y = fi.int8_linear(x, wq, ws)
    xq, xs = fk.quantize_rows(x.reshape(-1, 1024), rotate=False)
    y2 = fi.gemm(xq, wq, xs, ws)
    assert torch.equal(y.reshape(-1, 768), y2)
    fs._tls.qkv = fi._QuantScope()
    try:
        a = fi._int8_linear_shared(x, (wq, ws), None)
        b = fi._int8_linear_shared(x, (wq, ws), None)
        assert torch.equal(a, y) and torch.equal(b, y)
        # pending modulate: the quantiser applies bf16(bf16(x * (1 + scale)) + shift) itself
        scale = (torch.randn((2, 1, 1024), device="cuda", generator=g) * 0.1).to(torch.bfloat16)
        shift = (torch.randn((2, 1, 1024), device="cuda", generator=g) * 0.1).to(torch.bfloat16)
        fi._set_pre(x, "mod", scale, shift)
        c = fi._int8_linear_shared(x, (wq, ws), None)
        fi._clear_pre()
        real = x * (1 + scale) + shift
        d = fi.int8_linear(real, wq, ws)
        assert torch.equal(c, d)
    finally:
        fs._tls.qkv = None
        fi._clear_pre()


def _gemm_residual(xq, wq, xs, ws, resid, gate, rpg, out):
    ext = wf("_ext")
    m, k = xq.shape
    n = wq.shape[0]
    rc = ext.lib().wf_w8a8_gemm_residual(xq.data_ptr(), wq.data_ptr(), xs.data_ptr(), ws.data_ptr(),
                                         resid.data_ptr(), gate.data_ptr(), rpg, out.data_ptr(), m, n, k,
                                         ext.stream_of(xq.device))
    ext.check(rc, "wf_w8a8_gemm_residual")
    return out


@pytest.mark.parametrize("m,n,k,rpg", [(300, 520, 272, 100), (1024, 2048, 2048, 256), (64, 512, 256, 64),
                                       (257, 264, 64, 1000), (2048, 512, 4096, 7)])
def test_gemm_residual_equals_gemm_then_addcmul(cuda, m, n, k, rpg):
    """The residual epilogue gives exactly the plain GEMM followed by PyTorch's bf16 addcmul with each row's gate row,
    also written in place over the residual."""
    import torch
    xq, wq, xs, ws = _operands(m, n, k, seed=m + 3 * n + k)
    g = torch.Generator(device="cuda").manual_seed(m * n)
    resid = torch.randn((m, n), device="cuda", generator=g).to(torch.bfloat16)
    groups = (m + rpg - 1) // rpg
    gate = (torch.randn((groups, n), device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    y, _ = _gemm(xq, wq, xs, ws, with_acc=False)
    rows_gate = gate[torch.arange(m, device="cuda") // rpg]
    want = torch.addcmul(resid, rows_gate, y)
    assert torch.equal(want, (resid.float() + rows_gate.float() * y.float()).to(torch.bfloat16))
    out = _gemm_residual(xq, wq, xs, ws, resid, gate, rpg, torch.empty_like(resid))
    inplace = resid.clone()
    _gemm_residual(xq, wq, xs, ws, inplace, gate, rpg, inplace)
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    assert torch.equal(inplace, want)


def test_gemm_residual_rejections(cuda):
    import torch
    ext = wf("_ext")
    t = torch.zeros(1 << 16, dtype=torch.int8, device="cuda")
    p = t.data_ptr()
    st = ext.stream_of(t.device)
    L = ext.lib()
    assert L.wf_w8a8_gemm_residual(p, p, p, p, None, p, 1, p, 16, 16, 32, st) == -1      # no residual
    assert L.wf_w8a8_gemm_residual(p, p, p, p, p, None, 1, p, 16, 16, 32, st) == -1      # no gate
    assert L.wf_w8a8_gemm_residual(p, p, p, p, p, p, 0, p, 16, 16, 32, st) == -1         # rows_per_group
    assert L.wf_w8a8_gemm_residual(p, p, p, p, p + 2, p, 1, p, 16, 16, 32, st) == -1     # resid alignment
    assert L.wf_w8a8_gemm_residual(p, p, p, p, p, p + 8, 1, p, 16, 16, 32, st) == -1     # gate alignment


@pytest.mark.parametrize("five_d", [True, False])
def test_int8_linear_residual_entry_point(cuda, five_d):
    """_int8_linear_residual (the reference's residual sub-layer output) equals the plain int8 linear followed by the
    block's addcmul, for the block's (B, T, H, W, D) layout and the row layout (B, N, D)."""
    import torch
    fi = wf("enhancers.fused_int8")
    fs = wf("enhancers.fused_state")
    g = torch.Generator(device="cuda").manual_seed(21)
    B, T, H, W, D, k = 2, 2, 8, 16, 512, 768
    x = torch.randn((B, T, H, W, k) if five_d else (B, T * H * W, k), device="cuda", generator=g).to(torch.bfloat16)
    wq = torch.randint(-127, 128, (D, k), dtype=torch.int16, device="cuda", generator=g).to(torch.int8)
    ws = torch.rand(D, device="cuda", generator=g) * 1e-3
    xr = torch.randn((*x.shape[:-1], D), device="cuda", generator=g).to(torch.bfloat16)
    gshape = (B, T, 1, 1, D) if five_d else (B, 1, D)
    gate = (torch.randn(gshape, device="cuda", generator=g) * 0.3).to(torch.bfloat16)
    fs._tls.qkv = fi._QuantScope()
    try:
        out = fi._int8_linear_residual(x, (wq, ws), None, {"x": xr, "gate": gate})
        plain = fi._int8_linear_shared(x, (wq, ws), None)
    finally:
        fs._tls.qkv = None
    assert out is not None and out.shape == xr.shape
    want = torch.addcmul(xr, gate, plain.view(xr.shape))
    torch.cuda.synchronize()
    assert torch.equal(out, want)


@pytest.mark.parametrize("m,n,k", [(128, 512, 8192), (512, 512, 8192)])  # the one-CTA kernel, the CTA-pair kernel
def test_gemm_wait_expiry_reports_and_recovers(cuda, m, n, k):
    """A pipeline wait made to run out on purpose: with the wait limit shortened to 1 ns (the library's test hook), the
    kernel stops issuing, drains the copies and MMAs it started, frees its tensor memory and reports the wait's code
    (1 producer, 2 MMA issuer, 3 epilogue); a GEMM launched after it with the normal limit is exact again."""
    import ctypes
    import torch
    ext = wf("_ext")
    lib = ext.lib()
    xq, wq, xs, ws = _operands(m, n, k, seed=11 + m)
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    st = ctypes.c_int(-1)
    ext.check(lib.wf_w8a8_gemm_status(ctypes.byref(st)), "status")  # reading clears it
    ext.check(lib.wf_w8a8_gemm_set_wait_limit(1), "wf_w8a8_gemm_set_wait_limit")
    try:
        ext.check(lib.wf_w8a8_gemm(xq.data_ptr(), wq.data_ptr(), xs.data_ptr(), ws.data_ptr(), y.data_ptr(), None,
                                   m, n, k, ext.stream_of(xq.device)), "wf_w8a8_gemm")
        torch.cuda.synchronize()
    finally:
        ext.check(lib.wf_w8a8_gemm_set_wait_limit(0), "wf_w8a8_gemm_set_wait_limit")
    ext.check(lib.wf_w8a8_gemm_status(ctypes.byref(st)), "status")
    assert st.value in (1, 2, 3), f"no wait ran out (status {st.value})"
    y2, acc = _gemm(xq, wq, xs, ws)  # asserts the status reads 0 again
    _check(xq, wq, xs, ws, y2, acc)
