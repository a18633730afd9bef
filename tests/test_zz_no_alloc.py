"""The W8A8 linear entry point that allocates nothing (wf_w8a8_linear_noalloc), for callers that cannot allocate
device memory when they run a layer. Called through the C ABI twice in a row on different inputs, its output must
equal the regular path's (wf_quant_rows into caller-allocated int8 activations and scales, then wf_w8a8_gemm) bit for
bit -- the same kernels on the same data; and a problem beyond its fixed buffer is refused with WF_ERR_TOO_LARGE.
This file is collected last so that a stop at its first failure has already run every other test."""

import pytest

from conftest import wf

pytestmark = pytest.mark.gpu


def _regular(x, wq, ws):
    import torch
    ext = wf("_ext")
    m, k = x.shape
    n = wq.shape[0]
    xq = torch.empty((m, k), dtype=torch.int8, device="cuda")
    xs = torch.empty((m,), dtype=torch.float32, device="cuda")
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    st = ext.stream_of(x.device)
    ext.check(ext.lib().wf_quant_rows(x.data_ptr(), None, None, None, xq.data_ptr(), xs.data_ptr(), m, k, 1, 0.0, 0,
                                      0, st), "wf_quant_rows")
    ext.check(ext.lib().wf_w8a8_gemm(xq.data_ptr(), wq.data_ptr(), xs.data_ptr(), ws.data_ptr(), y.data_ptr(), None,
                                     m, n, k, st), "wf_w8a8_gemm")
    return y


def _noalloc(x, wq, ws):
    import torch
    ext = wf("_ext")
    m, k = x.shape
    n = wq.shape[0]
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    ext.check(ext.lib().wf_w8a8_linear_noalloc(x.data_ptr(), wq.data_ptr(), ws.data_ptr(), y.data_ptr(), m, n, k,
                                               ext.stream_of(x.device)), "wf_w8a8_linear_noalloc")
    return y


def _operands(torch, m, n, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((m, k), device="cuda", generator=g).to(torch.bfloat16)
    wq = torch.randint(-127, 128, (n, k), dtype=torch.int16, device="cuda", generator=g).to(torch.int8)
    ws = (torch.rand((n,), device="cuda", generator=g) * 1e-3 + 1e-5).contiguous()
    return x, wq, ws


def test_noalloc_linear_matches_regular_path_twice(cuda):
    import torch
    for m, n, k, seed in ((8192, 2048, 2048, 1), (777, 520, 1024, 2)):  # the second call reuses the same buffer
        x, wq, ws = _operands(torch, m, n, k, seed)
        got = _noalloc(x, wq, ws)
        want = _regular(x, wq, ws)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), (m, n, k)


def test_noalloc_linear_refuses_beyond_its_buffer(cuda):
    import torch
    ext = wf("_ext")
    t = torch.zeros(64, dtype=torch.int8, device="cuda")
    p = t.data_ptr()
    st = ext.stream_of(t.device)
    assert ext.lib().wf_w8a8_linear_noalloc(p, p, p, p, 8193, 16, 2048, st) == -5   # m * k > 16,777,216
    assert ext.lib().wf_w8a8_linear_noalloc(p, p, p, p, 65537, 16, 16, st) == -5    # m > 65,536
    assert ext.lib().wf_w8a8_linear_noalloc(p, p, p, p, 2, 16, 1 << 62, st) == -5   # m * k would overflow int64
    assert ext.lib().wf_w8a8_linear_noalloc(p, p, p, p, 2, 16, 51216, st) == -2     # k beyond the quantiser's row
    assert "fixed buffer" in ext.status_string(-5)
