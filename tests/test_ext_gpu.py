"""The launchers' stream and device helpers (_ext.stream_of, _ext.on_device) on the GPU: the stream is PyTorch's
current one -- the default stream, a side stream made current with torch.cuda.stream, on the device named by a
torch.device, an index or a string -- and the device guard makes a tensor's device current only for the launch."""

import pytest

from conftest import wf

pytestmark = pytest.mark.gpu


def test_stream_of_is_the_current_stream(cuda):
    import torch
    ext = wf("_ext")
    dev = torch.device("cuda", torch.cuda.current_device())
    assert ext.stream_of(dev) == torch.cuda.current_stream(dev).cuda_stream
    assert ext.stream_of(dev.index) == torch.cuda.current_stream(dev).cuda_stream
    assert ext.stream_of("cuda") == torch.cuda.current_stream().cuda_stream
    side = torch.cuda.Stream(dev)
    with torch.cuda.stream(side):
        assert ext.stream_of(dev) == side.cuda_stream != torch.cuda.default_stream(dev).cuda_stream
    assert ext.stream_of(dev) == torch.cuda.current_stream(dev).cuda_stream


def test_launch_on_a_side_stream_is_ordered_on_that_stream(cuda):
    """A quantiser launched inside `with torch.cuda.stream(side)` runs on `side`: its result is ready after
    side.synchronize() and matches a launch on the default stream."""
    import torch
    fk = wf("enhancers.fused_kernels")
    g = torch.Generator(device="cuda").manual_seed(5)
    x = (torch.randn((4096, 2048), device="cuda", generator=g) * 2).to(torch.bfloat16)
    q0, s0 = fk.quantize_rows(x)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        q1, s1 = fk.quantize_rows(x)
    side.synchronize()
    torch.cuda.synchronize()
    assert torch.equal(q0, q1) and torch.equal(s0.view(torch.int32), s1.view(torch.int32))


def test_on_device_guard(cuda):
    import torch
    ext = wf("_ext")
    cur = torch.cuda.current_device()
    with ext.on_device(torch.device("cuda", cur)):
        assert torch.cuda.current_device() == cur
    if torch.cuda.device_count() > 1:
        other = (cur + 1) % torch.cuda.device_count()
        with ext.on_device(other):
            assert torch.cuda.current_device() == other
        assert torch.cuda.current_device() == cur
