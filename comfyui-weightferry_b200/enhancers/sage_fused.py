"""RMSNorm-128 + split-half RoPE of the self-attention's q / k (the ``_rope_rows`` / ``rms_rope`` / ``rope_ok`` part
of enhancers/sage_fused.py of the reference, :159-176, :246-334) on the sm_100a kernel wf_rms_rope128 (wf_rms_rope128_pair for q and k in one launch).

The reference reproduces comfy_kitchen's rms_rope_split_half (lane t of 32 owns values t, t+32, t+64, t+96; the
squares summed by fma; rsqrt.approx; n = bf16((x * rr) * w); pairs (d, d + 64) rotated by a 2x2 float32 matrix per
token and frequency with nvcc's fma contraction). The SageAttention quantisers of that file are attention-side work
for an sm89 kernel and are not part of the weight path."""

import torch

from .. import _ext


def rope_ok(q, k, f, q_scale, k_scale, eps=1e-6):
    """The case the kernel covers: contiguous bf16 (batch, tokens, heads, 128) q and k of the same shape, float32
    rotations (1, tokens, 1, 64, 2, 2) on q's device, 128-value scales of one dtype (bf16 / fp16 / fp32)."""
    if f is None or q.dim() != 4:
        return False
    b, L, h, d = q.shape
    return bool(d == 128 and q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and k.shape == q.shape
                and q.is_contiguous() and k.is_contiguous() and q.is_cuda and f.dtype == torch.float32
                and f.dim() == 6 and tuple(f.shape) == (1, L, 1, 64, 2, 2) and f.device == q.device
                and all(s is not None and s.dim() == 1 and s.shape[0] == 128 and s.is_contiguous()
                        and s.device == q.device and s.dtype in (torch.bfloat16, torch.float16, torch.float32)
                        for s in (q_scale, k_scale))
                and q_scale.dtype == k_scale.dtype)


def rms_rope(x, f, w, eps):
    """comfy_kitchen's rms_rope_split_half for one of q / k (rope_ok's case): bf16 out, same bits as the
    reference's reproduction."""
    b, L, h, d = x.shape
    out = torch.empty_like(x)
    with _ext.on_device(x.device):
        rc = _ext.lib().wf_rms_rope128(x.data_ptr(), f.data_ptr(), f.stride(1), f.stride(3), f.stride(4), f.stride(5),
                                       w.data_ptr(), _ext.dtype_code(w.dtype), out.data_ptr(), b, L, h, float(eps),
                                       _ext.stream_of(x.device))
    _ext.check(rc, "wf_rms_rope128")
    return out


def rms_rope_pair(q, k, f, q_scale, k_scale, eps):
    """(rms_rope(q), rms_rope(k)): the self-attention's q and k after their norms and the 3D RoPE -- one launch for
    both when they have one shape and their scales one dtype (rope_ok's case), else one launch each."""
    if q.shape != k.shape or q_scale.dtype != k_scale.dtype or q.device != k.device:
        return rms_rope(q, f, q_scale, eps), rms_rope(k, f, k_scale, eps)
    b, L, h, d = q.shape
    qo, ko = torch.empty_like(q), torch.empty_like(k)
    with _ext.on_device(q.device):
        rc = _ext.lib().wf_rms_rope128_pair(q.data_ptr(), k.data_ptr(), f.data_ptr(), f.stride(1), f.stride(3),
                                            f.stride(4), f.stride(5), q_scale.data_ptr(), k_scale.data_ptr(),
                                            _ext.dtype_code(q_scale.dtype), qo.data_ptr(), ko.data_ptr(), b, L, h,
                                            float(eps), _ext.stream_of(q.device))
    _ext.check(rc, "wf_rms_rope128_pair")
    return qo, ko
