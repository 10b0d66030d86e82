"""Model-side neighbours of the operator: the caller's fused Q/K/V projection and the
RMS normalisation of the exact-local q and k (reference examples/common.py:6-20,
``ProjectedInputs``), with the same names and semantics.

The projection is a plain GEMM (``F.linear``, cuBLAS); the split into the five
operands and the two RMS norms run in one library kernel forward and one backward
(``tao_qkv_split_norm``), so the operator receives contiguous q, k, v, raw_q and raw_k
without five separate elementwise passes.  Positional transforms stay the caller's.
"""

import torch
from torch import nn
from torch.nn import functional as F

from . import _lib

_BF16 = torch.bfloat16
# F.rms_norm's default eps: the epsilon of its fp32 compute type (also for bf16 inputs)
RMS_EPS = float(torch.finfo(torch.float32).eps)


class _SplitNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, projected, heads, width):
        rows = projected.numel() // (3 * heads * width)
        shape = (*projected.shape[:-1], heads, width)
        outs = [torch.empty(shape, dtype=_BF16, device=projected.device) for _ in range(5)]
        q, k, v, raw_q, raw_k = outs
        stream = torch.cuda.current_stream(projected.device).cuda_stream
        _lib.check(_lib.lib().tao_qkv_split_norm(projected.data_ptr(), rows, heads, width, RMS_EPS, q.data_ptr(),
                                                 k.data_ptr(), v.data_ptr(), raw_q.data_ptr(), raw_k.data_ptr(),
                                                 stream))
        ctx.save_for_backward(raw_q, raw_k)
        ctx.dims = (rows, heads, width, projected.shape)
        return q, k, v, raw_q, raw_k

    @staticmethod
    def backward(ctx, dq, dk, dv, d_raw_q, d_raw_k):
        raw_q, raw_k = ctx.saved_tensors
        rows, heads, width, shape = ctx.dims
        grads = [torch.zeros_like(raw_q) if g is None else g.to(_BF16).contiguous()
                 for g in (dq, dk, dv, d_raw_q, d_raw_k)]
        d_proj = torch.empty(shape, dtype=_BF16, device=raw_q.device)
        stream = torch.cuda.current_stream(raw_q.device).cuda_stream
        _lib.check(_lib.lib().tao_qkv_split_norm_backward(raw_q.data_ptr(), raw_k.data_ptr(),
                                                          *(g.data_ptr() for g in grads), rows, heads, width,
                                                          RMS_EPS, d_proj.data_ptr(), stream))
        return d_proj, None, None


def split_norm(projected, heads, width):
    """[..., 3 * heads * width] bf16 CUDA -> (q, k, v, raw_q, raw_k), each [..., heads, width]."""
    if projected.dtype != _BF16 or not projected.is_cuda:
        raise ValueError("split_norm takes a bf16 CUDA projection (no CPU fallback)")
    if projected.shape[-1] != 3 * heads * width:
        raise ValueError("the projection's last dimension must be 3 * heads * width")
    return _SplitNorm.apply(projected.contiguous(), heads, width)


class ProjectedInputs(nn.Module):
    """Caller-owned projections feeding the operator (examples/common.py:6-20):
    x [B, T, heads * width] -> q, k, v, raw_q, raw_k [B, T, heads, width]; fusion_a and
    fusion_b are the pointwise gate's parameters."""

    def __init__(self, heads=2, width=64):
        super().__init__()
        self.heads, self.width = heads, width
        self.projection = nn.Linear(heads * width, 3 * heads * width, bias=False)
        self.fusion_a = nn.Parameter(torch.zeros(heads, width, 3))
        self.fusion_b = nn.Parameter(torch.zeros(heads, width, 3))

    def forward(self, x):
        projected = F.linear(x, self.projection.weight.to(x.dtype))
        return split_norm(projected, self.heads, self.width)


__all__ = ["ProjectedInputs", "split_norm", "RMS_EPS"]
