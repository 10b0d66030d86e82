"""Differentiable ``tao_attention`` on sm_100a (reference operator.py:42-54,
tao_stream.py:668-787 forward; selected_read.py:156-187 and the surrounding torch
autograd backward).

Every kernel runs in libtao_b200.so; torch provides device memory, streams and
the autograd graph.  Supported envelope: bf16 operands [B, T, H, D] with D in
{64, 128} and the index-only preset (the reference's own training path raises for
fp32 operands, selected_read.py:32, so fp32 is rejected here too).
"""

import ctypes

import torch

from . import _lib
from .stream import check_config

_BF16 = torch.bfloat16
TAO_TRAIN_CALLER_FINE_C = 1   # TaoTrainBuffers.flags (include/tao_b200.h)


class _Buffers(ctypes.Structure):
    _fields_ = [("local", ctypes.c_void_p), ("lse", ctypes.c_void_p), ("fine_z", ctypes.c_void_p),
                ("fine_c", ctypes.c_void_p), ("page_prefix", ctypes.c_void_p), ("num", ctypes.c_void_p),
                ("den", ctypes.c_void_p), ("sel", ctypes.c_void_p), ("err", ctypes.c_void_p),
                ("mmax", ctypes.c_int32), ("flags", ctypes.c_int32)]


def _geometry(tokens):
    s, p, m = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _lib.check(_lib.lib().tao_train_geometry(tokens, ctypes.byref(s), ctypes.byref(p), ctypes.byref(m)))
    return s.value, p.value, m.value


def _gains(alpha, heads, device):
    """gain_h = bf16(2 * alpha_h) (operator.py:34: torch.full((), 2 * alpha, dtype))."""
    if isinstance(alpha, (int, float)):
        vals = [float(alpha)] * heads
    else:
        vals = [float(a) for a in (alpha.tolist() if torch.is_tensor(alpha) else alpha)]
        if len(vals) != heads:
            raise ValueError("per-head alpha needs one value per head")
    g = torch.tensor([2 * a for a in vals], dtype=torch.float64).to(_BF16).float()
    return g.to(device)


def _regularized_matrices(raw_k, v, s):
    """fine_writer="regularized_association": C of the S sealed blocks
    (_seal_training_all, tao_stream.py:113-117): writer statistics on the tensor
    cores (``tao_writer_stats``), the regularised Cholesky solve in torch.linalg
    (association_matrix, association_writer.py:21-32).  Returns bf16 [B,H,S,D,D]."""
    b, t, h, d = raw_k.shape
    dev = raw_k.device
    gram = torch.empty(b, s, h, d, d, dtype=torch.float32, device=dev)
    cross = torch.empty_like(gram)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for i in range(b):
        _lib.check(_lib.lib().tao_writer_stats(raw_k[i].data_ptr(), v[i].data_ptr(), h * d, d, 256 * h * d, s, h, d,
                                               gram[i].data_ptr(), cross[i].data_ptr(), None, stream))
    gram, cross = gram.permute(0, 2, 1, 3, 4), cross.permute(0, 2, 1, 3, 4)
    reg = gram.diagonal(dim1=-2, dim2=-1).sum(-1) / d
    system = gram + reg[..., None, None] * torch.eye(d, dtype=torch.float32, device=dev)
    return torch.cholesky_solve(cross, torch.linalg.cholesky(system)).to(_BF16)


def _forward(q, k, v, raw_q, raw_k, fa, fb, gain, writer="softmax", flags=0):
    b, t, h, d = q.shape
    dev = q.device
    s, pages, mmax = _geometry(t)
    bufs = dict(
        local=torch.empty_like(q), lse=torch.empty(b, h, t, dtype=torch.float32, device=dev),
        fine_z=torch.empty(b, h, max(s, 1), d, dtype=_BF16, device=dev),
        fine_c=torch.empty(b, h, max(s, 1), d, d, dtype=_BF16, device=dev),
        page_prefix=torch.zeros(b, h, max(pages, 1), 8, d, dtype=_BF16, device=dev),
        num=torch.empty_like(q), den=torch.empty(b, t, h, dtype=torch.float32, device=dev),
        sel=torch.empty(b, t, h, mmax, dtype=torch.int16, device=dev),
        err=torch.zeros(1, dtype=torch.int32, device=dev))
    if writer != "softmax" and s > 0:
        bufs["fine_c"].copy_(_regularized_matrices(raw_k, v, s))
        flags |= TAO_TRAIN_CALLER_FINE_C
    desc = _Buffers(*(bufs[n].data_ptr() for n in ("local", "lse", "fine_z", "fine_c", "page_prefix",
                                                   "num", "den", "sel", "err")), mmax, flags)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(_lib.lib().tao_train_forward(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), raw_q.data_ptr(), raw_k.data_ptr(), fa.data_ptr(),
        fb.data_ptr(), gain.data_ptr(), b, t, h, d, out.data_ptr(), ctypes.byref(desc), stream))
    return out, bufs


class _TaoAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, raw_q, raw_k, fa, fb, gain, writer="softmax"):
        out, bufs = _forward(q, k, v, raw_q, raw_k, fa, fb, gain, writer)
        ctx.save_for_backward(q, k, v, raw_q, raw_k, fa, fb, gain, out, *bufs.values())
        ctx.names = tuple(bufs)
        ctx.writer = writer
        ctx.external = False
        return out

    @staticmethod
    def backward(ctx, grad):
        from .training_backward import backward
        return backward(ctx, grad)


def tao_attention_train(q, k, v, raw_q, raw_k, fusion_a, fusion_b, alpha, config):
    check_config(config, training=True)
    ops = (q, k, v, raw_q, raw_k)
    if any(t.dtype != _BF16 for t in ops):
        raise ValueError("tao_attention on B200 takes bf16 operands (the reference's selected read "
                         "needs bf16: Both operands must be same dtype)")
    if any(t.shape != q.shape for t in ops) or q.dim() != 4:
        raise ValueError("q, k, v, raw_q and raw_k must share one [batch, tokens, heads, width] shape")
    if not q.is_cuda:
        raise ValueError("tao_attention on B200 needs CUDA tensors (no CPU fallback)")
    heads, width = q.shape[2], q.shape[3]
    if width not in (64, 128):
        raise ValueError("head width must be 64 or 128")
    if fusion_a.shape != (heads, width, 3) or fusion_b.shape != (heads, width, 3):
        raise ValueError("fusion_a and fusion_b must have shape [heads, width, 3]")
    gain = _gains(alpha, heads, q.device)
    if not config.coarse_index_only:
        from .training_coarse import tao_attention_coarse
        return tao_attention_coarse(*(t.contiguous() for t in ops), fusion_a, fusion_b, gain)
    if config.fine_writer in ("feature_mass_association", "structured_gram_association") and q.shape[1] > 768:
        from .training_feature import tao_attention_feature
        return tao_attention_feature(*(t.contiguous() for t in ops), fusion_a, fusion_b, gain, config.fine_writer)
    fa = fusion_a.to(_BF16)
    fb = fusion_b.to(_BF16)
    writer = "softmax" if config.fine_writer in ("feature_mass_association", "structured_gram_association") \
        else config.fine_writer   # <= 768 tokens: no sealed fine, the output is the local attention
    return _TaoAttention.apply(*(t.contiguous() for t in ops), fa.contiguous(), fb.contiguous(), gain, writer)
