"""Backward of tao_attention through libtao_b200.so (tao_train_backward)."""

import ctypes

import torch

from . import _lib

_BF16 = torch.bfloat16


class _Grads(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("dq", "dk", "dv", "d_raw_q", "d_raw_k", "d_fusion_a",
                                             "d_fusion_b", "d_local", "gn", "d_rq_f", "gd", "row_dot",
                                             "dC", "dz", "dc_partial", "dq_acc")]


def _regularized_backward(saved, gr, s):
    """C path of fine_writer="regularized_association": the library returned dC
    (fp32 sum of the per-tile bf16 partials) and the z path; differentiate
    C = association_matrix(association_statistics(raw_k, v)) per sealed block
    (association_writer.py:11-32 under tao_stream.py:113-117): the statistics come
    from the library's writer-statistics kernel with their explicit adjoint
    (training_feature._WriterStats), torch autograd runs through the regularised
    Cholesky solve only; the result is added to d raw_k and dv in bf16."""
    from .training_feature import _WriterStats
    raw_k, v = saved["raw_k"], saved["v"]
    d = raw_k.shape[-1]
    with torch.enable_grad():
        kb = raw_k.detach().requires_grad_(True)
        vb = v.detach().requires_grad_(True)
        gram, cross, _ = _WriterStats.apply(kb, vb, s)
        reg = gram.diagonal(dim1=-2, dim2=-1).sum(-1) / d
        system = gram + reg[..., None, None] * torch.eye(d, dtype=torch.float32, device=raw_k.device)
        c = torch.cholesky_solve(cross, torch.linalg.cholesky(system)).to(_BF16)
        dk, dv = torch.autograd.grad(c, (kb, vb), gr["dC"].to(_BF16))
    gr["d_raw_k"] += dk
    gr["dv"] += dv


def backward(ctx, grad, d_local=None):
    """grad: gradient of the fused output, or with ctx.external of the unfused fine
    output; d_local: the caller's gradient of the local output (external fusion)."""
    from .training import _Buffers
    saved = dict(zip(("q", "k", "v", "raw_q", "raw_k", "fa", "fb", "gain", "out") + ctx.names,
                     ctx.saved_tensors))
    q = saved["q"]
    b, t, h, d = q.shape
    dev = q.device
    grad = grad.to(_BF16).contiguous()
    s = saved["fine_c"].shape[2] if t > 768 else 1
    e = lambda: torch.empty_like(q)
    gr = dict(dq=e(), dk=e(), dv=e(), d_raw_q=e(), d_raw_k=e(),
              d_fusion_a=torch.zeros(h, d, 3, dtype=torch.float32, device=dev),
              d_fusion_b=torch.zeros(h, d, 3, dtype=torch.float32, device=dev),
              d_local=e() if d_local is None else d_local, gn=e(), d_rq_f=e(),
              gd=torch.empty(b, t, h, dtype=torch.float32, device=dev),
              row_dot=torch.empty(b, h, t, dtype=torch.float32, device=dev),
              dC=torch.empty(b, h, s, d, d, dtype=torch.float32, device=dev),
              dz=torch.zeros(b, h, s, d, dtype=torch.float32, device=dev),
              dc_partial=torch.empty(b, h, max(1, _lib.lib().tao_train_pairs(t)), d, d, dtype=_BF16,
                                     device=dev),
              dq_acc=torch.empty(b, t, h, d, dtype=torch.float32, device=dev))
    gdesc = _Grads(*(gr[n].data_ptr() for n, _ in _Grads._fields_))
    caller_c = ctx.writer != "softmax" and t > 768
    from .training import TAO_TRAIN_CALLER_FINE_C
    from .training_coarse import TAO_TRAIN_EXTERNAL_FUSION
    flags = (TAO_TRAIN_CALLER_FINE_C if caller_c else 0) | (TAO_TRAIN_EXTERNAL_FUSION if ctx.external else 0)
    sdesc = _Buffers(*(saved[n].data_ptr() for n in ("local", "lse", "fine_z", "fine_c", "page_prefix",
                                                    "num", "den", "sel", "err")),
                     saved["sel"].shape[-1], flags)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(_lib.lib().tao_train_backward(
        grad.data_ptr(), *(saved[n].data_ptr() for n in ("q", "k", "v", "raw_q", "raw_k", "fa", "fb", "gain")),
        b, t, h, d, saved["out"].data_ptr(), ctypes.byref(sdesc), ctypes.byref(gdesc), stream))
    if caller_c:
        _regularized_backward(saved, gr, s)
    # parameter gradients: the reference sums bf16 products in fp32 and rounds once
    dfa = gr["d_fusion_a"].to(_BF16)
    dfb = gr["d_fusion_b"].to(_BF16)
    return gr["dq"], gr["dk"], gr["dv"], gr["d_raw_q"], gr["d_raw_k"], dfa, dfb, None, None
