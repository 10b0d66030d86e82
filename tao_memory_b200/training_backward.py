"""Backward of tao_attention through libtao_b200.so (tao_train_backward)."""

import ctypes

import torch

from . import _lib

_BF16 = torch.bfloat16


class _Grads(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("dq", "dk", "dv", "d_raw_q", "d_raw_k", "d_fusion_a",
                                             "d_fusion_b", "d_local", "gn", "d_rq_f", "gd", "row_dot",
                                             "dC", "dz", "dc_partial", "dq_acc")]


def backward(ctx, grad):
    from .training import _Buffers
    saved = dict(zip(("q", "k", "v", "raw_q", "raw_k", "fa", "fb", "gain", "out") + ctx.names,
                     ctx.saved_tensors))
    q = saved["q"]
    b, t, h, d = q.shape
    dev = q.device
    grad = grad.to(_BF16).contiguous()
    s = saved["fine_c"].shape[2] if t > 768 else 1
    e = lambda: torch.empty_like(q)
    gr = dict(dq=e(), dk=e(), dv=e(), d_raw_q=e(), d_raw_k=torch.zeros_like(q),
              d_fusion_a=torch.zeros(h, d, 3, dtype=torch.float32, device=dev),
              d_fusion_b=torch.zeros(h, d, 3, dtype=torch.float32, device=dev),
              d_local=e(), gn=e(), d_rq_f=e(),
              gd=torch.empty(b, t, h, dtype=torch.float32, device=dev),
              row_dot=torch.empty(b, h, t, dtype=torch.float32, device=dev),
              dC=torch.empty(b, h, s, d, d, dtype=torch.float32, device=dev),
              dz=torch.zeros(b, h, s, d, dtype=torch.float32, device=dev),
              dc_partial=torch.zeros(b, h, max(1, _lib.lib().tao_train_pairs(t)), d, d, dtype=_BF16,
                                     device=dev),
              dq_acc=torch.empty(b, t, h, d, dtype=torch.float32, device=dev))
    gdesc = _Grads(*(gr[n].data_ptr() for n, _ in _Grads._fields_))
    sdesc = _Buffers(*(saved[n].data_ptr() for n in ("local", "lse", "fine_z", "fine_c", "page_prefix",
                                                    "num", "den", "sel", "err")),
                     saved["sel"].shape[-1], 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(_lib.lib().tao_train_backward(
        grad.data_ptr(), *(saved[n].data_ptr() for n in ("q", "k", "v", "raw_q", "raw_k", "fa", "fb", "gain")),
        b, t, h, d, saved["out"].data_ptr(), ctypes.byref(sdesc), ctypes.byref(gdesc), stream))
    # parameter gradients: the reference sums bf16 products in fp32 and rounds once
    dfa = gr["d_fusion_a"].to(_BF16)
    dfb = gr["d_fusion_b"].to(_BF16)
    return gr["dq"], gr["dk"], gr["dv"], gr["d_raw_q"], gr["d_raw_k"], dfa, dfb, None
