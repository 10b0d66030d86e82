"""``tao_attention`` with the feature-read fine writers (``feature_mass_association``
and ``structured_gram_association``) on the index-only preset.

Reference: _seal_training_all (tao_stream.py:87-106) seals every complete block but
the last with u = bf16(fp32 softmax of raw_k) and the fp32 statistics Gram = u^T u,
X = u^T v and mass = sum_t u; z = bf16(log mass), C = the unchecked regularised
solve of (Gram, X) (feature-mass) or the structured inverse of (diag Gram, X, mass)
(structured-Gram).  _training_metadata (tao_stream.py:538-549) gives each page prefix
z = bf16(log of the fp32 mass summed in fine order).  _read_training_group
(tao_stream.py:600-601, 658-661) routes as for every writer and reads the selected
fines with the feature-mass coefficients and no denominator; the pointwise gate fuses
local and fine (operator.py:21-39).

Device work: the writer statistics (``tao_writer_stats``, tensor cores), the local
attention and the routing (``tao_train_forward`` with TAO_TRAIN_ROUTE_ONLY), the
feature read and its adjoints (``tao_feature_read_forward`` / ``_backward``,
tcgen05); the solve of the 256-token blocks runs in torch.linalg and the page
prefixes, the gate and the statistics' adjoints (batched GEMMs) are torch
operations on the device, all under torch autograd.
"""

import ctypes

import torch

from . import _lib
from .training import _Buffers, _geometry

_BF16 = torch.bfloat16
FINE, GROUP = 256, 8
TAO_TRAIN_ROUTE_ONLY = 4   # TaoTrainBuffers.flags (include/tao_b200.h)


def _blocks(x, s):
    """[B,T,H,D] -> the S sealed 256-token blocks [B,S,H,256,D] (a view's copy)."""
    b, _, h, d = x.shape
    return x[:, :s * FINE].reshape(b, s, FINE, h, d).permute(0, 1, 3, 2, 4)


class _WriterStats(torch.autograd.Function):
    """Statistics of the sealed blocks: Gram, X [B,H,S,D,D] and mass [B,H,S,D], fp32
    (association_statistics with mass, association_writer.py:11-18).  Forward on the
    tensor cores; backward: du = u (dG + dG^T) + v dX^T + d mass, then the bf16
    rounding of u and the fp32 softmax backward (d raw_k), and dv = u dX."""

    @staticmethod
    def forward(ctx, raw_k, v, s):
        b, t, h, d = raw_k.shape
        dev = raw_k.device
        gram = torch.empty(b, s, h, d, d, dtype=torch.float32, device=dev)
        cross = torch.empty_like(gram)
        mass = torch.empty(b, s, h, d, dtype=torch.float32, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        for i in range(b):
            _lib.check(_lib.lib().tao_writer_stats(raw_k[i].data_ptr(), v[i].data_ptr(), h * d, d, FINE * h * d, s,
                                                   h, d, gram[i].data_ptr(), cross[i].data_ptr(),
                                                   mass[i].data_ptr(), stream))
        ctx.save_for_backward(raw_k, v)
        ctx.s = s
        return gram.permute(0, 2, 1, 3, 4), cross.permute(0, 2, 1, 3, 4), mass.permute(0, 2, 1, 3)

    @staticmethod
    def backward(ctx, d_gram, d_cross, d_mass):
        raw_k, v = ctx.saved_tensors
        s = ctx.s
        y = _blocks(raw_k, s).float().softmax(dim=-1)               # [B,S,H,256,D] fp32
        u = y.to(_BF16).float()
        vals = _blocks(v, s).float()
        du = torch.zeros_like(u)
        if d_gram is not None:
            g = d_gram.permute(0, 2, 1, 3, 4)
            du = du + u @ (g + g.transpose(-1, -2))
        dv = None
        if d_cross is not None:
            x = d_cross.permute(0, 2, 1, 3, 4)
            du = du + vals @ x.transpose(-1, -2)
            dv = u @ x
        if d_mass is not None:
            du = du + d_mass.permute(0, 2, 1, 3).unsqueeze(-2)
        dy = du.to(_BF16).float()                                    # u = bf16(y): the cast's adjoint
        dk = y * (dy - (dy * y).sum(-1, keepdim=True))
        b, t, h, d = raw_k.shape
        d_raw_k = torch.zeros_like(raw_k)
        d_raw_k[:, :s * FINE] = dk.permute(0, 1, 3, 2, 4).reshape(b, s * FINE, h, d).to(_BF16)
        d_v = torch.zeros_like(v)
        if dv is not None:
            d_v[:, :s * FINE] = dv.permute(0, 1, 3, 2, 4).reshape(b, s * FINE, h, d).to(_BF16)
        return d_raw_k, d_v, None


def _association_matrix(gram, cross):
    """association_matrix(unchecked=True) (association_writer.py:21-32)."""
    d = gram.shape[-1]
    reg = gram.diagonal(dim1=-2, dim2=-1).sum(-1) / d
    system = gram + reg[..., None, None] * torch.eye(d, dtype=torch.float32, device=gram.device)
    factor, _ = torch.linalg.cholesky_ex(system, upper=False, check_errors=False)
    return torch.cholesky_solve(cross, factor).to(_BF16)


def _structured_matrix(square, cross, mass, count):
    """structured_matrix (structured_writer.py:17-34), fp32 in the reference's order."""
    var = (square - mass * mass / count).clamp_min(0)
    var_sum = var.sum(-1, keepdim=True)
    ridge = square.sum(-1, keepdim=True) / mass.shape[-1]
    diag = var + ridge
    t0 = var / diag
    flat = var_sum == 0
    t = torch.where(flat, torch.zeros_like(t0), t0)
    pos = (var * ridge / diag).sum(-1, keepdim=True)
    norm = torch.where(flat, torch.ones_like(pos), pos)
    tx = (t.unsqueeze(-1) * cross).sum(-2)
    hx = cross / diag.unsqueeze(-1) + t.unsqueeze(-1) * tx.unsqueeze(-2) / norm.unsqueeze(-1)
    hm = mass / diag + t * (t * mass).sum(-1, keepdim=True) / norm
    mhx = (mass.unsqueeze(-1) * hx).sum(-2)
    den = count + (mass * hm).sum(-1, keepdim=True)
    return (hx - hm.unsqueeze(-1) * mhx.unsqueeze(-2) / den.unsqueeze(-1)).to(_BF16)


def _page_prefixes(mass, pages):
    """[B,H,pages,8,D] bf16: entry (p, n-1) = bf16(log of the mass of the page's first
    n fines, summed one fine after another in fp32) (tao_stream.py:538-549)."""
    b, h, s, d = mass.shape
    padded = torch.ones(b, h, pages * GROUP, d, dtype=torch.float32, device=mass.device)
    padded[:, :, :s] = mass
    m = padded.reshape(b, h, pages, GROUP, d)
    out = torch.empty(b, h, pages, GROUP, d, dtype=_BF16, device=mass.device)
    acc = m[:, :, :, 0]
    out[:, :, :, 0] = acc.log().to(_BF16)
    for i in range(1, GROUP):
        acc = acc + m[:, :, :, i]
        out[:, :, :, i] = acc.log().to(_BF16)
    return out


class _FeatureCore(torch.autograd.Function):
    """Local attention and feature read: (local, fine).  z and C carry the writer's
    gradient back to the statistics; the page prefixes only steer the routing."""

    @staticmethod
    def forward(ctx, q, k, v, raw_q, z, c, page_prefix, fa, fb, gain):
        b, t, h, d = q.shape
        dev = q.device
        _, _, mmax = _geometry(t)
        one = lambda dtype: torch.empty(1, dtype=dtype, device=dev)
        bufs = dict(local=torch.empty_like(q), lse=torch.empty(b, h, t, dtype=torch.float32, device=dev),
                    fine_z=z.contiguous(), fine_c=c.contiguous(), page_prefix=page_prefix.contiguous(),
                    num=one(_BF16), den=torch.empty(b, t, h, dtype=torch.float32, device=dev),
                    sel=torch.empty(b, t, h, mmax, dtype=torch.int16, device=dev),
                    err=torch.zeros(1, dtype=torch.int32, device=dev))
        desc = _Buffers(*(bufs[n].data_ptr() for n in ("local", "lse", "fine_z", "fine_c", "page_prefix",
                                                       "num", "den", "sel", "err")), mmax, TAO_TRAIN_ROUTE_ONLY)
        stream = torch.cuda.current_stream(dev).cuda_stream
        lib = _lib.lib()
        _lib.check(lib.tao_train_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), raw_q.data_ptr(),
                                         raw_q.data_ptr(), fa.data_ptr(), fb.data_ptr(), gain.data_ptr(), b, t, h,
                                         d, bufs["num"].data_ptr(), ctypes.byref(desc), stream))
        fine = torch.empty_like(q)
        _lib.check(lib.tao_feature_read_forward(raw_q.data_ptr(), bufs["fine_z"].data_ptr(),
                                                bufs["fine_c"].data_ptr(), bufs["sel"].data_ptr(), b, t, h, d,
                                                mmax, fine.data_ptr(), bufs["err"].data_ptr(), stream))
        ctx.save_for_backward(q, k, v, raw_q, fa, fb, gain, *bufs.values())
        ctx.names = tuple(bufs)
        ctx.mmax = mmax
        return bufs["local"], fine

    @staticmethod
    def backward(ctx, d_local, d_fine):
        from .training_backward import _Grads
        saved = dict(zip(("q", "k", "v", "raw_q", "fa", "fb", "gain") + ctx.names, ctx.saved_tensors))
        q = saved["q"]
        b, t, h, d = q.shape
        dev = q.device
        lib = _lib.lib()
        stream = torch.cuda.current_stream(dev).cuda_stream
        d_local = torch.zeros_like(q) if d_local is None else d_local.to(_BF16).contiguous()
        d_fine = torch.zeros_like(q) if d_fine is None else d_fine.to(_BF16).contiguous()
        e = lambda: torch.empty_like(q)
        one = lambda dtype: torch.empty(1, dtype=dtype, device=dev)
        gr = dict(dq=e(), dk=e(), dv=e(), d_raw_q=e(), d_raw_k=e(),
                  d_fusion_a=torch.zeros(h, d, 3, dtype=torch.float32, device=dev),
                  d_fusion_b=torch.zeros(h, d, 3, dtype=torch.float32, device=dev),
                  d_local=d_local, gn=e(), d_rq_f=e(),
                  gd=torch.empty(b, t, h, dtype=torch.float32, device=dev),
                  row_dot=torch.empty(b, h, t, dtype=torch.float32, device=dev),
                  dC=one(torch.float32), dz=one(torch.float32), dc_partial=one(_BF16),
                  dq_acc=torch.empty(b, t, h, d, dtype=torch.float32, device=dev))
        gdesc = _Grads(*(gr[n].data_ptr() for n, _ in _Grads._fields_))
        sdesc = _Buffers(*(saved[n].data_ptr() for n in ("local", "lse", "fine_z", "fine_c", "page_prefix",
                                                        "num", "den", "sel", "err")), ctx.mmax, TAO_TRAIN_ROUTE_ONLY)
        _lib.check(lib.tao_train_backward(
            d_local.data_ptr(), *(saved[n].data_ptr() for n in ("q", "k", "v", "raw_q", "raw_q", "fa", "fb", "gain")),
            b, t, h, d, d_local.data_ptr(), ctypes.byref(sdesc), ctypes.byref(gdesc), stream))
        z, c = saved["fine_z"], saved["fine_c"]
        d_raw_q = torch.empty_like(q)
        dz = torch.zeros(z.shape, dtype=torch.float32, device=dev)
        dc = torch.zeros(c.shape, dtype=torch.float32, device=dev)
        _lib.check(lib.tao_feature_read_backward(d_fine.data_ptr(), saved["raw_q"].data_ptr(), z.data_ptr(),
                                                 c.data_ptr(), saved["sel"].data_ptr(), b, t, h, d, ctx.mmax,
                                                 d_raw_q.data_ptr(), dz.data_ptr(), dc.data_ptr(),
                                                 saved["err"].data_ptr(), stream))
        return (gr["dq"], gr["dk"], gr["dv"], d_raw_q, dz.to(_BF16), dc.to(_BF16), None, None, None, None)


def tao_attention_feature(q, k, v, raw_q, raw_k, fusion_a, fusion_b, gain, writer):
    """tao_attention for the feature-read writers; gain [H] fp32 = bf16(2 * alpha_h).
    Sequences of at most 768 tokens have no sealed fine: the caller serves them with
    the softmax path (the output is the local attention either way)."""
    from .training_coarse import fuse
    b, t, h, d = q.shape
    s, pages, _ = _geometry(t)
    gram, cross, mass = _WriterStats.apply(raw_k, v, s)
    if writer == "structured_gram_association":
        c = _structured_matrix(gram.diagonal(dim1=-2, dim2=-1), cross, mass, FINE)
    else:
        c = _association_matrix(gram, cross)
    z = mass.log().to(_BF16)
    prefix = _page_prefixes(mass.detach(), pages)
    fa = fusion_a.detach().to(_BF16).contiguous()
    fb = fusion_b.detach().to(_BF16).contiguous()
    local, fine = _FeatureCore.apply(q, k, v, raw_q, z, c, prefix, fa, fb, gain)
    return fuse(local, raw_q, torch.zeros_like(local), fine, fusion_a, fusion_b, gain, with_coarse=False)


__all__ = ["tao_attention_feature"]
