"""Coarse value branch of ``tao_attention`` in training (TaoConfig with
coarse_index_only=False, the historical default).

The library computes the exact local attention and the routed fine read as in
the index-only preset, but returns them unfused (TAO_TRAIN_EXTERNAL_FUSION): the
three-term pointwise gate needs the coarse read, which every query takes over
all completed pages.  The coarse branch and the gate are composed here from
torch operations on the device, following the reference's formulas and rounding
points:

* fine matrices and log-partitions of the completed pages' blocks, the softmax
  writer (tao_stream.py:80-123, 66-76);
* per completed page: page_z = bf16 logsumexp over its 8 fines and
  C_page = bf16(sum_s bf16(exp(bf16(z_s - page_z))) * C_s)
  (_training_metadata, tao_stream.py:552-573);
* per 256-query tile with `completed` pages: coarse = bf16(sum_p sum_d
  bf16(h * softmax_p(page_z)) * C_page) (_read_training_group,
  tao_stream.py:611-617), h = bf16 softmax of raw_q;
* the fusion with coarse present from position 512 + 8 * 256 on
  (_fuse_training, operator.py:21-39, 52).

Gradients of the coarse branch flow back through torch autograd into raw_q,
raw_k and v and are added to the library's (which cover the local attention,
the fine read and the library's writer).
"""

import torch
import torch.nn.functional as F

_BF16 = torch.bfloat16
FINE, GROUP, FIRST_COARSE, FIRST_FINE = 256, 8, 512 + 8 * 256, 768
TAO_TRAIN_EXTERNAL_FUSION = 2   # TaoTrainBuffers.flags (include/tao_b200.h)


class _LocalAndFine(torch.autograd.Function):
    """The library's local attention and fine read, unfused: (local, fine)."""

    @staticmethod
    def forward(ctx, q, k, v, raw_q, raw_k, fa, fb, gain):
        from .training import _forward
        fine, bufs = _forward(q, k, v, raw_q, raw_k, fa, fb, gain, flags=TAO_TRAIN_EXTERNAL_FUSION)
        ctx.save_for_backward(q, k, v, raw_q, raw_k, fa, fb, gain, fine, *bufs.values())
        ctx.names = tuple(bufs)
        ctx.writer = "softmax"
        ctx.external = True
        return bufs["local"], fine

    @staticmethod
    def backward(ctx, d_local, d_fine):
        from .training_backward import backward
        q = ctx.saved_tensors[0]
        d_local = torch.zeros_like(q) if d_local is None else d_local.to(_BF16).contiguous()
        d_fine = torch.zeros_like(q) if d_fine is None else d_fine.to(_BF16).contiguous()
        grads = backward(ctx, d_fine, d_local=d_local)
        return grads[:5] + (None, None, None)


def _seal_pages(raw_k, v, pages):
    """Softmax writer over the first pages * 8 blocks: z [B,H,S,D], C [B,H,S,D,D]."""
    b, _, heads, d = raw_k.shape
    s = pages * GROUP
    keys = raw_k[:, :s * FINE].reshape(b, s, FINE, heads, d)
    values = v[:, :s * FINE].reshape(b, s, FINE, heads, d)
    maximum = keys.amax(dim=2, keepdim=True)
    exponent = (keys - maximum).exp().to(_BF16)
    partition = exponent.sum(dim=2, keepdim=True).to(_BF16)
    prob = (exponent / partition).to(_BF16)
    z = (maximum.squeeze(2) + partition.squeeze(2).log()).to(_BF16).permute(0, 2, 1, 3)
    c = torch.einsum("bsihd,bsihe->bhsde", prob, values).to(_BF16)
    return z, c


def coarse_read(raw_q, raw_k, v):
    """Coarse value read of every query [B,T,H,D] (zero before the first complete page)."""
    b, t, heads, d = raw_q.shape
    sealed = t // FINE - 1 if t > FIRST_FINE else 0
    pages = sealed // GROUP
    coarse = torch.zeros_like(raw_q)
    if pages == 0:
        return coarse
    z, c = _seal_pages(raw_k, v, pages)
    zp = z.reshape(b, heads, pages, GROUP, d)
    page_z = torch.logsumexp(zp, dim=3).to(_BF16)                               # [B,H,P,D]
    weight = (zp - page_z.unsqueeze(3)).exp().to(_BF16)
    page_c = torch.einsum("bhpsd,bhpsde->bhpde", weight,
                          c.reshape(b, heads, pages, GROUP, d, d)).to(_BF16)      # [B,H,P,D,D]
    parts = []
    for completed in range(1, pages + 1):
        # tiles whose visible fines (tile - 2) span `completed` full pages
        first = max(GROUP * completed + 2, 0) * FINE
        last = min((GROUP * (completed + 1) + 2) * FINE, t)
        if first >= last:
            continue
        q = raw_q[:, first:last]
        h = F.softmax(q, dim=-1).to(_BF16)
        cw = F.softmax(page_z[:, :, :completed], dim=2).to(_BF16)
        chv = (h.unsqueeze(3) * cw[:, None]).to(_BF16)
        parts.append((first, last, torch.einsum("bthpd,bhpde->bthe", chv, page_c[:, :, :completed]).to(_BF16)))
    pieces = [coarse[:, :parts[0][0]]] + [p for _, _, p in parts]
    return torch.cat(pieces, dim=1)


def fuse(local, raw_q, coarse, fine, fusion_a, fusion_b, gains, with_coarse=True):
    """Three-term pointwise gate (operator.py:21-39); gains [H] = bf16(2 * alpha_h).
    with_coarse=False: index-only pages (the coarse term is absent everywhere)."""
    t = raw_q.shape[1]
    pos = torch.arange(t, device=raw_q.device)[None, :, None, None]
    fine_present = pos >= FIRST_FINE
    coarse_present = (pos >= FIRST_COARSE) & with_coarse
    score = (fusion_a.to(_BF16) * raw_q.unsqueeze(-1)).to(_BF16)
    score = (score + fusion_b.to(_BF16)).to(_BF16)
    count = coarse_present.to(torch.int32) + fine_present.to(torch.int32)
    local_bias = count.clamp_min(1).to(_BF16).log().to(_BF16)
    score = torch.stack(((score[..., 0] + local_bias).to(_BF16), score[..., 1], score[..., 2]), dim=-1)
    score = torch.stack((score[..., 0], score[..., 1].masked_fill(~coarse_present, -torch.inf),
                         score[..., 2].masked_fill(~fine_present, -torch.inf)), dim=-1)
    rho = F.softmax(score, dim=-1).to(_BF16)
    gain = gains.to(_BF16).view(1, 1, -1, 1)
    local_term = (rho[..., 0] * (2 * local).to(_BF16)).to(_BF16)
    coarse_term = (rho[..., 1] * (gain * coarse).to(_BF16)).to(_BF16)
    fine_term = (rho[..., 2] * (gain * fine).to(_BF16)).to(_BF16)
    fused = ((local_term + coarse_term).to(_BF16) + fine_term).to(_BF16)
    return torch.where(coarse_present | fine_present, fused, local)


def tao_attention_coarse(q, k, v, raw_q, raw_k, fusion_a, fusion_b, gains):
    """tao_attention with coarse_index_only=False (softmax writer); gains [H] float32."""
    local, fine = _LocalAndFine.apply(q, k, v, raw_q, raw_k, fusion_a.detach().to(_BF16).contiguous(),
                                      fusion_b.detach().to(_BF16).contiguous(), gains)
    coarse = coarse_read(raw_q, raw_k, v)
    return fuse(local, raw_q, coarse, fine, fusion_a, fusion_b, gains)


__all__ = ["tao_attention_coarse", "coarse_read", "fuse"]
