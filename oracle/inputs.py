"""Seeded synthetic operands shared by the golden generator, the parity tests and
the CPU baselines (test infrastructure, not product code).

Draw order follows the measurement plan: q, k, v, raw_q, raw_k, fusion_a,
fusion_b, then (training only) alpha per head and the upstream gradient.  All
draws are fp32 from a CPU ``torch.Generator`` and then cast, so the CPU oracle
and the GPU see identical bits.
"""

import hashlib

import torch


def make_inputs(batch, tokens, heads, width, seed=0, dtype=torch.bfloat16,
                fusion_std=0.02):
    g = torch.Generator().manual_seed(seed)
    q, k, v, raw_q, raw_k = (torch.randn(batch, tokens, heads, width, generator=g).to(dtype)
                             for _ in range(5))
    fa = (torch.randn(heads, width, 3, generator=g) * fusion_std).to(dtype)
    fb = (torch.randn(heads, width, 3, generator=g) * fusion_std).to(dtype)
    return dict(q=q, k=k, v=v, raw_q=raw_q, raw_k=raw_k, fusion_a=fa, fusion_b=fb), g


def digest(*tensors):
    """Short content hash, used to detect RNG drift between machines."""
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.detach().contiguous().view(torch.uint8).numpy().tobytes()
                 if t.dtype != torch.bfloat16 else
                 t.detach().contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()[:16]
