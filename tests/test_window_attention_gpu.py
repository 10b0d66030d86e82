"""Windowed causal attention kernel vs the reference's local attention
(tao_stream.py:760-787 through torch SDPA), fp32 oracle on CPU.
Tolerance: bf16 output, |a-b| <= 2e-2 + 2e-2|b|."""
import ctypes

import pytest
import torch

from oracle import tao_oracle as o
from oracle.inputs import make_inputs

pytestmark = pytest.mark.gpu


def _run(q, k, v, variant):
    """tao_window_attention with the given kernel variant (1: tcgen05, 0: mma.sync)."""
    from tao_memory_b200 import _lib
    b, t, h, d = q.shape
    out = torch.empty_like(q)
    lse = torch.empty(b, h, t, dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib().tao_attention_variant(variant))
    try:
        rc = _lib.lib().tao_window_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                             lse.data_ptr(), b, t, h, d,
                                             torch.cuda.current_stream().cuda_stream)
        _lib.check(rc)
        torch.cuda.synchronize()
    finally:
        _lib.lib().tao_attention_variant(1)
    return out, lse


@pytest.mark.parametrize("variant", [1, 0])
@pytest.mark.parametrize("b,t,h,d", [(1, 2048, 2, 64), (2, 1536, 3, 128), (1, 2000, 2, 64), (1, 300, 1, 64),
                                     (3, 1100, 2, 64)])
def test_window_attention_matches_oracle(b, t, h, d, variant):
    x, _ = make_inputs(b, t, h, d, seed=5)
    q, k, v = (x[n].cuda() for n in ("q", "k", "v"))
    out, lse = _run(q, k, v, variant)
    ref = o._local_training(x["q"].float(), x["k"].float(), x["v"].float())
    got = out.float().cpu()
    bad = ((got - ref).abs() > 2e-2 + 2e-2 * ref.abs()).float().mean().item()
    assert bad == 0.0, bad
    # log-sum-exp of scaled scores, checked on a few rows
    for tq in (tq for tq in (0, 255, 700, t - 1) if tq < t):
        start = max(0, 256 * (tq // 256) - 512)
        s = (x["q"][0, tq, 0].float() @ x["k"][0, start:tq + 1, 0].float().T) / d ** 0.5
        assert abs(torch.logsumexp(s, 0).item() - lse[0, 0, tq].item()) < 1e-2


@pytest.mark.parametrize("b,t,h,d", [(1, 8192, 12, 64), (2, 3000, 4, 64), (1, 100, 3, 64), (1, 4096, 6, 128),
                                     (2, 1000, 2, 128)])
def test_tcgen05_matches_mma_sync(b, t, h, d):
    """The tcgen05/TMEM kernel and the mma.sync kernel agree on every row (widths 64 and
    128): outputs to one bf16 rounding (|a-b| <= 1e-2 + 1e-2|b|), log-sum-exp to 1e-3."""
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn(b, t, h, d, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    o1, l1 = _run(q, k, v, 1)
    o0, l0 = _run(q, k, v, 0)
    diff = (o1.float() - o0.float()).abs()
    assert (diff <= 1e-2 + 1e-2 * o0.float().abs()).all(), diff.max().item()
    assert (l1 - l0).abs().max().item() < 1e-3
