"""Windowed causal attention kernel vs the reference's local attention
(tao_stream.py:760-787 through torch SDPA), fp32 oracle on CPU.
Tolerance: bf16 output, |a-b| <= 2e-2 + 2e-2|b|."""
import ctypes

import pytest
import torch

from oracle import tao_oracle as o
from oracle.inputs import make_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("b,t,h,d", [(1, 2048, 2, 64), (2, 1536, 3, 128), (1, 2000, 2, 64), (1, 300, 1, 64)])
def test_window_attention_matches_oracle(b, t, h, d):
    from tao_memory_b200 import _lib
    x, _ = make_inputs(b, t, h, d, seed=5)
    q, k, v = (x[n].cuda() for n in ("q", "k", "v"))
    out = torch.empty_like(q)
    lse = torch.empty(b, h, t, dtype=torch.float32, device="cuda")
    rc = _lib.lib().tao_window_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                         lse.data_ptr(), b, t, h, d,
                                         torch.cuda.current_stream().cuda_stream)
    _lib.check(rc)
    ref = o._local_training(x["q"].float(), x["k"].float(), x["v"].float())
    got = out.float().cpu()
    bad = ((got - ref).abs() > 2e-2 + 2e-2 * ref.abs()).float().mean().item()
    assert bad == 0.0, bad
    # log-sum-exp of scaled scores, checked on a few rows
    for tq in (tq for tq in (0, 255, 700, t - 1) if tq < t):
        start = max(0, 256 * (tq // 256) - 512)
        s = (x["q"][0, tq, 0].float() @ x["k"][0, start:tq + 1, 0].float().T) / d ** 0.5
        assert abs(torch.logsumexp(s, 0).item() - lse[0, 0, tq].item()) < 1e-2
