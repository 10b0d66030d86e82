"""Model-side neighbours on the GPU: ProjectedInputs (the caller's Q/K/V projection
with the split and RMS norms in one library kernel) against the reference's own torch
composition (examples/common.py:6-20: F.linear, reshape/unbind, F.rms_norm over the
width), forward within one bf16 rounding (|a-b| <= 1e-2 + 1e-2|b|) and gradients of x,
the projection weight and the five outputs' consumers rel-L2 <= 1e-2; then the
reference examples' training step and streaming loop run through the module."""
import pytest
import torch
from torch.nn import functional as F

pytestmark = pytest.mark.gpu


def _reference(x, weight, heads, width):
    projected = F.linear(x, weight.to(x.dtype))
    raw_q, raw_k, v = projected.reshape(*x.shape[:2], 3, heads, width).unbind(2)
    return F.rms_norm(raw_q, (width,)), F.rms_norm(raw_k, (width,)), v, raw_q, raw_k


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("heads,width", [(2, 64), (6, 128)])
def test_projected_inputs_match_the_reference_composition(heads, width):
    from tao_memory_b200.model import ProjectedInputs
    torch.manual_seed(5)
    model = ProjectedInputs(heads, width).cuda()
    x = torch.randn(2, 300, heads * width, device="cuda", dtype=torch.bfloat16)
    xa, xb = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
    w_ref = model.projection.weight.detach().clone().requires_grad_(True)
    mine = model(xa)
    ref = _reference(xb, w_ref, heads, width)
    grads = [torch.randn_like(t) for t in ref]
    for a, b in zip(mine, ref):
        assert a.shape == b.shape and a.is_contiguous()
        bad = (a.float() - b.float()).abs() > 1e-2 + 1e-2 * b.float().abs()
        assert not bad.any(), int(bad.sum())
    torch.autograd.backward(mine, grads)
    torch.autograd.backward(ref, grads)
    assert _rel(xa.grad, xb.grad) <= 1e-2
    assert _rel(model.projection.weight.grad, w_ref.grad) <= 1e-2


def test_reference_examples_run_through_the_module():
    """examples/train.py (one update) and examples/stream.py (prefill, decode,
    snapshot) with this package in place of the reference's."""
    import tao_memory_b200 as tb
    from tao_memory_b200.model import ProjectedInputs
    from tao_memory_b200.presets import index_only_page_memo
    torch.manual_seed(42)
    model = ProjectedInputs().cuda()
    optimizer = torch.optim.AdamW(model.parameters(), lr=1e-3)
    x = torch.randn(1, 1024, 128, device="cuda", dtype=torch.bfloat16)
    q, k, v, raw_q, raw_k = model(x)
    heads = tb.tao_attention(q, k, v, raw_q=raw_q, raw_k=raw_k, fusion_a=model.fusion_a,
                             fusion_b=model.fusion_b, alpha=0.1, config=index_only_page_memo())
    loss = heads.float().square().mean()
    loss.backward()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in model.parameters())
    optimizer.step()

    model = ProjectedInputs(heads=6, width=128).cuda().eval()
    state = tb.new_state(0, index_only_page_memo(graph=True))
    with torch.inference_mode():
        x = torch.randn(1, 2112, 768, device="cuda", dtype=torch.bfloat16)
        for start in range(0, 2048, 256):
            q, k, v, raw_q, raw_k = model(x[:, start:start + 256])
            out, state = tb.tao_attention_prefill(q, k, v, raw_q=raw_q, raw_k=raw_k, fusion_a=model.fusion_a,
                                                  fusion_b=model.fusion_b, alpha=0.1, state=state,
                                                  position=state.get_pos())
        for index in range(2048, 2112):
            q, k, v, raw_q, raw_k = model(x[:, index:index + 1])
            out, state = tb.tao_attention_decode(q, k, v, raw_q=raw_q, raw_k=raw_k, fusion_a=model.fusion_a,
                                                 fusion_b=model.fusion_b, alpha=0.1, state=state,
                                                 position=state.get_pos())
        restored = tb.StreamCache.from_export(state.export())
    assert state.get_pos() == restored.get_pos() == 2112 and out.shape == (1, 1, 6, 128)
    assert torch.isfinite(out.float()).all()
