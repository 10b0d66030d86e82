"""Training with the feature-read fine writers (feature-mass, structured-Gram) on the
GPU.

* The tcgen05 feature read itself (tao_feature_read_forward / _backward) on given
  raw_q, z, C and selections against the oracle's feature read and its adjoints
  (the reference's rounding points, tests/golden pinned): outputs within bf16
  tolerance |a-b| <= 2e-2 + 2e-2|b| for every element, d raw_q / dz / dC rel-L2 <=
  1e-2.
* tao_attention end to end against the reference's goldens (TaoConfig with the
  writer, made by tests/golden/make_golden.py) and against the oracle at other
  shapes: outputs within the bf16 tolerance, gradients rel-L2 <= 2e-2.
"""
import os

import pytest
import torch

from oracle import tao_oracle as o
from oracle.inputs import make_inputs
from _parity import assert_close

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
KEYS = ("q", "k", "v", "raw_q", "raw_k")


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def _random_selection(b, t, h, mmax, gen):
    """Selections as the routing makes them: query t of tile (t // 256) >= 3 picks
    min(mmax, V) distinct fines among V = tile - 2 (-1 padded); earlier tiles none."""
    sel = torch.full((b, t, h, mmax), -1, dtype=torch.int16)
    for tile in range(3, (t + 255) // 256):
        v = tile - 2
        m = min(mmax, v)
        for q in range(tile * 256, min(t, tile * 256 + 256)):
            for bb in range(b):
                for hh in range(h):
                    sel[bb, q, hh, :m] = torch.randperm(v, generator=gen)[:m].to(torch.int16)
    return sel


@pytest.mark.parametrize("width,tokens,mmax", [(64, 2304, 5), (128, 1800, 4)])
def test_feature_read_kernels_match_oracle(width, tokens, mmax, one_thread):
    from tao_memory_b200 import _lib
    b, h = 2, 2
    s = tokens // 256 - 1
    gen = torch.Generator().manual_seed(width + tokens)
    raw_q = torch.randn(b, tokens, h, width, generator=gen).to(torch.bfloat16)
    z = (torch.randn(b, h, s, width, generator=gen) * 0.5 + 3.0).to(torch.bfloat16)
    c = (torch.randn(b, h, s, width, width, generator=gen) * 0.3).to(torch.bfloat16)
    sel = _random_selection(b, tokens, h, mmax, gen)
    grad = torch.randn(b, tokens, h, width, generator=gen).to(torch.bfloat16)
    # oracle: the feature read of every query with its selections, and the adjoints
    leaves = {"raw_q": raw_q.clone().requires_grad_(True), "z": z.clone().requires_grad_(True),
              "c": c.clone().requires_grad_(True)}
    hq = torch.softmax(leaves["raw_q"].float(), dim=-1).to(torch.bfloat16)
    first = 3 * 256
    ids = sel[:, first:].long()
    parts = []
    for tile in range(3, (tokens + 255) // 256):
        lo, hi = tile * 256 - first, min(tokens, tile * 256 + 256) - first
        mt = min(mmax, tile - 2)
        idt = ids[:, lo:hi, :, :mt]
        # expand + gather as the reference: the adjoint sums the queries in fp32
        sel_z = leaves["z"][:, None].expand(-1, hi - lo, -1, -1, -1).gather(
            3, idt.unsqueeze(-1).expand(-1, -1, -1, -1, width))
        parts.append(o.feature_read(hq[:, first + lo:first + hi], sel_z, idt, leaves["c"]))
    ref = torch.cat([torch.zeros(b, first, h, width, dtype=torch.bfloat16)] + parts, 1)
    ref.backward(grad)
    # the library's kernels
    dev = torch.device("cuda")
    d = {k: t.to(dev).contiguous() for k, t in (("raw_q", raw_q), ("z", z), ("c", c), ("sel", sel),
                                                ("g", grad))}
    out = torch.empty(b, tokens, h, width, dtype=torch.bfloat16, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.tao_feature_read_forward(d["raw_q"].data_ptr(), d["z"].data_ptr(), d["c"].data_ptr(),
                                            d["sel"].data_ptr(), b, tokens, h, width, mmax, out.data_ptr(),
                                            err.data_ptr(), stream))
    d_raw_q = torch.empty_like(out)
    dz = torch.zeros(b, h, s, width, dtype=torch.float32, device=dev)
    dc = torch.zeros(b, h, s, width, width, dtype=torch.float32, device=dev)
    _lib.check(lib.tao_feature_read_backward(d["g"].data_ptr(), d["raw_q"].data_ptr(), d["z"].data_ptr(),
                                             d["c"].data_ptr(), d["sel"].data_ptr(), b, tokens, h, width, mmax,
                                             d_raw_q.data_ptr(), dz.data_ptr(), dc.data_ptr(), err.data_ptr(),
                                             stream))
    torch.cuda.synchronize()
    assert err.item() == 0
    assert_close(out, ref.detach(), f"feature read d{width}")
    assert _rel(d_raw_q, leaves["raw_q"].grad) <= 1e-2
    assert _rel(dz.to(torch.bfloat16), leaves["z"].grad) <= 1e-2
    assert _rel(dc.to(torch.bfloat16), leaves["c"].grad) <= 1e-2


def _train(x, alpha, grad, writer):
    import tao_memory_b200 as tb
    from tao_memory_b200.presets import index_only_page_memo
    config = tb.TaoConfig(**{**index_only_page_memo().export(), "fine_writer": writer})
    leaves = {k: t.cuda().requires_grad_(True) for k, t in x.items()}
    out = tb.tao_attention(*(leaves[k] for k in KEYS[:3]), raw_q=leaves["raw_q"], raw_k=leaves["raw_k"],
                           fusion_a=leaves["fusion_a"], fusion_b=leaves["fusion_b"], alpha=alpha, config=config)
    out.backward(grad.cuda())
    return out.detach().cpu(), {k: leaves[k].grad.cpu() for k in leaves}


def _check(out, grads, ref_out, ref_grads, what, stride=1):
    assert_close(out[:, ::stride], ref_out, what)
    for k, r in ref_grads.items():
        mine = grads[k][:, ::stride] if k in KEYS else grads[k]
        rel = _rel(mine, r)
        assert rel <= 2e-2, (what, k, rel)


@pytest.mark.parametrize("name", ["train_feature_mass", "train_structured_gram"])
def test_feature_training_matches_reference_golden(name, one_thread):
    g = torch.load(os.path.join(GOLDEN, name + ".pt"), weights_only=False)
    b, t, h, d, alpha, seed = g["case"]
    x, gen = make_inputs(b, t, h, d, seed)
    grad = torch.randn(b, t, h, d, generator=gen).to(torch.bfloat16)
    out, grads = _train(x, alpha, grad, g["config"]["fine_writer"])
    _check(out, grads, g["output"], g["grads"], name, g.get("row_stride", 1))


@pytest.mark.parametrize("writer,b,t,h,d,alpha", [
    ("feature_mass_association", 2, 3328, 2, 64, [0.3, 0.7]),
    ("structured_gram_association", 1, 2304, 1, 128, 0.5),
])
def test_feature_training_matches_oracle(writer, b, t, h, d, alpha, one_thread):
    x, gen = make_inputs(b, t, h, d, seed=61 + d)
    grad = torch.randn(b, t, h, d, generator=gen).to(torch.bfloat16)
    out, grads = _train(x, alpha, grad, writer)
    leaves = {k: v.clone().requires_grad_(True) for k, v in x.items()}
    ref = o.tao_attention(*(leaves[k] for k in KEYS), leaves["fusion_a"], leaves["fusion_b"], alpha, writer)
    ref.backward(grad)
    _check(out, grads, ref.detach(), {k: v.grad for k, v in leaves.items()}, f"{writer} vs oracle")
