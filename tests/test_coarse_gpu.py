"""The coarse value branch (coarse_index_only=False, the historical TaoConfig()
default) on the GPU.

Completed pages carry a coarse matrix C_page = bf16(sum_s w_s * C_s) built when the
page closes (tao_stream.py:486-500); every query reads all completed pages'
matrices through the softmax over completed pages (tao_stream.py:299-305); the
fusion gains its coarse term and the local bias becomes log 2 (operator.py:21-39,
fusion_pointwise.py:10-92).  Checked against the reference's own outputs (golden
produced by tests/golden/make_golden.py under TaoConfig()), the oracle at other
sizes with page closes inside prefill chunks and inside decode, a reference-made
snapshot imported and continued, and graph decode against eager decode; in
training, forward and backward against the reference golden and the oracle.
Tolerance (bf16): |a-b| <= 2e-2 + 2e-2|b| for every element, routes exact (training:
queries whose selection differs at a proven near-tie are exempt, tests/_parity.py);
gradients rel-L2 <= 2e-2.
"""
import os

import pytest
import torch

from oracle import tao_oracle as o
from oracle.inputs import make_inputs
from _parity import assert_close
from test_stream_gpu import GOLDEN, KEYS, run_gpu

pytestmark = pytest.mark.gpu


def _config(graph=False):
    from tao_memory_b200 import TaoConfig
    return TaoConfig(q1_history_region_graph=graph)


def _oracle(x, layer, chunks, alpha):
    st = o.OracleStream(layer, coarse_index_only=False)
    outs, ids, pos = [], [], 0
    for n in chunks:
        sl = slice(pos, pos + n)
        outs.append(st.step(*(x[k][:, sl] for k in KEYS), x["fusion_a"], x["fusion_b"], alpha))
        if n == 1:
            ids.append(st.route_ids[1].clone())
        pos += n
    return torch.cat(outs, 1), ids, st


def test_coarse_stream_matches_reference_golden(one_thread):
    g = torch.load(os.path.join(GOLDEN, "stream_coarse.pt"), weights_only=False)
    from tao_memory_b200 import TaoConfig
    heads, width, layer, splits, steps, seed = g["case"]
    assert g["config"]["coarse_index_only"] is False
    x, _ = make_inputs(1, sum(splits) + steps, heads, width, seed)
    out, ids, st, _ = run_gpu(x, layer, splits, steps, g["alpha"], config=TaoConfig(**g["config"]))
    stride = g["row_stride"]
    assert_close(out[:, ::stride], g["output"], "coarse golden")
    assert_close(out[:, -steps:], g["decode_output"], "coarse golden decode")
    for i, (a, b) in enumerate(zip(ids, g["decode_route_ids"])):
        assert torch.equal(a, b), f"decode step {i}"
    snap, ref = st.export(), g["snapshot_final"]
    assert len(snap["pages"]) == len(ref["pages"]) >= 2
    for (pz, pc, fz), (rpz, rpc, rfz) in zip(snap["pages"], ref["pages"]):
        assert_close(pz, rpz, "page z")
        assert_close(fz, rfz, "fine z")
        assert_close(pc, rpc, "page matrix")


@pytest.mark.parametrize("heads,width,layer,splits,steps", [
    (3, 64, 2, (2000, 2550), 80),     # page 0 closes inside a prefill chunk, page 1 inside decode (4607)
    (2, 128, 5, (2700,), 40),
])
def test_coarse_stream_matches_oracle(heads, width, layer, splits, steps, one_thread):
    x, _ = make_inputs(1, sum(splits) + steps, heads, width, seed=33 + layer)
    out, ids, st, _ = run_gpu(x, layer, splits, steps, 0.45, config=_config())
    ref, ref_ids, orc = _oracle(x, layer, list(splits) + [1] * steps, 0.45)
    assert_close(out, ref, f"coarse h{heads} d{width}")
    assert all(torch.equal(a, b) for a, b in zip(ids, ref_ids))
    snap = st.export()
    assert len(snap["pages"]) == len(orc.page_c)
    for (_, pc, _), rpc in zip(snap["pages"], orc.page_c):
        assert_close(pc, rpc, "page matrix")


def test_coarse_snapshot_from_the_reference_continues_like_the_oracle(one_thread):
    import tao_memory_b200 as tb
    from tao_memory_b200 import StreamCache
    from tao_memory_b200.stream import check_device
    g = torch.load(os.path.join(GOLDEN, "stream_coarse.pt"), weights_only=False)
    heads, width, layer, splits, steps, seed = g["case"]
    total = sum(splits) + steps
    x, _ = make_inputs(1, total + 200, heads, width, seed)
    dev = torch.device("cuda")
    xs = {k: t.to(dev) for k, t in x.items()}
    kw = dict(fusion_a=xs["fusion_a"], fusion_b=xs["fusion_b"], alpha=g["alpha"])
    st = StreamCache.from_export(g["snapshot_final"], device=dev)     # produced by the reference
    orc = o.OracleStream.from_export(g["snapshot_final"])
    assert not orc.coarse_index_only and orc.page_c
    pos = total
    for n in [150] + [1] * 50:      # a prefill chunk, then decode across the seal at 5119
        sl = slice(pos, pos + n)
        call = tb.tao_attention_prefill if n > 1 else tb.tao_attention_decode
        mine, st = call(*(xs[k][:, sl] for k in KEYS[:3]), raw_q=xs["raw_q"][:, sl], raw_k=xs["raw_k"][:, sl],
                        state=st, position=pos, **kw)
        ref = orc.step(*(x[k][:, sl] for k in KEYS), x["fusion_a"], x["fusion_b"], g["alpha"])
        assert_close(mine, ref, f"continued at {pos}")
        pos += n
    assert check_device() == 0
    assert st.export()["fine_seal_events"] == orc.state_version


def test_coarse_graph_decode_equals_eager(monkeypatch):
    """Graph decode (one captured step, route/seal/page-close decided on the device)
    equals eager decode bit for bit across a page close (position 2559) and a
    fine-bank growth."""
    import tao_memory_b200 as tb
    from tao_memory_b200 import stream
    from tao_memory_b200.stream import check_device
    monkeypatch.setattr(stream, "MIN_CAP", 8)
    dev = torch.device("cuda")
    H, D, P, N = 2, 64, 2300, 600
    x = {k: t.to(dev) for k, t in make_inputs(1, P + N, H, D, seed=78)[0].items()}
    kw = dict(fusion_a=x["fusion_a"], fusion_b=x["fusion_b"], alpha=0.35)
    outs, states = {}, {}
    for graph in (False, True):
        st = tb.new_state(1, _config(graph))
        got = [tb.tao_attention_prefill(*(x[k][:, :P] for k in KEYS[:3]), raw_q=x["raw_q"][:, :P],
                                        raw_k=x["raw_k"][:, :P], state=st, position=0, **kw)[0]]
        for t in range(P, P + N):
            sl = slice(t, t + 1)
            got.append(tb.tao_attention_decode(*(x[k][:, sl] for k in KEYS[:3]), raw_q=x["raw_q"][:, sl],
                                               raw_k=x["raw_k"][:, sl], state=st, position=t, **kw)[0])
        outs[graph], states[graph] = torch.cat(got, 1), st
    assert check_device() == 0
    assert states[True]._graph is not None and states[True].cap_fines > 8
    assert torch.equal(outs[False], outs[True])
    ea, eb = states[False].export(), states[True].export()
    assert len(ea["pages"]) == 1
    assert torch.equal(ea["pages"][0][1], eb["pages"][0][1])
    assert torch.equal(ea["packed_fine_c"], eb["packed_fine_c"])


def _train(x, alpha, grad, config):
    import tao_memory_b200 as tb
    leaves = {k: t.cuda().requires_grad_(True) for k, t in x.items()}
    out = tb.tao_attention(*(leaves[k] for k in KEYS[:3]), raw_q=leaves["raw_q"], raw_k=leaves["raw_k"],
                           fusion_a=leaves["fusion_a"], fusion_b=leaves["fusion_b"], alpha=alpha, config=config)
    out.backward(grad.cuda())
    return out.detach().cpu(), {k: leaves[k].grad.cpu() for k in leaves}


def _check_training(x, alpha, out, grads, ref_out, ref_grads, what, stride=1):
    from test_train_gpu import selections
    from _parity import training_route_flips
    heads = list(range(x["q"].shape[2]))
    flipped, _, problems = training_route_flips(selections(x, alpha), o.training_routes(
        x["raw_q"], x["raw_k"], x["v"]), heads)
    assert not problems, problems[:5]
    assert_close(out[:, ::stride], ref_out, what, exempt=flipped[:, ::stride])
    for k, r in ref_grads.items():
        mine = grads[k][:, ::stride] if k in KEYS else grads[k]
        rel = ((mine.float() - r.float()).norm() / r.float().norm().clamp_min(1e-30)).item()
        assert rel <= 2e-2, (what, k, rel)


def test_coarse_training_matches_reference_golden(one_thread):
    from tao_memory_b200 import TaoConfig
    g = torch.load(os.path.join(GOLDEN, "train_coarse.pt"), weights_only=False)
    b, t, h, d, alpha, seed = g["case"]
    assert g["config"]["coarse_index_only"] is False
    x, gen = make_inputs(b, t, h, d, seed)
    grad = torch.randn(b, t, h, d, generator=gen).to(torch.bfloat16)
    out, grads = _train(x, alpha, grad, TaoConfig(**g["config"]))
    _check_training(x, alpha, out, grads, g["output"], g["grads"], "coarse training golden", g["row_stride"])


def test_coarse_training_matches_oracle(one_thread):
    """Two batch rows, two heads with their own alpha, T = 5376 (two complete pages
    at the last tiles), forward and backward against the oracle."""
    b, t, h, d, alpha = 2, 5376, 2, 64, [0.3, 0.8]
    x, gen = make_inputs(b, t, h, d, seed=57)
    grad = torch.randn(b, t, h, d, generator=gen).to(torch.bfloat16)
    out, grads = _train(x, alpha, grad, _config())
    leaves = {k: v.clone().requires_grad_(True) for k, v in x.items()}
    ref = o.tao_attention(*(leaves[k] for k in KEYS), leaves["fusion_a"], leaves["fusion_b"], alpha,
                          coarse_index_only=False)
    ref.backward(grad)
    _check_training(x, alpha, out, grads, ref.detach(), {k: v.grad for k, v in leaves.items()},
                    "coarse training vs oracle")
