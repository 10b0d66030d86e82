"""Parity at the full sizes of the benchmark workloads.

* Long-context decode (the decode benchmark's shape): a 131,072-token context,
  H=12, D=64, bf16, then 280 decode steps, so the window seals a block at position
  131,327 and the routes refresh a dozen times inside the decoded span.
* Training forward + backward at B4 T8192 H12 D64 bf16 (the training benchmark's
  shape), per-head alpha, with the routing selections of every query compared.

The library runs every head; heads are independent in the algorithm (routing,
pages, reads and fusion parameters are per head), so the CPU oracle checks a
subset of heads on the same inputs sliced to those heads.  Tolerance (bf16):
|a-b| <= 2e-2 + 2e-2|b| for every element; routing selections exact, except
queries whose selections differ at a proven near-tie of the oracle's scores
(tests/_parity.py), which are counted and exempted from the output check.
"""
import pytest
import torch

from oracle import tao_oracle as o
from oracle.inputs import make_inputs
from _parity import assert_close, training_route_flips, out_of_tolerance

pytestmark = pytest.mark.gpu
KEYS = ("q", "k", "v", "raw_q", "raw_k")


def _heads(x, heads):
    return {k: (t[:, :, heads] if t.dim() == 4 else t[heads]) for k, t in x.items()}


def _route_ids(st):
    """Selected fine ids of a library state in rank order, [H, M] int64 (no clone of the bank)."""
    n = st._download().n_route
    return st._buf["route_ids"][:, :n].to(torch.int64).cpu()


def test_decode_at_128k_context_across_a_seal(one_thread):
    import tao_memory_b200 as tb
    from tao_memory_b200.presets import index_only_page_memo
    from tao_memory_b200.stream import check_device, is_refresh, window_start
    H, D, P, N, layer, alpha = 12, 64, 131072, 280, 0, 0.5
    x, _ = make_inputs(1, P + N, H, D, seed=64)
    dev = torch.device("cuda")
    xs = {k: t.to(dev) for k, t in x.items()}
    kw = dict(fusion_a=xs["fusion_a"], fusion_b=xs["fusion_b"], alpha=alpha)
    st = tb.new_state(layer, index_only_page_memo(graph=True))
    pos = 0
    while pos < P:                       # the prompt in 16K pieces, as a server would feed it
        n = min(16384, P - pos)
        sl = slice(pos, pos + n)
        tb.tao_attention_prefill(*(xs[k][:, sl] for k in KEYS[:3]), raw_q=xs["raw_q"][:, sl],
                                 raw_k=xs["raw_k"][:, sl], state=st, position=pos, **kw)
        pos += n
    outs, ids = [], []
    for t in range(P, P + N):
        sl = slice(t, t + 1)
        y, st = tb.tao_attention_decode(*(xs[k][:, sl] for k in KEYS[:3]), raw_q=xs["raw_q"][:, sl],
                                        raw_k=xs["raw_k"][:, sl], state=st, position=t, **kw)
        outs.append(y)
        ids.append(_route_ids(st))
    out = torch.cat(outs, 1).cpu()
    assert check_device() == 0
    assert st._graph is not None
    seal = next(t for t in range(P, P + N) if t + 1 - window_start(t) == 768)
    assert seal == 131327
    assert sum(is_refresh(t, layer, st.config) for t in range(P, P + N)) >= 10

    heads = [0, 7]
    ref_x = _heads(x, heads)
    orc = o.OracleStream(layer)
    pos = 0
    while pos < P:
        n = min(16384, P - pos)
        orc.step(*(ref_x[k][:, pos:pos + n] for k in KEYS), ref_x["fusion_a"], ref_x["fusion_b"], alpha)
        pos += n
    ref, ref_ids = [], []
    for t in range(P, P + N):
        sl = slice(t, t + 1)
        ref.append(orc.step(*(ref_x[k][:, sl] for k in KEYS), ref_x["fusion_a"], ref_x["fusion_b"], alpha))
        ref_ids.append(orc.route_ids[1][0, 0].clone())
    ref = torch.cat(ref, 1)
    bad_steps = [i for i, (a, b) in enumerate(zip(ids, ref_ids)) if not torch.equal(a[heads], b)]
    assert not bad_steps, f"routes differ at decode steps {bad_steps[:8]}"
    assert_close(out[:, :, heads], ref, "decode output at 128K")
    snap = st.export()
    assert snap["fine_seal_events"] == orc.state_version == 511
    assert_close(snap["packed_fine_c"][:, heads][:, :, -1], orc.fine_c[:, :, -1], "fine sealed at 131327")


def test_training_full_config_selections_outputs_and_gradients(one_thread):
    import tao_memory_b200 as tb
    from tao_memory_b200 import training
    from tao_memory_b200.presets import index_only_page_memo
    B, T, H, D = 4, 8192, 12, 64
    x, gen = make_inputs(B, T, H, D, seed=2)
    alpha = torch.rand(H, generator=gen).tolist()
    grad = torch.randn(B, T, H, D, generator=gen).to(torch.bfloat16)
    dev = torch.device("cuda")
    leaves = {k: t.to(dev).requires_grad_(True) for k, t in x.items()}
    out = tb.tao_attention(*(leaves[k] for k in KEYS[:3]), raw_q=leaves["raw_q"], raw_k=leaves["raw_k"],
                           fusion_a=leaves["fusion_a"], fusion_b=leaves["fusion_b"], alpha=alpha,
                           config=index_only_page_memo())
    out.backward(grad.to(dev))
    with torch.no_grad():
        gains = training._gains(alpha, H, dev)
        _, bufs = training._forward(*(leaves[k].detach() for k in KEYS), leaves["fusion_a"].detach(),
                                    leaves["fusion_b"].detach(), gains)
    sel = bufs["sel"].cpu()
    out = out.detach().cpu()
    grads = {k: leaves[k].grad.cpu() for k in leaves}

    heads = [0, 11]
    ref_x = _heads(x, heads)
    tiles = o.training_routes(ref_x["raw_q"], ref_x["raw_k"], ref_x["v"])
    flipped, n_flip, problems = training_route_flips(sel, tiles, heads)
    assert not problems, problems[:5]
    assert n_flip <= 1e-3 * B * T * len(heads), n_flip
    ref_leaves = {k: t.clone().requires_grad_(True) for k, t in ref_x.items()}
    ref = o.tao_attention(*(ref_leaves[k] for k in KEYS), ref_leaves["fusion_a"], ref_leaves["fusion_b"],
                          [alpha[h] for h in heads])
    ref.backward(grad[:, :, heads])
    print(f"training selections: {n_flip} of {B * T * len(heads)} queries differ at near-ties; "
          f"outputs out of tolerance at {int(out_of_tolerance(out[:, :, heads], ref.detach()).sum())} elements")
    assert_close(out[:, :, heads], ref.detach(), "training output", exempt=flipped)
    for k, g in ref_leaves.items():
        mine = grads[k][:, :, heads] if g.grad.dim() == 4 else grads[k][heads]
        rel = ((mine.float() - g.grad.float()).norm() / g.grad.float().norm()).item()
        assert rel <= 2e-2, (k, rel)
