"""Parity at the shapes of the streaming workloads of the measurement plan.

* Streaming inference: a 16,384-token prompt through ``tao_attention_prefill`` then
  512 ``tao_attention_decode`` steps, batch 1, H=12, D=64, page memo on, graph=True
  (the whole-step decode graph).
* Mixed-length serving decode: requests with prompt lengths log-uniform in 2K-16K
  (the workload's range is 2K-128K; the oracle bounds it here), H=16, D=128, decoded
  together through ``tao_attention_decode_batch``, every state exported and imported
  mid-stream.

The GPU runs every head; heads are independent in the algorithm (routing, pages and
reads are per head), so the CPU oracle checks a subset of heads against the same
inputs sliced to those heads.  Tolerance (bf16 outputs): |a-b| <= 2e-2 + 2e-2*|b| per
element, at most 1e-4 of the elements outside it; routing selections exact.
"""
import math

import pytest
import torch

from oracle import tao_oracle as o
from oracle.inputs import make_inputs
from test_stream_gpu import KEYS, close_frac

pytestmark = pytest.mark.gpu


def _heads(x, heads):
    """The inputs of a subset of heads (token tensors and fusion parameters)."""
    return {k: (t[:, :, heads] if t.dim() == 4 else t[heads]) for k, t in x.items()}


def _oracle_run(x, layer, chunks, alpha):
    st = o.OracleStream(layer)
    outs, ids, pos = [], [], 0
    for n in chunks:
        sl = slice(pos, pos + n)
        outs.append(st.step(*(x[k][:, sl] for k in KEYS), x["fusion_a"], x["fusion_b"], alpha))
        ids.append(None if st.route_ids is None else st.route_ids[1].clone())
        pos += n
    return torch.cat(outs, 1), ids, st


def test_streaming_inference_16k_prompt_512_decodes_graph(one_thread):
    import tao_memory_b200 as tb
    from tao_memory_b200.presets import index_only_page_memo
    from tao_memory_b200.stream import check_device
    H, D, P, N, layer, alpha = 12, 64, 16384, 512, 3, 0.4
    x, _ = make_inputs(1, P + N, H, D, seed=61)
    dev = torch.device("cuda")
    xs = {k: t.to(dev) for k, t in x.items()}
    kw = dict(fusion_a=xs["fusion_a"], fusion_b=xs["fusion_b"], alpha=alpha)
    st = tb.new_state(layer, index_only_page_memo(graph=True))
    out, st = tb.tao_attention_prefill(*(xs[k][:, :P] for k in KEYS[:3]), raw_q=xs["raw_q"][:, :P],
                                       raw_k=xs["raw_k"][:, :P], state=st, position=0, **kw)
    outs, ids = [out], []
    for t in range(P, P + N):
        sl = slice(t, t + 1)
        o1, st = tb.tao_attention_decode(*(xs[k][:, sl] for k in KEYS[:3]), raw_q=xs["raw_q"][:, sl],
                                         raw_k=xs["raw_k"][:, sl], state=st, position=t, **kw)
        outs.append(o1)
        ids.append(st.export()["route_ids"][1].cpu() if t % 37 == 0 else None)
    out = torch.cat(outs, 1).cpu()
    torch.cuda.synchronize()
    assert check_device() == 0
    assert st._graph is not None            # the decode steps ran as the captured graph
    heads = [0, 7]
    ref, ref_ids, orc = _oracle_run(_heads(x, heads), layer, [P] + [1] * N, alpha)
    assert close_frac(out[:, :, heads], ref) <= 1e-4
    for i, mine in enumerate(ids):
        if mine is not None:
            assert torch.equal(mine[:, :, heads], ref_ids[1 + i]), f"decode step {i}"
    snap = st.export()
    assert snap["position"] == P + N and snap["fine_seal_events"] == orc.state_version
    assert close_frac(snap["packed_fine_c"][:, heads], orc.fine_c) == 0.0


def test_mixed_length_serving_decode_with_midstream_snapshots(one_thread):
    import tao_memory_b200 as tb
    from tao_memory_b200 import StreamCache
    from tao_memory_b200.presets import index_only_page_memo
    from tao_memory_b200.stream import check_device
    R, H, D, N, layer, alpha = 5, 16, 128, 48, 1, 0.6
    g = torch.Generator().manual_seed(71)
    lo, hi = math.log(2048), math.log(16384)
    prompts = [int(math.exp(lo + (hi - lo) * torch.rand(1, generator=g).item())) for _ in range(R)]
    xs_cpu = [make_inputs(1, p + N, H, D, seed=80 + r)[0] for r, p in enumerate(prompts)]
    fa, fb = xs_cpu[0]["fusion_a"], xs_cpu[0]["fusion_b"]   # one layer's parameters for every request
    dev = torch.device("cuda")
    xs = [{k: t.to(dev) for k, t in x.items()} for x in xs_cpu]
    kw = dict(fusion_a=fa.to(dev), fusion_b=fb.to(dev), alpha=alpha)
    states, prefill_out = [], []
    for r, p in enumerate(prompts):
        st = tb.new_state(layer, index_only_page_memo())
        out, st = tb.tao_attention_prefill(*(xs[r][k][:, :p] for k in KEYS[:3]), raw_q=xs[r]["raw_q"][:, :p],
                                           raw_k=xs[r]["raw_k"][:, :p], state=st, position=0, **kw)
        states.append(st)
        prefill_out.append(out.cpu())
    dec = [[] for _ in range(R)]
    for i in range(N):
        if i == N // 2:   # snapshot every request and continue from the imports
            states = [StreamCache.from_export(st.export()) for st in states]
        stack = {k: torch.cat([xs[r][k][:, prompts[r] + i:prompts[r] + i + 1] for r in range(R)], 0)
                 for k in KEYS}
        many, states = tb.tao_attention_decode_batch(*(stack[k] for k in KEYS[:3]), raw_q=stack["raw_q"],
                                                     raw_k=stack["raw_k"], states=states, **kw)
        for r in range(R):
            dec[r].append(many[r:r + 1].cpu())
    torch.cuda.synchronize()
    assert check_device() == 0
    for r, p in enumerate(prompts):
        head = [(3 * r) % H]
        x = _heads({**xs_cpu[r], "fusion_a": fa, "fusion_b": fb}, head)
        ref, _, orc = _oracle_run(x, layer, [p] + [1] * N, alpha)
        mine = torch.cat([prefill_out[r]] + dec[r], 1)[:, :, head]
        assert close_frac(mine, ref) <= 1e-4, f"request {r} (prompt {p})"
        snap = states[r].export()
        assert snap["position"] == p + N
        if orc.route_ids is not None:
            assert torch.equal(snap["route_ids"][1][:, :, head].cpu(), orc.route_ids[1])
