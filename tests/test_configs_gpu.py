"""Parity at the shapes of the streaming workloads of the measurement plan.

* Streaming inference: a 16,384-token prompt through ``tao_attention_prefill`` then
  512 ``tao_attention_decode`` steps, batch 1, H=12, D=64, page memo on, graph=True
  (the whole-step decode graph).
* Mixed-length serving decode: 64 requests with prompt lengths log-uniform in
  2K-128K, H=16, D=128, 128 steps decoded together through
  ``tao_attention_decode_batch``, every state exported and imported after step 64.

The GPU runs every head; heads are independent in the algorithm (routing, pages and
reads are per head), so the CPU oracle checks a subset of heads against the same
inputs sliced to those heads.  Tolerance (bf16 outputs): |a-b| <= 2e-2 + 2e-2*|b| per
element, for every element; routing selections exact at every decode step.
"""
import math

import pytest
import torch

from oracle import tao_oracle as o
from oracle.inputs import make_inputs
from test_stream_gpu import KEYS
from _parity import assert_close

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
        n = st._download().n_route
        ids.append(st._buf["route_ids"][:, :n].to(torch.int64).cpu().view(1, 1, H, n))
    out = torch.cat(outs, 1).cpu()
    torch.cuda.synchronize()
    assert check_device() == 0
    assert st._graph is not None            # the decode steps ran as the captured graph
    heads = [0, 7]
    ref, ref_ids, orc = _oracle_run(_heads(x, heads), layer, [P] + [1] * N, alpha)
    assert_close(out[:, :, heads], ref, "16K prompt + 512 graph decodes")
    for i, mine in enumerate(ids):
        assert torch.equal(mine[:, :, heads], ref_ids[1 + i]), f"decode step {i}"
    snap = st.export()
    assert snap["position"] == P + N and snap["fine_seal_events"] == orc.state_version
    assert_close(snap["packed_fine_c"][:, heads], orc.fine_c, "fine bank")


def test_mixed_length_serving_decode_with_midstream_snapshots(one_thread):
    """The serving workload at its full shape: 64 requests with prompt lengths
    log-uniform in 2K-128K, H=16, D=128, 128 decode steps through
    tao_attention_decode_batch, every state exported and imported after decode step
    64.  All requests run on the GPU; the oracle checks one head of four of them
    (the longest and shortest prompts and two others), whose inputs are drawn on
    the CPU and written into that head of the GPU operands."""
    import tao_memory_b200 as tb
    from tao_memory_b200 import StreamCache
    from tao_memory_b200.presets import index_only_page_memo
    from tao_memory_b200.stream import check_device
    R, H, D, N, layer, alpha = 64, 16, 128, 128, 1, 0.6
    g = torch.Generator().manual_seed(71)
    lo, hi = math.log(2048), math.log(131072)
    prompts = [int(round(math.exp(lo + (hi - lo) * torch.rand(1, generator=g).item()))) for _ in range(R)]
    fa = (torch.randn(H, D, 3, generator=g) * 0.02).to(torch.bfloat16)
    fb = (torch.randn(H, D, 3, generator=g) * 0.02).to(torch.bfloat16)
    order = sorted(range(R), key=lambda r: prompts[r])
    checked = {order[-1]: 5, order[0]: 11, order[R // 2]: 0, order[R // 4]: 15}   # request -> head
    dev = torch.device("cuda")
    kw = dict(fusion_a=fa.to(dev), fusion_b=fb.to(dev), alpha=alpha)
    dgen = torch.Generator(device=dev)
    states, prefill_out, decode_in, cpu_x = [], {}, [], {}
    for r, p in enumerate(prompts):
        dgen.manual_seed(1000 + r)
        x = torch.randn(5, 1, p + N, H, D, device=dev, generator=dgen).to(torch.bfloat16)
        if r in checked:
            xc, _ = make_inputs(1, p + N, 1, D, seed=300 + r)
            cpu_x[r] = xc
            for i, k in enumerate(KEYS):
                x[i, :, :, checked[r]] = xc[k][:, :, 0].to(dev)
        st = tb.new_state(layer, index_only_page_memo())
        out, st = tb.tao_attention_prefill(x[0, :, :p], x[1, :, :p], x[2, :, :p], raw_q=x[3, :, :p],
                                           raw_k=x[4, :, :p], state=st, position=0, **kw)
        if r in checked:
            prefill_out[r] = out[:, :, checked[r]].cpu()
        decode_in.append(x[:, :, p:].clone())
        states.append(st)
        del x, out
    decode_in = torch.cat(decode_in, 1)          # [5, R, N, H, D]
    dec = []
    for i in range(N):
        if i == N // 2:   # snapshot every request and continue from the imports
            states = [StreamCache.from_export(st.export()) for st in states]
        step = decode_in[:, :, i:i + 1]
        many, states = tb.tao_attention_decode_batch(step[0], step[1], step[2], raw_q=step[3], raw_k=step[4],
                                                     states=states, **kw)
        dec.append(many.cpu())
    dec = torch.cat(dec, 1)                      # [R, N, H, D]
    assert check_device() == 0
    for r, head in checked.items():
        p = prompts[r]
        x = {**cpu_x[r], "fusion_a": fa[head:head + 1], "fusion_b": fb[head:head + 1]}
        ref, _, orc = _oracle_run(x, layer, [p] + [1] * N, alpha)
        mine = torch.cat([prefill_out[r], dec[r:r + 1, :, head]], 1).unsqueeze(2)
        assert_close(mine, ref, f"request {r} (prompt {p}, head {head})")
        snap = states[r].export()
        assert snap["position"] == p + N
        if orc.route_ids is not None:
            assert torch.equal(snap["route_ids"][1][:, :, [head]].cpu(), orc.route_ids[1])
