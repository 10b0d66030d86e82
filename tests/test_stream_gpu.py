"""Streaming prefill/decode on the GPU vs the reference goldens and the CPU oracle.

Tolerance (bf16 outputs): |a-b| <= 2e-2 + 2e-2*|b| per element; routing
selections are integers and must match exactly.  A CUDA result is compared with
the reference's own outputs (golden fixtures) and with the oracle at other sizes.
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
ATOL = RTOL = 2e-2


def _tb():
    import tao_memory_b200 as tb
    from tao_memory_b200.presets import index_only_page_memo
    from tao_memory_b200.stream import check_device
    return tb, index_only_page_memo, check_device


def close_frac(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    bad = (a - b).abs() > ATOL + RTOL * b.abs()
    return bad.float().mean().item()


def run_gpu(x, layer, splits, steps, alpha, snapshot_at=None, config=None):
    tb, preset, check_device = _tb()
    dev = torch.device("cuda")
    xs = {k: t.to(dev) for k, t in x.items()}
    st = tb.new_state(layer, preset() if config is None else config)
    outs, ids, pos = [], [], 0
    snap = None
    kw = dict(fusion_a=xs["fusion_a"], fusion_b=xs["fusion_b"], alpha=alpha)
    for n in splits:
        sl = slice(pos, pos + n)
        out, st = tb.tao_attention_prefill(*(xs[k][:, sl] for k in KEYS[:3]), raw_q=xs["raw_q"][:, sl],
                                           raw_k=xs["raw_k"][:, sl], state=st, position=pos, **kw)
        outs.append(out)
        pos += n
    for i in range(steps):
        sl = slice(pos, pos + 1)
        out, st = tb.tao_attention_decode(*(xs[k][:, sl] for k in KEYS[:3]), raw_q=xs["raw_q"][:, sl],
                                          raw_k=xs["raw_k"][:, sl], state=st, position=pos, **kw)
        outs.append(out)
        e = st.export()["route_ids"]
        ids.append(None if e is None else e[1].cpu())
        pos += 1
        if snapshot_at is not None and i + 1 == snapshot_at:
            snap = st.export()
    torch.cuda.synchronize()
    assert check_device() == 0
    return torch.cat(outs, 1), ids, st, snap


@pytest.mark.parametrize("name", ["stream_h2d64", "stream_h1d128", "stream_pages", "stream_regularized",
                                  "stream_feature_mass", "stream_structured_gram"])
def test_stream_matches_reference_golden(name):
    from tao_memory_b200 import TaoConfig
    g = torch.load(os.path.join(GOLDEN, name + ".pt"), weights_only=False)
    heads, width, layer, splits, steps, seed = g["case"]
    x, _ = make_inputs(1, sum(splits) + steps, heads, width, seed)
    config = TaoConfig(**g["config"]) if "config" in g else None
    out, ids, st, _ = run_gpu(x, layer, splits, steps, g["alpha"], config=config)
    stride = g.get("row_stride", 1)
    assert_close(out[:, ::stride], g["output"], name)
    if "decode_output" in g:
        assert_close(out[:, -steps:], g["decode_output"], name + " decode")
    mism = sum(int(not torch.equal(a, b)) for a, b in zip(ids, g["decode_route_ids"]) if b is not None)
    assert mism == 0, f"{mism} decode steps with different routes"
    snap = st.export()
    ref = g["snapshot_final"]
    assert snap["position"] == ref["position"]
    for (pz, _, fz), (rpz, _, rfz) in zip(snap["pages"], ref["pages"]):
        assert_close(pz, rpz, "page z")
        assert_close(fz, rfz, "fine z")
    assert_close(snap["packed_fine_c"], ref["packed_fine_c"], "fine bank")
    # fp32 writer statistics (association writers): u = bf16(softmax) can land on the
    # other side of a bf16 rounding boundary between torch's CPU softmax and the
    # kernel's (a few values per block), so the sums agree to 1e-3 in relative norm
    for key in ("pending_gram", "pending_cross", "pending_mass", "pending_square_mass"):
        assert (snap[key] is None) == (ref[key] is None), key
        if ref[key] is not None:
            err = (snap[key].cpu() - ref[key]).norm() / ref[key].norm()
            assert err <= 1e-3, (key, err.item())


@pytest.mark.parametrize("heads,width,layer,splits,steps", [
    (4, 64, 2, (300, 1500, 1333), 60),
    (3, 128, 5, (2100,), 40),
])
def test_stream_matches_oracle(heads, width, layer, splits, steps, one_thread):
    x, _ = make_inputs(1, sum(splits) + steps, heads, width, seed=11 + layer)
    out, ids, _, _ = run_gpu(x, layer, splits, steps, 0.4)
    st = o.OracleStream(layer)
    ref, ref_ids, pos = [], [], 0
    for n in list(splits) + [1] * steps:
        sl = slice(pos, pos + n)
        ref.append(st.step(*(x[k][:, sl] for k in KEYS), x["fusion_a"], x["fusion_b"], 0.4))
        if n == 1:
            ref_ids.append(st.route_ids[1].clone())
        pos += n
    ref = torch.cat(ref, 1)
    assert_close(out, ref, f"h{heads} d{width} layer {layer}")
    assert sum(int(not torch.equal(a, b)) for a, b in zip(ids, ref_ids)) == 0


@pytest.mark.parametrize("width", [64, 128])
def test_prefill_ring_attention_tcgen05_matches_mma_sync_and_oracle(width, one_thread):
    """The streaming prefill's chunk attention over the ring runs on tcgen05 (attention
    variant 1) or on mma.sync (variant 0): both prefill the same prompt (chunks that
    start mid-tile, fill a window and wrap the ring) to outputs within the bf16
    tolerance of the oracle, with identical routes."""
    from tao_memory_b200 import _lib
    heads, layer = 2, 1
    splits = (300, 500, 1200, 77, 1000)      # 3077 tokens: seals, wraps, ragged chunks
    x, _ = make_inputs(1, sum(splits) + 4, heads, width, seed=70 + width)
    outs = {}
    for variant in (0, 1):
        _lib.check(_lib.lib().tao_attention_variant(variant))
        try:
            outs[variant] = run_gpu(x, layer, splits, 4, 0.4)
        finally:
            _lib.check(_lib.lib().tao_attention_variant(1))
    orc = o.OracleStream(layer)
    ref = torch.cat([orc.step(*(x[k][:, sl] for k in KEYS), x["fusion_a"], x["fusion_b"], 0.4)
                     for sl in [slice(a, a + n) for a, n in zip((0, 300, 800, 2000, 2077), splits)]], 1)
    n = sum(splits)
    for variant in (0, 1):
        assert_close(outs[variant][0][:, :n], ref, f"prefill attention variant {variant} d{width}")
    assert all(torch.equal(a, b) for a, b in zip(outs[0][1], outs[1][1]))
    e0, e1 = outs[0][2].export(), outs[1][2].export()
    assert torch.equal(e0["packed_fine_c"], e1["packed_fine_c"])


@pytest.mark.parametrize("variant", [1, 3, 4, 0, 2])
@pytest.mark.parametrize("width", [64, 128])
def test_decode_kernel_variants_match_oracle(variant, width, one_thread):
    """Every decode kernel of tao_decode_variant against the oracle: 40 decode steps
    after a 3050-token prefill, across route refreshes and the seal at position 3071."""
    from tao_memory_b200 import _lib
    heads, layer, prefill, steps = 2, 1, 3050, 40
    x, _ = make_inputs(1, prefill + steps, heads, width, seed=90 + width)
    _lib.check(_lib.lib().tao_decode_variant(variant))
    try:
        out, ids, st, _ = run_gpu(x, layer, (prefill,), steps, 0.4)
    finally:
        _lib.check(_lib.lib().tao_decode_variant(1))
    orc = o.OracleStream(layer)
    orc.step(*(x[k][:, :prefill] for k in KEYS), x["fusion_a"], x["fusion_b"], 0.4)
    ref, ref_ids = [], []
    for pos in range(prefill, prefill + steps):
        sl = slice(pos, pos + 1)
        ref.append(orc.step(*(x[k][:, sl] for k in KEYS), x["fusion_a"], x["fusion_b"], 0.4))
        ref_ids.append(orc.route_ids[1].clone())
    assert_close(out[:, prefill:], torch.cat(ref, 1), f"decode variant {variant} d{width}")
    assert all(torch.equal(a, b) for a, b in zip(ids, ref_ids))
    assert st.export()["fine_seal_events"] == orc.state_version


def test_batch_decode_equals_single_requests():
    tb, preset, check_device = _tb()
    dev = torch.device("cuda")
    R, H, D, P = 3, 2, 64, 1100
    xs = [make_inputs(1, P + 30, H, D, seed=40 + r)[0] for r in range(R)]
    xs = [{k: t.to(dev) for k, t in x.items()} for x in xs]
    fa, fb = xs[0]["fusion_a"], xs[0]["fusion_b"]
    singles, batch = [], []
    for r in range(R):
        for lst in (singles, batch):
            st = tb.new_state(r, preset())
            tb.tao_attention_prefill(*(xs[r][k][:, :P] for k in KEYS[:3]), raw_q=xs[r]["raw_q"][:, :P],
                                     raw_k=xs[r]["raw_k"][:, :P], fusion_a=fa, fusion_b=fb, alpha=0.3,
                                     state=st, position=0)
            lst.append(st)
    for t in range(P, P + 30):
        sl = slice(t, t + 1)
        one = [tb.tao_attention_decode(*(xs[r][k][:, sl] for k in KEYS[:3]), raw_q=xs[r]["raw_q"][:, sl],
                                       raw_k=xs[r]["raw_k"][:, sl], fusion_a=fa, fusion_b=fb, alpha=0.3,
                                       state=singles[r], position=t)[0] for r in range(R)]
        stack = {k: torch.cat([xs[r][k][:, sl] for r in range(R)], 0) for k in KEYS}
        many, _ = tb.tao_attention_decode_batch(*(stack[k] for k in KEYS[:3]), raw_q=stack["raw_q"],
                                                raw_k=stack["raw_k"], fusion_a=fa, fusion_b=fb,
                                                alpha=0.3, states=batch)
        assert torch.equal(torch.cat(one, 0), many)
    assert check_device() == 0


def test_export_import_roundtrip_and_reference_snapshot(one_thread):
    tb, preset, check_device = _tb()
    from tao_memory_b200 import StreamCache
    dev = torch.device("cuda")
    g = torch.load(os.path.join(GOLDEN, "stream_h2d64.pt"), weights_only=False)
    heads, width, layer, splits, steps, seed = g["case"]
    total = sum(splits) + steps
    x, _ = make_inputs(1, total + 20, heads, width, seed)
    out, _, st, snap = run_gpu({k: t[:, :total] if t.dim() == 4 else t for k, t in x.items()},
                               layer, splits, steps, g["alpha"], snapshot_at=steps)
    xs = {k: t.to(dev) for k, t in x.items()}
    kw = dict(fusion_a=xs["fusion_a"], fusion_b=xs["fusion_b"], alpha=g["alpha"])
    a = StreamCache.from_export(st.export())
    b = StreamCache.from_export(g["snapshot_final"], device=dev)   # produced by the reference
    orc = o.OracleStream.from_export(g["snapshot_final"])
    for t in range(total, total + 20):
        sl = slice(t, t + 1)
        args = [xs[k][:, sl] for k in KEYS[:3]]
        o1, st = tb.tao_attention_decode(*args, raw_q=xs["raw_q"][:, sl], raw_k=xs["raw_k"][:, sl],
                                         state=st, position=t, **kw)
        o2, a = tb.tao_attention_decode(*args, raw_q=xs["raw_q"][:, sl], raw_k=xs["raw_k"][:, sl],
                                        state=a, position=t, **kw)
        o3, b = tb.tao_attention_decode(*args, raw_q=xs["raw_q"][:, sl], raw_k=xs["raw_k"][:, sl],
                                        state=b, position=t, **kw)
        ref = orc.step(*(x[k][:, sl] for k in KEYS), x["fusion_a"], x["fusion_b"], g["alpha"])
        assert torch.equal(o1, o2)
        assert_close(o3, ref, f"decode {t} from the reference snapshot")
    st.reset()
    assert st.get_pos() == 0 and a.get_pos() == total + 20
    assert check_device() == 0


def test_stream_errors():
    tb, preset, _ = _tb()
    dev = torch.device("cuda")
    x, _ = make_inputs(1, 4, 1, 64)
    xs = {k: t.to(dev) for k, t in x.items()}
    st = tb.new_state(0, preset())
    kw = dict(fusion_a=xs["fusion_a"], fusion_b=xs["fusion_b"], alpha=0.5)
    with pytest.raises(ValueError):
        tb.tao_attention_prefill(*(xs[k] for k in KEYS[:3]), raw_q=xs["raw_q"], raw_k=xs["raw_k"],
                                 state=st, position=3, **kw)
    with pytest.raises(ValueError):
        tb.tao_attention_decode(*(xs[k][:, :2] for k in KEYS[:3]), raw_q=xs["raw_q"][:, :2],
                                raw_k=xs["raw_k"][:, :2], state=st, position=0, **kw)
    with pytest.raises(ValueError):
        tb.tao_attention_prefill(*(xs[k].float() for k in KEYS[:3]), raw_q=xs["raw_q"].float(),
                                 raw_k=xs["raw_k"].float(), state=st, position=0, **kw)


def test_graph_decode_equals_eager(monkeypatch):
    """config.q1_history_region_graph: decode replays one captured CUDA graph per
    fine-bank capacity.  Outputs and exported states equal eager decode bit for bit
    across route refreshes, seals and a fine-bank growth (initial capacity lowered to
    8 fines so the growth happens within the test)."""
    tb, preset, check_device = _tb()
    from tao_memory_b200 import stream
    monkeypatch.setattr(stream, "MIN_CAP", 8)
    dev = torch.device("cuda")
    H, D, P, N = 2, 64, 1000, 1700
    x = {k: t.to(dev) for k, t in make_inputs(1, P + N, H, D, seed=77)[0].items()}
    kw = dict(fusion_a=x["fusion_a"], fusion_b=x["fusion_b"], alpha=0.45)
    outs = {}
    states = {}
    for graph in (False, True):
        st = tb.new_state(3, preset(graph=graph))
        got = [tb.tao_attention_prefill(*(x[k][:, :P] for k in KEYS[:3]), raw_q=x["raw_q"][:, :P],
                                        raw_k=x["raw_k"][:, :P], state=st, position=0, **kw)[0]]
        for t in range(P, P + N):
            sl = slice(t, t + 1)
            got.append(tb.tao_attention_decode(*(x[k][:, sl] for k in KEYS[:3]), raw_q=x["raw_q"][:, sl],
                                               raw_k=x["raw_k"][:, sl], state=st, position=t, **kw)[0])
        outs[graph] = torch.cat(got, 1)
        states[graph] = st
    torch.cuda.synchronize()
    assert check_device() == 0
    assert states[True].cap_fines > 8 and states[True]._graph is not None
    assert torch.equal(outs[False], outs[True])
    def same(a, b):
        if isinstance(a, torch.Tensor):
            return torch.equal(a, b)
        if isinstance(a, (list, tuple)):
            return len(a) == len(b) and all(same(u, w) for u, w in zip(a, b))
        if isinstance(a, dict):
            return a.keys() == b.keys() and all(same(a[k], b[k]) for k in a)
        return a == b
    ea, eb = states[False].export(), states[True].export()
    ca, cb = dict(ea.pop("config")), dict(eb.pop("config"))
    assert cb.pop("q1_history_region_graph") and not ca.pop("q1_history_region_graph") and ca == cb
    for key in ea:
        assert same(ea[key], eb[key]), key


def test_writer_stats_match_oracle():
    """tao_writer_stats (u = bf16 channel softmax, G = u^T u, X = u^T v on the tensor
    cores) against the oracle's fp32 restatement of association_statistics; the
    regularised matrix built from them agrees to bf16 rounding.  Tolerances: a few
    u values may round to the neighbouring bf16 value (torch's CPU softmax and the
    kernel's fp32 softmax differ in the last bits), so G and X agree to 1e-4 and
    1e-3 in relative norm."""
    from tao_memory_b200 import _lib
    g = torch.Generator().manual_seed(31)
    for heads, width in ((3, 64), (2, 128)):
        k = torch.randn(1, 256, heads, width, generator=g).to(torch.bfloat16)
        v = torch.randn(1, 256, heads, width, generator=g).to(torch.bfloat16)
        kd, vd = k.cuda(), v.cuda()
        gram = torch.empty(1, heads, width, width, dtype=torch.float32, device="cuda")
        cross = torch.empty_like(gram)
        mass = torch.empty(1, heads, width, dtype=torch.float32, device="cuda")
        _lib.check(_lib.lib().tao_writer_stats(kd.data_ptr(), vd.data_ptr(), heads * width, width, 0, 1, heads,
                                               width, gram.data_ptr(), cross.data_ptr(), mass.data_ptr(),
                                               torch.cuda.current_stream().cuda_stream))
        rg, rx, rm = o.association_statistics(k, v, with_mass=True)
        assert ((gram.cpu() - rg).norm() / rg.norm()).item() <= 1e-4
        assert ((cross.cpu() - rx).norm() / rx.norm()).item() <= 1e-3
        assert ((mass.cpu() - rm).norm() / rm.norm()).item() <= 1e-4
        c = o.association_matrix(gram.cpu(), cross.cpu()).float()
        rc = o.association_matrix(rg, rx).float()
        assert ((c - rc).abs() <= 1e-2 + 1e-2 * rc.abs()).all()


def test_batch_graph_decode_equals_eager():
    """tao_attention_decode_batch with graph-configured states and reused operand
    buffers replays one captured step (from the second call on); outputs equal the
    eager batch bit for bit across refreshes and a seal."""
    tb, preset, check_device = _tb()
    from tao_memory_b200 import stream
    dev = torch.device("cuda")
    R, H, D, P, N = 3, 2, 64, 1000, 300
    xs = [{k: t.to(dev) for k, t in make_inputs(1, P + N, H, D, seed=90 + r)[0].items()} for r in range(R)]
    fa, fb = xs[0]["fusion_a"], xs[0]["fusion_b"]
    outs = {}
    for graph in (False, True):
        states = []
        for r in range(R):
            st = tb.new_state(r, preset(graph=graph))
            tb.tao_attention_prefill(*(xs[r][k][:, :P] for k in KEYS[:3]), raw_q=xs[r]["raw_q"][:, :P],
                                     raw_k=xs[r]["raw_k"][:, :P], fusion_a=fa, fusion_b=fb, alpha=0.3,
                                     state=st, position=0)
            states.append(st)
        stage = torch.empty(5, R, 1, H, D, dtype=torch.bfloat16, device=dev)
        out = torch.empty(R, 1, H, D, dtype=torch.bfloat16, device=dev)
        got = []
        for t in range(P, P + N):
            for i, k in enumerate(KEYS):
                stage[i].copy_(torch.cat([xs[r][k][:, t:t + 1] for r in range(R)], 0))
            tb.tao_attention_decode_batch(stage[0], stage[1], stage[2], raw_q=stage[3], raw_k=stage[4],
                                          fusion_a=fa, fusion_b=fb, alpha=0.3, states=states, out=out)
            got.append(out.clone())
        outs[graph] = torch.stack(got)
    torch.cuda.synchronize()
    assert check_device() == 0
    assert len(stream._BatchGraph.cache) >= 1
    assert torch.equal(outs[False], outs[True])


def test_host_transfers_by_the_sms():
    """copy_to_device / copy_to_host move page-locked host bytes exactly; pageable
    host memory is refused before anything is accessed; a decode step fed and read
    back this way equals the one fed from device memory."""
    import tao_memory_b200 as tb
    from tao_memory_b200.presets import index_only_page_memo
    from tao_memory_b200.stream import check_device
    dev = torch.device("cuda")
    host = torch.randint(0, 1 << 15, (5, 8, 1, 12, 64), dtype=torch.int16).view(torch.bfloat16).pin_memory()
    d = torch.empty(host.shape, dtype=host.dtype, device=dev)
    tb.copy_to_device(d, host)
    back = torch.empty_like(host).pin_memory()
    tb.copy_to_host(back, d)
    torch.cuda.synchronize()
    assert torch.equal(d.cpu().view(torch.int16), host.view(torch.int16))
    assert torch.equal(back.view(torch.int16), host.view(torch.int16))
    with pytest.raises(ValueError):
        tb.copy_to_device(d, torch.from_numpy(host.view(torch.int16).numpy().copy()).view(torch.bfloat16))
    from tao_memory_b200 import _lib
    rc = _lib.lib().tao_copy_host_to_device(d.data_ptr(), torch.empty(64, dtype=torch.uint8).data_ptr(), 64,
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.TAO_ERR_ARG                    # the C entry checks the pointer kind itself
    # one decode step both ways
    R, H, D, P = 2, 3, 64, 900
    xs = [{k: t.to(dev) for k, t in make_inputs(1, P + 1, H, D, seed=90 + r)[0].items()} for r in range(R)]
    fa, fb = xs[0]["fusion_a"], xs[0]["fusion_b"]
    outs = []
    for via_host in (False, True):
        states = []
        for r in range(R):
            st = tb.new_state(r, index_only_page_memo())
            tb.tao_attention_prefill(*(xs[r][k][:, :P] for k in KEYS[:3]), raw_q=xs[r]["raw_q"][:, :P],
                                     raw_k=xs[r]["raw_k"][:, :P], fusion_a=fa, fusion_b=fb, alpha=0.3,
                                     state=st, position=0)
            states.append(st)
        stack = torch.stack([torch.cat([xs[r][k][:, P:P + 1] for r in range(R)], 0) for k in KEYS])
        if via_host:
            pinned = stack.cpu().pin_memory()
            stack = torch.empty_like(stack)
            tb.copy_to_device(stack, pinned)
        y, _ = tb.tao_attention_decode_batch(*stack[:3], raw_q=stack[3], raw_k=stack[4], fusion_a=fa,
                                             fusion_b=fb, alpha=0.3, states=states)
        if via_host:
            res = torch.empty(y.shape, dtype=y.dtype).pin_memory()
            tb.copy_to_host(res, y)
            torch.cuda.synchronize()
            y = res
        outs.append(y.cpu())
    assert torch.equal(outs[0], outs[1])
    assert check_device() == 0


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("width", [64, 128])
def test_decode_session_equals_decode_batch(graph, width):
    """DecodeSession (operands and results in page-locked host memory, brought in by
    the routing launch and written back by the fused kernel, completion signalled by a
    word in host memory; one graph launch per step for graph-configured states)
    decodes exactly like tao_attention_decode_batch, across route refreshes and a
    seal."""
    tb, preset, check_device = _tb()
    dev = torch.device("cuda")
    R, H, D, P, N = 3, 2, width, 1000, 40
    xs = [{k: t.to(dev) for k, t in make_inputs(1, P + N, H, D, seed=95 + r)[0].items()} for r in range(R)]
    fa, fb = xs[0]["fusion_a"], xs[0]["fusion_b"]
    sets = []
    for _ in range(2):
        states = []
        for r in range(R):
            st = tb.new_state(r, preset(graph=graph))
            tb.tao_attention_prefill(*(xs[r][k][:, :P] for k in KEYS[:3]), raw_q=xs[r]["raw_q"][:, :P],
                                     raw_k=xs[r]["raw_k"][:, :P], fusion_a=fa, fusion_b=fb, alpha=0.3,
                                     state=st, position=0)
            states.append(st)
        sets.append(states)
    session = tb.DecodeSession(sets[1], fa, fb, 0.3, reserve=N)
    for t in range(P, P + N):
        stack = torch.stack([torch.cat([xs[r][k][:, t:t + 1] for r in range(R)], 0) for k in KEYS])
        ref, _ = tb.tao_attention_decode_batch(*stack[:3], raw_q=stack[3], raw_k=stack[4], fusion_a=fa,
                                               fusion_b=fb, alpha=0.3, states=sets[0])
        session.inputs.copy_(stack.cpu())
        session.step()
        got = session.wait()
        assert torch.equal(got, ref.cpu()), f"position {t}"
    assert (session.graph is not None) == graph
    assert int(session.done[0]) == session.seq == N
    session.check()
    assert check_device() == 0
    for a, b in zip(*sets):
        assert a.position == b.position == P + N
        assert torch.equal(a.export()["packed_fine_c"], b.export()["packed_fine_c"])


def test_decode_session_grows_its_banks(monkeypatch):
    """A session whose states reach their fine-bank capacity mid-loop grows the banks
    before the step that seals past it (and captures its graph again), decoding
    exactly like tao_attention_decode_batch."""
    from tao_memory_b200 import stream
    tb, preset, check_device = _tb()
    monkeypatch.setattr(stream, "MIN_CAP", 8)
    dev = torch.device("cuda")
    R, H, D, P, N = 2, 2, 64, 2300, 300     # capacity 8 fines: the seal at 2559 needs a ninth
    xs = [{k: t.to(dev) for k, t in make_inputs(1, P + N, H, D, seed=97 + r)[0].items()} for r in range(R)]
    fa, fb = xs[0]["fusion_a"], xs[0]["fusion_b"]
    sets = []
    for _ in range(2):
        states = []
        for r in range(R):
            st = tb.new_state(r, preset(graph=True))
            tb.tao_attention_prefill(*(xs[r][k][:, :P] for k in KEYS[:3]), raw_q=xs[r]["raw_q"][:, :P],
                                     raw_k=xs[r]["raw_k"][:, :P], fusion_a=fa, fusion_b=fb, alpha=0.3,
                                     state=st, position=0)
            states.append(st)
        sets.append(states)
    session = tb.DecodeSession(sets[1], fa, fb, 0.3, reserve=1)
    caps = [st.cap_fines for st in sets[1]]
    for t in range(P, P + N):
        stack = torch.stack([torch.cat([xs[r][k][:, t:t + 1] for r in range(R)], 0) for k in KEYS])
        ref, _ = tb.tao_attention_decode_batch(*stack[:3], raw_q=stack[3], raw_k=stack[4], fusion_a=fa,
                                               fusion_b=fb, alpha=0.3, states=sets[0])
        session.inputs.copy_(stack.cpu())
        session.step()
        assert torch.equal(session.wait(), ref.cpu()), f"position {t}"
    assert all(st.cap_fines > c for st, c in zip(sets[1], caps))
    session.check()
    assert check_device() == 0
