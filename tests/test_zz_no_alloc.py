"""The allocation-free decode entry point (tao_stream_decode_noalloc).

Some callers cannot call cudaMalloc -- their device memory belongs to another
runtime's pool, or they run loops where an allocation could synchronise the
device -- so they cannot provide the workspace tao_stream_step needs.  The
no-alloc variant keeps its scratch in a static device array in the library.

These tests call it through the C ABI, step after step (each call reuses the
scratch the previous one left behind), over decode positions that include a
route refresh and a seal, at widths 64 and 128.  Both entry points run the same
kernels on the same inputs, so their outputs and the states they leave must be
bit-identical; the outputs are also checked against the CPU oracle
(|a-b| <= 2e-2 + 2e-2|b| for every element, routes exact).  A policy whose route
capacity is too small for the states is reported through the error word
(tao_stream_decode_noalloc_check).  The file is named to be collected last.
"""
import ctypes

import pytest
import torch

from oracle import tao_oracle as o
from oracle.inputs import make_inputs
from _parity import assert_close

pytestmark = pytest.mark.gpu
KEYS = ("q", "k", "v", "raw_q", "raw_k")


def _prefilled(tb, preset, xs, prompt, fa, fb, alpha):
    states = []
    for r, x in enumerate(xs):
        st = tb.new_state(0, preset())
        tb.tao_attention_prefill(*(x[k][:, :prompt] for k in KEYS[:3]), raw_q=x["raw_q"][:, :prompt],
                                 raw_k=x["raw_k"][:, :prompt], fusion_a=fa, fusion_b=fb, alpha=alpha,
                                 state=st, position=0)
        st._ensure(st.heads, st.width, st.device, 16)
        states.append(st)
    return states


@pytest.mark.parametrize("width", [64, 128])
def test_noalloc_decode_matches_workspace_entry_point_across_refresh_and_seal(width, one_thread):
    import tao_memory_b200 as tb
    from tao_memory_b200 import _lib
    from tao_memory_b200.presets import index_only_page_memo
    from tao_memory_b200.stream import policy_for, ROUTE_CAP, is_refresh, window_start

    dev = torch.device("cuda", torch.cuda.current_device())
    R, H, P, N, alpha = 2, 2, 1270, 12, 0.3
    cpu = [make_inputs(1, P + N, H, width, seed=70 + r)[0] for r in range(R)]
    xs = [{k: t.to(dev) for k, t in x.items()} for x in cpu]
    fa, fb = xs[0]["fusion_a"], xs[0]["fusion_b"]
    sets = [_prefilled(tb, index_only_page_memo, xs, P, fa, fb, alpha) for _ in range(2)]
    cfg = sets[0][0].config
    assert any(is_refresh(t, 0, cfg) for t in range(P, P + N))
    assert any(t + 1 - window_start(t) == 768 for t in range(P, P + N))
    lib = _lib.lib()
    policy = policy_for(cfg)
    assert policy.route_cap == ROUTE_CAP
    stream = torch.cuda.current_stream(dev).cuda_stream
    ws = torch.zeros(lib.tao_stream_workspace_bytes(R, 1, H, width, ROUTE_CAP, ctypes.byref(policy)),
                     dtype=torch.uint8, device=dev)
    got = [[], []]
    for t in range(P, P + N):
        x = {k: torch.cat([xs[r][k][:, t:t + 1] for r in range(R)], 0).contiguous() for k in KEYS}
        for which, states in enumerate(sets):
            ptrs = torch.tensor([st._desc.data_ptr() for st in states], dtype=torch.int64, device=dev)
            pos = (ctypes.c_int64 * R)(*[st.position for st in states])
            cap = (ctypes.c_int32 * R)(*[st.cap_fines for st in states])
            out = torch.empty(R, 1, H, width, dtype=torch.bfloat16, device=dev)
            args = [x[k].data_ptr() for k in KEYS] + [fa.data_ptr(), fb.data_ptr(), alpha, out.data_ptr()]
            if which == 0:
                rc = lib.tao_stream_step(ptrs.data_ptr(), R, pos, cap, ctypes.byref(policy), 1, H, width,
                                         *args, ws.data_ptr(), ws.numel(), stream)
            else:
                rc = lib.tao_stream_decode_noalloc(ptrs.data_ptr(), R, pos, cap, ctypes.byref(policy),
                                                   H, width, *args, stream)
            _lib.check(rc)
            torch.cuda.synchronize()
            for st in states:
                st.position += 1
            got[which].append(out.cpu())
        assert torch.equal(got[0][-1], got[1][-1]), f"outputs differ at position {t}"
    flags = ctypes.c_int(-1)
    _lib.check(lib.tao_stream_decode_noalloc_check(ctypes.byref(flags), stream))
    assert flags.value == 0
    _lib.check(lib.tao_stream_check(ws.data_ptr(), ctypes.byref(flags), stream))
    for a, b in zip(sets[0], sets[1]):
        ea, eb = a.export(), b.export()
        assert ea["position"] == eb["position"] == P + N
        assert ea["fine_seal_events"] == eb["fine_seal_events"]
        assert torch.equal(ea["packed_fine_c"], eb["packed_fine_c"])
        assert torch.equal(ea["route_ids"][1], eb["route_ids"][1])
    for r in range(R):
        orc = o.OracleStream(0)
        orc.step(*(cpu[r][k][:, :P] for k in KEYS), cpu[r]["fusion_a"], cpu[r]["fusion_b"], alpha)
        ref = [orc.step(*(cpu[r][k][:, t:t + 1] for k in KEYS), cpu[r]["fusion_a"], cpu[r]["fusion_b"], alpha)
               for t in range(P, P + N)]
        mine = torch.cat([g[r:r + 1] for g in got[1]], 1)
        assert_close(mine, torch.cat(ref, 1), f"no-alloc decode, request {r}, width {width}")
        assert torch.equal(sets[1][r].export()["route_ids"][1].cpu(), orc.route_ids[1])


def test_noalloc_reports_route_overflow_through_its_error_word():
    """States holding more routes than the call's route capacity: the kernels skip
    the fine read, set the route-overflow bit, and the check entry point returns it
    once (then the word is clear)."""
    import tao_memory_b200 as tb
    from tao_memory_b200 import _lib
    from tao_memory_b200.presets import index_only_page_memo
    from tao_memory_b200.stream import policy_for

    dev = torch.device("cuda", torch.cuda.current_device())
    R, H, D, P = 2, 2, 64, 1100
    xs = [{k: t.to(dev) for k, t in make_inputs(1, P + 1, H, D, seed=90 + r)[0].items()} for r in range(R)]
    fa, fb = xs[0]["fusion_a"], xs[0]["fusion_b"]
    states = _prefilled(tb, index_only_page_memo, xs, P, fa, fb, 0.3)
    assert all(st._download().n_route >= 2 for st in states)
    lib = _lib.lib()
    policy = policy_for(states[0].config)
    policy.route_cap = 1
    stream = torch.cuda.current_stream(dev).cuda_stream
    x = {k: torch.cat([xs[r][k][:, P:P + 1] for r in range(R)], 0).contiguous() for k in KEYS}
    ptrs = torch.tensor([st._desc.data_ptr() for st in states], dtype=torch.int64, device=dev)
    pos = (ctypes.c_int64 * R)(*[st.position for st in states])
    cap = (ctypes.c_int32 * R)(*[st.cap_fines for st in states])
    out = torch.empty(R, 1, H, D, dtype=torch.bfloat16, device=dev)
    _lib.check(lib.tao_stream_decode_noalloc(ptrs.data_ptr(), R, pos, cap, ctypes.byref(policy), H, D,
                                             *(x[k].data_ptr() for k in KEYS), fa.data_ptr(), fb.data_ptr(),
                                             0.3, out.data_ptr(), stream))
    flags = ctypes.c_int(0)
    rc = lib.tao_stream_decode_noalloc_check(ctypes.byref(flags), stream)
    assert rc == _lib.TAO_ERR_DEVICE and flags.value & 2
    assert lib.tao_stream_decode_noalloc_check(ctypes.byref(flags), stream) == _lib.TAO_OK
    assert flags.value == 0
