"""The allocation-free decode entry point (tao_stream_decode_noalloc).

Some callers cannot call cudaMalloc -- their device memory belongs to another
runtime's pool, or they run loops where an allocation could synchronise the
device -- so they cannot provide the workspace tao_stream_step needs.  The
no-alloc variant keeps its scratch in a static device array in the library.
This test calls it through the C ABI and checks it against tao_stream_step on
the same inputs, for two calls in a row (the second call reuses the scratch the
first one left behind).  Tolerance: |a-b| <= 2e-2 + 2e-2|b| (bf16), as the other
parity tests.  The file is named to be collected last.
"""
import ctypes

import pytest
import torch

from oracle.inputs import make_inputs

pytestmark = pytest.mark.gpu
KEYS = ("q", "k", "v", "raw_q", "raw_k")


def test_noalloc_decode_matches_workspace_entry_point():
    import tao_memory_b200 as tb
    from tao_memory_b200 import _lib
    from tao_memory_b200.presets import index_only_page_memo
    from tao_memory_b200.stream import policy_for, ROUTE_CAP

    dev = torch.device("cuda", torch.cuda.current_device())
    R, H, D, P = 2, 2, 64, 1100
    xs = [{k: t.to(dev) for k, t in make_inputs(1, P + 2, H, D, seed=70 + r)[0].items()} for r in range(R)]
    fa, fb = xs[0]["fusion_a"], xs[0]["fusion_b"]
    sets = []
    for _ in range(2):
        states = []
        for r in range(R):
            st = tb.new_state(r, index_only_page_memo())
            tb.tao_attention_prefill(*(xs[r][k][:, :P] for k in KEYS[:3]), raw_q=xs[r]["raw_q"][:, :P],
                                     raw_k=xs[r]["raw_k"][:, :P], fusion_a=fa, fusion_b=fb, alpha=0.3,
                                     state=st, position=0)
            st._ensure(H, D, dev, 4)
            states.append(st)
        sets.append(states)
    lib = _lib.lib()
    policy = policy_for(sets[0][0].config)
    assert policy.route_cap == ROUTE_CAP
    stream = torch.cuda.current_stream(dev).cuda_stream
    for t in (P, P + 1):
        x = {k: torch.cat([xs[r][k][:, t:t + 1] for r in range(R)], 0).contiguous() for k in KEYS}
        outs = []
        for which, states in enumerate(sets):
            ptrs = torch.tensor([st._desc.data_ptr() for st in states], dtype=torch.int64, device=dev)
            pos = (ctypes.c_int64 * R)(*[st.position for st in states])
            cap = (ctypes.c_int32 * R)(*[st.cap_fines for st in states])
            out = torch.empty(R, 1, H, D, dtype=torch.bfloat16, device=dev)
            args = [x[k].data_ptr() for k in KEYS] + [fa.data_ptr(), fb.data_ptr(), 0.3, out.data_ptr()]
            if which == 0:
                ws = torch.zeros(lib.tao_stream_workspace_bytes(R, 1, H, D, ROUTE_CAP, ctypes.byref(policy)),
                                 dtype=torch.uint8, device=dev)
                rc = lib.tao_stream_step(ptrs.data_ptr(), R, pos, cap, ctypes.byref(policy), 1, H, D,
                                         *args, ws.data_ptr(), ws.numel(), stream)
            else:
                rc = lib.tao_stream_decode_noalloc(ptrs.data_ptr(), R, pos, cap, ctypes.byref(policy),
                                                   H, D, *args, stream)
            _lib.check(rc)
            torch.cuda.synchronize()
            for st in states:
                st.position += 1
            outs.append(out.float().cpu())
        a, b = outs[1], outs[0]
        assert ((a - b).abs() > 2e-2 + 2e-2 * b.abs()).sum().item() == 0
        assert torch.isfinite(a).all()
