"""The serving caller on the GPU: a two-layer model's decode loop through
DecodeScheduler with requests joining and leaving between tokens and one request
saved to disk and reloaded mid-stream, against each request served alone through
tao_attention_prefill / tao_attention_decode (bit for bit: batched decode equals
single-request decode), and the reloaded request against its uninterrupted twin
(bf16 tolerance |a-b| <= 2e-2 + 2e-2|b|: an import rebuilds the page memo from the
exported state)."""
import pytest
import torch

from oracle.inputs import make_inputs
from _parity import assert_close

pytestmark = pytest.mark.gpu
KEYS = ("q", "k", "v", "raw_q", "raw_k")


def test_scheduler_matches_single_requests(tmp_path):
    import tao_memory_b200 as tb
    from tao_memory_b200.stream import check_device
    dev = torch.device("cuda")
    L, H, D, N = 2, 2, 64, 40
    prompts = {"a": 1500, "b": 900, "c": 2200}
    joins = {"a": 0, "b": 0, "c": 10}          # token at which the request joins
    leaves = {"a": 25}                         # token after which it leaves
    inputs = {rid: [{k: t.to(dev) for k, t in make_inputs(1, P + N, H, D, seed=70 + 5 * i + l)[0].items()}
                    for l in range(L)] for i, (rid, P) in enumerate(prompts.items())}
    fa = torch.stack([inputs["a"][l]["fusion_a"] for l in range(L)])
    fb = torch.stack([inputs["a"][l]["fusion_b"] for l in range(L)])
    alpha = [0.3, 0.6]
    cfg = tb.TaoConfig(coarse_index_only=True)
    sch = tb.DecodeScheduler(L, fa, fb, alpha, max_batch=2)
    reqs, alone = {}, {}
    for rid, P in prompts.items():
        reqs[rid] = tb.RequestStates(L, cfg)
        alone[rid] = tb.RequestStates(L, cfg)
        if joins[rid] == 0:
            sch.add(rid, reqs[rid])
        for l in range(L):
            x = inputs[rid][l]
            if rid in sch.requests:
                sch_out = sch.prefill(rid, l, *(x[k][:, :P] for k in KEYS))
            else:                              # prefilled before it is scheduled
                sch_out = tb.tao_attention_prefill(*(x[k][:, :P] for k in KEYS[:3]), raw_q=x["raw_q"][:, :P],
                                                   raw_k=x["raw_k"][:, :P], fusion_a=fa[l], fusion_b=fb[l],
                                                   alpha=alpha[l], state=reqs[rid][l], position=0)[0]
            one = tb.tao_attention_prefill(*(x[k][:, :P] for k in KEYS[:3]), raw_q=x["raw_q"][:, :P],
                                           raw_k=x["raw_k"][:, :P], fusion_a=fa[l], fusion_b=fb[l],
                                           alpha=alpha[l], state=alone[rid][l], position=0)[0]
            assert torch.equal(sch_out, one)
    step = {rid: 0 for rid in prompts}         # decode steps taken by each request
    expected = ["a", "b"]                      # the batch's row order
    b_out = {}                                 # (step, layer) -> output of "b"
    reloaded = None
    for token in range(N):
        if token == 10:
            sch.add("c", reqs["c"])
            expected.append("c")
        if token == 15:                        # "b" to disk and back: it continues as a new request
            path = tmp_path / "b.pt"
            tb.save_snapshot(reqs["b"], path)
            reloaded, reload_step = tb.load_snapshot(path, device=dev), step["b"]
        for l in range(L):
            rows = {k: torch.cat([inputs[r][l][k][:, prompts[r] + step[r]:prompts[r] + step[r] + 1]
                                  for r in expected], 0) for k in KEYS}
            out = sch.decode(l, *(rows[k] for k in KEYS))
            assert list(sch.active) == expected
            for i, r in enumerate(expected):
                sl = slice(prompts[r] + step[r], prompts[r] + step[r] + 1)
                x = inputs[r][l]
                ref = tb.tao_attention_decode(*(x[k][:, sl] for k in KEYS[:3]), raw_q=x["raw_q"][:, sl],
                                              raw_k=x["raw_k"][:, sl], fusion_a=fa[l], fusion_b=fb[l],
                                              alpha=alpha[l], state=alone[r][l],
                                              position=prompts[r] + step[r])[0]
                assert torch.equal(out[i:i + 1], ref), (token, l, r)
                if r == "b":
                    b_out[(step[r], l)] = ref
        for r in expected:
            step[r] += 1
        if token == leaves["a"]:
            sch.remove("a")
            expected.remove("a")
    assert step["a"] == 26 and step["c"] == N - 10 and step["b"] == N
    assert "a" not in sch.requests
    # the reloaded copy of "b" continues like "b" did from token 15
    for s_ in range(reload_step, N):
        for l in range(L):
            x = inputs["b"][l]
            sl = slice(prompts["b"] + s_, prompts["b"] + s_ + 1)
            got = tb.tao_attention_decode(*(x[k][:, sl] for k in KEYS[:3]), raw_q=x["raw_q"][:, sl],
                                          raw_k=x["raw_k"][:, sl], fusion_a=fa[l], fusion_b=fb[l],
                                          alpha=alpha[l], state=reloaded[l], position=prompts["b"] + s_)[0]
            assert_close(got, b_out[(s_, l)], f"reloaded b, step {s_}, layer {l}")
    assert reloaded.positions == reqs["b"].positions
    assert check_device() == 0
