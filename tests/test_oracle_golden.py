"""Pin the CPU oracle (oracle/tao_oracle.py) to golden vectors produced by the
unmodified reference (tests/golden/make_golden.py).  No GPU needed."""
import os

import pytest
import torch

from oracle import tao_oracle as o
from oracle.inputs import make_inputs, digest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
STREAM = ["stream_h2d64", "stream_h1d128", "stream_pages", "stream_regularized", "stream_feature_mass",
          "stream_structured_gram", "stream_coarse"]
TRAIN = ["train_t2048_h2", "train_t3072_b2", "train_t2000_ragged", "train_pages", "train_regularized",
         "train_coarse", "train_feature_mass", "train_structured_gram"]
KEYS = ("q", "k", "v", "raw_q", "raw_k")


def load(name):
    return torch.load(os.path.join(GOLDEN, name + ".pt"), weights_only=False)


@pytest.mark.parametrize("name", STREAM)
def test_stream_oracle_matches_reference(name, one_thread):
    g = load(name)
    heads, width, layer, splits, steps, seed = g["case"]
    x, _ = make_inputs(1, sum(splits) + steps, heads, width, seed)
    assert digest(*(x[k] for k in (*KEYS, "fusion_a", "fusion_b"))) == g["input_digest"]
    config = g.get("config", {})
    st = o.OracleStream(layer, config.get("fine_writer", "softmax"), config.get("coarse_index_only", True))
    outs, ids, pos = [], [], 0
    for n in list(splits) + [1] * steps:
        sl = slice(pos, pos + n)
        outs.append(st.step(*(x[k][:, sl] for k in KEYS), x["fusion_a"], x["fusion_b"], g["alpha"]))
        if n == 1:
            ids.append(st.route_ids[1].clone())
        pos += n
    out = torch.cat(outs, 1)
    stride = g.get("row_stride", 1)
    ref = g["output"]
    mine = out[:, ::stride]
    assert mine.shape == ref.shape
    bad = (mine != ref).sum().item()
    # the reference's Triton fine read sums in its own fp32 order: a handful of 1-ulp flips
    assert bad <= max(8, ref.numel() // 50000), bad
    assert (mine.float() - ref.float()).abs().max().item() <= 2e-3
    if "decode_output" in g:
        assert (out[:, -steps:] != g["decode_output"]).sum().item() <= 4
    # routing selections are integer results: bit-exact
    for a, b in zip(ids, g["decode_route_ids"]):
        assert torch.equal(a, b)
    snap = g["snapshot_final"]
    mine_snap = st.export()
    assert mine_snap["position"] == snap["position"]
    assert torch.equal(mine_snap["packed_fine_c"], snap["packed_fine_c"])
    for (pz, pc, fz), (rpz, rpc, rfz) in zip(mine_snap["pages"], snap["pages"]):
        assert torch.equal(pz, rpz) and torch.equal(fz, rfz)
        assert (pc is None) == (rpc is None)
        if rpc is not None:   # coarse page matrix (coarse_index_only=False)
            assert torch.equal(pc, rpc)
    for z, rz in zip(mine_snap["pending_z"], snap["pending_z"]):
        assert torch.equal(z, rz)
    for key in ("pending_gram", "pending_cross", "pending_mass", "pending_square_mass"):
        assert (mine_snap[key] is None) == (snap.get(key) is None)
        if snap[key] is not None:
            assert torch.equal(mine_snap[key], snap[key]), key


@pytest.mark.parametrize("name", TRAIN)
def test_training_oracle_matches_reference(name, one_thread):
    g = load(name)
    b, t, h, d, alpha, seed = g["case"]
    x, gen = make_inputs(b, t, h, d, seed)
    grad = torch.randn(b, t, h, d, generator=gen).to(torch.bfloat16)
    assert digest(*(x[k] for k in (*KEYS, "fusion_a", "fusion_b")), grad) == g["input_digest"]
    leaves = {k: x[k].clone().requires_grad_(True) for k in x}
    writer = g.get("config", {}).get("fine_writer", "softmax")
    index_only = g.get("config", {}).get("coarse_index_only", True)
    out = o.tao_attention(*(leaves[k] for k in KEYS), leaves["fusion_a"], leaves["fusion_b"], alpha, writer,
                          coarse_index_only=index_only)
    out.backward(grad)
    s = g.get("row_stride", 1)
    ref = g["output"]
    assert (out.detach()[:, ::s] != ref).sum().item() <= 16
    assert (out.detach()[:, ::s].float() - ref.float()).abs().max().item() <= 2e-3
    for k in leaves:
        mine = leaves[k].grad
        if k in KEYS:
            mine = mine[:, ::s]
        r = g["grads"][k].float()
        rel = ((mine.float() - r).norm() / r.norm().clamp_min(1e-30)).item()
        # dC / dw are rounded per checkpoint group in the reference; the oracle
        # rounds per tile: raw_k and v gradients differ at the 1e-2 level
        assert rel <= (2e-2 if k in ("raw_k", "v") else 1e-3), (k, rel)
