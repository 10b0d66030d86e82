"""The feature-read writers ("feature_mass_association", "structured_gram_association")
streaming on the GPU against the oracle and the reference's snapshots.

Both writers (tao_stream.py:56-65, 463-500) store z = bf16(log mass) per fine and
bf16(log accumulated mass) per page, and read the selected fines with the
feature-mass mixture (association_writer.py:43-53); they differ in C (unchecked
regularised solve, structured_writer.py:17-34 closed-form inverse).  Tolerance (bf16
outputs): |a-b| <= 2e-2 + 2e-2*|b| for every element.  The fp32 masses are sums in
another order than torch's CPU sum, so a z value can round to the neighbouring
bf16 value; routing selections are compared exactly all the same.
"""
import os

import pytest
import torch

from oracle import tao_oracle as o
from oracle.inputs import make_inputs
from test_stream_gpu import GOLDEN, KEYS, run_gpu
from _parity import assert_close

pytestmark = pytest.mark.gpu
WRITERS = ("feature_mass_association", "structured_gram_association")
GOLDEN_OF = {"feature_mass_association": "stream_feature_mass",
             "structured_gram_association": "stream_structured_gram"}


def _config(writer):
    from tao_memory_b200 import TaoConfig
    from tao_memory_b200.presets import index_only_page_memo
    return TaoConfig(**{**index_only_page_memo().export(), "fine_writer": writer})


@pytest.mark.parametrize("writer", WRITERS)
@pytest.mark.parametrize("heads,width,layer,splits,steps", [
    (4, 64, 2, (300, 1500, 1333), 40),
    (3, 128, 5, (2100,), 30),
])
def test_feature_writer_stream_matches_oracle(writer, heads, width, layer, splits, steps, one_thread):
    x, _ = make_inputs(1, sum(splits) + steps, heads, width, seed=21 + layer)
    out, ids, st, _ = run_gpu(x, layer, splits, steps, 0.4, config=_config(writer))
    orc = o.OracleStream(layer, fine_writer=writer)
    ref, ref_ids, pos = [], [], 0
    for n in list(splits) + [1] * steps:
        sl = slice(pos, pos + n)
        ref.append(orc.step(*(x[k][:, sl] for k in KEYS), x["fusion_a"], x["fusion_b"], 0.4))
        if n == 1:
            ref_ids.append(orc.route_ids[1].clone())
        pos += n
    ref = torch.cat(ref, 1)
    assert_close(out, ref, f"{writer} h{heads} d{width}")
    assert sum(int(not torch.equal(a, b)) for a, b in zip(ids, ref_ids)) == 0
    snap = st.export()
    err = (snap["pending_mass"].cpu() - orc.pending_mass).norm() / orc.pending_mass.norm()
    assert err <= 1e-4
    assert st.bytes()["pending_feature_mass_bytes"] == heads * width * 4
    if writer == "structured_gram_association":
        err = ((snap["pending_square_mass"].cpu() - orc.pending_square_mass).norm()
               / orc.pending_square_mass.norm())
        assert err <= 1e-4 and snap["pending_gram"] is None


@pytest.mark.parametrize("writer", WRITERS)
def test_feature_writer_snapshot_roundtrip(writer, one_thread):
    """Own export -> import continues bit-identically; the reference's snapshot
    imported on the device continues like the oracle imported from it."""
    import tao_memory_b200 as tb
    from tao_memory_b200 import StreamCache
    from tao_memory_b200.stream import check_device
    dev = torch.device("cuda")
    g = torch.load(os.path.join(GOLDEN, GOLDEN_OF[writer] + ".pt"), weights_only=False)
    heads, width, layer, splits, steps, seed = g["case"]
    total = sum(splits) + steps
    x, _ = make_inputs(1, total + 300, heads, width, seed)
    _, _, st, _ = run_gpu({k: t[:, :total] if t.dim() == 4 else t for k, t in x.items()},
                          layer, splits, steps, g["alpha"], config=_config(writer))
    xs = {k: t.to(dev) for k, t in x.items()}
    kw = dict(fusion_a=xs["fusion_a"], fusion_b=xs["fusion_b"], alpha=g["alpha"])
    a = StreamCache.from_export(st.export())
    b = StreamCache.from_export(g["snapshot_final"], device=dev)   # produced by the reference
    orc = o.OracleStream.from_export(g["snapshot_final"])
    pos = total
    # a 200-token chunk, then decode across the next seal (the window fills at 3072)
    for n in [200] + [1] * 100:
        sl = slice(pos, pos + n)
        args = [xs[k][:, sl] for k in KEYS[:3]]
        call = tb.tao_attention_prefill if n > 1 else tb.tao_attention_decode
        o1, st = call(*args, raw_q=xs["raw_q"][:, sl], raw_k=xs["raw_k"][:, sl], state=st, position=pos, **kw)
        o2, a = call(*args, raw_q=xs["raw_q"][:, sl], raw_k=xs["raw_k"][:, sl], state=a, position=pos, **kw)
        o3, b = call(*args, raw_q=xs["raw_q"][:, sl], raw_k=xs["raw_k"][:, sl], state=b, position=pos, **kw)
        ref = orc.step(*(x[k][:, sl] for k in KEYS), x["fusion_a"], x["fusion_b"], g["alpha"])
        assert torch.equal(o1, o2)
        assert_close(o3, ref, f"{writer} from the reference snapshot at {pos}")
        pos += n
    sb = b.export()
    assert sb["fine_seal_events"] == orc.state_version
    err = (sb["pending_mass"].cpu() - orc.pending_mass).norm() / orc.pending_mass.norm()
    assert err <= 1e-4
    assert check_device() == 0
