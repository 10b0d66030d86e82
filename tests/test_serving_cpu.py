"""Serving caller host logic on the CPU: per-layer state binding, the on-disk
snapshot format (torch.save / torch.load(weights_only=True) of every layer's export
dictionary) and the scheduler's membership and layer-order rules.  No decode runs
here: the decode itself is covered by tests/test_serving_gpu.py."""
import pytest
import torch

from tao_memory_b200 import DecodeScheduler, RequestStates, TaoConfig, load_snapshot, new_state, save_snapshot


def test_request_states_bind_one_state_per_layer():
    req = RequestStates(3, TaoConfig(coarse_index_only=True))
    assert len(req) == 3 and [st.layer_index for st in req.layers] == [0, 1, 2]
    assert req.positions == [0, 0, 0]
    with pytest.raises(ValueError):
        RequestStates(states=[new_state(1)])          # layer 0 must hold layer_index 0
    st = new_state(0)
    with pytest.raises(ValueError):
        RequestStates(states=[st, st])
    with pytest.raises(ValueError):
        RequestStates(0)
    total = req.bytes()["total"]
    assert total["history_bytes"] == 0 and len(req.bytes()["layers"]) == 3


def test_snapshot_roundtrip_on_disk(tmp_path):
    cfg = TaoConfig(coarse_index_only=True, q1_history_region_graph=True)
    req = RequestStates(4, cfg)
    path = tmp_path / "req.pt"
    save_snapshot(req, path)
    back = load_snapshot(path)
    assert len(back) == 4 and back.positions == [0, 0, 0, 0]
    assert all(b.config == cfg and b.layer_index == i for i, b in enumerate(back.layers))
    assert all(a is not b for a, b in zip(req.layers, back.layers))
    # the file holds plain containers and tensors: it loads with weights_only
    raw = torch.load(path, weights_only=True)
    assert raw["format"] == 1 and len(raw["layers"]) == 4
    # a single layer-0 state is saved as a one-layer request
    save_snapshot(new_state(0), tmp_path / "one.pt")
    assert len(load_snapshot(tmp_path / "one.pt")) == 1
    with pytest.raises(ValueError):
        save_snapshot(new_state(2), tmp_path / "two.pt")


@pytest.mark.parametrize("mutate", ["kind", "format", "layers", "order"])
def test_snapshot_refuses_malformed_files(tmp_path, mutate):
    saved = RequestStates(2).export()
    if mutate == "kind":
        saved["kind"] = "something else"
    elif mutate == "format":
        saved["format"] = 99
    elif mutate == "layers":
        saved["layers"] = []
    else:
        saved["layers"] = saved["layers"][::-1]
    path = tmp_path / "bad.pt"
    torch.save(saved, path)
    with pytest.raises(ValueError):
        load_snapshot(path)


def test_scheduler_membership_and_layer_order():
    fa = torch.zeros(2, 2, 64, 3, dtype=torch.bfloat16)
    sch = DecodeScheduler(2, fa, fa, [0.3, 0.5])
    assert sch.alpha == [0.3, 0.5]
    a, b = RequestStates(2), RequestStates(2)
    sch.add("a", a)
    with pytest.raises(ValueError):
        sch.add("a", b)
    with pytest.raises(ValueError):
        sch.add("c", RequestStates(3))      # layer count differs from the model's
    assert sch.remove("a") is a and "a" not in sch.requests   # never joined: dropped at once
    with pytest.raises(KeyError):
        sch.remove("a")
    x = torch.zeros(1, 1, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        sch.decode(1, x, x, x, x, x)        # layer 1 before layer 0 of the token
    with pytest.raises(RuntimeError):
        sch.decode(0, x, x, x, x, x)        # nobody is active
    sch.add("b", b)
    b.layers[1].position = 5                # layers of a request must agree at a token start
    with pytest.raises(RuntimeError):
        sch.decode(0, x, x, x, x, x)
    with pytest.raises(ValueError):
        DecodeScheduler(2, fa, fa, [0.1])
