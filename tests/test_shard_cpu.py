"""Multi-GPU partitioning and the output gather, on the CPU (no GPU needed).

* The request split and the LPT plan (requests x head groups by decode bytes per
  token) cover every (request, head) exactly once and balance the load.
* Two ranks over gloo: each decodes its shards (a stand-in computation that
  depends on the request, the head and the step), the outputs are all-gathered
  and rank 0 assembles the global [requests, 1, heads, width] tensor.
* Host-side failures: a rank that raises before the gather tells the other
  through the store (it stops at once); a rank that leaves silently is reported
  by the step check's timeout; a collective the peer never joins ends with an
  error when the process group's short timeout expires.
"""
import math
import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tao_memory_b200.shard import (OutputGather, PeerCheck, RankFailure, assemble, decode_bytes_per_token,
                                   plan_imbalance, plan_lpt, requests_of_rank)


def test_request_split_covers_every_request_once():
    for n in (1, 7, 8, 64):
        for world in (1, 2, 4, 8):
            got = [r for k in range(world) for r in requests_of_rank(n, world, k)]
            assert got == list(range(n))
            sizes = [len(requests_of_rank(n, world, k)) for k in range(world)]
            assert max(sizes) - min(sizes) <= 1


def _serving_lengths(n=64, seed=71):
    g = torch.Generator().manual_seed(seed)
    lo, hi = math.log(2048), math.log(131072)
    return [int(round(math.exp(lo + (hi - lo) * torch.rand(1, generator=g).item()))) for _ in range(n)]


def test_lpt_plan_covers_every_head_once_and_balances():
    lengths = _serving_lengths()
    for world in (1, 2, 4, 8):
        plan = plan_lpt(lengths, 16, 128, world)
        assert plan == plan_lpt(lengths, 16, 128, world)            # deterministic
        seen = {}
        for s in plan:
            for h in range(s.head_lo, s.head_hi):
                seen[(s.request, h)] = seen.get((s.request, h), 0) + 1
        assert len(seen) == 64 * 16 and set(seen.values()) == {1}
        assert plan_imbalance(plan, world) <= 1.05, (world, plan_imbalance(plan, world))
    # the longest request is split by head group once a rank's share is below its load
    plan8 = plan_lpt(lengths, 16, 128, 8)
    longest = max(range(64), key=lambda r: lengths[r])
    assert any(s.request == longest and s.head_hi - s.head_lo < 16 for s in plan8) or \
        decode_bytes_per_token(lengths[longest], 16, 128) <= sum(
            decode_bytes_per_token(c, 16, 128) for c in lengths) / 8


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, fn, *args):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(rank, world, port, q, fn, args)) for rank in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, value = q.get(timeout=120)
        results[rank] = value
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode is not None, "a rank did not exit"
    return results


def _entry(rank, world, port, q, fn, args):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=3))
        q.put((rank, fn(rank, world, *args)))
    except Exception as e:   # noqa: BLE001 - reported to the parent
        q.put((rank, ("error", type(e).__name__, str(e), traceback.format_exc())))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:   # noqa: BLE001
                pass


def _fake_output(shard, step, width):
    """Stand-in for a shard's decode output: depends on request, head and step."""
    heads = torch.arange(shard.head_lo, shard.head_hi, dtype=torch.float32)
    val = shard.request * 1000 + heads * 10 + step
    return val.view(1, -1, 1).expand(1, -1, width).clone()


def _gather_worker(rank, world, lengths, heads, width, steps):
    plan = plan_lpt(lengths, heads, width, world)
    rows = [[s for s in plan if s.rank == k] for k in range(world)]
    max_rows = max(len(r) for r in rows)
    gather = OutputGather(dist.group.WORLD, (max_rows, 1, heads, width), torch.float32, "cpu")
    results = []
    for step in range(steps):
        local = torch.zeros(max_rows, 1, heads, width)
        for row, s in enumerate(rows[rank]):
            local[row, :, :s.head_hi - s.head_lo] = _fake_output(s, step, width)
        gather.start(local)
        got = gather.finish()
        if rank == 0:
            results.append(assemble(got, plan, rows, len(lengths), heads))
    return results


def test_two_ranks_gather_every_requests_outputs():
    lengths = [2048, 131072, 9000, 40000, 3000]
    heads, width, steps = 8, 4, 3
    res = _run(2, _gather_worker, lengths, heads, width, steps)
    assert not isinstance(res[1], tuple), res[1]
    out = res[0]
    assert not isinstance(out, tuple), out
    for step, glob in enumerate(out):
        for r in range(len(lengths)):
            for h in range(heads):
                assert torch.all(glob[r, 0, h] == r * 1000 + h * 10 + step)


def _failing_worker(rank, world, mode):
    # a peer that aborts is seen at once, whatever the timeout; a silent one only at the timeout
    check = PeerCheck(dist.distributed_c10d._get_default_store(), rank, world,
                      timeout_s=30.0 if mode == "raise" else 2.0, prefix=f"tao/{mode}")
    if rank == 1:
        check.wait(0)                                   # step 0 runs on both ranks
        if mode == "raise":
            try:
                raise RuntimeError("decode failed on rank 1")
            except RuntimeError as e:
                check.abort(str(e))                    # tell the others, then leave
                return ("left", str(e))
        return ("left", "silently")
    try:
        # rank 1 never posts step 1; its abort may already show while rank 0 checks step 0
        check.wait(0)
        check.wait(1)
    except RankFailure as e:
        return ("failure", str(e))
    return ("no failure detected",)


@pytest.mark.parametrize("mode", ["raise", "silent"])
def test_peer_failure_is_detected_before_the_next_collective(mode):
    res = _run(2, _failing_worker, mode)
    assert res[1][0] == "left"
    assert res[0][0] == "failure", res[0]
    if mode == "raise":
        assert "decode failed on rank 1" in res[0][1]
    else:
        assert "[1]" in res[0][1]


def _collective_timeout_worker(rank, world):
    if rank == 1:
        return ("left",)
    t0 = torch.zeros(2, 3)
    out = torch.empty(2, 2, 3)
    try:
        dist.all_gather_into_tensor(out, t0)            # rank 1 never joins: the group's timeout ends it
    except RuntimeError as e:
        return ("error", type(e).__name__)
    return ("completed",)


def test_gather_without_the_peer_ends_with_an_error():
    res = _run(2, _collective_timeout_worker)
    assert res[0][0] == "error", res[0]
