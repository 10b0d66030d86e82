"""Partitioning of decode work over the GPUs of one node, and the output gather.

Requests are independent (each owns its state; the reference forbids sharing a
state between concurrent requests, docs/usage.md:35-36) and so are heads (routing,
pages, fine reads and the fusion parameters are all per head, tao_stream.py:299-360),
so decode work splits by request and by head group with no exchange during a
step.  The only collective is the gather of each step's outputs to the caller's
rank: one NCCL all-gather on a side stream, overlapped with the next step.

* ``requests_of_rank``: equal contiguous blocks of requests (requests of equal
  length, e.g. 8 requests at 128K context).
* ``plan_lpt``: mixed lengths.  A request's load is its decode bytes per token
  (local window + selected fines, ``decode_bytes_per_token``); requests heavier
  than the mean load per rank are split into 2 or 4 head groups, then the units
  go to ranks longest-first, each to the least-loaded rank (LPT).
* ``OutputGather``: all-gather of [rows, 1, heads, width] outputs into a
  [world, rows, ...] buffer on a side stream; rank 0 reads it after ``finish``.
* ``PeerCheck``: host-side liveness through the process group's store, so ranks
  learn that a peer has gone before they launch the next collective; collectives
  themselves end with an error when the process group's timeout expires.
"""

from dataclasses import dataclass
import time

import torch
import torch.distributed as dist

from .config import TaoConfig, routed_counts

WINDOW, FINE, KEEP, GROUP = 768, 256, 512, 8


def requests_of_rank(n_requests, world, rank):
    """Contiguous block of request indices served by ``rank`` (sizes differ by at most one)."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    base, extra = divmod(n_requests, world)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (rank < extra)))


def decode_bytes_per_token(context, heads, width, config=TaoConfig()):
    """HBM bytes one decode token of a request at ``context`` reads and writes: local
    K and V of every window key, the selected fines' matrices with their z / page z /
    page weight rows, q and raw_q in, the output out."""
    pos = context
    start = 0 if pos < WINDOW else FINE * ((pos - KEEP) // FINE)
    keys = pos - start + 1
    sealed = (pos - WINDOW) // FINE + 1 if pos >= WINDOW else 0
    m = routed_counts(sealed // GROUP, sealed % GROUP, config)[2] if sealed else 0
    return heads * (keys * width * 4 + m * (width * width * 2 + 3 * width * 2) + 3 * width * 2)


@dataclass(frozen=True)
class Shard:
    request: int
    head_lo: int
    head_hi: int
    rank: int
    load: float


def plan_lpt(contexts, heads, width, world, config=TaoConfig(), splits=(1, 2, 4)):
    """Assign (request, head group) units to ranks.

    contexts: context length of each request.  Returns a list of ``Shard`` sorted by
    (rank, request, head_lo).  A request whose load exceeds the mean load per rank is
    split into the smallest head-group count from ``splits`` that brings each part
    under that mean (or the largest that divides ``heads``); units are placed
    longest-first on the least-loaded rank, ties to the lower rank, so the plan is
    deterministic."""
    if world <= 0:
        raise ValueError("world must be positive")
    loads = [decode_bytes_per_token(c, heads, width, config) for c in contexts]
    mean = sum(loads) / world
    units = []
    for r, load in enumerate(loads):
        usable = [g for g in sorted(splits) if heads % g == 0]
        g = usable[0]
        for cand in usable:
            g = cand
            if load / cand <= mean:
                break
        step = heads // g
        for i in range(g):
            units.append((load / g, r, i * step, (i + 1) * step))
    units.sort(key=lambda u: (-u[0], u[1], u[2]))
    rank_load = [0.0] * world
    shards = []
    for load, r, lo, hi in units:
        target = min(range(world), key=lambda k: (rank_load[k], k))
        rank_load[target] += load
        shards.append(Shard(r, lo, hi, target, load))
    shards.sort(key=lambda s: (s.rank, s.request, s.head_lo))
    return shards


def plan_imbalance(shards, world):
    """max rank load / mean rank load of a plan (1.0 = perfectly balanced)."""
    per = [0.0] * world
    for s in shards:
        per[s.rank] += s.load
    mean = sum(per) / world
    return max(per) / mean if mean else 1.0


class OutputGather:
    """All-gather of each step's local outputs to every rank (rank 0 consumes them).

    ``start(local)`` enqueues the all-gather of ``local`` (shape ``shape``) on a side
    stream after the work the current stream has queued so far, so it overlaps the
    next step; ``finish()`` makes the current stream wait for the gathers in flight
    and returns the last gathered buffer, [world, *shape].  With a CPU (gloo) group
    the gather runs synchronously.  With ``group=None`` (one process) both are no-ops.
    """

    def __init__(self, group, shape, dtype, device, slots=2):
        self.group = group
        self.world = 1 if group is None else dist.get_world_size(group)
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        shape = tuple(shape)
        self.shape = shape
        # flat [world * rows, ...] buffers (the layout every backend accepts), read as [world, rows, ...]
        self.bufs = [torch.empty((self.world * shape[0],) + shape[1:], dtype=dtype, device=self.device)
                     for _ in range(slots)] if group is not None else []
        self.side = torch.cuda.Stream(self.device) if (self.cuda and group is not None) else None
        self.n = 0
        self.last = None

    def start(self, local):
        if self.group is None:
            return
        buf = self.bufs[self.n % len(self.bufs)]
        self.n += 1
        if self.side is None:
            dist.all_gather_into_tensor(buf, local.contiguous(), group=self.group)
        else:
            self.side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.side):
                dist.all_gather_into_tensor(buf, local, group=self.group)
                local.record_stream(self.side)
        self.last = buf.view((self.world,) + self.shape)

    def finish(self):
        if self.side is not None:
            torch.cuda.current_stream(self.device).wait_stream(self.side)
        return self.last


def assemble(gathered, shards, rows_of_rank, n_requests, heads):
    """Global [n_requests, 1, heads, width] output from an LPT plan's gathered buffer.
    gathered: [world, max_rows, 1, H_max, width]; rows_of_rank[k]: the shards of rank k
    in the order its rows were written."""
    width = gathered.shape[-1]
    out = torch.empty(n_requests, 1, heads, width, dtype=gathered.dtype, device=gathered.device)
    for k, mine in enumerate(rows_of_rank):
        for row, s in enumerate(mine):
            out[s.request, :, s.head_lo:s.head_hi] = gathered[k, row, :, :s.head_hi - s.head_lo]
    return out


class RankFailure(RuntimeError):
    """A peer rank stopped taking part (it raised, exited or never joined)."""


class PeerCheck:
    """Step-by-step liveness over the process group's store: every rank posts the
    step it is about to run; ``wait(step)`` returns once all ranks have posted it,
    or raises ``RankFailure`` naming the ranks missing after ``timeout_s``.  A rank
    that fails posts ``abort`` so the others stop at once instead of waiting out
    the timeout.  Runs on the host between steps, before any collective launch."""

    def __init__(self, store, rank, world, timeout_s=5.0, prefix="tao/step"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = timeout_s, prefix

    def post(self, step):
        self.store.set(f"{self.prefix}/{self.rank}", str(step))

    def abort(self, why):
        self.store.set(f"{self.prefix}/abort", f"{self.rank}: {why}")

    def wait(self, step):
        self.post(step)
        deadline = time.monotonic() + self.timeout_s
        missing = list(range(self.world))
        while True:
            if self.store.check([f"{self.prefix}/abort"]):
                raise RankFailure("peer aborted: " + self.store.get(f"{self.prefix}/abort").decode())
            still = []
            for k in missing:
                key = f"{self.prefix}/{k}"
                if not self.store.check([key]) or int(self.store.get(key)) < step:
                    still.append(k)
            missing = still
            if not missing:
                return
            if time.monotonic() > deadline:
                raise RankFailure(f"ranks {missing} did not reach step {step} within {self.timeout_s} s")
            time.sleep(0.005)


def shard_heads(x, shard):
    """The head slice of [..., H, D] operands (or [H, D, 3] fusion parameters) that a shard serves."""
    if x.dim() == 3:
        return x[shard.head_lo:shard.head_hi]
    return x[..., shard.head_lo:shard.head_hi, :]


def balanced_heads(heads, groups):
    """Equal contiguous head groups (``heads`` divisible by ``groups``)."""
    if heads % groups:
        raise ValueError("heads must divide evenly into head groups")
    step = heads // groups
    return [(i * step, (i + 1) * step) for i in range(groups)]


__all__ = ["requests_of_rank", "decode_bytes_per_token", "Shard", "plan_lpt", "plan_imbalance",
           "OutputGather", "assemble", "RankFailure", "PeerCheck", "shard_heads", "balanced_heads"]
