#!/usr/bin/env python
"""Benchmark of the TaoMemory attention hot path on B200.

Headline workload ("decode128k"): per GPU, 8 independent
requests (one state each), H=12, D=64, bf16, each prefilled with 131,072
synthetic tokens ~N(0,1) through the public prefill API, then decoded one token
per request per step for the config's 256 decode steps.  A step is one decode
token for every request on the rank (weak scaling: 8 requests per GPU); the
timed window is the last K of the 256 steps, so it holds the seal at position
131,327 and the route refreshes before it.

Reported (one JSON line on rank 0):
* value      -- decode tokens/s over all ranks, inputs resident in HBM, steps
                launched through the C ABI (BatchDecoder), L2 flushed between
                timed steps (1 GiB memset outside the timed window);
* e2e        -- the same metric through the public Python API (DecodeSession:
                the step's inputs handed over in page-locked host memory, the
                output back in host memory, one captured graph per step); host
                clock per step, the device synchronised at the end of every step
                (a caller that needs each token's output before the next);
* parity     -- the timed steps' outputs and route ids against the CPU oracle
                continuing the same states (exported before the window) on the
                same inputs: every element, every request, every head;
* roofline   -- achieved HBM GB/s of the main decode kernel = algorithmic bytes /
                CUDA-event duration, against the measured copy bandwidth;
* cpu_baseline -- the CPU oracle (reference port) on a bounded sample;
* serving    -- BASELINE.json config 5 (64 requests, prompts 2K-128K, H16 D128,
                snapshots mid-stream), requests x head groups planned over the
                ranks by LPT, with the whole step's HBM roofline;
* train8k    -- BASELINE.json config 2 (tao_attention forward + backward, B4 T8192
                H12 D64 bf16) with its own value / e2e / roofline / cpu_baseline.
With N > 1 ranks every rank decodes its own 8 requests and the step's outputs are
gathered to rank 0 over NCCL on a side stream (tao_memory_b200.shard).

``--impl reference`` times the reference's algorithm on the host CPU (the oracle
port in oracle/tao_oracle.py) on the same config and prints the same line, with a
``reference_triton`` object: the unmodified reference (installed in baseline/_ref)
running its own Triton path on one B200.
"""

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s @128K ctx"
UNIT = "tok/s"
REQUESTS, HEADS, WIDTH, CONTEXT, LAYER, DECODE_STEPS = 8, 12, 64, 131072, 0, 256
L2_FLUSH_BYTES = 1 << 30   # also keeps the GPU busy while the host enqueues the step
L2_CLEAN_BYTES = 1 << 28   # read after the memset: its dirty lines are written back before timing
# DRAM bytes (read + write) of one decode_fused_kernel launch at this workload (the
# timed window's last steps), from the full capture
#   ncu --set full --clock-control none -k regex:decode_fused_kernel --nvtx --nvtx-include "timed_decode/" \
#       -c 1 -o fused64 python bench.py --no-train --no-serving --no-parity --steps 6 --warmup 3
# (dram__bytes_read.sum + dram__bytes_write.sum of that capture).
DECODE_TRAFFIC_BYTES = 46640896
# The same for read_bwd_kernel in the train8k workload, one launch of
#   ncu --section SpeedOfLight --section MemoryWorkloadAnalysis --section WarpStateStats \
#       --metrics dram__bytes_read.sum,dram__bytes_write.sum --clock-control none \
#       -k regex:read_bwd_kernel -s 3 -c 1 python bench.py --workload train8k --steps 2 --warmup 3
# (dram__bytes_read.sum + dram__bytes_write.sum of that capture).
READ_BWD_TRAFFIC_BYTES = 348393216


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--requests", type=int, default=REQUESTS)
    ap.add_argument("--context", type=int, default=CONTEXT)
    ap.add_argument("--cpu-sample-steps", type=int, default=4)
    ap.add_argument("--workload", default="decode128k", choices=["decode128k", "train8k", "serving"])
    ap.add_argument("--serving-requests", type=int, default=None,
                    help="serving leg: the first N requests of the 64 (profiling captures of a smaller case)")
    ap.add_argument("--no-train", action="store_true", help="leave the nested train8k leg out")
    ap.add_argument("--no-serving", action="store_true", help="leave the nested serving (config 5) leg out")
    ap.add_argument("--no-parity", action="store_true", help="leave the oracle parity check out")
    ap.add_argument("--decode-variant", type=int, default=None,
                    help="decode kernel of tao_decode_step (tao_decode_variant: 1 default, 0, 2, 3, 4)")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed loops run."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.samples = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for s in self.samples for n, v in zip(names, s[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


class Events:
    """CUDA events through the library (recorded on the launching stream)."""

    def __init__(self, lib, n):
        from tao_memory_b200 import _lib
        self.lib, self._lib = lib, _lib
        self.ev = []
        for _ in range(n):
            e = ctypes.c_void_p()
            _lib.check(lib.tao_event_create(ctypes.byref(e)))
            self.ev.append(e)

    def __getitem__(self, i):
        return self.ev[i]

    def elapsed(self, a, b):
        ms = ctypes.c_float()
        self._lib.check(self.lib.tao_event_elapsed(self.ev[a], self.ev[b], ctypes.byref(ms)))
        return ms.value

    def close(self):
        for e in self.ev:
            self.lib.tao_event_destroy(e)


# ---------------------------------------------------------------------------
# B200 arm: decode128k
# ---------------------------------------------------------------------------

def prefill_states(tb, preset, n, context, device, seed):
    """n fresh states, each advanced through `context` synthetic tokens with the
    public prefill API (pieces of 16K tokens to bound input memory)."""
    import torch
    gen = torch.Generator(device=device)
    states = []
    fa = (torch.randn(HEADS, WIDTH, 3, device=device, generator=gen.manual_seed(seed)) * 0.02).to(torch.bfloat16)
    fb = (torch.randn(HEADS, WIDTH, 3, device=device, generator=gen) * 0.02).to(torch.bfloat16)
    piece = 16384
    for r in range(n):
        st = tb.new_state(LAYER, preset(graph=True))   # graph mode: the e2e leg replays one captured step
        gen.manual_seed(seed * 1000 + r + 1)
        pos = 0
        while pos < context:
            w = min(piece, context - pos)
            x = [torch.randn(1, w, HEADS, WIDTH, device=device, generator=gen).to(torch.bfloat16)
                 for _ in range(5)]
            tb.tao_attention_prefill(x[0], x[1], x[2], raw_q=x[3], raw_k=x[4], fusion_a=fa,
                                     fusion_b=fb, alpha=0.5, state=st, position=pos)
            pos += w
        states.append(st)
    return states, fa, fb


def decode_parity(exported, inputs, outs, fa, fb, states):
    """Continue the exported states on the CPU oracle with the timed steps' inputs;
    compare every output element and the final route ids with the GPU's."""
    import torch
    from oracle import tao_oracle as o
    torch.set_num_threads(os.cpu_count() or 1)
    fa, fb = fa.cpu(), fb.cpu()
    xs = inputs.cpu()                 # [K, 5, R, 1, H, D]
    got = outs.float().cpu()          # [K, R, 1, H, D]
    bad, worst, elems, route_bad = 0, 0.0, 0, 0
    hosts = []
    for r, snap in enumerate(exported):
        st = o.OracleStream.from_export(snap)
        ref = torch.cat([st.step(*(xs[i, j, r:r + 1] for j in range(5)), fa, fb, 0.5)
                         for i in range(xs.shape[0])], 1).float()          # [1, K, H, D]
        mine = got[:, r].permute(1, 0, 2, 3)                                # [1, K, H, D]
        err = (mine - ref).abs()
        bad += int((err > 2e-2 + 2e-2 * ref.abs()).sum())
        worst = max(worst, err.max().item())
        elems += ref.numel()
        gpu_ids = states[r].export()["route_ids"][1].cpu()
        route_bad += int(not torch.equal(gpu_ids, st.route_ids[1]))
        hosts.append(st)
    return {"checked": "every output element of the timed steps, all requests and heads, and the "
                       "final route ids, against oracle/tao_oracle.py continuing the states "
                       "exported before the window on the same inputs",
            "requests": len(exported), "steps": int(xs.shape[0]), "elements": elems,
            "tolerance": "|a-b| <= 2e-2 + 2e-2|b|", "out_of_tolerance": bad,
            "max_abs_err": round(worst, 6), "route_mismatches": route_bad}, hosts


def run_b200(args, world, rank, local):
    import torch
    import torch.distributed as dist
    import tao_memory_b200 as tb
    from tao_memory_b200 import _lib
    from tao_memory_b200.presets import index_only_page_memo
    from tao_memory_b200.shard import OutputGather
    from tao_memory_b200.stream import BatchDecoder, decode_bytes, is_refresh, window_start

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    R, K, W = args.requests, args.steps, args.warmup
    lib = _lib.lib()
    if args.decode_variant is not None:
        _lib.check(lib.tao_decode_variant(args.decode_variant))
    stream = torch.cuda.current_stream(device).cuda_stream

    t0 = time.time()
    states, fa, fb = prefill_states(tb, index_only_page_memo, R, args.context, device, seed=rank + 1)
    torch.cuda.synchronize()
    prefill_s = time.time() - t0

    # decode schedule: [lead untimed][e2e: E2E_WARM + K][warm-up W][kernel window K][timed K],
    # ending at the config's last decode step (256) when it fits.  The kernel window times
    # the fused kernel alone (events around it, for the roofline); the timed window has
    # events around whole steps only, since every event pair recorded inside a step adds
    # its own latency to the step (about 5 us on this GPU).
    E2E_WARM = 3                      # untimed e2e steps: graph capture, first replays
    n_e2e = E2E_WARM + K
    lead = max(0, DECODE_STEPS - (n_e2e + W + 2 * K))
    total_steps = lead + n_e2e + W + 2 * K
    gen = torch.Generator(device=device).manual_seed(10_000 + rank)
    inputs = torch.randn(total_steps, 5, R, 1, HEADS, WIDTH, device=device, generator=gen).to(torch.bfloat16)
    outs = torch.empty(K, R, 1, HEADS, WIDTH, dtype=torch.bfloat16, device=device)
    scratch_out = torch.empty(R, 1, HEADS, WIDTH, dtype=torch.bfloat16, device=device)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    clean = torch.ones(L2_CLEAN_BYTES // 4, dtype=torch.float32, device=device)
    gather = OutputGather(dist.group.WORLD if world > 1 else None, (R, 1, HEADS, WIDTH), torch.bfloat16, device)

    def flush_l2():
        """Evict L2 outside the timed window: write 1 GiB, then read 256 MB of clean
        lines so the memset's dirty lines are written back now, not by the step."""
        flush.zero_()
        clean.sum()

    dec = BatchDecoder(states, fa, fb, 0.5, device)
    dec.reserve(total_steps + 1)

    def step_ptrs(i):
        x = inputs[i]
        return [x[j].data_ptr() for j in range(5)]

    for i in range(lead):
        dec.step(*step_ptrs(i), scratch_out.data_ptr())
    torch.cuda.synchronize()
    dec.check()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)

    # ---- e2e: public API, operands in page-locked host memory, output back to host,
    # host clock per step with the device synchronised at the end of each step
    host_in = inputs[lead:lead + n_e2e].cpu().pin_memory()
    session = tb.DecodeSession(states, fa, fb, 0.5, reserve=total_steps + 1)
    e2e_s = []
    for i in range(n_e2e):
        flush_l2()
        torch.cuda.synchronize()
        if world > 1 and i == E2E_WARM:
            dist.barrier()
        t_a = time.perf_counter()
        session.inputs.copy_(host_in[i])                          # the caller's bytes into the session
        session.step()
        session.wait()                                            # the step's output is in host memory
        e2e_s.append(time.perf_counter() - t_a)
    session.check()
    e2e_s = e2e_s[E2E_WARM:]
    dec._sync_ptrs()

    def window_bytes():
        base = [st.position for st in states]
        per = []
        for i in range(K):
            for st, p in zip(states, base):
                st.position = p + i
            per.append(decode_bytes(states))
        for st, p in zip(states, base):
            st.position = p
        return per

    # ---- warm-up, the kernel window and the timed window (C ABI, inputs resident in HBM)
    for i in range(W):
        dec.step(*step_ptrs(lead + n_e2e + i), scratch_out.data_ptr())
    torch.cuda.synchronize()
    dec.check()
    kern0 = lead + n_e2e + W
    algo_bytes = window_bytes()
    ev = Events(lib, 4 * K)
    torch.cuda.synchronize()
    for i in range(K):
        flush_l2()
        lib.tao_stream_profile_next(ev[4 * i + 2], ev[4 * i + 3])
        dec.step(*step_ptrs(kern0 + i), scratch_out.data_ptr())
    torch.cuda.synchronize()
    dec.check()
    main_ms = [ev.elapsed(4 * i + 2, 4 * i + 3) for i in range(K)]
    kernel_positions = [states[0].position - K, states[0].position - 1]
    exported = [st.export() for st in states] if (rank == 0 and not args.no_parity) else None
    timed0 = kern0 + K
    timed_bytes = window_bytes()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("timed_decode")
    for i in range(K):
        flush_l2()                        # evict L2 (outside the timed window)
        lib.tao_event_record(ev[4 * i], stream)
        dec.step(*step_ptrs(timed0 + i), outs[i].data_ptr())
        gather.start(outs[i])            # side stream; overlaps the next step
        lib.tao_event_record(ev[4 * i + 1], stream)
    gather.finish()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    dec.check()
    clocks.stop()
    step_ms = [ev.elapsed(4 * i, 4 * i + 1) for i in range(K)]
    ev.close()
    cfg = states[0].config
    p0 = states[0].position - K
    gpu_launches = sum(1 + any(is_refresh(p0 + i, st.layer_index, cfg) for st in states)
                       + any(p0 + i + 1 - window_start(p0 + i) == 768 for st in states) for i in range(K))
    seals = sum(p0 + i + 1 - window_start(p0 + i) == 768 for i in range(K))
    refreshes = sum(is_refresh(p0 + i, LAYER, cfg) for i in range(K))
    total_ms = sum(step_ms)
    e2e_ms = sum(e2e_s) * 1e3

    tot = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms = tot.tolist()
    tokens = world * R * K

    peaks, peak_kind = measured_peaks()
    peak = float(peaks["hbm_gbs"])
    achieved = sum(algo_bytes) / (sum(main_ms) * 1e-3) / 1e9
    result = {
        "metric": METRIC, "value": round(tokens / (total_ms * 1e-3), 1), "unit": UNIT,
        "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(total_ms / K, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic ~N(0,1), seeded",
        "config": {"workload": "decode128k (BASELINE.json config 4)", "requests_per_gpu": R,
                   "context": args.context, "heads": HEADS, "head_dim": WIDTH, "layer_index": LAYER,
                   "preset": "index_only_page_memo(graph=True)",
                   "timed_positions": [p0, p0 + K - 1], "seals_in_window": seals,
                   "refreshes_in_window": refreshes,
                   "l2": "flushed between timed steps (1 GiB memset, then a 256 MB read so the memset's "
                         "dirty lines are written back outside the timed window)",
                   "parallelism": f"{world} GPU(s), requests sharded, outputs gathered to rank 0 over NCCL"
                                  if world > 1 else "1 GPU",
                   "prefill_s": round(prefill_s, 2),
                   "prefill_tok_s": round(R * args.context / prefill_s, 1)},
        "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 1), "unit": UNIT,
                "h2d_bytes_per_step": 5 * R * HEADS * WIDTH * 2,
                "d2h_bytes_per_step": R * HEADS * WIDTH * 2,
                "timing": "host clock per step: the caller's bytes into the session's page-locked "
                          "buffer, DecodeSession.step() (one captured graph: copy in, decode, copy out), "
                          "wait() for the output in host memory; max over ranks",
                "ms_per_step_median": round(statistics.median(e2e_s) * 1e3, 4)},
        "roofline": {"bound": "hbm", "kernel": "decode_fused_kernel (tao_decode_step main kernel, variant %s)"
                     % (1 if args.decode_variant is None else args.decode_variant),
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind + " (copy bandwidth)",
                     "algorithmic_bytes_per_launch": int(statistics.mean(algo_bytes)),
                     "kernel_ms_mean": round(statistics.mean(main_ms), 5),
                     "kernel_timing": "CUDA events around the fused kernel on its stream, L2 flushed "
                                      "before each launch, over the K steps just before the timed "
                                      "window (positions %d-%d), step bytes %.1f MB there and %.1f MB "
                                      "in the timed window" % (kernel_positions[0], kernel_positions[1],
                                                               statistics.mean(algo_bytes) / 1e6,
                                                               statistics.mean(timed_bytes) / 1e6),
                     "traffic": DECODE_TRAFFIC_BYTES},
        "gpu_launches": gpu_launches,
        "clocks": clocks.summary(),
    }
    return result, states, exported, inputs[timed0:timed0 + K], outs, fa, fb


# ---------------------------------------------------------------------------
# CPU legs (reference port = oracle/tao_oracle.py)
# ---------------------------------------------------------------------------

def synthetic_oracle_state(layer, context, seed):
    """A reference-port state at `context` tokens with seeded random contents of
    the exact shapes a real prefill leaves (values do not change decode cost)."""
    import torch
    from oracle import tao_oracle as o
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    st = o.OracleStream(layer)
    st.position = context
    start = 0 if context < 768 else 256 * ((context - 512) // 256)
    n = context - start
    st.local = tuple(torch.randn(1, n, HEADS, WIDTH, generator=g).to(bf) for _ in range(3))
    s = (context - 768) // 256 + 1 if context >= 768 else 0
    z = (torch.randn(1, HEADS, s, WIDTH, generator=g) + 5).to(bf)
    st.fine_c = (torch.randn(1, HEADS, s, WIDTH, WIDTH, generator=g) * 0.05).to(bf)
    full = s // 8
    st.pages = [(torch.logsumexp(z[:, :, 8 * p:8 * p + 8], dim=2).to(bf), z[:, :, 8 * p:8 * p + 8])
                for p in range(full)]
    st.pending = [z[:, :, i] for i in range(8 * full, s)]
    st.state_version = s
    q = torch.randn(1, 1, HEADS, WIDTH, generator=g).to(bf)
    st._read_segment(q, refresh=True)          # populate route ids as a refresh would
    return st


def time_oracle_decode(states, steps, seed, budget_s=None):
    """Decode `steps` tokens round-robin over the oracle states; return
    (tokens, seconds)."""
    import torch
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    fa = (torch.randn(HEADS, WIDTH, 3, generator=g) * 0.02).to(bf)
    fb = (torch.randn(HEADS, WIDTH, 3, generator=g) * 0.02).to(bf)
    toks = [torch.randn(5, 1, 1, HEADS, WIDTH, generator=g).to(bf) for _ in range(8)]
    done, t0 = 0, time.perf_counter()
    for i in range(steps):
        st = states[i % len(states)]
        x = toks[i % len(toks)]
        st.step(x[0], x[1], x[2], x[3], x[4], fa, fb, 0.5)
        done += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s:
            break
    return done, time.perf_counter() - t0


def cpu_baseline_decode(host_states, sample_steps):
    """Time the CPU oracle on a bounded sample of the same workload: GPU states
    exported and continued on the host cores."""
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    picked = host_states[:2]
    time_oracle_decode(picked, 2, seed=7)                       # warm-up
    n, secs = time_oracle_decode(picked, sample_steps * len(picked), seed=8, budget_s=30)
    return {"value": round(n / secs, 2), "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{n} decode tokens over {len(picked)} exported 128K-context requests "
                      f"(H{HEADS} D{WIDTH}), oracle/tao_oracle.py on the host CPU"}


# ---------------------------------------------------------------------------
# Serving workload: 64 requests, prompts log-uniform in
# 2K-128K, H16 D128, 128 decode steps, snapshots exported / imported after step 64,
# requests x head groups planned over the ranks by LPT (tao_memory_b200.shard)
# ---------------------------------------------------------------------------
SV_REQUESTS, SV_HEADS, SV_WIDTH, SV_STEPS, SV_SNAPSHOT_AT = 64, 16, 128, 128, 64


def serving_lengths(n=SV_REQUESTS, seed=71):
    import math
    import torch
    g = torch.Generator().manual_seed(seed)
    lo, hi = math.log(2048), math.log(131072)
    return [int(round(math.exp(lo + (hi - lo) * torch.rand(1, generator=g).item()))) for _ in range(n)]


def run_serving(args, world, rank, local):
    """Config 5 on this rank's LPT shards: prefill every shard (its head group of its
    request), decode the config's 128 steps with every request's state exported and
    imported after step 64, time the last K steps (device events, L2 flushed between
    steps).  A step decodes one token of every request on the rank; states of one head
    count decode as one batch."""
    import torch
    import torch.distributed as dist
    import tao_memory_b200 as tb
    from tao_memory_b200 import StreamCache
    from tao_memory_b200.presets import index_only_page_memo
    from tao_memory_b200.shard import plan_imbalance, plan_lpt
    from tao_memory_b200 import _lib
    from tao_memory_b200.stream import decode_bytes
    device = torch.device("cuda", local)
    if args.decode_variant is not None:
        _lib.check(_lib.lib().tao_decode_variant(args.decode_variant))
    lengths = serving_lengths()[:args.serving_requests or SV_REQUESTS]
    n_req = len(lengths)
    plan = plan_lpt(lengths, SV_HEADS, SV_WIDTH, world)
    mine = [s for s in plan if s.rank == rank]
    K, W = args.steps, args.warmup
    lead = max(0, SV_STEPS - W - K)
    gen = torch.Generator(device=device)
    fa = (torch.randn(SV_HEADS, SV_WIDTH, 3, device=device, generator=gen.manual_seed(5)) * 0.02).to(torch.bfloat16)
    fb = (torch.randn(SV_HEADS, SV_WIDTH, 3, device=device, generator=gen) * 0.02).to(torch.bfloat16)
    t0 = time.time()
    states, groups = [], {}
    for i, sh in enumerate(mine):
        hh = sh.head_hi - sh.head_lo
        st = tb.new_state(1, index_only_page_memo())
        gen.manual_seed(20_000 + sh.request)
        pos, L = 0, lengths[sh.request]
        while pos < L:
            w = min(16384, L - pos)
            x = torch.randn(5, 1, w, SV_HEADS, SV_WIDTH, device=device, generator=gen).to(torch.bfloat16)
            x = x[:, :, :, sh.head_lo:sh.head_hi].contiguous()
            tb.tao_attention_prefill(x[0], x[1], x[2], raw_q=x[3], raw_k=x[4], fusion_a=fa[sh.head_lo:sh.head_hi],
                                     fusion_b=fb[sh.head_lo:sh.head_hi], alpha=0.6, state=st, position=pos)
            pos += w
        states.append(st)
        groups.setdefault((hh, sh.head_lo), []).append(i)
    torch.cuda.synchronize()
    prefill_s = time.time() - t0
    steps = lead + W + K
    tokens_in = {key: torch.randn(steps, 5, len(idx), 1, key[0], SV_WIDTH, device=device,
                                  generator=gen.manual_seed(30_000 + rank * 97 + key[1])).to(torch.bfloat16)
                 for key, idx in groups.items()}
    outs = {key: torch.empty(len(idx), 1, key[0], SV_WIDTH, dtype=torch.bfloat16, device=device)
            for key, idx in groups.items()}
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    clean = torch.ones(L2_CLEAN_BYTES // 4, dtype=torch.float32, device=device)

    def step(i):
        for (hh, lo), idx in groups.items():
            x = tokens_in[(hh, lo)][i]
            tb.tao_attention_decode_batch(x[0], x[1], x[2], raw_q=x[3], raw_k=x[4], fusion_a=fa[lo:lo + hh],
                                          fusion_b=fb[lo:lo + hh], alpha=0.6,
                                          states=[states[j] for j in idx], out=outs[(hh, lo)])

    for i in range(lead + W):
        if i == min(SV_SNAPSHOT_AT, lead):
            states[:] = [StreamCache.from_export(st.export()) for st in states]
        step(i)
    torch.cuda.synchronize()
    algo = 0
    base = [st.position for st in states]
    for i in range(K):
        for st, p in zip(states, base):
            st.position = p + i
        algo += decode_bytes(states)
    for st, p in zip(states, base):
        st.position = p
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    if world > 1:
        dist.barrier()
    for i in range(K):
        flush.zero_()
        clean.sum()
        starts[i].record()
        step(lead + W + i)
        stops[i].record()
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in zip(starts, stops))
    tot = torch.tensor([ms, algo], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(tot[:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(tot[1:], op=dist.ReduceOp.SUM)
    ms, algo = tot.tolist()
    peaks, kind = measured_peaks()
    # all ranks' bytes over the slowest rank's time, against the peak of all ranks' HBM
    achieved = algo / (ms * 1e-3) / 1e9
    peak_all = float(peaks["hbm_gbs"]) * world
    return {
        "metric": "serving decode tok/s (64 requests, 2K-128K prompts)", "unit": "tok/s",
        "value": round(n_req * K / (ms * 1e-3), 1), "steps": K, "warmup": W,
        "ms_per_step": round(ms / K, 4), "n_gpus": world, "scaling": "strong",
        "config": {"workload": "serving (BASELINE.json config 5)", "requests": n_req, "heads": SV_HEADS,
                   "head_dim": SV_WIDTH, "prompts": "log-uniform 2K-128K (seed 71)",
                   "decode_steps": SV_STEPS, "timed": f"steps {lead + W}..{lead + W + K - 1}",
                   "snapshot": f"every state exported and imported after decode step {min(SV_SNAPSHOT_AT, lead)}",
                   "plan": f"LPT over requests x head groups, {len(plan)} shards, imbalance "
                           f"{plan_imbalance(plan, world):.3f}" if world > 1 else "1 GPU",
                   "prefill_s": round(prefill_s, 1),
                   "l2": "flushed between timed steps"},
        "roofline_step": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak_all,
                          "unit": "GB/s", "frac": round(achieved / peak_all, 4),
                          "peak_kind": kind + f" (copy bandwidth x {world} GPU(s))",
                          "algorithmic_bytes_per_step": int(algo / K),
                          "basis": "whole decode step (all launches of every batch) on the device clock"},
    }


# ---------------------------------------------------------------------------
# Training workload: tao_attention fwd+bwd, B4 T8192 H12 D64
# ---------------------------------------------------------------------------
TB, TT, TH, TD = 4, 8192, 12, 64


def local_attention_flops(tokens, heads, width, batch):
    """Exact forward FLOPs of the windowed local attention: 4*D per (query, key)."""
    total = 0
    for t in range(tokens):
        lo = max(0, 256 * (t // 256) - 512)
        total += t - lo + 1
    return 4 * width * total * heads * batch


def read_backward_flops(tokens, heads, width, batch, cfg):
    """Algorithmic FLOPs of the selected-read backward: every query of 256-query tile t
    selects exactly M(t) fines, and each (query, fine) pair costs dA = gn.C^T and its
    share of dC = A^T.gn, 2 x 2 x width^2 FLOPs."""
    from tao_memory_b200.config import routed_counts
    pairs = 0
    for tile in range((tokens + 255) // 256):
        visible = max(0, tile - 2)
        if visible == 0:
            continue
        m = routed_counts(visible // 8, visible % 8, cfg)[2]
        pairs += min(256, tokens - tile * 256) * m
    return 4 * width * width * pairs * heads * batch


def train_inputs(device, seed, batch=TB, tokens=TT):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    x = [torch.randn(batch, tokens, TH, TD, device=device, generator=g).to(torch.bfloat16) for _ in range(5)]
    fa = (torch.randn(TH, TD, 3, device=device, generator=g) * 0.02).to(torch.bfloat16)
    fb = (torch.randn(TH, TD, 3, device=device, generator=g) * 0.02).to(torch.bfloat16)
    alpha = torch.rand(TH, device=device, generator=g).tolist()
    grad = torch.randn(batch, tokens, TH, TD, device=device, generator=g).to(torch.bfloat16)
    return x, fa, fb, alpha, grad


def run_train_bench(args, world, rank, local):
    import torch
    import torch.distributed as dist
    import tao_memory_b200 as tb
    from tao_memory_b200 import _lib
    from tao_memory_b200.presets import index_only_page_memo
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    lib = _lib.lib()
    cfg = index_only_page_memo()
    x, fa, fb, alpha, grad = train_inputs(device, seed=1 + rank)
    leaves = [t.requires_grad_(True) for t in x] + [fa.requires_grad_(True), fb.requires_grad_(True)]

    def step():
        for t in leaves:
            t.grad = None
        out = tb.tao_attention(leaves[0], leaves[1], leaves[2], raw_q=leaves[3], raw_k=leaves[4],
                               fusion_a=leaves[5], fusion_b=leaves[6], alpha=alpha, config=cfg)
        out.backward(grad)
        return out

    K, W = args.steps, max(args.warmup, 3)
    for _ in range(W):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device).cuda_stream
    ev = Events(lib, 6 * K)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("timed_train")
    for i in range(K):
        lib.tao_event_record(ev[6 * i], stream)
        lib.tao_stream_profile_next(ev[6 * i + 2], ev[6 * i + 3])   # forward: local attention kernel
        for t in leaves:
            t.grad = None
        out = tb.tao_attention(leaves[0], leaves[1], leaves[2], raw_q=leaves[3], raw_k=leaves[4],
                               fusion_a=leaves[5], fusion_b=leaves[6], alpha=alpha, config=cfg)
        lib.tao_stream_profile_next(ev[6 * i + 4], ev[6 * i + 5])   # backward: selected-read backward
        out.backward(grad)
        lib.tao_event_record(ev[6 * i + 1], stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    step_ms = [ev.elapsed(6 * i, 6 * i + 1) for i in range(K)]
    attn_ms = [ev.elapsed(6 * i + 2, 6 * i + 3) for i in range(K)]
    rbwd_ms = [ev.elapsed(6 * i + 4, 6 * i + 5) for i in range(K)]
    ev.close()
    # e2e: operands from pinned host memory each step, loss scalar back to the host.
    # The next step's host->device copies run on a copy stream into the other half of
    # a double buffer while this step computes (an input pipeline); every step's
    # copies and its loss read-back are inside the timed window (host clock).
    host = [t.detach().cpu().pin_memory() for t in x] + [grad.cpu().pin_memory()]
    bufs = [[torch.empty_like(h, device=device) for h in host] for _ in range(2)]
    copy_stream = torch.cuda.Stream(device)
    main = torch.cuda.current_stream(device)
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()

    def stage_inputs(i):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[i % 2])      # step i-2 is done with this half
            for d, h in zip(bufs[i % 2], host):
                d.copy_(h, non_blocking=True)
            ready[i % 2].record(copy_stream)

    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_a = time.perf_counter()
    stage_inputs(0)
    for i in range(K):
        if i + 1 < K:
            stage_inputs(i + 1)
        main.wait_event(ready[i % 2])
        ops = [d.detach().requires_grad_(True) for d in bufs[i % 2][:5]]
        out = tb.tao_attention(ops[0], ops[1], ops[2], raw_q=ops[3], raw_k=ops[4], fusion_a=leaves[5],
                               fusion_b=leaves[6], alpha=alpha, config=cfg)
        loss = (out.float() * bufs[i % 2][5].float()).sum()
        loss.backward()
        loss_host.copy_(loss.detach(), non_blocking=True)
        free[i % 2].record(main)
    torch.cuda.synchronize()
    e2e_ms = (time.perf_counter() - t_a) * 1e3
    clocks.stop()
    total_ms = sum(step_ms)
    tot = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms = tot.tolist()
    tokens = world * TB * TT * K
    flops = local_attention_flops(TT, TH, TD, TB)
    achieved = flops / (statistics.mean(attn_ms) * 1e-3) / 1e12
    rb_flops = read_backward_flops(TT, TH, TD, TB, cfg)
    rb_achieved = rb_flops / (statistics.mean(rbwd_ms) * 1e-3) / 1e12
    step_flops = 260.9e9  # per step, fwd + bwd = 3 x the forward's 86.96 GFLOP (config 2 work count)
    step_achieved = step_flops / (total_ms / K * 1e-3) / 1e12
    peaks, kind = measured_peaks()
    peak = float(peaks["bf16_tflops_sustained"])
    kind += " (cuBLAS bf16, sustained)"
    return {
        "metric": "train fwd+bwd tokens/s @8K", "value": round(tokens / (total_ms * 1e-3), 1),
        "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(total_ms / K, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic ~N(0,1), seeded",
        "config": {"workload": "train8k (BASELINE.json config 2)", "batch": TB, "seq_len": TT,
                   "heads": TH, "head_dim": TD, "alpha": "U(0,1) per head",
                   "preset": "index_only_page_memo", "l2": "inputs (5 x 50 MB) larger than L2",
                   "parallelism": f"{world} GPU(s), one batch of 4 per GPU" if world > 1 else "1 GPU"},
        "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": 6 * TB * TT * TH * TD * 2, "d2h_bytes_per_step": 4,
                "timing": "host clock over the K steps, device synchronised at both ends; next step's "
                          "inputs copied on a second stream during this step"},
        # the step's dominant kernel (about a third of the step): selected-read backward
        "roofline": {"bound": "tensor", "kernel": "read_bwd_kernel (selected-read backward)",
                     "achieved": round(rb_achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(rb_achieved / peak, 4), "peak_kind": kind,
                     "algorithmic_flops_per_launch": rb_flops,
                     "kernel_ms_mean": round(statistics.mean(rbwd_ms), 4), "traffic": READ_BWD_TRAFFIC_BYTES},
        "roofline_step": {"bound": "tensor", "achieved": round(step_achieved, 1), "peak": peak,
                          "unit": "TFLOP/s", "frac": round(step_achieved / peak, 4),
                          "algorithmic_flops_per_step": step_flops},
        "roofline_local_attention": {"bound": "tensor", "kernel": "tc_window_attention_kernel (forward, tcgen05)",
                                     "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                                     "frac": round(achieved / peak, 4), "algorithmic_flops_per_launch": flops,
                                     "kernel_ms_mean": round(statistics.mean(attn_ms), 4)},
        "gpu_launches": 10 * K,
        "clocks": clocks.summary(),
    }


def cpu_train_baseline(budget_tokens=8192):
    """Oracle fwd+bwd on one batch row and one head of the 8K workload."""
    import torch
    from oracle import tao_oracle as o
    from oracle.inputs import make_inputs
    torch.set_num_threads(os.cpu_count() or 1)
    x, g = make_inputs(1, budget_tokens, 1, TD, seed=3)
    grad = torch.randn(1, budget_tokens, 1, TD, generator=g).to(torch.bfloat16)
    leaves = {k: v.clone().requires_grad_(True) for k, v in x.items()}
    t0 = time.perf_counter()
    out = o.tao_attention(leaves["q"], leaves["k"], leaves["v"], leaves["raw_q"], leaves["raw_k"],
                          leaves["fusion_a"], leaves["fusion_b"], 0.5)
    out.backward(grad)
    secs = time.perf_counter() - t0
    # one head of 12 and one batch row of 4: tokens/s of the full workload
    value = budget_tokens / (secs * TH)
    return {"value": round(value, 2), "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"fwd+bwd of 1 row x 1 head x {budget_tokens} tokens (of {TB} x {TH} heads), "
                      f"oracle/tao_oracle.py; value scaled to all {TH} heads"}


# ---------------------------------------------------------------------------
# Reference arm: the oracle port on the host CPU, plus the unmodified reference's
# own Triton path on one B200 (reference_triton)
# ---------------------------------------------------------------------------

def run_reference_cpu(args):
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    t0 = time.time()
    states = [synthetic_oracle_state(LAYER, args.context, seed=100 + r) for r in range(args.requests)]
    setup_s = time.time() - t0
    time_oracle_decode(states, max(args.warmup, 1), seed=1)
    n, secs = time_oracle_decode(states, args.steps, seed=2, budget_s=240)
    value = n / secs
    cores = torch.get_num_threads()
    return {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": args.gpus,
        "steps": n, "warmup": args.warmup, "ms_per_step": round(secs * 1e3 / n, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic ~N(0,1), seeded", "impl": "reference",
        "config": {"workload": "decode128k (BASELINE.json config 4)", "requests": args.requests,
                   "context": args.context, "heads": HEADS, "head_dim": WIDTH,
                   "preset": "index_only_page_memo", "step": "one decode token of one request (round robin)",
                   "state": "synthetic 128K-context states of the prefilled shapes (a CPU prefill of "
                            "131,072 tokens takes minutes; values do not change decode cost)",
                   "setup_s": round(setup_s, 1)},
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{n} decode tokens round-robin over {args.requests} synthetic "
                                   f"128K-context states (oracle/tao_oracle.py: the reference's "
                                   f"algorithm restated in PyTorch CPU ops)"},
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def reference_triton(args):
    """The unmodified reference (baseline/_ref) through its own public API on one
    B200: decode at 128K context (graph=True, one request at a time as its batch-1
    API serves them) and tao_attention forward + backward at the training config.
    Returns a dict (or {"unavailable": why})."""
    import torch
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "tao_attention")):
        return {"unavailable": "baseline/_ref is not installed"}
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    sys.path.insert(0, ref_root)
    try:
        import triton
        import tao_attention as ref
        from tao_attention.presets import index_only_page_memo as ref_preset
    except Exception as e:   # noqa: BLE001 - report why the comparator cannot run
        return {"unavailable": f"import failed: {type(e).__name__}: {e}"}
    out = {"versions": {"torch": torch.__version__, "triton": triton.__version__},
           "source": "baseline/_ref (pip install --no-deps of the reference, unmodified)"}
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    # decode @128K: one request prefilled, then timed decode steps in both configurations
    # (eager and graph); the state moves between them through export / from_export.  The
    # local attention of this torch build runs through cuDNN, which plans once per new
    # (query, key) length: a decode token's key count cycles through 513..768, so one full
    # cycle of 256 untimed decode steps first leaves every plan built and the timed steps
    # measure the steady state.
    try:
        gen = torch.Generator(device=dev).manual_seed(4242)
        fa = (torch.randn(HEADS, WIDTH, 3, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        fb = (torch.randn(HEADS, WIDTH, 3, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        K, W = args.steps, max(args.warmup, 3)
        t0 = time.time()
        with torch.inference_mode():
            st = ref.new_state(LAYER, ref_preset(graph=False))
            pos = 0
            while pos < args.context:
                w = min(16384, args.context - pos)
                x = [torch.randn(1, w, HEADS, WIDTH, device=dev, generator=gen).to(torch.bfloat16)
                     for _ in range(5)]
                _, st = ref.tao_attention_prefill(x[0], x[1], x[2], raw_q=x[3], raw_k=x[4], fusion_a=fa,
                                                  fusion_b=fb, alpha=0.5, state=st, position=pos)
                pos += w
            torch.cuda.synchronize()
            prefill_s = time.time() - t0
            snap = st.export()
            t0 = time.time()
            warm = torch.randn(256, 5, 1, 1, HEADS, WIDTH, device=dev, generator=gen).to(torch.bfloat16)
            for i in range(256):
                _, st = ref.tao_attention_decode(*warm[i, :3], raw_q=warm[i, 3], raw_k=warm[i, 4], fusion_a=fa,
                                                 fusion_b=fb, alpha=0.5, state=st, position=st.get_pos())
            torch.cuda.synchronize()
            plan_warm_s = time.time() - t0
            st.release_execution()
            modes = {}
            for graph in (False, True):
                saved = dict(snap, config=dict(snap["config"], q1_history_region_graph=graph))
                run = ref.StreamCache.from_export(saved)
                xs = torch.randn(W + K, 5, 1, 1, HEADS, WIDTH, device=dev, generator=gen).to(torch.bfloat16)
                for i in range(W):
                    _, run = ref.tao_attention_decode(*xs[i, :3], raw_q=xs[i, 3], raw_k=xs[i, 4], fusion_a=fa,
                                                      fusion_b=fb, alpha=0.5, state=run, position=run.get_pos())
                torch.cuda.synchronize()
                starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
                stops = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
                t_host = time.perf_counter()
                for i in range(K):
                    starts[i].record()
                    _, run = ref.tao_attention_decode(*xs[W + i, :3], raw_q=xs[W + i, 3], raw_k=xs[W + i, 4],
                                                      fusion_a=fa, fusion_b=fb, alpha=0.5, state=run,
                                                      position=run.get_pos())
                    stops[i].record()
                torch.cuda.synchronize()
                host_s = time.perf_counter() - t_host
                ms = [a.elapsed_time(b) for a, b in zip(starts, stops)]
                run.release_execution()
                per_tok = max(sum(ms) / K, host_s * 1e3 / K)
                modes["graph" if graph else "eager"] = {
                    "value": round(1e3 / per_tok, 1), "ms_per_token": round(per_tok, 4),
                    "device_ms_per_token": round(sum(ms) / K, 4), "host_ms_per_token": round(host_s * 1e3 / K, 4)}
        best = max(modes.values(), key=lambda m: m["value"])
        out["decode128k"] = {
            "value": best["value"], "unit": UNIT, "modes": modes, "steps": K, "warmup": W,
            "prefill_s": round(prefill_s, 1), "plan_warmup_s": round(plan_warm_s, 1),
            "how": "one 131,072-token request (H12 D64 bf16, index_only_page_memo(graph=False) for the prefill), "
                   "256 untimed decode steps (one cycle of key lengths, so torch's cuDNN attention plans are "
                   "built), then decoded from the 131,072-token snapshot in index_only_page_memo(graph=False) "
                   "and (graph=True) through export / from_export; "
                   "the reference serves batch 1, so 8 requests run one after another and the rate is "
                   "1 / time per token (the larger of the device and host time); value = the faster mode"}
    except Exception as e:   # noqa: BLE001
        out["decode128k"] = {"unavailable": f"{type(e).__name__}: {e}"}
    torch.cuda.empty_cache()
    # training fwd+bwd at config 2
    try:
        x, fa, fb, alpha, grad = train_inputs(dev, seed=77)
        leaves = [t.requires_grad_(True) for t in x] + [fa.requires_grad_(True), fb.requires_grad_(True)]
        # the reference API takes one Python alpha for all heads; the work does not depend on its value
        a0 = float(sum(alpha) / len(alpha))

        def step():
            for t in leaves:
                t.grad = None
            y = ref.tao_attention(leaves[0], leaves[1], leaves[2], raw_q=leaves[3], raw_k=leaves[4],
                                  fusion_a=leaves[5], fusion_b=leaves[6], alpha=a0, config=ref_preset())
            y.backward(grad)

        K, W = max(3, min(args.steps, 10)), 2
        for _ in range(W):
            step()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(K):
            step()
        s1.record()
        torch.cuda.synchronize()
        ms = s0.elapsed_time(s1) / K
        out["train8k"] = {"value": round(TB * TT / (ms * 1e-3), 1), "unit": "tok/s",
                          "ms_per_step": round(ms, 3), "steps": K, "warmup": W,
                          "how": "tao_attention forward + backward, B4 T8192 H12 D64 bf16, "
                                 "index_only_page_memo(), one scalar alpha (the API's form)"}
    except Exception as e:   # noqa: BLE001
        out["train8k"] = {"unavailable": f"{type(e).__name__}: {e}"}
    return out


def main():
    args = parse()
    world, rank, local = dist_env()
    if args.impl == "reference":
        if rank != 0:
            return 0
        if args.workload == "train8k":
            cb = cpu_train_baseline()
            line = {"metric": "train fwd+bwd tokens/s @8K", "value": cb["value"], "unit": "tok/s",
                    "n_gpus": args.gpus, "steps": 1, "warmup": 0, "higher_is_better": True,
                    "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                    "data": "synthetic ~N(0,1), seeded", "impl": "reference",
                    "config": {"workload": "train8k (BASELINE.json config 2)"},
                    "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "tok/s",
                                                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        else:
            line = run_reference_cpu(args)
        line["reference_triton"] = reference_triton(args)
        print(json.dumps(line), flush=True)
        return 0
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    try:
        if args.workload == "train8k":
            result = run_train_bench(args, world, rank, local)
            if rank == 0:
                result["cpu_baseline"] = cpu_train_baseline() if world == 1 else None
        elif args.workload == "serving":
            result = run_serving(args, world, rank, local)
        else:
            result, states, exported, timed_inputs, outs, fa, fb = run_b200(args, world, rank, local)
            if rank == 0 and exported is not None:
                result["parity"], hosts = decode_parity(exported, timed_inputs, outs, fa, fb, states)
                result["cpu_baseline"] = cpu_baseline_decode(hosts, args.cpu_sample_steps) if world == 1 else None
            elif rank == 0:
                result["cpu_baseline"] = None
            del states, exported, timed_inputs, outs
            torch.cuda.empty_cache()
            if not args.no_serving:
                serving = run_serving(args, world, rank, local)
                if rank == 0:
                    result["serving"] = serving
                torch.cuda.empty_cache()
            if not args.no_train:
                train = run_train_bench(args, world, rank, local)
                if rank == 0:
                    train["cpu_baseline"] = cpu_train_baseline() if world == 1 else None
                    result["train8k"] = train
        if rank == 0:
            print(json.dumps(result), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
