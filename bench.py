"""Benchmark of the device path (one JSON line on rank 0).

Headline workload: BrFS of the 4x4 sliding-tile task (60 seeded random blank moves from the solved layout, seed 0) to
depth 22, the whole reachable space below that depth, witness pruning and canonical order on (mymyr::brfs defaults),
stop_at_goal off. One step = one complete BrFS (22 expanded layers). Metric: BrFS expanded states/s. Every search is
checked against the reference's layer counts and states at its depth (tests/golden/tile4x4_brfs.json), the first one
also against its fingerprint; a mismatch ends the run with a non-zero exit code. Further legs in the same line: the
batched env step (65,536 envs of the two-room, 40-ball transport task, 1,000 random-policy steps), the lifted
successor-generation stress batch (1,048,576 random states of the seeded 16-schema domain at 5 % atom density) and A*
with h^max.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--depth D]

N > 1 runs under torchrun, one process per GPU, and shards the search by state-hash owner (NCCL reductions, NVLink
peer-memory exchange of successors). Without --depth, N GPUs search to depth 22 + log2(N) (weak scaling: each layer
of this space holds about 2.1 times the states of the one before, so the states per GPU stay about constant); with
--depth the search is the same at every N (strong scaling). --impl reference times the reference's own CPU BrFS
(oracle/_ref, mymyr::brfs with deterministic ids, all host threads) on the same workload at the same depth.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "BrFS expanded states/sec"
UNIT = "states/s"
DEPTH = 22


def workload(depth: int) -> str:
    return f"sliding-tile 4x4 BrFS to depth {depth} (seed 0, 60 scramble moves, whole space below the depth)"


def bench_depth(args, world: int) -> tuple[int, str]:
    """The search depth at `world` GPUs and the scaling it gives."""
    if args.depth is not None:
        return args.depth, "strong" if world > 1 else "weak"
    return DEPTH + max(0, round(math.log2(world))), "weak"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--env-steps", type=int, default=1000)
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--depth", type=int, default=None,
                    help="BrFS depth at every N (default: 22 + log2(N), weak scaling; profiling runs use a smaller case)")
    ap.add_argument("--quick", action="store_true", help="timed BrFS only: no e2e, CPU baseline or env leg")
    ap.add_argument("--no-astar", action="store_true", help="skip the A* leg")
    ap.add_argument("--no-expand", action="store_true", help="skip the successor-generation stress leg")
    ap.add_argument("--leg", choices=["all", "astar", "env", "expand"], default="all",
                    help="run one leg alone and print its JSON (profiling runs)")
    return ap.parse_args()


def algorithmic_bytes(layer_counts, W):
    """Per-layer algorithmic bytes of expansion + dedup: parent rows 8W*E, one 32-byte sector per probe 32*G, a stored
    row compare per duplicate 32*ceil(8W/32)*D, and per new state its row, slot sector and node record."""
    total = 0
    for E, G, N in layer_counts:
        D = G - N
        total += 8 * W * E + 32 * G + 32 * -(-8 * W // 32) * D + (8 * W + 32 + 8) * N
    return total


GOLDEN = ROOT / "tests" / "golden" / "tile4x4_brfs.json"


def golden(depth: int):
    """The reference's result at `depth` (tests/golden/make_brfs_golden.py), or None past the file's depths."""
    if not GOLDEN.exists():
        return None
    return json.loads(GOLDEN.read_text())["depths"].get(str(depth))


def check_golden(r, depth: int, fingerprint: bool) -> bool:
    """Compares a search with the reference's at its depth; exits with status 3 on a mismatch. False: no golden."""
    g = golden(depth)
    if g is None:
        return False
    got = {"states": r.states, "expanded": r.expanded, "generated": r.generated,
           "layer_counts": [list(x) for x in r.layer_counts]}
    want = {k: g[k] for k in got}
    if fingerprint:
        got["fingerprint"], want["fingerprint"] = f"{r.fingerprint:#018x}", g["fingerprint"]
    if got != want:
        print(json.dumps({"error": f"the search to depth {depth} differs from the reference's", "got": got,
                          "want": want}), flush=True)
        sys.exit(3)
    return True


def random_accesses(layer_counts):
    """Random DRAM accesses of expansion + dedup per search: one hash-set probe per candidate and one stored-row
    compare per duplicate (G + D over the layers); parent rows and new states' rows are streams, not counted."""
    return sum(G + (G - N) for _E, G, N in layer_counts)


# DRAM traffic of one depth-22 search's expansion + resolve + winners scan (one-GPU, compiled matcher), from the ncu
# launch list of profiles/launches_bench_tile4x4_depth22.md (dram__bytes_read.sum + dram__bytes_write.sum, the
# presized search's launches)
TRAFFIC_DEPTH22 = 5_573e6


def random_read_peak(device) -> float:
    """Random 8-byte reads per second over a 1 GiB table (torch.take of 2^25 random indices, CUDA events, best of 5):
    the denominator of the random-access roofline. Every such read costs a DRAM burst, so a random-access-bound
    kernel is bounded by this rate, not by the streaming copy bandwidth."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(0)
    table = torch.zeros(1 << 27, dtype=torch.int64, device=device)
    idx = torch.randint(0, 1 << 27, (1 << 25,), device=device, generator=g)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = float("inf")
    for rep in range(7):
        a.record()
        torch.take(table, idx)
        b.record()
        b.synchronize()
        if rep >= 2:
            best = min(best, a.elapsed_time(b))
    del table, idx
    torch.cuda.empty_cache()
    return (1 << 25) / (best / 1000.0)


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """SM clocks and clock-event reasons during the timed region, sampled by NVML every 200 ms from a thread of rank 0
    (set up before the timed region, so that no driver start-up cost falls inside it) for the GPUs of all ranks; the
    other ranks sample nothing, so that their search loops share no driver time with it."""

    REASONS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
               "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
               "sw_power_cap": "nvmlClocksEventReasonSwPowerCap"}

    def __init__(self, cuda_indices, enabled: bool = True):
        self.samples = []
        self.error = None
        self.h = None
        self.stop = threading.Event()
        if not enabled:
            self.error = "sampled by rank 0"
            return
        try:
            import pynvml
            import torch

            self.nv = pynvml
            pynvml.nvmlInit()
            self.hs = []
            for idx in cuda_indices:
                p = torch.cuda.get_device_properties(idx)
                try:
                    bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
                    self.hs.append(pynvml.nvmlDeviceGetHandleByPciBusId(bus))
                except Exception:
                    self.hs.append(pynvml.nvmlDeviceGetHandleByIndex(idx))
            self.h = self.hs[0]
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.bits = {k: getattr(pynvml, v) for k, v in self.REASONS.items()}
        except Exception as e:  # no NVML: the line says so
            self.error = f"nvml unavailable: {e}"

    def _run(self):
        nv = self.nv
        while not self.stop.is_set():
            try:
                for h in self.hs:
                    mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((mhz, reasons))
            except Exception as e:
                self.error = str(e)
                return
            self.stop.wait(0.2)

    def __enter__(self):
        if self.h is not None:
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        return self

    def __exit__(self, *a):
        self.stop.set()
        if self.h is not None:
            self.thread.join(timeout=5)

    def summary(self):
        if self.h is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.error or "no samples"]}
        reasons = sorted({k for _, r in self.samples for k, bit in self.bits.items() if r & bit})
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples), "gpus": len(self.hs), "source": "nvml"}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args, world, rank):
    """The reference arm: mymyr::brfs on the host cores (rank 0 only), on the same workload at the same depth as this
    repository's arm. A step is one whole search; when K such steps would take more than about four minutes, fewer
    are timed (the line's "steps" says how many)."""
    if rank != 0:
        return
    from mymyr_b200 import tasks
    from oracle import ref

    if not ref.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built (make -C oracle)"}))
        return
    threads = os.cpu_count() or 1
    depth, scaling = bench_depth(args, world)
    rt = ref.RefTask(tasks.sliding_tile(4, 4, 60, 0))
    t0 = time.perf_counter()
    first = rt.brfs(threads=threads, max_depth=depth, stop_at_goal=False, store="concurrent", fingerprint=True)
    one_s = time.perf_counter() - t0
    g = golden(depth)
    if g is not None and (first["states"] != g["states"] or f"{first['fingerprint']:#018x}" != g["fingerprint"]):
        print(json.dumps({"impl": "reference", "error": "the reference's search differs from its golden values"}))
        sys.exit(3)
    budget = 240.0
    steps = max(1, min(args.steps, int(budget / max(one_s, 1e-3))))
    warmup = max(0, min(args.warmup - 1, int(budget / 4 / max(one_s, 1e-3))))
    for _ in range(warmup):
        rt.brfs(threads=threads, max_depth=depth, stop_at_goal=False, store="concurrent")
    times, expanded = [], 0
    for _ in range(steps):
        t0 = time.perf_counter()
        r = rt.brfs(threads=threads, max_depth=depth, stop_at_goal=False, store="concurrent")
        times.append(time.perf_counter() - t0)
        expanded = r["expanded"]
    total = sum(times)
    value = expanded * steps / total
    sample = f"the full workload (depth {depth}, {expanded} expanded) x {steps} runs"
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
            "warmup": warmup + 1, "ms_per_step": 1000 * total / steps, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "u64", "data": "synthetic",
            "config": {"workload": workload(depth), "depth": depth, "threads": threads, "store": "concurrent",
                       "deterministic_ids": True, "steps_requested": args.steps,
                       "golden": "matches tests/golden/tile4x4_brfs.json" if g is not None else "no golden"},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline(steps_hint=1):
    from mymyr_b200 import tasks
    from oracle import ref

    if not ref.available():
        return None
    threads = os.cpu_count() or 1
    rt = ref.RefTask(tasks.sliding_tile(4, 4, 60, 0))
    t0 = time.perf_counter()
    r = rt.brfs(threads=threads, max_depth=DEPTH, stop_at_goal=False, store="concurrent")
    dt = time.perf_counter() - t0  # the headline depth: cpu_baseline is taken at N = 1 only
    return {"value": r["expanded"] / dt, "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": f"one full BrFS to depth {DEPTH} ({r['expanded']} expanded, {dt:.2f} s, mymyr::brfs "
                      f"concurrent store, {threads} threads)"}


ENV_BYTES_PER_STEP = 126  # algorithmic bytes of one env step at W = 3 words, label width 3 (see env_secondary)


def env_secondary(args, device, world=1, rank=0, pg=None, with_cpu=False):
    """Env steps/s of the 65,536-env pool over --env-steps random-policy steps (1,000 by default); at N > 1 each rank
    steps its shard of the env ids (first_env = rank x rows; an env's trajectory depends only on its global id), with
    no communication. Device time, max over ranks. Roofline: 126 algorithmic bytes per env step (state read and
    write 2 x 8W = 48, draw counter 16, step counter 8, goal flag 2, reward 4, four flags 4, schema 4, binding 12,
    count 4, final state 8W = 24). e2e: the same steps through BatchedEnv with the step's result (reward, terminated,
    truncated, count) read back to pinned host memory after every step."""
    import torch

    from mymyr_b200 import rl as b2rl
    from mymyr_b200 import tasks
    from mymyr_b200.task import Task

    text = tasks.transport(2, 40, 2, 0)
    t = Task.from_text(text)
    total = 65536
    n = total // world
    env = b2rl.BatchedEnv(t, n, seed=0, device=device, first_env=rank * n)
    stream = torch.cuda.Stream(device)
    launches = 0
    with torch.cuda.stream(stream):
        env.reset(stream=stream.cuda_stream)
        for _ in range(20):
            env.step(stream=stream.cuda_stream)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.env_steps):
            env.step(stream=stream.cuda_stream)
            launches += 1
        b.record(stream)
    stream.synchronize()
    ms_launch = a.elapsed_time(b)
    # the same steps as CUDA graphs of 50 steps each (the step launches one kernel and waits for nothing, so a graph
    # holds it as it is): the launches' host cost drops out
    per_graph = 50
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(per_graph):
            env.step(stream=stream.cuda_stream)
    replays = max(1, args.env_steps // per_graph)
    with torch.cuda.stream(stream):  # replay() launches on the current stream
        graph.replay()
        stream.synchronize()
        a.record(stream)
        for _ in range(replays):
            graph.replay()
        b.record(stream)
    stream.synchronize()
    ms_graph = a.elapsed_time(b) * args.env_steps / (replays * per_graph)
    launches += replays * per_graph
    ms = min(ms_launch, ms_graph)
    # e2e: the step's result to the host every step
    host = {k: torch.empty(n, dtype=getattr(env, k).dtype, pin_memory=True)
            for k in ("reward", "terminated", "truncated", "count")}
    e2e_steps = min(args.env_steps, 200)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for _ in range(e2e_steps):
            env.step(stream=stream.cuda_stream)
            for k, h in host.items():
                h.copy_(getattr(env, k), non_blocking=True)
            stream.synchronize()
    e2e_s = time.perf_counter() - t0
    d2h = sum(h.numel() * h.element_size() for h in host.values())
    if pg is not None:
        x = torch.tensor([ms, e2e_s], dtype=torch.float64, device=device)
        pg.all_reduce(x, op=pg.ReduceOp.MAX)
        ms, e2e_s = float(x[0]), float(x[1])
    value = n * world * args.env_steps / (ms / 1000.0)
    peak, peak_kind = measured_peaks()
    achieved = n * ENV_BYTES_PER_STEP / (ms / 1000.0 / args.env_steps) / 1e9
    out = {"metric": "env steps/sec (65,536 envs, transport 2 rooms/40 balls/2 grippers)",
           "value": value, "unit": "steps/s", "steps_timed": args.env_steps,
           "ms_per_step": ms / args.env_steps, "envs_per_rank": n, "gpu_launches": launches,
           "ms_per_step_launched": ms_launch / args.env_steps, "ms_per_step_graph": ms_graph / args.env_steps,
           "timing": "the faster of one launch per step and CUDA graphs of 50 steps (both timed over --env-steps)",
           "parallelism": f"env ids sharded over {world} GPUs" if world > 1 else "single",
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                        "traffic": None, "kernel": "b2j_env_step_nw", "peak_source": peak_kind,
                        "algorithmic_bytes_per_env_step": ENV_BYTES_PER_STEP,
                        "note": "the per-env arrays (8.3 MB per step) stay in L2: latency-bound, no HBM target"},
           "e2e": {"value": n * world * e2e_steps / e2e_s, "unit": "steps/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": d2h, "steps": e2e_steps}}
    if with_cpu:
        from oracle import ref

        if ref.available():
            threads = os.cpu_count() or 1
            csteps = 50
            sec, _ = ref.RefTask(text).pool_bench(total, csteps, threads, 0)
            out["cpu_baseline"] = {"value": total * csteps / sec, "unit": "steps/s", "cores": threads,
                                   "kind": "reference",
                                   "sample": f"rl::CpuEnvPool, {total} envs x {csteps} random-policy steps, "
                                             f"{threads} threads ({sec:.2f} s)"}
    return out


EXPAND_STATES = 1 << 20


def expand_secondary(args, device, world=1, rank=0, pg=None, with_cpu=False):
    """The lifted successor-generation stress test: b2_expand (rl::expand) of 1,048,576 random states of the seeded
    16-schema random domain (24 predicates of arity 1-3, 200 typed objects, 165-word rows), every fluent slot set at
    5 % density (tasks.bernoulli_rows, seed 0), witness pruning off, canonical order; a step is one call over the
    resident batch into preallocated outputs (offsets, parent, schema, binding, successor hash). At N > 1 each rank
    expands its shard of the rows (no communication). Roofline: 8W + 4 bytes per state (its row, its offset) plus 36
    per successor (schema 4, binding 4 x 5, hash 8, parent 4). e2e: the same call from pinned host memory, the batch
    copied in and the CSR copied out every step."""
    import ctypes as C

    import torch

    from mymyr_b200 import _lib, tasks
    from mymyr_b200.task import Task, default_context

    text = tasks.random_domain(0)
    t = Task.from_text(text, default_context(device.index))
    n = EXPAND_STATES // world
    states = tasks.bernoulli_rows(n, t.words, t.fluent_slots, 0.05, seed=0, device=device, first=rank * n,
                                  chunk=1 << 13)
    L = _lib.lib()
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))  # the rows were drawn on the current stream
    sp = stream.cuda_stream
    W, lw = t.words, max(1, t.label_width)
    probe = _lib.Expansion()
    offsets = torch.empty(n + 1, dtype=torch.int32, device=device)
    probe.offsets = offsets.data_ptr()
    _lib.check(L.b2_expand(t.handle, states.data_ptr(), n, W, 0, C.byref(probe), sp))
    m = probe.generated
    outs = {"parent": torch.empty(m, dtype=torch.int32, device=device),
            "schema": torch.empty(m, dtype=torch.int32, device=device),
            "binding": torch.empty((m, lw), dtype=torch.int32, device=device),
            "succ_hash": torch.empty(m, dtype=torch.int64, device=device)}
    e = _lib.Expansion()
    e.capacity, e.words, e.label_width = m, W, lw
    for k, v in outs.items():
        setattr(e, k, v.data_ptr())
    e.offsets = offsets.data_ptr()

    def call(src):
        _lib.check(L.b2_expand(t.handle, src.data_ptr(), n, W, 0, C.byref(e), sp))

    for _ in range(max(3, args.warmup)):
        call(states)
    steps = max(3, min(args.steps, 20))
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        call(states)
    b.record(stream)
    stream.synchronize()
    ms = a.elapsed_time(b) / steps
    # e2e from host memory: batch in, CSR out
    hstates = torch.empty_like(states, device="cpu").pin_memory()
    hstates.copy_(states)
    dstates = torch.empty_like(states)
    hout = {k: torch.empty_like(v, device="cpu").pin_memory() for k, v in outs.items()}
    hoff = torch.empty_like(offsets, device="cpu").pin_memory()
    e2e_steps = max(2, min(steps, 5))
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for _ in range(e2e_steps):
            dstates.copy_(hstates, non_blocking=True)
            call(dstates)
            hoff.copy_(offsets, non_blocking=True)
            for k, v in outs.items():
                hout[k].copy_(v, non_blocking=True)
            stream.synchronize()
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    h2d = hstates.numel() * 8
    d2h = hoff.numel() * 4 + sum(v.numel() * v.element_size() for v in hout.values())
    if pg is not None:
        x = torch.tensor([ms, e2e_s, float(m)], dtype=torch.float64, device=device)
        y = x.clone()
        pg.all_reduce(x, op=pg.ReduceOp.MAX)
        pg.all_reduce(y, op=pg.ReduceOp.SUM)
        ms, e2e_s, m_all = float(x[0]), float(x[1]), int(y[2])
    else:
        m_all = m
    peak, peak_kind = measured_peaks()
    bytes_call = n * (8 * W + 4) + m * 36
    achieved = bytes_call / (ms / 1000.0) / 1e9
    out = {"metric": "lifted successor generation states/sec (1,048,576 random states, 16 schemas, 200 objects)",
           "value": EXPAND_STATES / (ms / 1000.0), "unit": "states/s",
           "successors_per_s": m_all / (ms / 1000.0), "successors": m_all, "ms_per_batch": ms,
           "words": W, "states_per_rank": n, "steps_timed": steps, "gpu_launches": 5 * steps,
           "parallelism": f"rows sharded over {world} GPUs" if world > 1 else "single",
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                        "traffic": None, "kernel": "b2j_expand_count + scan + b2j_expand_write (one b2_expand call)",
                        "algorithmic_bytes_per_call": bytes_call, "peak_source": peak_kind},
           "e2e": {"value": EXPAND_STATES / e2e_s, "unit": "states/s", "h2d_bytes_per_step": h2d,
                   "d2h_bytes_per_step": d2h, "steps": e2e_steps}}
    if with_cpu:
        from oracle import ref

        if ref.available():
            threads = os.cpu_count() or 1
            k = 1 << 17
            r = ref.RefTask(text).expand(states[:k].cpu().numpy().view("uint64"), witness_pruning=False,
                                         threads=threads, capacity=m)
            out["cpu_baseline"] = {"value": k / r["seconds"], "unit": "states/s", "cores": threads,
                                   "kind": "reference",
                                   "sample": f"rl::expand (ThreadPool overload) of the batch's first {k} states, "
                                             f"{threads} threads ({r['seconds']:.2f} s, {r['generated']} successors)"}
    return out


def astar_secondary(args, device, with_cpu: bool, comm=None, pg=None):
    """A* with h^max on the logistics workload (logistics, 8 cities x 4 locations, 6 trucks, 2 airplanes, 2 packages): the time
    to the optimal plan and the expansions/s (device events around each search; at N > 1 the states are partitioned
    over the ranks by state-hash owner and the time is the slowest rank's), next to the reference's CPU A*
    (search::astar_eager, one thread: it has no thread option) on the same task."""
    import torch

    from mymyr_b200 import cuda as b2cuda
    from mymyr_b200 import tasks
    from mymyr_b200.task import Task

    cfg = (8, 4, 6, 2, 2, 0)
    text = tasks.logistics(*cfg)
    from mymyr_b200.task import default_context

    t = Task.from_text(text, default_context(device.index))
    H = b2cuda.Heuristic(t)
    stream = torch.cuda.Stream(device)
    r = b2cuda.astar(t, heuristic=H, stream=stream.cuda_stream, comm=comm)
    expected = r.states
    r.close()
    runs = []
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        r = b2cuda.astar(t, heuristic=H, stream=stream.cuda_stream, expected_states=expected, timings=True,
                         comm=comm)
        b.record(stream)
        stream.synchronize()
        runs.append((a.elapsed_time(b), r.expanded, r.generated, r.cost, r.stats, r.search_s))
        r.close()
    ms = statistics.median(x[0] for x in runs)
    if pg is not None:
        x = torch.tensor([ms], dtype=torch.float64, device=device)
        pg.all_reduce(x, op=pg.ReduceOp.MAX)
        ms = float(x.item())
    out = {"metric": "A* expansions/sec (h^max, logistics 8x4 cities/locations, 6 trucks, 2 airplanes, 2 packages)",
           "value": runs[-1][1] / (ms / 1000.0), "unit": "expansions/s", "ms_per_search": ms,
           "cost": runs[-1][3], "expanded": runs[-1][1], "generated": runs[-1][2],
           "phases_ms": {k: runs[-1][4][k] for k in ("count_ms", "expand_ms", "eval_ms")},
           "host_ms_per_search": statistics.median(x[5] for x in runs) * 1000,
           "parallelism": f"states sharded by hash owner over {comm.world} GPUs" if comm is not None else "single",
           "note": "each device step expands a whole f layer, so it expands more states than the one-at-a-time "
                   "reference; the time to the optimal plan compares the two"}
    if with_cpu:
        from oracle import ref

        if ref.available():
            rr = ref.RefTask(text).astar()
            out["cpu_baseline"] = {"ms_per_search": rr["seconds"] * 1000, "expanded": rr["expanded"],
                                   "value": rr["expanded"] / rr["seconds"], "unit": "expansions/s", "cores": 1,
                                   "kind": "reference", "cost": rr["cost"],
                                   "sample": "one full search (search::astar_eager, h^max, unit costs)"}
    return out


def main():
    args = parse()
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    import torch

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
        pg = dist
    if args.leg != "all":
        leg_comm = None
        if world > 1 and args.leg == "astar":
            from mymyr_b200.dist import Communicator
            from mymyr_b200.task import default_context

            leg_comm = Communicator(default_context(local))
        if args.leg == "astar":
            out = astar_secondary(args, device, with_cpu=False, comm=leg_comm, pg=pg)
        elif args.leg == "env":
            out = env_secondary(args, device, world, rank, pg)
        else:
            out = expand_secondary(args, device, world, rank, pg)
        if leg_comm is not None:
            leg_comm.close()
        if rank == 0:
            print(json.dumps(out), flush=True)
        if pg is not None:
            pg.destroy_process_group()
        return
    from mymyr_b200 import cuda as b2cuda
    from mymyr_b200 import tasks
    from mymyr_b200.task import Context, Task

    ctx = Context(local)
    comm = None
    if world > 1:
        from mymyr_b200.dist import Communicator

        comm = Communicator(ctx)
    depth, scaling = bench_depth(args, world)
    text = tasks.sliding_tile(4, 4, 60, 0)
    task = Task.from_text(text, ctx)
    stream = torch.cuda.Stream(device)
    sp = stream.cuda_stream

    def one(expected=None, timings=False, fingerprint=False):
        r = b2cuda.brfs(task, max_depth=depth, stop_at_goal=False, timings=timings, expected_states=expected,
                        stream=sp, comm=comm, fingerprint=fingerprint)
        r.close()  # free the search's device buffers now (back to the pool for the next step)
        return r

    # NVML set up before the warm-up (no driver start-up inside the timed region); rank 0 samples every rank's GPU
    clk = Clocks(list(range(world)), enabled=rank == 0)
    r = one(fingerprint=True)
    checked = check_golden(r, depth, fingerprint=True)  # exits on a mismatch
    expected = r.states
    # the warm-up searches also give the per-phase device times (per-layer events; the timed searches run without
    # them, as a user's would)
    phased = [one(expected, timings=True) for _ in range(max(1, args.warmup - 1))]

    def barrier():
        torch.cuda.synchronize(device)
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(device)

    # ---------------------------------------------------------------- timed region (device events)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    results = []
    # rank 0's sampler thread starts before the barrier: its start-up and first NVML queries overlap the barrier, not
    # the first search (whose collectives would make every other rank wait for it)
    with clk:
        barrier()
        ev0.record(stream)
        for _ in range(args.steps):
            results.append(one(expected))
        ev1.record(stream)
        stream.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)
    clocks = clk.summary()
    for rr in results + phased:
        check_golden(rr, depth, fingerprint=False)
    if pg is not None:
        t = torch.tensor([ms], dtype=torch.float64, device=device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    expanded = results[-1].expanded
    # every rank's search is the same one (sharded): the whole job expands `expanded` states per step
    value = expanded * args.steps / (ms / 1000.0)
    # roofline of expansion + dedup from its device events (a rank's share of the algorithmic bytes at N > 1, and its
    # expansion + exchange + insert + id phases, the slowest rank's)
    W = task.words
    bytes_run = algorithmic_bytes(results[-1].layer_counts, W) / world
    kern_ms = statistics.mean(r.stats.gen_ms + r.stats.dedup_ms for r in phased)
    exchanged = statistics.mean(r.stats.exchanged for r in phased)
    if pg is not None:
        t = torch.tensor([kern_ms, exchanged], dtype=torch.float64, device=device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        kern_ms, exchanged = float(t[0]), float(t[1])
    peak, peak_kind = measured_peaks()
    achieved = bytes_run / (kern_ms / 1000.0) / 1e9
    launches = sum(r.stats.kernel_launches for r in results)
    rand_run = random_accesses(results[-1].layer_counts) / world
    rand_peak = random_read_peak(device)

    phases = {"rehashes": results[-1].stats.rehashes,
              "count": statistics.mean(r.stats.count_ms for r in phased),
              "expand": statistics.mean(r.stats.gen_ms for r in phased),
              "rank": statistics.mean(r.stats.dedup_ms for r in phased),
              "source": "the warm-up searches, with per-layer events",
              "wall": statistics.mean(r.search_s * 1000 for r in results),
              "host_wait": statistics.mean(r.stats.wait_ms for r in results)}
    if world > 1:
        phases["exchange"] = statistics.mean(r.stats.exchange_ms for r in phased)  # part of "expand"
    if args.quick:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                              "depth": depth, "ms_per_step": ms / args.steps, "roofline_achieved": achieved,
                              "frac": achieved / peak, "phases_ms_per_run": phases, "quick": True}), flush=True)
        if comm is not None:
            comm.close()
        if pg is not None:
            pg.destroy_process_group()
        return
    # ---------------------------------------------------------------- end to end through the public API
    # every step: the task text becomes a Task (compiled on the host, uploaded), cuda.brfs runs the search (the
    # initial row goes up, the layer counts and totals come back) and the search is released, timed on the host
    barrier()
    e2e_times = []
    h2d = len(text.encode()) + 8 * W
    d2h = 0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        t2 = Task.from_text(text, ctx)
        rr = b2cuda.brfs(t2, max_depth=depth, stop_at_goal=False, expected_states=expected, stream=sp, comm=comm)
        counts = rr.layer_counts
        rr.close()
        e2e_times.append(time.perf_counter() - t0)
        d2h = 24 * len(counts) + 160  # the layer counts and the result struct
    e2e_s = sum(e2e_times)
    if pg is not None:
        t = torch.tensor([e2e_s], dtype=torch.float64, device=device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = expanded * args.steps / e2e_s

    secondary = None if args.no_secondary else env_secondary(args, device, world, rank, pg, with_cpu=world == 1)
    expand_line = None if args.no_expand else expand_secondary(args, device, world, rank, pg, with_cpu=world == 1)
    astar_line = None if args.no_astar else astar_secondary(args, device, with_cpu=world == 1, comm=comm, pg=pg)
    base = cpu_baseline() if rank == 0 and world == 1 else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": "u64", "data": "synthetic",
            "config": {"workload": workload(depth), "depth": depth, "states": results[-1].states,
                       "expanded": expanded, "generated": results[-1].generated, "layers": results[-1].layers,
                       "words": W,
                       "parallelism": (f"hash-owner sharded over {world} GPUs (NCCL all-reduce of counts and flags, "
                                       "NVLink peer-memory push of successors)") if world > 1 else "single",
                       "exchanged_per_rank": exchanged,
                       "l2": "working set > L2 (rows, table and frontiers are several hundred MB)",
                       "expected_states": "presized from the warm-up run",
                       "golden": (f"every search's states and layer counts, and the first one's fingerprint, equal "
                                  f"the reference's at depth {depth} (tests/golden/tile4x4_brfs.json)") if checked
                                 else f"no golden values for depth {depth}"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": TRAFFIC_DEPTH22 if world == 1 and depth == 22 else None,
                         "traffic_source": ("ncu launch list of the depth-22 search (expansion + resolve + winners "
                                            "scan), profiles/launches_bench_tile4x4_depth22.md")
                                           if world == 1 and depth == 22 else "not captured for this depth",
                         "kernel": "b2j_brfs_expand + k_resolve + winners scan" if world == 1 else
                                   "b2j_dbrfs_expand + k_push + k_dinsert + id scan (per rank)",
                         "algorithmic_bytes_per_run": bytes_run, "kernel_ms_per_run": kern_ms,
                         "peak_source": peak_kind,
                         "random_access": {"achieved": rand_run / (kern_ms / 1000.0) / 1e9,
                                           "peak": rand_peak / 1e9, "unit": "G accesses/s",
                                           "frac": rand_run / (kern_ms / 1000.0) / rand_peak,
                                           "accesses_per_run": rand_run,
                                           "peak_source": "random 8-byte reads over a 1 GiB table (torch.take), "
                                                          "measured in this run"}},
            "cpu_baseline": base,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "clocks": clocks,
            "phases_ms_per_run": phases,
            "secondary": secondary,
            "expand": expand_line,
            "astar": astar_line,
        }
        print(json.dumps(line), flush=True)
    if comm is not None:
        comm.close()
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
