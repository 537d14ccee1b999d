"""Benchmark of the device path (one JSON line on rank 0).

Headline workload: BrFS of the 4x4 sliding-tile task (60 seeded random blank moves from the solved layout, seed 0) to
depth 22, the whole reachable space below that depth, witness pruning and canonical order on (mymyr::brfs defaults),
stop_at_goal off. One step = one complete BrFS (22 expanded layers). Metric: BrFS expanded states/s. Secondary: env
steps/s of 65,536 envs of the two-room, 40-ball transport task.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--depth D]

N > 1 runs under torchrun, one process per GPU, and shards the search by state-hash owner (NCCL reductions, NVLink
peer-memory exchange of successors). Without --depth, N GPUs search to depth 22 + log2(N) (weak scaling: each layer
of this space holds about 2.1 times the states of the one before, so the states per GPU stay about constant); with
--depth the search is the same at every N (strong scaling). --impl reference times the reference's own CPU BrFS
(oracle/_ref, mymyr::brfs with deterministic ids, all host threads) on the same workload.
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
    ap.add_argument("--env-steps", type=int, default=200)
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--depth", type=int, default=None,
                    help="BrFS depth at every N (default: 22 + log2(N), weak scaling; profiling runs use a smaller case)")
    ap.add_argument("--quick", action="store_true", help="timed BrFS only: no e2e, CPU baseline or env leg")
    ap.add_argument("--no-astar", action="store_true", help="skip the A* leg")
    ap.add_argument("--leg", choices=["all", "astar", "env"], default="all",
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


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """SM clocks and clock-event reasons during the timed region, sampled by NVML every 50 ms from a thread (set up
    before the timed region, so that no driver start-up cost falls inside it)."""

    REASONS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
               "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
               "sw_power_cap": "nvmlClocksEventReasonSwPowerCap"}

    def __init__(self, cuda_index: int):
        self.samples = []
        self.error = None
        self.h = None
        self.stop = threading.Event()
        try:
            import pynvml
            import torch

            self.nv = pynvml
            pynvml.nvmlInit()
            p = torch.cuda.get_device_properties(cuda_index)
            try:
                bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.bits = {k: getattr(pynvml, v) for k, v in self.REASONS.items()}
        except Exception as e:  # no NVML: the line says so
            self.error = f"nvml unavailable: {e}"

    def _run(self):
        nv = self.nv
        while not self.stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, reasons))
            except Exception as e:
                self.error = str(e)
                return
            self.stop.wait(0.05)

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
                "reasons": reasons, "samples": len(self.samples), "source": "nvml"}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args, world, rank):
    """The reference arm: mymyr::brfs on the host cores (rank 0 only)."""
    if rank != 0:
        return
    from mymyr_b200 import tasks
    from oracle import ref

    if not ref.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built (make -C oracle)"}))
        return
    threads = os.cpu_count() or 1
    depth, scaling = bench_depth(args, world)
    # a step is one reference BrFS; past depth 23 it takes a bounded sample of the workload (the same space to depth
    # 23, the first 23 of its layers), so that the whole run ends within minutes
    sample_depth = min(depth, 23)
    rt = ref.RefTask(tasks.sliding_tile(4, 4, 60, 0))
    for _ in range(args.warmup):
        rt.brfs(threads=threads, max_depth=sample_depth, stop_at_goal=False, store="concurrent")
    times, expanded = [], 0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        r = rt.brfs(threads=threads, max_depth=sample_depth, stop_at_goal=False, store="concurrent")
        times.append(time.perf_counter() - t0)
        expanded = r["expanded"]
    total = sum(times)
    value = expanded * args.steps / total
    sample = (f"the full workload x {args.steps} runs" if sample_depth == depth else
              f"the workload's first {sample_depth} layers ({expanded} expanded) x {args.steps} runs")
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "u64", "data": "synthetic",
            "config": {"workload": workload(depth), "threads": threads, "store": "concurrent",
                       "deterministic_ids": True},
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


def env_secondary(args, device, world=1, rank=0, pg=None):
    """Env steps/s of the 65,536-env pool; at N > 1 each rank steps its shard of the env ids (first_env = rank x rows;
    an env's trajectory depends only on its global id), with no communication. Device time, max over ranks."""
    import torch

    from mymyr_b200 import rl as b2rl
    from mymyr_b200 import tasks
    from mymyr_b200.task import Task

    t = Task.from_text(tasks.transport(2, 40, 2, 0))
    total = 65536
    n = total // world
    env = b2rl.BatchedEnv(t, n, seed=0, device=device, first_env=rank * n)
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        env.reset(stream=stream.cuda_stream)
        for _ in range(20):
            env.step(stream=stream.cuda_stream)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.env_steps):
            env.step(stream=stream.cuda_stream)
        b.record(stream)
    stream.synchronize()
    ms = a.elapsed_time(b)
    if pg is not None:
        x = torch.tensor([ms], dtype=torch.float64, device=device)
        pg.all_reduce(x, op=pg.ReduceOp.MAX)
        ms = float(x.item())
    return {"metric": "env steps/sec (65,536 envs, transport 2 rooms/40 balls/2 grippers)",
            "value": n * world * args.env_steps / (ms / 1000.0), "unit": "steps/s", "steps_timed": args.env_steps,
            "ms_per_step": ms / args.env_steps, "envs_per_rank": n,
            "parallelism": f"env ids sharded over {world} GPUs" if world > 1 else "single"}


def astar_secondary(args, device, with_cpu: bool, comm=None, pg=None):
    """A* with h^max on config [5] (logistics, 8 cities x 4 locations, 6 trucks, 2 airplanes, 2 packages): the time
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
        out = astar_secondary(args, device, with_cpu=False, comm=leg_comm, pg=pg) if args.leg == "astar" else \
            env_secondary(args, device, world, rank, pg)
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

    def one(expected=None, timings=False):
        r = b2cuda.brfs(task, max_depth=depth, stop_at_goal=False, timings=timings, expected_states=expected,
                        stream=sp, comm=comm)
        r.close()  # free the search's device buffers now (back to the pool for the next step)
        return r

    clk = Clocks(local)  # NVML set up before the warm-up: no driver start-up inside the timed region
    r = one()
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
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    results = []
    with clk:
        ev0.record(stream)
        for _ in range(args.steps):
            results.append(one(expected))
        ev1.record(stream)
        stream.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)
    clocks = clk.summary()
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

    secondary = None if args.no_secondary else env_secondary(args, device, world, rank, pg)
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
                       "expected_states": "presized from the warm-up run"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None,
                         "kernel": "b2j_brfs_expand + k_resolve + winners scan" if world == 1 else
                                   "b2j_dbrfs_expand + k_push + k_dinsert + id scan (per rank)",
                         "algorithmic_bytes_per_run": bytes_run, "kernel_ms_per_run": kern_ms,
                         "peak_source": peak_kind},
            "cpu_baseline": base,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "clocks": clocks,
            "phases_ms_per_run": phases,
            "secondary": secondary,
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
