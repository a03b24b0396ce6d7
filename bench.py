"""Benchmark of the block-Gibbs sweep path (node-updates/s).

Workload (the sparse random-graph Ising configuration): Erdos-Renyi graph
with N = 2^20 nodes and mean degree 8, J_ij ~ N(0, 1/8) symmetric, h_i ~ N(0,
0.1) (variances), beta = 1, greedy colouring into k blocks (one sampling group
each), 256 chains per GPU, seeded synthetic data.  One bench step = one run of
200 sweeps over all k groups for all chains of every GPU.

* `value`: steps on device-resident state (CUDA-graph replay of 200 sweeps),
  one CUDA event pair per step on the executor's stream, barrier + synchronize
  on both sides, max over ranks.  The bit-packed state (32 MiB) and the CSR
  tables fit in L2, so L2 is flushed (256 MiB write) before every step,
  outside the timed windows.
* `e2e`: the same metric through the public API: each step is one
  `Executor.sample_states` call (pinned host initial state -> 200 sweeps ->
  final state back on the host), wall clock with synchronize on both sides.
* `roofline`: the sparse spin kernel, algorithmic bytes per launch (neighbour
  state rows read, own row written, CSR tables read once; a row is 32 B
  bit-packed or 256 B as int8) over the CUDA-event duration of each launch,
  against the measured HBM copy bandwidth.
* `cpu_baseline`: the CPU oracle (C restatement of the reference's group
  math) on this host's cores over a bounded sample of the same workload.

`--impl reference` times only the CPU oracle (the reference itself needs JAX,
thrml and Tenstorrent hardware, none of which exist here) on all host cores.
Multi-GPU: launched by torchrun, one rank per GPU; chains are sharded (weak
scaling, no collective inside the timed loop).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
N_NODES = 1 << 20
MEAN_DEGREE = 8.0
CHAINS_PER_GPU = 256
SWEEPS_PER_STEP = 200
SEED = 0
WORKLOAD = "er-ising-n1048576-deg8-c256pergpu-s200"
METRIC = "node-updates/sec (sites x chains x sweeps / s)"


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _traffic_per_launch(avg_algorithmic_bytes: float):
    """DRAM bytes of an average sparse-spin launch, from the committed ncu summary.

    The summary holds one captured launch (DRAM read + write bytes and its
    algorithmic bytes); the figure is scaled to the average launch of a sweep
    by algorithmic bytes.  None when no summary is committed.
    """
    f = ROOT / "profiles" / "spin_bits_er1m_c256.md"
    if not f.exists():
        return None
    vals = {}
    for line in f.read_text().splitlines():
        if ":" in line and line.split(":", 1)[0] in ("traffic_bytes_per_launch", "algorithmic_bytes_captured_launch"):
            try:
                vals[line.split(":", 1)[0]] = float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    if len(vals) != 2:
        return None
    return vals["traffic_bytes_per_launch"] * avg_algorithmic_bytes / vals["algorithmic_bytes_captured_launch"]


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(f"/tmp/tthrml_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"],
                stdout=open(self.path, "w"),
                stderr=subprocess.DEVNULL,
            )
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = [r.split(",") for r in self.path.read_text().strip().splitlines() if r.strip()]
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
                for name, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        try:
            self.path.unlink()
        except OSError:
            pass
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


def build_workload():
    from tt_thrml_b200 import workloads

    return workloads.erdos_renyi_ising(N_NODES, MEAN_DEGREE, seed=SEED)


def algorithmic_bytes(prog, n_chains: int, layout: str):
    """Per block launch: state bytes (each neighbour row read once, own row written once) plus the
    CSR tables read once (8 B per edge: column + weight; 4 B bias and 8 B offset per row).
    A state row is n_chains bytes in the int8 layout and n_chains/8 bytes bit-packed."""
    row_bytes = n_chains // 8 if layout == "bits" else n_chains
    out = []
    for s in prog.specs:
        n = s.n_nodes
        nnz = int(s.interactions[1].row_ptr[-1])
        out.append(row_bytes * (nnz + n) + 8 * nnz + 4 * n + 8 * (n + 1))
    return out


def cpu_oracle_sample(prog, n_chains: int, n_sweeps: int, threads: int):
    """Times the CPU oracle on `n_sweeps` full sweeps of `n_chains` chains; returns (updates/s, seconds)."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as orc

    o = orc.OracleSampler(prog, n_chains=n_chains, n_threads=threads)
    rng = np.random.default_rng(1)
    o.load_state([rng.integers(0, 2, (n_chains, len(b.nodes))).astype(bool) for b in prog.gibbs_spec.free_blocks])
    o.sweep(0, seed=7)  # warm
    t0 = time.perf_counter()
    for s in range(n_sweeps):
        o.sweep(1 + s, seed=7)
    dt = time.perf_counter() - t0
    return N_NODES * n_chains * n_sweeps / dt, dt


def run_reference(args):
    """CPU arm: the oracle restatement of the reference's group kernel on all host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    prog = build_workload()
    chains = 32  # bounded sample: all 2^20 nodes, 32 chains, one sweep per step
    for _ in range(args.warmup):
        cpu_oracle_sample(prog, chains, 1, threads)
    times = []
    for _ in range(args.steps):
        _, dt = cpu_oracle_sample(prog, chains, 1, threads)
        times.append(dt)
    tot = sum(times)
    value = N_NODES * chains * args.steps / tot
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "node-updates/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * tot / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded Erdos-Renyi graph, random init)",
        "config": {"workload": WORKLOAD, "sample": f"all {N_NODES} nodes x {chains} chains x 1 sweep per step"},
        "cpu_baseline": {
            "value": value,
            "unit": "node-updates/s",
            "cores": threads,
            "kind": "port",
            "sample": f"CPU oracle (C restatement, float32 state), {N_NODES} nodes x {chains} chains, 1 sweep/step",
        },
        "e2e": {"value": value, "unit": "node-updates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)

    from tt_thrml_b200 import Executor, make_cuda_config
    from tt_thrml_b200.backend import CudaDevice

    prog = build_workload()
    k = len(prog.specs)
    C = CHAINS_PER_GPU
    device = CudaDevice(local)
    cfg = make_cuda_config(n_chains=C, cuda_graphs=True)
    total_sweeps = SWEEPS_PER_STEP * (args.steps + args.warmup) + 16
    ex = Executor(None, device, prog, cfg, n_sweeps=total_sweeps, n_chains=C, chain_offset=rank * C)
    kinds = {g.kernel_artifact.kind for g in ex.compiled.sampling_groups}
    assert kinds <= {"spin_csr", "spin_bits"}, kinds
    rng = np.random.default_rng(100 + rank)
    init = [rng.integers(0, 2, (C, len(b.nodes))).astype(bool) for b in prog.gibbs_spec.free_blocks]
    ex.load_state(init, [])
    ex.prepare_rng(SEED)
    stream = ex.stream

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # ---- device-resident steps: warmup, then K timed steps
    for _ in range(args.warmup):
        ex.run_sweeps(SWEEPS_PER_STEP)
    barrier()
    # Each step is timed by its own event pair; between steps a 256 MiB buffer is
    # written so every step starts with a cold L2 (the bit-packed state and the
    # CSR tables together fit in the 126 MB L2).
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        for e0, e1 in events:
            with torch.cuda.stream(stream):
                flush.fill_(1)
            e0.record(stream)
            ex.run_sweeps(SWEEPS_PER_STEP)
            e1.record(stream)
        barrier()
    dt_ms = sum(e0.elapsed_time(e1) for e0, e1 in events)
    del flush
    if dist is not None:
        t = torch.tensor([dt_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt_ms = float(t.item())
    updates = world * N_NODES * C * SWEEPS_PER_STEP * args.steps
    value = updates / (dt_ms / 1000.0)
    gpu_launches = args.steps * (SWEEPS_PER_STEP * k + 1)

    # ---- roofline: per-launch CUDA events on the launch stream (eager sweeps)
    layout = ex.compiled.state_dtype
    per_block_bytes = algorithmic_bytes(prog, C, layout)
    ex.profile = True
    ex._timing_log.clear()
    n_prof = 5
    for _ in range(n_prof):
        ex.run_sweep()
    ex.profile = False
    kernel_ms = [kms for _, _, kms in ex._timing_log]
    launch_bytes = per_block_bytes * n_prof
    achieved = sum(launch_bytes) / (sum(kernel_ms) / 1000.0) / 1e9
    peak, peak_kind = _peaks()
    traffic = _traffic_per_launch(sum(per_block_bytes) / len(per_block_bytes)) if layout == "bits" else None

    # ---- end to end through the public API (pinned host state in, final state out)
    from tt_thrml_b200.observers import StateObserver

    pinned = [torch.from_numpy(s.astype(np.int8) * 2 - 1).pin_memory() for s in init]

    class _Sched:
        n_warmup, n_samples, steps_per_sample = SWEEPS_PER_STEP, 1, 1

    nodes = prog.gibbs_spec.free_blocks
    ex.sample_states(SEED + 1, _Sched, nodes, init_state_free=pinned)  # warm the graph for this schedule
    barrier()
    e2e_times = []
    for s in range(args.steps):
        barrier()
        t0 = time.perf_counter()
        out = ex.sample_states(SEED + 2 + s, _Sched, nodes, init_state_free=pinned)
        torch.cuda.synchronize(dev)
        e2e_times.append(time.perf_counter() - t0)
    assert out[0].shape == (1, C, len(nodes[0].nodes))
    e2e_s = sum(e2e_times)
    if dist is not None:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = updates / e2e_s
    h2d = N_NODES * C  # int8 ±1 initial state
    d2h = N_NODES * C  # bool final state

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, _ = cpu_oracle_sample(prog, 32, 1, threads)
        cpu = {
            "value": v,
            "unit": "node-updates/s",
            "cores": threads,
            "kind": "port",
            "sample": f"CPU oracle (C restatement, float32 state), {N_NODES} nodes x 32 chains x 1 sweep",
        }

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "node-updates/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": dt_ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "u32 bit-packed spins, f32 fields" if ex.compiled.state_dtype == "bits" else "int8 spins, f32 fields",
            "data": "synthetic (seeded Erdos-Renyi graph, random init)",
            "config": {
                "workload": WORKLOAD,
                "n_nodes": N_NODES,
                "mean_degree": MEAN_DEGREE,
                "colour_blocks": k,
                "chains_per_gpu": C,
                "sweeps_per_step": SWEEPS_PER_STEP,
                "rng": "philox4x32-10 on device",
                "state_layout": ex.compiled.state_dtype,
                "l2": "flushed before every timed step (256 MiB write)",
                "parallelism": f"chain-sharded x{world}",
            },
            "roofline": {
                "kernel": "k_spin_bits" if layout == "bits" else "k_spin_csr_async",
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "peak_source": peak_kind,
                "traffic": traffic,
                "algorithmic_bytes_per_update": sum(per_block_bytes) / (N_NODES * C),
            },
            "e2e": {
                "value": e2e_value,
                "unit": "node-updates/s",
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
            },
            "gpu_launches": gpu_launches,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-sweeps", type=int, default=0,
                    help="run this many eager sweeps of the workload and exit (profiler target, no timing)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.profile_sweeps:
        return run_profile_target(args.profile_sweeps)
    return run_ours(args)


def run_profile_target(n_sweeps: int) -> int:
    """Eager sweeps of the bench workload: one kernel launch per colour block per sweep."""
    import torch

    from tt_thrml_b200 import Executor, make_cuda_config

    prog = build_workload()
    C = CHAINS_PER_GPU
    ex = Executor(None, 0, prog, make_cuda_config(n_chains=C, cuda_graphs=False), n_sweeps=n_sweeps, n_chains=C)
    rng = np.random.default_rng(100)
    ex.load_state([rng.integers(0, 2, (C, len(b.nodes))).astype(bool) for b in prog.gibbs_spec.free_blocks], [])
    ex.prepare_rng(SEED)
    for _ in range(n_sweeps):
        ex.run_sweep()
    torch.cuda.synchronize()
    print(f"profile target: {n_sweeps} sweeps x {len(prog.specs)} blocks", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
