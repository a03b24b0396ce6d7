"""Benchmark of the block-Gibbs sweep path (node-updates/s).

Default workload (`--workload er`, the headline: the sparse random-graph
Ising configuration): Erdos-Renyi graph with N = 2^20 nodes and mean degree 8,
J_ij ~ N(0, 1/8) symmetric, h_i ~ N(0, 0.1) (variances), beta = 1, greedy
colouring into k blocks (one sampling group each), 256 chains per GPU, seeded
synthetic data.  One bench step = one run of 200 sweeps over all k groups for
all chains of every GPU.  Other workloads: `--workload rbm` (Gauss-Bernoulli
RBM, 4096 gaussian visible x 8192 spin hidden, 8192 chains, 100 sweeps per
step; tensor-core roofline) and `--workload lattice` (64x64 Ising, 1024
chains, the schedule n_warmup=32 n_samples=64 steps_per_sample=2 per step).

* `value`: steps on device-resident state (CUDA-graph replay of the step's
  sweeps), one CUDA event pair per step on the executor's stream, barrier +
  synchronize on both sides, max over ranks.  L2 is flushed (256 MiB write)
  before every step, outside the timed windows.
* `e2e`: the same metric through the public API: each step is one
  `Executor.sample_states` call (pinned host initial state -> the sweeps ->
  final state back on the host; for the lattice, `sample_with_observation`
  with the magnetisation observed on device), wall clock with synchronize on
  both sides.
* `roofline`: the step's dominant kernel over per-launch CUDA events of eager
  sweeps: algorithmic bytes (sparse spin kernel: neighbour state rows read,
  own row written, CSR tables read once) against the measured HBM copy
  bandwidth, or algorithmic FLOPs (dense kernel: 2 x chains x visible x
  hidden per GEMM, two per sweep) against the measured bf16 GEMM peak.
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
SEED = 0


class ErIsing:
    """Sparse random-graph Ising: N = 2^20, Erdos-Renyi mean degree 8, greedy colouring, 256 chains/GPU, 200 sweeps."""

    name = "er"
    workload = "er-ising-n1048576-deg8-c256pergpu-s200"
    metric = "node-updates/sec (sites x chains x sweeps / s)"
    chains = 256
    sweeps = 200
    data = "synthetic (seeded Erdos-Renyi graph, random init)"
    cpu_chains, cpu_sweeps = 32, 1

    def build(self):
        from tt_thrml_b200 import workloads

        return workloads.erdos_renyi_ising(1 << 20, 8.0, seed=SEED)

    def init(self, prog, C, seed):
        rng = np.random.default_rng(seed)
        return [rng.integers(0, 2, (C, len(b.nodes))).astype(bool) for b in prog.gibbs_spec.free_blocks]

    def host_inputs(self, init):
        import torch

        return [torch.from_numpy(s.astype(np.int8) * 2 - 1).pin_memory() for s in init]

    def check(self, ex):
        kinds = {g.kernel_artifact.kind for g in ex.compiled.sampling_groups}
        assert kinds <= {"spin_csr", "spin_bits"}, kinds

    def config(self, prog, ex, world):
        return {
            "workload": self.workload,
            "n_nodes": _n_nodes(prog),
            "mean_degree": 8.0,
            "colour_blocks": len(prog.specs),
            "chains_per_gpu": self.chains,
            "sweeps_per_step": self.sweeps,
            "rng": "philox4x32-10 on device",
            "state_layout": ex.compiled.state_dtype,
            "l2": "flushed before every timed step (256 MiB write)",
            "parallelism": f"chain-sharded x{world}",
        }

    def dtype(self, ex):
        return "u32 bit-packed spins, f32 fields" if ex.compiled.state_dtype == "bits" else "int8 spins, f32 fields"

    def roofline(self, ex, prog, C, kernel_ms_per_group, n_prof):
        layout = ex.compiled.state_dtype
        per_block = algorithmic_bytes(prog, C, layout)
        achieved = sum(per_block) * n_prof / (sum(kernel_ms_per_group) / 1000.0) / 1e9
        peak, kind = _peaks()["hbm"]
        traffic = _traffic_per_launch(sum(per_block) / len(per_block)) if layout == "bits" else None
        return {
            "kernel": "k_spin_bits16" if layout == "bits" else "k_spin_csr_async",
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "peak_source": kind,
            "traffic": traffic,
            "algorithmic_bytes_per_update": sum(per_block) / (_n_nodes(prog) * C),
        }


class GaussBernoulliRBM:
    """Gauss-Bernoulli RBM: 4096 gaussian visible x 8192 spin hidden, W ~ N(0, 0.01^2), 8192 chains, 100 sweeps."""

    name = "rbm"
    workload = "gauss-bernoulli-rbm-v4096-h8192-c8192-s100"
    metric = "node-updates/sec (sites x chains x sweeps / s)"
    chains = 8192
    sweeps = 100
    data = "synthetic (seeded RBM weights rounded to bf16, random init)"
    cpu_chains, cpu_sweeps = 8, 1
    V, H = 4096, 8192

    def build(self):
        from tt_thrml_b200 import workloads

        return workloads.gaussian_bernoulli_rbm(self.V, self.H, seed=SEED)

    def init(self, prog, C, seed):
        rng = np.random.default_rng(seed)
        return [rng.standard_normal((C, self.V)).astype(np.float32), rng.integers(0, 2, (C, self.H)).astype(bool)]

    def host_inputs(self, init):
        import torch

        return [torch.from_numpy(init[0]).pin_memory(), torch.from_numpy(init[1]).pin_memory()]

    def check(self, ex):
        kinds = {g.kernel_artifact.kind for g in ex.compiled.sampling_groups}
        assert kinds == {"dense"}, kinds

    def config(self, prog, ex, world):
        return {
            "workload": self.workload,
            "n_visible": self.V,
            "n_hidden": self.H,
            "chains_per_gpu": self.chains,
            "sweeps_per_step": self.sweeps,
            "rng": "philox4x32-10 on device",
            "state_layout": "bf16 chain-major blocks (tcgen05 GEMM operands)",
            "l2": "operands (64-128 MiB per launch) exceed L2; flushed before every timed step (256 MiB write)",
            "parallelism": f"chain-sharded x{world}",
        }

    def dtype(self, ex):
        return "bf16 operands, f32 accumulate (tcgen05)"

    def roofline(self, ex, prog, C, kernel_ms_per_group, n_prof):
        flops = 2.0 * 2.0 * C * self.V * self.H * n_prof  # two GEMMs per sweep
        achieved = flops / (sum(kernel_ms_per_group) / 1000.0) / 1e12
        peaks = _peaks()
        peak, kind = peaks["bf16"]
        return {
            "kernel": "k_dense_field_sample",
            "bound": "tensor",
            "achieved": achieved,
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": achieved / peak,
            "peak_source": kind + " burst (kernels timed launch by launch)",
            "frac_of_sustained": achieved / peaks["bf16_sustained"][0],
            "traffic": _dense_traffic_per_launch(),
            "algorithmic_flops_per_update": 2.0 * 2.0 * self.V * self.H / (self.V + self.H),
        }


class Lattice2D:
    """2-D Ising 64x64 periodic, J=1, h=0, beta=0.44, 1024 chains; one step = the sampling schedule
    n_warmup=32, n_samples=64, steps_per_sample=2 with the per-chain magnetisation observed on device."""

    name = "lattice"
    workload = "ising2d-64x64-c1024-w32-n64-s2"
    metric = "node-updates/sec (sites x chains x sweeps / s)"
    chains = 1024
    sweeps = 32 + 63 * 2
    data = "synthetic (uniform +-1 init from seed 0)"
    cpu_chains, cpu_sweeps = 1024, 4

    def build(self):
        from tt_thrml_b200 import workloads

        return workloads.ising_lattice_2d(64, 64, J=1.0, h=0.0, beta=0.44)

    def init(self, prog, C, seed):
        rng = np.random.default_rng(seed)
        return [rng.integers(0, 2, (C, len(b.nodes))).astype(bool) for b in prog.gibbs_spec.free_blocks]

    def host_inputs(self, init):
        import torch

        return [torch.from_numpy(s.astype(np.int8) * 2 - 1).pin_memory() for s in init]

    def check(self, ex):
        kinds = {g.kernel_artifact.kind for g in ex.compiled.sampling_groups}
        assert kinds <= {"spin_csr", "spin_bits", "ising2d_resident"}, kinds

    def config(self, prog, ex, world):
        return {
            "workload": self.workload,
            "lattice": "64x64 periodic",
            "kernel": ex.compiled.sampling_groups[0].kernel_artifact.kind,
            "chains_per_gpu": self.chains,
            "sweeps_per_step": self.sweeps,
            "observable": "per-chain magnetisation, 64 samples, summed on device",
            "state_layout": ex.compiled.state_dtype,
            "l2": "state (512 KiB) is L2-resident by design; flushed before every timed step (256 MiB write)",
            "parallelism": f"chain-sharded x{world}",
        }

    def dtype(self, ex):
        return ErIsing.dtype(self, ex)

    def roofline(self, ex, prog, C, kernel_ms_per_group, n_prof, step_ms=None):
        if ex.compiled.sampling_groups[0].kernel_artifact.kind != "ising2d_resident":
            return ErIsing.roofline(self, ex, prog, C, kernel_ms_per_group, n_prof) | {"traffic": None}
        # shared-memory resident: one launch runs every sweep of a step; state bits read and written once per
        # half-sweep as if from memory (the algorithmic bytes), over the device time of the timed steps
        per_update = 2.0 / 8.0
        achieved = _n_nodes(prog) * C * self.sweeps * per_update / (step_ms / 1000.0) / 1e9
        peak, kind = _peaks()["hbm"]
        return {
            "kernel": "k_ising2d_resident",
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "peak_source": kind,
            "traffic": _profile_traffic("ising2d_resident_64x64_c1024.md"),
            "algorithmic_bytes_per_update": per_update,
            "note": "state resident in shared memory for the whole step; DRAM is touched only at launch start/end",
        }


class Potts3D:
    """3-D q=8 Potts 128^3 periodic, per-axis symmetric 8x8 couplings ~ N(0, 1), bias ~ N(0, 0.5), 64 chains,
    100 sweeps per step."""

    name = "potts"
    workload = "potts3d-128cube-q8-c64-s100"
    metric = "node-updates/sec (sites x chains x sweeps / s)"
    chains = 64
    sweeps = 100
    data = "synthetic (seeded couplings and biases, uniform random categories)"
    cpu_chains, cpu_sweeps = 64, 1
    side, q = 128, 8

    def build(self):
        from tt_thrml_b200 import workloads

        return workloads.potts_lattice_3d(self.side, self.q, seed=SEED)

    def cpu_program(self, prog):
        # the oracle runs on per-term tables, which a 128^3 lattice cannot afford: a 32^3 lattice of the
        # same model family gives the per-update CPU rate
        from tt_thrml_b200 import workloads

        return workloads.potts_lattice_3d(32, self.q, seed=SEED)

    def init(self, prog, C, seed):
        rng = np.random.default_rng(seed)
        return [rng.integers(0, self.q, (C, len(b.nodes))).astype(np.int8) for b in prog.gibbs_spec.free_blocks]

    def host_inputs(self, init):
        import torch

        return [torch.from_numpy(s).pin_memory() for s in init]

    def check(self, ex):
        kinds = {g.kernel_artifact.kind for g in ex.compiled.sampling_groups}
        assert kinds == {"potts3d"}, kinds

    def config(self, prog, ex, world):
        return {
            "workload": self.workload,
            "lattice": f"{self.side}^3 periodic",
            "q": self.q,
            "chains_per_gpu": self.chains,
            "sweeps_per_step": self.sweeps,
            "rng": "philox4x32-10 on device, inverse-CDF draw",
            "state_layout": "int8 categories [rows][chains]",
            "l2": "state 128 MiB + bias 32 MiB exceed L2; flushed before every timed step (256 MiB write)",
            "parallelism": f"chain-sharded x{world}",
        }

    def dtype(self, ex):
        return "int8 categories, f32 fields"

    def roofline(self, ex, prog, C, kernel_ms_per_group, n_prof):
        half = prog.n_sites // 2
        per_block = half * C * 2 + half * self.q * 4  # source rows read once, target rows written, bias read
        achieved = per_block * len(kernel_ms_per_group) / (sum(kernel_ms_per_group) / 1000.0) / 1e9
        peak, kind = _peaks()["hbm"]
        return {
            "kernel": "k_potts3d",
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "peak_source": kind,
            "traffic": _profile_traffic("potts3d_128cube_q8_c64.md") if C == self.chains else None,
            "algorithmic_bytes_per_update": per_block / (half * C),
        }


class BigIsing:
    """Single-chain 2-D Ising 32768^2 periodic, J=1, h=0, beta=0.4407, int8 spins, 1000 sweeps per step,
    domain-decomposed into row strips over the GPUs (deep halos exchanged every halo/2 sweeps)."""

    name = "ising"
    scaling = "strong"
    workload = "ising2d-32768sq-1chain-s1000-strips"
    metric = "node-updates/sec (sites x chains x sweeps / s)"
    side = 32768
    sweeps = 1000
    halo = 40  # 20 sweeps per exchange, 1000 = 50 exchanges
    data = "synthetic (uniform +-1 spins from a seeded hash of the site)"
    cpu_chains, cpu_sweeps = 1, 2

    def build(self):
        from tt_thrml_b200 import workloads

        return workloads.IsingLattice2D(self.side, self.side, beta=0.4407)

    def cpu_program(self, prog):
        # per-edge tables of the full lattice would take ~48 GB: a 1024^2 lattice gives the per-update rate
        from tt_thrml_b200 import workloads

        return workloads.IsingLattice2D(1024, 1024, beta=0.4407)

    def init(self, prog, C, seed):
        rng = np.random.default_rng(seed)
        return [rng.integers(0, 2, (C, len(b.nodes))).astype(bool) for b in prog.gibbs_spec.free_blocks]


WORKLOADS = {w.name: w for w in (ErIsing(), GaussBernoulliRBM(), Lattice2D(), Potts3D(), BigIsing())}


def run_ising(args, W):
    """The domain-decomposed lattice: strong scaling (the lattice is fixed, the strips shrink with N)."""
    import torch

    from tt_thrml_b200.domain import LatticeStrips

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    prog = W.build()
    S = W.sweeps
    st = LatticeStrips(prog, device=dev, halo=W.halo)
    st.load_random(SEED)
    st.prepare_rng(SEED, S * (args.steps + args.warmup) + S)
    stream = st._stream

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        st.run_sweeps(S)
    barrier()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    with ClockSampler(local) as clocks:
        for e0, e1 in events:
            with torch.cuda.stream(stream):
                flush.fill_(1)
            e0.record(stream)
            st.run_sweeps(S)
            e1.record(stream)
        barrier()
    del flush
    st.check_errors()
    dt_ms = sum(e0.elapsed_time(e1) for e0, e1 in events)
    if dist is not None:
        t = torch.tensor([dt_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt_ms = float(t.item())
    n_sites = W.side * W.side
    updates = n_sites * S * args.steps
    value = updates / (dt_ms / 1000.0)
    periods = S // (W.halo // 2)
    gpu_launches = args.steps * (periods * (W.halo + 2) + 1)  # import + half-sweeps + signal per period, ctl advance
    em = st.energy_magnetisation()

    # roofline: one eager half-sweep of the own rows, CUDA events on the launch stream
    hw = W.side // 2
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    n_prof = 10
    nat_bytes = 0
    st.cuda_graphs = False
    from tt_thrml_b200 import _native as nat

    nat.bind_device(local)
    with torch.cuda.stream(stream):
        ev[0].record(stream)
        for k in range(n_prof):
            st._cuda_halfsweep(k & 1, st.D, st.D + st.h, st.sweep, stream)
            nat_bytes += 2 * st.h * st.row_bytes  # other colour read once + own colour written once
        ev[1].record(stream)
    stream.synchronize()
    kms = ev[0].elapsed_time(ev[1]) / n_prof
    achieved = nat_bytes / n_prof / (kms / 1000.0) / 1e9
    peak, kind = _peaks()["hbm"]

    # end to end: pinned host split-colour lattice in, 1000 sweeps, energy/magnetisation trace out
    host = [torch.empty((W.side, hw), dtype=torch.int8).pin_memory() for _ in range(2)]
    for c in range(2):
        host[c].copy_(st._own_rows(c).cpu().repeat(W.side // st.h, 1))
    st.cuda_graphs = True
    e2e_times = []
    for s in range(args.steps):
        barrier()
        t0 = time.perf_counter()
        st.load_split_colours(host[0], host[1])
        st.prepare_rng(SEED + 1 + s, S)
        st.run_sweeps(S)
        trace = st.energy_magnetisation()
        torch.cuda.synchronize(dev)
        e2e_times.append(time.perf_counter() - t0)
    e2e_s = sum(e2e_times)
    if dist is not None:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    h2d = st.rows_local * hw * 2
    d2h = int(trace.nbytes)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, _ = cpu_oracle_sample(W, prog, W.cpu_chains, W.cpu_sweeps, threads)
        cpu = {"value": v, "unit": "node-updates/s", "cores": threads, "kind": "port",
               "sample": _cpu_sample_text(W, prog, W.cpu_chains, W.cpu_sweeps)}
    if rank == 0:
        line = {
            "metric": W.metric,
            "value": value,
            "unit": "node-updates/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": dt_ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "int8 spins" if st.storage == "int8" else "bit-packed spins (32 sites per uint32)",
            "data": W.data,
            "config": {
                "workload": W.workload,
                "lattice": f"{W.side}x{W.side} periodic, 1 chain",
                "sweeps_per_step": S,
                "strips": world,
                "halo_rows": W.halo,
                "exchange": "boundary rows stored into the neighbours' mailboxes by the half-sweep kernel (peer "
                            "memory over NVLink), flag per period, every halo/2 sweeps",
                "rng": "philox4x32-10 on device",
                "l2": "state 1 GiB exceeds L2; flushed before every timed step (256 MiB write)",
                "parallelism": f"row strips x{world}",
                "final_energy_per_site": float(em[-1, 0]),
                "final_magnetisation_per_site": float(em[-1, 1]),
            },
            "roofline": {
                "kernel": ("k_ising2d_bits" if st.storage == "bits" else
                           "k_ising2d_planes" if st.rng_layout == "planes" else "k_ising2d"),
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "peak_source": kind,
                "traffic": _profile_traffic("ising2d_32768.md") if st.storage == "bits" and world == 1 else None,
                "algorithmic_bytes_per_update": 2.0 * st.row_bytes / hw,
                "note": ("bit-packed rows move 0.25 B per update; the kernel is bound by instruction issue "
                         "(bit-sliced decision), not by HBM" if st.storage == "bits" else None),
            },
            "e2e": {"value": updates / e2e_s, "unit": "node-updates/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": gpu_launches,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0



def _n_nodes(prog):
    return sum(len(b.nodes) for b in prog.gibbs_spec.blocks)


def _peaks():
    """Roofline denominators: (value, "measured" | "fallback") per kind."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {
            "hbm": (float(d["hbm_gbs"]), "measured"),
            "bf16": (float(d["bf16_tflops"]), "measured"),
            "bf16_sustained": (float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"),
        }
    return {"hbm": (6650.0, "fallback"), "bf16": (1590.0, "fallback"), "bf16_sustained": (1400.0, "fallback")}


def _profile_figures(name: str, keys):
    """Machine-readable `key: value` lines of a committed ncu summary, or None."""
    f = ROOT / "profiles" / name
    if not f.exists():
        return None
    vals = {}
    for line in f.read_text().splitlines():
        k = line.split(":", 1)[0]
        if ":" in line and k in keys:
            try:
                vals[k] = float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return vals if len(vals) == len(keys) else None


def _profile_traffic(name: str):
    """DRAM bytes per launch recorded in a committed ncu summary (captured at the bench's full size), or None."""
    vals = _profile_figures(name, ("traffic_bytes_per_launch",))
    return None if vals is None else vals["traffic_bytes_per_launch"]


def _traffic_per_launch(avg_algorithmic_bytes: float):
    """DRAM bytes of an average sparse-spin launch, from the committed ncu summary.

    The summary holds one captured launch (DRAM read + write bytes and its
    algorithmic bytes); the figure is scaled to the average launch of a sweep
    by algorithmic bytes.  None when no summary is committed.
    """
    vals = _profile_figures(
        "spin_bits_er1m_c256.md", ("traffic_bytes_per_launch", "algorithmic_bytes_captured_launch")
    )
    if vals is None:
        return None
    return vals["traffic_bytes_per_launch"] * avg_algorithmic_bytes / vals["algorithmic_bytes_captured_launch"]


def _dense_traffic_per_launch():
    """DRAM bytes of an average dense launch of the RBM sweep, from the committed ncu summary (None if absent)."""
    vals = _profile_figures("dense_tc_rbm.md", ("traffic_bytes_per_launch_full_size",))
    return None if vals is None else vals["traffic_bytes_per_launch_full_size"]


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


def cpu_oracle_sample(W, prog, n_chains: int, n_sweeps: int, threads: int):
    """Times the CPU oracle on `n_sweeps` full sweeps of `n_chains` chains; returns (updates/s, seconds)."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as orc

    prog = W.cpu_program(prog) if hasattr(W, "cpu_program") else prog
    o = orc.OracleSampler(prog, n_chains=n_chains, n_threads=threads)
    o.load_state(W.init(prog, n_chains, 1))
    o.sweep(0, seed=7)  # warm
    t0 = time.perf_counter()
    for s in range(n_sweeps):
        o.sweep(1 + s, seed=7)
    dt = time.perf_counter() - t0
    return _n_nodes(prog) * n_chains * n_sweeps / dt, dt


def _cpu_sample_text(W, prog, chains, sweeps):
    prog = W.cpu_program(prog) if hasattr(W, "cpu_program") else prog
    return (f"CPU oracle (C restatement, float32 state), {_n_nodes(prog)} nodes x {chains} chains x "
            f"{sweeps} sweep(s) per sample")


def run_reference(args, W):
    """CPU arm: the oracle restatement of the reference's group kernel on all host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    prog = W.build()
    cprog = W.cpu_program(prog) if hasattr(W, "cpu_program") else prog
    chains, sweeps = W.cpu_chains, W.cpu_sweeps  # bounded sample of the workload per step
    for _ in range(args.warmup):
        cpu_oracle_sample(W, prog, chains, sweeps, threads)
    times = []
    for _ in range(args.steps):
        _, dt = cpu_oracle_sample(W, prog, chains, sweeps, threads)
        times.append(dt)
    tot = sum(times)
    value = _n_nodes(cprog) * chains * sweeps * args.steps / tot
    line = {
        "impl": "reference",
        "metric": W.metric,
        "value": value,
        "unit": "node-updates/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * tot / args.steps,
        "higher_is_better": True,
        "scaling": getattr(W, "scaling", "weak"),
        "vs_baseline": None,
        "dtype": "f32",
        "data": W.data,
        "config": {"workload": W.workload, "sample": f"all {_n_nodes(cprog)} nodes x {chains} chains x {sweeps} "
                                                      "sweep(s) per step"},
        "cpu_baseline": {
            "value": value,
            "unit": "node-updates/s",
            "cores": threads,
            "kind": "port",
            "sample": _cpu_sample_text(W, prog, chains, sweeps),
        },
        "e2e": {"value": value, "unit": "node-updates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args, W):
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
    from tt_thrml_b200.observers import MagnetizationObserver

    prog = W.build()
    n_nodes = _n_nodes(prog)
    C, S = W.chains, W.sweeps
    device = CudaDevice(local)
    cfg = make_cuda_config(n_chains=C, cuda_graphs=True)
    total_sweeps = S * (args.steps + args.warmup) + 16
    ex = Executor(None, device, prog, cfg, n_sweeps=total_sweeps, n_chains=C, chain_offset=rank * C)
    W.check(ex)
    n_groups = len(ex.compiled.sampling_groups)
    init = W.init(prog, C, 100 + rank)
    ex.load_state(init, [])
    ex.prepare_rng(SEED)
    stream = ex.stream

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # ---- device-resident steps: warmup, then K timed steps
    for _ in range(args.warmup):
        ex.run_sweeps(S)
    barrier()
    # Each step is timed by its own event pair; between steps a 256 MiB buffer is
    # written so every step starts with a cold L2 (126 MB).
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        for e0, e1 in events:
            with torch.cuda.stream(stream):
                flush.fill_(1)
            e0.record(stream)
            ex.run_sweeps(S)
            e1.record(stream)
        barrier()
    ex.check_device_errors()
    dt_ms = sum(e0.elapsed_time(e1) for e0, e1 in events)
    del flush
    if dist is not None:
        t = torch.tensor([dt_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt_ms = float(t.item())
    updates = world * n_nodes * C * S * args.steps
    value = updates / (dt_ms / 1000.0)
    resident = ex._resident_plans() is not None
    # group kernels + the run-control advance of each graph, or one launch per step (resident lattice)
    gpu_launches = args.steps * (1 if resident else S * n_groups + 1)

    # ---- roofline: per-launch CUDA events on the launch stream (eager sweeps)
    ex.profile = True
    ex._timing_log.clear()
    n_prof = 5
    for _ in range(n_prof):
        ex.run_sweep()
    ex.profile = False
    kernel_ms = [kms for _, _, kms in ex._timing_log]
    roofline = (W.roofline(ex, prog, C, kernel_ms, n_prof, step_ms=dt_ms / args.steps) if W.name == "lattice"
                else W.roofline(ex, prog, C, kernel_ms, n_prof))

    # ---- end to end through the public API (pinned host state in, results out)
    host_init = W.host_inputs(init)
    h2d = sum(t.numel() * t.element_size() for t in host_init)
    nodes = prog.gibbs_spec.free_blocks
    from types import SimpleNamespace

    if W.name == "lattice":
        sched = SimpleNamespace(n_warmup=32, n_samples=64, steps_per_sample=2)
        obs = MagnetizationObserver(nodes)

        def e2e_call(key):
            _, m = ex.sample_with_observation(key, sched, obs, init_state_free=host_init)
            return [m]  # float64 magnetisation per chain per sample
    else:
        sched = SimpleNamespace(n_warmup=S, n_samples=1, steps_per_sample=1)

        def e2e_call(key):
            return ex.sample_states(key, sched, nodes, init_state_free=host_init)

    e2e_call(SEED + 1)  # warm the graph for this schedule
    barrier()
    e2e_times = []
    for s in range(args.steps):
        barrier()
        t0 = time.perf_counter()
        out = e2e_call(SEED + 2 + s)
        torch.cuda.synchronize(dev)
        e2e_times.append(time.perf_counter() - t0)
    d2h = int(sum(np.asarray(a).nbytes for a in out))  # bytes the call returned to the host
    del out
    ex.check_device_errors()
    e2e_s = sum(e2e_times)
    if dist is not None:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = updates / e2e_s

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, _ = cpu_oracle_sample(W, prog, W.cpu_chains, W.cpu_sweeps, threads)
        cpu = {
            "value": v,
            "unit": "node-updates/s",
            "cores": threads,
            "kind": "port",
            "sample": _cpu_sample_text(W, prog, W.cpu_chains, W.cpu_sweeps),
        }

    if rank == 0:
        line = {
            "metric": W.metric,
            "value": value,
            "unit": "node-updates/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": dt_ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": W.dtype(ex),
            "data": W.data,
            "config": W.config(prog, ex, world),
            "roofline": roofline,
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
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default 5; 2000 for the lattice workload, whose 0.5 ms step would otherwise "
                         "give a timed region shorter than the clock sampler's period)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="er",
                    help="er: sparse random-graph Ising (default, the headline); rbm: Gauss-Bernoulli RBM; "
                         "lattice: 64x64 Ising with magnetisation samples; potts: 3-D q=8 Potts 128^3; "
                         "ising: one-chain 32768^2 Ising in row strips over the GPUs")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-sweeps", type=int, default=0,
                    help="run this many eager sweeps of the workload and exit (profiler target, no timing)")
    ap.add_argument("--chains", type=int, default=0, help="profiler target only: chains (default: the workload's)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    W = WORKLOADS[args.workload]
    if args.steps is None:
        args.steps = 2000 if W.name == "lattice" and args.impl != "reference" else 5
    if args.impl == "reference":
        return run_reference(args, W)
    if W.name == "ising" and not args.profile_sweeps:
        return run_ising(args, W)
    if args.profile_sweeps:
        return run_profile_target(args, W)
    return run_ours(args, W)


def run_profile_target(args, W) -> int:
    """Eager sweeps of the workload: one kernel launch per sampling group per sweep."""
    import torch

    from tt_thrml_b200 import Executor, make_cuda_config

    prog = W.build()
    n = args.profile_sweeps
    if W.name == "ising":
        from tt_thrml_b200.domain import LatticeStrips

        st = LatticeStrips(prog, device=torch.device("cuda", 0), halo=W.halo, cuda_graphs=False)
        st.load_random(SEED)
        st.prepare_rng(SEED, n)
        st.run_sweeps(n)
        st.synchronize()
        print(f"profile target: {W.workload}, {n} sweeps (eager half-sweeps)", flush=True)
        return 0
    C = args.chains or W.chains
    ex = Executor(None, 0, prog, make_cuda_config(n_chains=C, cuda_graphs=False), n_sweeps=n, n_chains=C)
    ex.load_state(W.init(prog, C, 100), [])
    ex.prepare_rng(SEED)
    if ex._resident_plans() is not None:
        ex.run_sweeps(n)  # one persistent launch for all n sweeps
    else:
        for _ in range(n):
            ex.run_sweep()
    torch.cuda.synchronize()
    ex.check_device_errors()
    print(f"profile target: {W.workload}, {C} chains, {n} sweeps x {len(ex.compiled.sampling_groups)} groups", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
