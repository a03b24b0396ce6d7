"""Benchmark of the block-Gibbs sweep path (node-updates/s).

One default run (`python bench.py`) prints one JSON line: the headline
configuration at top level and the other four configurations under
`workloads`, each with its own value, e2e, roofline, clocks and CPU baseline.

* er (headline): sparse random-graph Ising, Erdos-Renyi N = 2^20 nodes, mean
  degree 8, J_ij ~ N(0, 1/8) symmetric, h_i ~ N(0, 0.1) (variances), beta = 1,
  greedy colouring into k blocks (one sampling group each), 256 chains per
  GPU, one step = 200 sweeps over all k groups;
* lattice: 64x64 periodic Ising, J = 1, h = 0, beta = 0.44, 1024 chains per
  GPU, one step = the schedule n_warmup = 32, n_samples = 64,
  steps_per_sample = 2 with the per-chain magnetisation observed on device;
* rbm: Gauss-Bernoulli RBM, 4096 gaussian visible x 8192 spin hidden,
  W ~ N(0, 0.01^2), 8192 chains per GPU, one step = 100 sweeps;
* potts: 3-D q = 8 Potts 128^3 periodic, per-axis symmetric couplings, bias
  variance 0.5, 64 chains per GPU, one step = 100 sweeps;
* ising: single-chain 2-D Ising 32768^2, beta = 0.4407, one step = 1000
  sweeps, row strips over the GPUs with the halo exchange fused into the
  half-sweep kernel (strong scaling).

`--workload NAME` runs one configuration alone.  Chain-sharded workloads
keep their chains per GPU fixed (weak scaling) and run through
`make_mesh_executor` (one process per GPU, no collective inside a sweep).

* `value`: steps on device-resident state (CUDA-graph replay of the step's
  sweeps), one CUDA event pair per step on the executor's stream, barrier +
  synchronize on both sides, max over ranks.  L2 is flushed (256 MiB write)
  before every step, outside the timed windows.
* `e2e`: the same metric through the public API with pinned host buffers:
  `sample_states` (initial state in, final state out), the lattice's
  `sample_with_observation` with the magnetisation observed on device, the
  strips' `load_split_colours` + `run_sweeps` + `energy_magnetisation`.
* `roofline`: the dominant kernel over per-launch CUDA events on its launch
  stream: algorithmic bytes against the measured HBM copy bandwidth, or
  algorithmic FLOPs against the measured bf16 GEMM peak; `traffic` from the
  committed ncu summaries.
* `cpu_baseline`: the CPU oracle (a C restatement of the reference's group
  math, built from the configuration's raw parameters) on this host's cores
  over a bounded sample of the same configuration.

`--impl reference` runs only the CPU oracle (the reference itself needs JAX,
thrml and Tenstorrent hardware; neither JAX nor thrml exists on these hosts)
on all host cores; it loads nothing of the product package.
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
L2_FLUSH = "flushed before every timed step (256 MiB write)"


def _orc():
    sys.path.insert(0, str(ROOT))
    from oracle import models
    from oracle import oracle as orc

    return orc, models


def _spin_init(blocks_nodes, C, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 2, (C, n)).astype(bool) for n in blocks_nodes]


class Workload:
    name = ""
    workload = ""
    metric = "node-updates/sec (sites x chains x sweeps / s)"
    scaling = "weak"
    chains = 1
    sweeps = 1
    steps_alone = 5   # default timed steps when run alone
    steps_extra = 5   # timed steps as an entry of the default run's `workloads`
    e2e_steps = 5
    data = ""

    def free_nodes(self, prog):
        return [len(b.nodes) for b in prog.gibbs_spec.free_blocks]

    def init(self, prog, C, seed):
        return _spin_init(self.free_nodes(prog), C, seed)

    def host_inputs(self, init):
        import torch

        return [torch.from_numpy(s.astype(np.int8) * 2 - 1).pin_memory() for s in init]

    # CPU sample of the configuration for the oracle: (program, chains, sweeps, description)
    def cpu_sample(self):
        raise NotImplementedError


class ErIsing(Workload):
    """Sparse random-graph Ising: N = 2^20, Erdos-Renyi mean degree 8, greedy colouring, 256 chains/GPU, 200 sweeps."""

    name = "er"
    workload = "er-ising-n1048576-deg8-c256pergpu-s200"
    chains = 256
    sweeps = 200
    steps_alone = 20  # 2.4 s of timed work
    data = "synthetic (seeded Erdos-Renyi graph, random init)"

    def build(self):
        from tt_thrml_b200 import workloads

        return workloads.erdos_renyi_ising(1 << 20, 8.0, seed=SEED)

    def cpu_sample(self):
        _, models = _orc()
        raw = models.er_ising_raw(1 << 20, 8.0, seed=SEED)
        prog = models.graph_ising(raw["row_ptr"], raw["cols"], raw["J"], raw["h"], raw["colours"], raw["beta"])
        return prog, 256, 1, "the configuration's graph (own construction), all 256 chains x 1 sweep per sample"

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
            "l2": L2_FLUSH,
            "parallelism": f"chain-sharded x{world}",
        }

    def dtype(self, ex):
        return "u32 bit-packed spins, f32 fields" if ex.compiled.state_dtype == "bits" else "int8 spins, f32 fields"

    def roofline(self, ex, prog, C, kernel_ms, n_prof, step_ms):
        layout = ex.compiled.state_dtype
        per_block = algorithmic_bytes(prog, C, layout)
        achieved = sum(per_block) * n_prof / (sum(kernel_ms) / 1000.0) / 1e9
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
            "issue": _issue_ceiling("spin_bits_er1m_c256.md", _n_nodes(prog) * C * n_prof / (sum(kernel_ms) / 1e3)),
        }


class GaussBernoulliRBM(Workload):
    """Gauss-Bernoulli RBM: 4096 gaussian visible x 8192 spin hidden, W ~ N(0, 0.01^2), 8192 chains, 100 sweeps."""

    name = "rbm"
    workload = "gauss-bernoulli-rbm-v4096-h8192-c8192-s100"
    chains = 8192
    sweeps = 100
    steps_alone = 20  # a 100 ms step: 2 s of timed work
    steps_extra = 20
    data = "synthetic (seeded RBM weights rounded to bf16, random init)"
    V, H = 4096, 8192

    def build(self):
        from tt_thrml_b200 import workloads

        return workloads.gaussian_bernoulli_rbm(self.V, self.H, seed=SEED)

    def cpu_sample(self):
        _, models = _orc()
        raw = models.rbm_raw(self.V, self.H, seed=SEED)
        prog = models.dense_bipartite(raw["W"], raw["b_v"], raw["b_h"])
        return prog, 64, 1, "the configuration's RBM (own construction), 64 of 8192 chains x 1 sweep per sample"

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
            "l2": "operands (64-128 MiB per launch) exceed L2; " + L2_FLUSH,
            "parallelism": f"chain-sharded x{world}",
        }

    def dtype(self, ex):
        return "bf16 operands, f32 accumulate (tcgen05)"

    def roofline(self, ex, prog, C, kernel_ms, n_prof, step_ms):
        flops = 2.0 * 2.0 * C * self.V * self.H * n_prof  # two GEMMs per sweep
        achieved = flops / (sum(kernel_ms) / 1000.0) / 1e12
        peaks = _peaks()
        # the launches are timed inside long graph-replayed steps under the power cap: the sustained GEMM peak
        peak, kind = peaks["bf16_sustained"]
        return {
            # the group launches cover the GEMM and, for spin blocks, the near-threshold settle kernel
            "kernel": ("k_dense_field_sample_pair" if C % 256 == 0 else "k_dense_field_sample") + " + k_dense_settle",
            "bound": "tensor",
            "achieved": achieved,
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": achieved / peak,
            "peak_source": kind + " sustained (launches timed inside the long step)",
            "frac_of_burst": achieved / peaks["bf16"][0],
            "traffic": _dense_traffic_per_launch(),
            "algorithmic_flops_per_update": 2.0 * 2.0 * self.V * self.H / (self.V + self.H),
        }


class Lattice2D(Workload):
    """2-D Ising 64x64 periodic, J=1, h=0, beta=0.44, 1024 chains; one step = the sampling schedule
    n_warmup=32, n_samples=64, steps_per_sample=2 with the per-chain magnetisation observed on device."""

    name = "lattice"
    workload = "ising2d-64x64-c1024-w32-n64-s2"
    chains = 1024
    sweeps = 32 + 63 * 2
    steps_alone = 4000
    steps_extra = 4000  # a 0.5 ms step: 2 s of timed work, 10 clock samples
    e2e_steps = 500
    data = "synthetic (uniform +-1 init from seed 0)"

    def build(self):
        from tt_thrml_b200 import workloads

        return workloads.ising_lattice_2d(64, 64, J=1.0, h=0.0, beta=0.44)

    def cpu_sample(self):
        _, models = _orc()
        prog = models.ising2d(64, 64, J=1.0, h=0.0, beta=0.44)
        return prog, 1024, 8, "the configuration's lattice (own construction), all 1024 chains x 8 sweeps per sample"

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
            "l2": "state (512 KiB) is L2-resident by design; " + L2_FLUSH,
            "parallelism": f"chain-sharded x{world}",
        }

    def dtype(self, ex):
        return ErIsing.dtype(self, ex)

    def roofline(self, ex, prog, C, kernel_ms, n_prof, step_ms):
        if ex.compiled.sampling_groups[0].kernel_artifact.kind != "ising2d_resident":
            return ErIsing.roofline(self, ex, prog, C, kernel_ms, n_prof, step_ms) | {"traffic": None}
        # shared-memory resident: one launch runs every sweep of a step; state bits read and written once per
        # half-sweep as if from memory (the algorithmic bytes), over the device time of the timed steps
        per_update = 2.0 / 8.0
        rate = _n_nodes(prog) * C * self.sweeps / (step_ms / 1000.0)
        achieved = rate * per_update / 1e9
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
            "issue": _issue_ceiling("ising2d_resident_64x64_c1024.md", rate),
        }


class Potts3D(Workload):
    """3-D q=8 Potts 128^3 periodic, per-axis symmetric 8x8 couplings ~ N(0, 1), bias ~ N(0, 0.5), 64 chains,
    100 sweeps per step."""

    name = "potts"
    workload = "potts3d-128cube-q8-c64-s100"
    chains = 64
    sweeps = 100
    data = "synthetic (seeded couplings and biases, uniform random categories)"
    side, q = 128, 8
    steps_alone = 40  # a 70 ms step: 2.8 s of timed work
    steps_extra = 40

    def build(self):
        from tt_thrml_b200 import workloads

        return workloads.potts_lattice_3d(self.side, self.q, seed=SEED)

    def cpu_sample(self):
        _, models = _orc()
        raw = models.potts_raw(self.side, self.q, seed=SEED)
        prog = models.potts3d(raw["dims"], raw["J"], raw["bias"])
        return prog, 16, 1, "the configuration's lattice (own construction), 16 of 64 chains x 1 sweep per sample"

    def init(self, prog, C, seed):
        rng = np.random.default_rng(seed)
        return [rng.integers(0, self.q, (C, n)).astype(np.int8) for n in self.free_nodes(prog)]

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
            "l2": "state 128 MiB + bias 32 MiB exceed L2; " + L2_FLUSH,
            "parallelism": f"chain-sharded x{world}",
        }

    def dtype(self, ex):
        return "int8 categories, f32 fields"

    def roofline(self, ex, prog, C, kernel_ms, n_prof, step_ms):
        half = prog.n_sites // 2
        per_block = half * C * 2 + half * self.q * 4  # source rows read once, target rows written, bias read
        achieved = per_block * len(kernel_ms) / (sum(kernel_ms) / 1000.0) / 1e9
        rate = half * C * len(kernel_ms) / (sum(kernel_ms) / 1000.0)
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
            "issue": _issue_ceiling("potts3d_128cube_q8_c64.md", rate),
            "sfu": _sfu_ceiling("potts3d_128cube_q8_c64.md", rate),
        }


class BigIsing(Workload):
    """Single-chain 2-D Ising 32768^2 periodic, J=1, h=0, beta=0.4407, 1000 sweeps per step, domain-decomposed
    into row strips over the GPUs (deep halos exchanged every halo/2 sweeps)."""

    name = "ising"
    scaling = "strong"
    workload = "ising2d-32768sq-1chain-s1000-strips"
    side = 32768
    sweeps = 1000
    steps_alone = 5
    steps_extra = 5
    e2e_steps = 3
    halo = 40  # 20 sweeps per exchange, 1000 = 50 exchanges
    data = "synthetic (uniform +-1 spins from a seeded hash of the site)"

    def build(self):
        from tt_thrml_b200 import workloads

        return workloads.IsingLattice2D(self.side, self.side, beta=0.4407)

    def cpu_sample(self):
        _, models = _orc()
        prog = models.ising2d(1024, self.side, J=1.0, h=0.0, beta=0.4407)
        return prog, 1, 2, ("1024 of the 32768 rows (full 32768-wide rows, same couplings; own construction) x "
                            "2 sweeps per sample")


WORKLOADS = {w.name: w for w in (ErIsing(), Lattice2D(), GaussBernoulliRBM(), Potts3D(), BigIsing())}
HEADLINE = "er"


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


def _issue_figures(name: str):
    return _profile_figures(name, ("thread_instructions_per_update",))


def _issue_ceiling(profile: str, rate: float):
    """Instruction-issue ceiling of a kernel from its committed ncu summary: 148 SMs x 4 schedulers x 32
    lanes per cycle at the maximum SM clock, over the thread instructions one update executes."""
    vals = _issue_figures(profile)
    if vals is None:
        return None
    per = vals["thread_instructions_per_update"]
    ceiling = 148 * 4 * 32 * 1.965e9 / per
    return {"thread_instructions_per_update": per, "ceiling_updates_per_s": ceiling, "frac": rate / ceiling,
            "source": f"profiles/{profile}"}


def _sfu_ceiling(profile: str, rate: float):
    """Special-function (XU) ceiling: 16 results per SM per cycle at the maximum SM clock over the XU
    instructions (ex2) one update executes, from the committed ncu summary."""
    vals = _profile_figures(profile, ("xu_instructions_per_update",))
    if vals is None:
        return None
    per = vals["xu_instructions_per_update"]
    if per <= 0:
        return {"xu_instructions_per_update": 0.0, "ceiling_updates_per_s": None, "frac": 0.0,
                "source": f"profiles/{profile}"}
    ceiling = 148 * 16 * 1.965e9 / per
    return {"xu_instructions_per_update": per, "ceiling_updates_per_s": ceiling, "frac": rate / ceiling,
            "source": f"profiles/{profile}"}


def _n_nodes(prog):
    return sum(len(b.nodes) for b in prog.gibbs_spec.blocks)


class DistCtx:
    """One process per GPU (torchrun env) or a single process."""

    def __init__(self, backend_ok: bool = True):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dist = None
        if not backend_ok:
            return
        import torch

        self.dev = torch.device("cuda", self.local)
        torch.cuda.set_device(self.dev)
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=self.dev)
            self.dist = dist

    def barrier(self):
        import torch

        if self.dist is not None:
            self.dist.barrier()
        torch.cuda.synchronize(self.dev)

    def max(self, x: float) -> float:
        if self.dist is None:
            return float(x)
        import torch

        t = torch.tensor([float(x)], device=self.dev, dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.dist is not None:
            self.dist.barrier()
            self.dist.destroy_process_group()


def _oracle_init(oprog, C, seed):
    rng = np.random.default_rng(seed)
    out = []
    for b in oprog.blocks[: oprog.n_free]:
        if b.family == "spin":
            out.append(rng.integers(0, 2, (C, b.n_nodes)).astype(bool))
        elif b.family == "categorical":
            out.append(rng.integers(0, b.q, (C, b.n_nodes)))
        else:
            out.append(rng.standard_normal((C, b.n_nodes)).astype(np.float32))
    return out


def cpu_oracle_time(oprog, C, n_sweeps, threads, seed=1):
    """Seconds of `n_sweeps` sweeps of the CPU oracle over C chains (after one untimed sweep)."""
    orc, _ = _orc()
    o = orc.OracleSampler(oprog, n_chains=C, n_threads=threads)
    o.load_state(_oracle_init(oprog, C, seed))
    o.sweep(0, seed=7)
    t0 = time.perf_counter()
    for s in range(n_sweeps):
        o.sweep(1 + s, seed=7)
    return time.perf_counter() - t0


def cpu_baseline(W):
    threads = os.cpu_count() or 1
    oprog, C, S, what = W.cpu_sample()
    dt = cpu_oracle_time(oprog, C, S, threads)
    return {"value": oprog.total * C * S / dt, "unit": "node-updates/s", "cores": threads, "kind": "port",
            "sample": f"CPU oracle (C restatement of the reference's group math, float32 state): {what}"}


def run_chain_sharded(ctx, args, W, steps, warmup, cpu):
    """Chains sharded over the GPUs (weak scaling: W.chains per GPU), through make_mesh_executor."""
    import torch

    from tt_thrml_b200 import make_cuda_config, make_mesh_executor
    from tt_thrml_b200.backend import CudaDevice
    from tt_thrml_b200.observers import MagnetizationObserver

    dev = ctx.dev
    prog = W.build()
    n_nodes = _n_nodes(prog)
    C, S = W.chains, W.sweeps
    cfg = make_cuda_config(n_chains=C * ctx.world, cuda_graphs=True)
    total_sweeps = S * (steps + warmup) + 16
    mesh = make_mesh_executor(None, CudaDevice(ctx.local), prog, cfg, n_sweeps=total_sweeps, n_chains=C * ctx.world,
                              gather=False)
    ex = mesh.shards[0]  # this process's chains
    assert ex.n_chains == C and ex.chain_offset == ctx.rank * C
    W.check(ex)
    # a dense spin group launches the GEMM and the near-threshold settle kernel
    n_group_launches = sum(2 if g.kernel_artifact.kind == "dense" and g.kernel_artifact.family == "spin" else 1
                           for g in ex.compiled.sampling_groups)
    init = W.init(prog, C, 100 + ctx.rank)
    mesh.load_state(init, [])
    mesh.prepare_rng(SEED)
    stream = ex.stream

    # ---- device-resident steps: warmup, then `steps` timed steps, each with its own event pair; a 256 MiB
    # write between steps starts every step with a cold L2 (126 MB)
    for _ in range(warmup):
        mesh.run_sweeps(S)
    ctx.barrier()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    with ClockSampler(ctx.local) as clocks:
        for e0, e1 in events:
            with torch.cuda.stream(stream):
                flush.fill_(1)
            e0.record(stream)
            mesh.run_sweeps(S)
            e1.record(stream)
        ctx.barrier()
    ex.check_device_errors()
    dt_ms = ctx.max(sum(e0.elapsed_time(e1) for e0, e1 in events))
    del flush
    updates = ctx.world * n_nodes * C * S * steps
    value = updates / (dt_ms / 1000.0)
    resident = ex._resident_plans() is not None
    # group kernels + the run-control advance of each graph, or one launch per step (resident lattice)
    gpu_launches = steps * (1 if resident else S * n_group_launches + 1)

    # ---- roofline: the average launch duration over the timed region (graph-replayed steps, events on the
    # launch stream): step time / group launches per step.  Per-launch events around eager sweeps are kept
    # as a cross-check; they also count the GPU's wait for each eager launch.
    n_prof = 5
    n_sites = len(ex.compiled.sampling_groups)
    timed_ms = [dt_ms / steps / (S * n_sites)] * (n_sites * n_prof)
    roofline = W.roofline(ex, prog, C, timed_ms, n_prof, dt_ms / steps)
    ex.profile = True
    ex._timing_log.clear()
    for _ in range(n_prof):
        ex.run_sweep()
    ex.profile = False
    kernel_ms = [kms for _, _, kms in ex._timing_log]
    eager = W.roofline(ex, prog, C, kernel_ms, n_prof, dt_ms / steps)
    roofline["duration_source"] = ("timed region: step time / launches per step" if not resident
                                   else "timed region: step time (one launch per step)")
    roofline["eager_launch_frac"] = eager["frac"]

    # ---- end to end through the public API (pinned host state in, results out)
    host_init = W.host_inputs(init)
    h2d = sum(t.numel() * t.element_size() for t in host_init)
    nodes = prog.gibbs_spec.free_blocks
    from types import SimpleNamespace

    if W.name == "lattice":
        sched = SimpleNamespace(n_warmup=32, n_samples=64, steps_per_sample=2)
        obs = MagnetizationObserver(nodes)

        def e2e_call(key):
            _, m = mesh.sample_with_observation(key, sched, obs, init_state_free=host_init)
            return [m]  # float64 magnetisation per chain per sample
    else:
        sched = SimpleNamespace(n_warmup=S, n_samples=1, steps_per_sample=1)

        def e2e_call(key):
            return mesh.sample_states(key, sched, nodes, init_state_free=host_init)

    # warm the graph for this schedule; a timed call runs while the previous call's result is still held,
    # so two warm calls leave both alternating pinned result buffers in torch's host-allocator cache
    out = e2e_call(SEED)
    out = e2e_call(SEED + 1)
    ctx.barrier()
    n_e2e = min(steps, W.e2e_steps)
    e2e_times = []
    for s in range(n_e2e):
        ctx.barrier()
        t0 = time.perf_counter()
        out = e2e_call(SEED + 2 + s)
        torch.cuda.synchronize(dev)
        e2e_times.append(time.perf_counter() - t0)
    d2h = int(sum(np.asarray(a).nbytes for a in out))  # bytes the call returned to the host
    del out
    ex.check_device_errors()
    e2e_s = ctx.max(sum(e2e_times))
    e2e_value = ctx.world * n_nodes * C * S * n_e2e / e2e_s
    dtype, config = W.dtype(ex), W.config(prog, ex, ctx.world)
    del mesh, ex
    torch.cuda.empty_cache()
    if ctx.rank != 0:
        return None
    return {
        "metric": W.metric,
        "value": value,
        "unit": "node-updates/s",
        "n_gpus": ctx.world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": dt_ms / steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": dtype,
        "data": W.data,
        "config": config,
        "roofline": roofline,
        "e2e": {"value": e2e_value, "unit": "node-updates/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": n_e2e,
                "api": "make_mesh_executor(...).sample_with_observation" if W.name == "lattice"
                       else "make_mesh_executor(...).sample_states"},
        "gpu_launches": gpu_launches,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
    }


def run_strips(ctx, args, W, steps, warmup, cpu):
    """The domain-decomposed lattice: strong scaling (the lattice is fixed, the strips shrink with N)."""
    import torch

    from tt_thrml_b200 import _native as nat
    from tt_thrml_b200.domain import LatticeStrips

    dev = ctx.dev
    prog = W.build()
    S = W.sweeps
    st = LatticeStrips(prog, device=dev, halo=W.halo)
    st.load_random(SEED)
    st.prepare_rng(SEED, S * (steps + warmup) + S)
    stream = st._stream
    for _ in range(warmup):
        st.run_sweeps(S)
    ctx.barrier()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    with ClockSampler(ctx.local) as clocks:
        for e0, e1 in events:
            with torch.cuda.stream(stream):
                flush.fill_(1)
            e0.record(stream)
            st.run_sweeps(S)
            e1.record(stream)
        ctx.barrier()
    del flush
    st.check_errors()
    dt_ms = ctx.max(sum(e0.elapsed_time(e1) for e0, e1 in events))
    n_sites = W.side * W.side
    updates = n_sites * S * steps
    value = updates / (dt_ms / 1000.0)
    periods = S // (W.halo // 2)
    gpu_launches = steps * (periods * (W.halo + 2) + 1)  # import + half-sweeps + signal per period, ctl advance
    em = st.energy_magnetisation()

    # roofline: eager half-sweeps of the own rows, CUDA events on the launch stream
    hw = W.side // 2
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    n_prof = 10
    nat_bytes = 0
    st.cuda_graphs = False
    nat.bind_device(ctx.local)
    with torch.cuda.stream(stream):
        ev[0].record(stream)
        for k in range(n_prof):
            st._cuda_halfsweep(k & 1, st.D, st.D + st.h, st.sweep, stream)
            nat_bytes += 2 * st.h * st.row_bytes  # other colour read once + own colour written once
        ev[1].record(stream)
    stream.synchronize()
    kms = ev[0].elapsed_time(ev[1]) / n_prof
    achieved = nat_bytes / n_prof / (kms / 1000.0) / 1e9
    rate = st.h * W.side / 2 / (kms / 1000.0)
    peak, kind = _peaks()["hbm"]

    # end to end: pinned host split-colour lattice in, 1000 sweeps, energy/magnetisation trace out
    host = [torch.empty((W.side, hw), dtype=torch.int8).pin_memory() for _ in range(2)]
    for c in range(2):
        host[c].copy_(st._own_rows(c).cpu().repeat(W.side // st.h, 1))
    st.cuda_graphs = True
    n_e2e = min(steps, W.e2e_steps)
    e2e_times = []
    for s in range(-1, n_e2e):  # call -1 (untimed) captures the CUDA graph of the S-sweep run
        ctx.barrier()
        t0 = time.perf_counter()
        st.load_split_colours(host[0], host[1])
        st.prepare_rng(SEED + 1 + s, S)
        st.run_sweeps(S)
        trace = st.energy_magnetisation()
        torch.cuda.synchronize(dev)
        if s >= 0:
            e2e_times.append(time.perf_counter() - t0)
    e2e_s = ctx.max(sum(e2e_times))
    h2d = st.rows_local * hw * 2
    d2h = int(trace.nbytes)
    storage, layout, h_rows, row_bytes = st.storage, st.rng_layout, st.h, st.row_bytes
    st.close()
    del st, host
    torch.cuda.empty_cache()
    if ctx.rank != 0:
        return None
    return {
        "metric": W.metric,
        "value": value,
        "unit": "node-updates/s",
        "n_gpus": ctx.world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": dt_ms / steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8 spins" if storage == "int8" else "bit-packed spins (32 sites per uint32)",
        "data": W.data,
        "config": {
            "workload": W.workload,
            "lattice": f"{W.side}x{W.side} periodic, 1 chain",
            "sweeps_per_step": S,
            "strips": ctx.world,
            "rows_per_strip": h_rows,
            "halo_rows": W.halo,
            "exchange": "boundary rows stored into the neighbours' mailboxes by the half-sweep kernel (peer "
                        "memory over NVLink), flag per period, every halo/2 sweeps",
            "rng": "philox4x32-10 on device",
            "l2": "state 1 GiB exceeds L2; " + L2_FLUSH,
            "parallelism": f"row strips x{ctx.world}",
            "final_energy_per_site": float(em[-1, 0]),
            "final_magnetisation_per_site": float(em[-1, 1]),
        },
        "roofline": {
            "kernel": ("k_ising2d_bits" if storage == "bits" else
                       "k_ising2d_planes" if layout == "planes" else "k_ising2d"),
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "peak_source": kind,
            "traffic": _profile_traffic("ising2d_32768.md") * h_rows / W.side
                       if storage == "bits" and _profile_traffic("ising2d_32768.md") else None,
            "algorithmic_bytes_per_update": 2.0 * row_bytes / hw,
            "note": ("bit-packed rows move 0.25 B per update; the kernel is bound by instruction issue "
                     "(bit-sliced decision), not by HBM" if storage == "bits" else None),
            "issue": _issue_ceiling("ising2d_32768.md", rate) if storage == "bits" else None,
        },
        "e2e": {"value": updates / steps * n_e2e / e2e_s, "unit": "node-updates/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": n_e2e,
                "api": "LatticeStrips.load_split_colours + run_sweeps + energy_magnetisation"},
        "gpu_launches": gpu_launches,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
    }


def run_reference(args, W):
    """CPU arm: the oracle restatement of the reference's group math on all host cores, built from the
    configuration's raw parameters by the oracle itself (nothing of the product package is loaded)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    oprog, C, S, what = W.cpu_sample()
    orc, _ = _orc()
    o = orc.OracleSampler(oprog, n_chains=C, n_threads=threads)
    o.load_state(_oracle_init(oprog, C, 1))
    sweep = 0

    def step():
        nonlocal sweep
        t0 = time.perf_counter()
        for _ in range(S):
            o.sweep(sweep, seed=7)
            sweep += 1
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        step()
    times = [step() for _ in range(args.steps)]
    tot = sum(times)
    value = oprog.total * C * S * args.steps / tot
    loaded = sorted({Path(m.__file__).name for m in list(sys.modules.values())
                     if getattr(m, "__file__", None) and "tt_thrml_b200" in str(m.__file__)})
    assert not loaded, f"the reference arm imported the product: {loaded}"
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
        "scaling": W.scaling,
        "vs_baseline": None,
        "dtype": "f32",
        "data": W.data,
        "config": {"workload": W.workload, "sample": what},
        "cpu_baseline": {"value": value, "unit": "node-updates/s", "cores": threads, "kind": "port",
                         "sample": f"CPU oracle (C restatement of the reference's group math): {what}"},
        "e2e": {"value": value, "unit": "node-updates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps of the headline workload (default 5); the other workloads of the default "
                         "run use their own step counts (about 2-4 s of timed work each)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["all", *WORKLOADS], default="all",
                    help="all (default): er as the headline plus lattice, rbm, potts and ising under 'workloads'; "
                         "or one of them alone")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-sweeps", type=int, default=0,
                    help="run this many eager sweeps of the workload and exit (profiler target, no timing)")
    ap.add_argument("--chains", type=int, default=0, help="profiler target only: chains (default: the workload's)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    names = list(WORKLOADS) if args.workload == "all" else [args.workload]
    if args.impl == "reference":
        W = WORKLOADS[HEADLINE if args.workload == "all" else args.workload]
        if args.steps is None:
            args.steps = 5
        return run_reference(args, W)
    if args.profile_sweeps:
        return run_profile_target(args, WORKLOADS[HEADLINE if args.workload == "all" else args.workload])
    ctx = DistCtx()
    lines = {}
    for i, name in enumerate(names):
        W = WORKLOADS[name]
        if i == 0:
            steps = args.steps if args.steps is not None else W.steps_alone
        else:
            steps = W.steps_extra
        cpu = None
        if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(W)
        run = run_strips if W.name == "ising" else run_chain_sharded
        lines[name] = run(ctx, args, W, steps, args.warmup, cpu)
    if ctx.rank == 0:
        out = lines[names[0]]
        if len(names) > 1:
            out["workloads"] = {n: lines[n] for n in names[1:]}
        print(json.dumps(out), flush=True)
    ctx.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
