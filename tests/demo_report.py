"""CPU-vs-GPU report over four small thrml programs (the reference's demo
harness, scripts/demo.py:270-381, with the CPU oracle in place of thrml's
JAX CPU path).

Programs: the reference's four parity scenarios (spin chain, categorical EBM,
gaussian chain, mixed spin + categorical + gaussian superblocks), each run
over its own sampling schedule with many independent chains:

* GPU: `make_executor(...).sample_states(key, schedule, ...)` on cuda:0,
  Philox mode (the timed mode of the backend);
* CPU: the oracle (C restatement of the reference's kernel math) stepping the
  same schedule with the same Philox counters, so both sides draw the same
  uniforms and the samples agree chain by chain, up to decisions within the
  1e-5 threshold band (a chain whose draw fell inside the band follows its own
  path from there on).

The report prints, per program, the wall time of each side, per-block sample
statistics (spin means, categorical modes and entropies, gaussian means and
standard deviations, as in scripts/demo.py:313-333), the speed-up and the
fraction of chains whose whole trajectory matches the oracle.  `--profile`
adds the executor's per-family dispatch and kernel timing
(tt_thrml/executor.py:411-431).

This is test infrastructure: it imports the oracle, which the product never
does.  Usage: python tests/demo_report.py [--chains C] [--profile]
"""

from __future__ import annotations

import argparse
import sys
import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
for p in (HERE, HERE.parent):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

import gpu_harness as gh  # noqa: E402
import thrml_shim as th  # noqa: E402
from oracle import oracle as orc  # noqa: E402

DEMOS = {
    "spin chain (4 spins, bias + pair factors)": th.make_spin_case,
    "categorical EBM (4 nodes, 3 categories)": th.make_categorical_case,
    "gaussian chain (3 continuous nodes)": th.make_gaussian_case,
    "mixed (spin + categorical + gaussian superblocks)": th.make_mixed_case,
}


@dataclass
class DemoResult:
    name: str
    schedule: object
    gpu: list
    gpu_s: float
    cpu: list
    cpu_s: float
    chains_matching: float
    timing: dict


def _broadcast(states, C):
    return [np.broadcast_to(np.asarray(s), (C,) + np.asarray(s).shape).copy() for s in states]


def _node_locations(spec):
    loc = {}
    for bi, b in enumerate(list(spec.free_blocks) + list(spec.clamped_blocks)):
        for pos, node in enumerate(b.nodes):
            loc[node] = (bi, pos)
    return loc


def run_oracle(case, C, seed, rng_layout):
    """The schedule of thrml.sample_states on the oracle: sample 0 after the
    warm-up sweeps, then one sample after every steps_per_sample sweeps
    (tt_thrml/executor.py:367-409); returns [n_samples, C, n] per sampled block."""
    sched = case.schedule
    o = orc.OracleSampler(case.program, n_chains=C, rng_layout=rng_layout)
    o.load_state(_broadcast(case.init_state_free, C), _broadcast(case.state_clamp, C))
    loc = _node_locations(case.program.gibbs_spec)
    out = [[] for _ in case.nodes_to_sample]
    sweep = 0

    def observe():
        decoded = {}
        for k, block in enumerate(case.nodes_to_sample):
            cols = []
            for node in block.nodes:
                bi, pos = loc[node]
                if bi not in decoded:
                    decoded[bi] = o.block_state(bi)
                cols.append(decoded[bi][:, pos])
            out[k].append(np.stack(cols, axis=-1))

    for _ in range(sched.n_warmup):
        o.sweep(sweep, seed=seed)
        sweep += 1
    observe()
    for _ in range(sched.n_samples - 1):
        for _ in range(sched.steps_per_sample):
            o.sweep(sweep, seed=seed)
            sweep += 1
        observe()
    return [np.stack(v) for v in out]


def chains_matching(gpu, cpu) -> float:
    """Fraction of chains whose every sample of every block agrees (discrete:
    equal; gaussian: within 1e-4 relative, 1e-6 absolute)."""
    ok = None
    for g, c in zip(gpu, cpu):
        g = np.asarray(g)
        c = np.asarray(c)
        if np.issubdtype(g.dtype, np.floating):
            same = np.isclose(g, c.astype(g.dtype), rtol=1e-4, atol=1e-6)
        else:
            same = g == c.astype(g.dtype)
        per_chain = same.reshape(same.shape[0], same.shape[1], -1).all(axis=(0, 2))
        ok = per_chain if ok is None else ok & per_chain
    return float(ok.mean())


def run_demo(name, make_case, C, key, *, profile=False) -> DemoResult:
    import torch

    from tt_thrml_b200 import make_cuda_config, make_executor
    from tt_thrml_b200.rng import seed_from_key

    case = make_case()
    ex = make_executor(None, 0, case.program, make_cuda_config(n_chains=C), profile=profile)
    init = _broadcast(case.init_state_free, C)
    clamp = _broadcast(case.state_clamp, C)
    # one untimed run compiles nothing more but warms the CUDA context and graphs
    ex.sample_states(key, case.schedule, case.nodes_to_sample, init_state_free=init, state_clamp=clamp)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    gpu = ex.sample_states(key, case.schedule, case.nodes_to_sample, init_state_free=init, state_clamp=clamp)
    torch.cuda.synchronize()
    gpu_s = time.perf_counter() - t0
    gpu = [np.asarray(s) for s in gpu]
    t0 = time.perf_counter()
    cpu = run_oracle(case, C, seed_from_key(key), gh.rng_layouts(ex.compiled))
    cpu_s = time.perf_counter() - t0
    return DemoResult(name, case.schedule, gpu, gpu_s, cpu, cpu_s, chains_matching(gpu, cpu),
                      ex.timing_summary() if profile else {})


def _row(label, value):
    print(f"  {label:<22} {value}")


def _block_stats(s: np.ndarray):
    flat = s.reshape(-1, s.shape[-1])  # samples x chains pooled
    if s.dtype == np.bool_:
        _row("spin mean", np.array2string(np.where(flat, 1.0, -1.0).mean(0), precision=3, suppress_small=True))
    elif np.issubdtype(s.dtype, np.integer):
        q = int(flat.max()) + 1
        counts = np.stack([np.bincount(flat[:, i], minlength=q) for i in range(flat.shape[1])]).astype(float)
        p = counts / counts.sum(1, keepdims=True)
        _row("cat mode", np.array2string(counts.argmax(1)))
        _row("cat entropy/node", f"{float(-(p * np.log(p + 1e-12)).sum() / flat.shape[1]):.4f} nats")
    else:
        _row("gauss mean", np.array2string(flat.mean(0), precision=4, suppress_small=True))
        _row("gauss std", np.array2string(flat.std(0), precision=4, suppress_small=True))


def report(results, C):
    print("=" * 64)
    print(f"  thrml programs: CPU oracle vs B200 (tt_thrml_b200), {C} chains each")
    print("=" * 64)
    for r in results:
        sc = r.schedule
        print(f"\n{'-' * 64}\n  {r.name}")
        print(f"  {sc.n_samples} samples, {sc.n_warmup} warmup, {sc.steps_per_sample} steps/sample\n")
        for label, out, secs in (("CPU (oracle)", r.cpu, r.cpu_s), ("B200", r.gpu, r.gpu_s)):
            print(f"  [{label}]  {secs * 1e3:.1f} ms")
            for s in out:
                _block_stats(np.asarray(s))
        print(f"\n  speedup: {r.cpu_s / r.gpu_s:.1f}x   chains identical to the oracle: {100 * r.chains_matching:.2f} %")
        for family, s in sorted(r.timing.items()):
            print(f"    {family:<12} n={s['n']:>4}  dispatch {s['dispatch_mean_ms']:.3f} ms/call  "
                  f"kernel {s['kernel_mean_ms']:.3f} ms/call")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--chains", type=int, default=4096)
    ap.add_argument("--profile", action="store_true")
    args = ap.parse_args(argv)
    results = [run_demo(name, make, args.chains, 999 + i, profile=args.profile)
               for i, (name, make) in enumerate(DEMOS.items())]
    report(results, args.chains)
    return results


if __name__ == "__main__":
    main()
