"""Edge cases of the sweep kernels against the oracle.

* hub nodes (degrees 40 and 300: past the partial-sum table, past the staged
  rows, past one warp's worth of neighbours) and isolated nodes, on the
  bit-packed, int8 and generic kernels;
* chain counts that are not multiples of the vector widths (generic kernel);
* Potts states holding out-of-range categories, which the reference's one-hot
  selection weighs with zero (stencil and generic kernels alike);
* schedules without warm-up.
"""

from __future__ import annotations

import numpy as np
import pytest

import gpu_harness as gh
import thrml_shim as th
from tt_thrml_b200 import Executor, make_cuda_config, workloads
from tt_thrml_b200.compiler import compile_program

pytestmark = pytest.mark.gpu


def _hub_graph(n=3000, seed=0):
    rng = np.random.default_rng(seed)
    ei, ej = workloads.erdos_renyi_edges(n, 4.0, seed)
    hubs = [(0, 300), (1, 40)]  # node, degree
    extra_i, extra_j = [], []
    for node, deg in hubs:
        others = rng.choice(np.arange(10, n), size=deg, replace=False)
        extra_i += [node] * deg
        extra_j += list(others)
    ei = np.concatenate([ei, np.asarray(extra_i, ei.dtype)])
    ej = np.concatenate([ej, np.asarray(extra_j, ej.dtype)])
    key = np.minimum(ei, ej) * n + np.maximum(ei, ej)
    _, keep = np.unique(key, return_index=True)
    ei, ej = ei[keep], ej[keep]
    ok = ei != ej
    ei, ej = ei[ok], ej[ok]
    J = (rng.standard_normal(ei.shape[0]) * 0.3).astype(np.float32)
    h = (rng.standard_normal(n) * 0.3).astype(np.float32)
    rp, cols, vals = workloads.symmetric_csr(n, ei, ej, J)
    colours = workloads.greedy_colouring(rp, cols)
    prog = workloads.spin_graph_program(rp, cols, vals, h, colours, beta=0.8)
    assert np.diff(rp).max() >= 300
    return prog


@pytest.mark.parametrize("C,kind", [(256, "spin_bits"), (64, "spin_csr"), (3, "generic")])
@pytest.mark.parametrize("mode", ["philox", "variates"])
def test_hub_nodes_match_oracle(cuda_device, C, kind, mode):
    prog = _hub_graph()
    rep, ex, _ = gh.run_parity(prog, C, 3, mode=mode)
    assert {g.kernel_artifact.kind for g in ex.compiled.sampling_groups} == {kind}
    assert rep.hard_mismatches == 0, rep
    assert rep.band_fraction < 1e-4, rep


@pytest.mark.parametrize("force_generic", [False, True])
def test_out_of_range_categories_weigh_zero(cuda_device, force_generic):
    prog = workloads.potts_lattice_3d(6, 5, seed=9)
    C = 32
    rng = np.random.default_rng(1)
    half = prog.n_sites // 2
    init = [rng.integers(0, 5, (C, half)).astype(np.int32) for _ in range(2)]
    init[1][:, ::7] = 7  # out of range (q = 5)
    init[1][:, 3::11] = -1  # negative
    # sample only colour 0 from these states and compare with the oracle
    cfg = make_cuda_config(n_chains=C, cuda_graphs=False)
    compiled = compile_program(None, 0, prog, cfg, n_sweeps=2, n_chains=C, force_generic=force_generic)
    ex = Executor(None, 0, prog, cfg, compiled, n_sweeps=2, n_chains=C)
    ex.load_state(init, [])
    ex.prepare_rng(4)
    from oracle import oracle as orc
    from tt_thrml_b200.rng import seed_from_key

    o = orc.OracleSampler(prog, n_chains=C, rng_layout=gh.rng_layouts(compiled))
    o.load_state(init)
    gi = [g.block_indices for g in compiled.sampling_groups].index((0,))
    ex._run_sampling_group(compiled.sampling_groups[gi], 0)
    margin = o.group_step(gi, 0, seed=seed_from_key(4), return_margin=True)
    got = ex.raw_state()[:half]
    want = o.state[:half]
    tie = np.abs(margin) < gh.BAND
    assert int(((got != want) & ~tie).sum()) == 0
    assert tie.mean() < 1e-3


def test_schedule_without_warmup_observes_the_initial_state(cuda_device):
    from tt_thrml_b200.observers import MagnetizationObserver

    prog = workloads.ising_lattice_2d(16, 16)
    C = 64
    rng = np.random.default_rng(2)
    init = [rng.integers(0, 2, (C, len(b.nodes))).astype(bool) for b in prog.gibbs_spec.free_blocks]
    ex = Executor(None, 0, prog, make_cuda_config(n_chains=C), n_sweeps=16, n_chains=C)
    sched = th.SamplingSchedule(n_warmup=0, n_samples=3, steps_per_sample=2)
    _, m = ex.sample_with_observation(1, sched, MagnetizationObserver(prog.gibbs_spec.free_blocks),
                                      init_state_free=init)
    want0 = sum(np.where(s, 1.0, -1.0).sum(-1) for s in init)
    np.testing.assert_array_equal(m[0], want0)
    states = ex.sample_states(1, sched, prog.gibbs_spec.free_blocks, init_state_free=init)
    np.testing.assert_array_equal(states[0][0], init[0])
