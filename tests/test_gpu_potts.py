"""3-D Potts lattices on the stencil kernel (tthrml_potts3d_step) against the oracle.

Categorical criteria: states bit-exact outside the 1e-5 threshold band (the
Philox-mode inverse-CDF draw is restated operation for operation in the
oracle, so its decisions agree exactly; variates mode takes argmax(theta + g)
over the same uploaded Gumbels).  The stencil kernel must also reproduce the
generic table-driven kernel bit for bit, and sample the exact Boltzmann
distribution of a lattice small enough to enumerate.
"""

from __future__ import annotations

import itertools

import numpy as np
import pytest

import gpu_harness as gh
from tt_thrml_b200 import Executor, make_cuda_config, workloads
from tt_thrml_b200.compiler import compile_program

pytestmark = pytest.mark.gpu


def _init(prog, C, seed=1):
    rng = np.random.default_rng(seed)
    half = prog.n_sites // 2
    return [rng.integers(0, prog.q, (C, half)).astype(np.int32) for _ in range(2)]


def _assert_parity(rep):
    assert rep.hard_mismatches == 0, rep
    assert rep.band_fraction < 1e-4, rep


@pytest.mark.parametrize("mode", ["variates", "philox"])
@pytest.mark.parametrize("side,q,C", [(8, 8, 64), (6, 3, 32)])
def test_potts_stencil_matches_oracle(cuda_device, mode, side, q, C):
    prog = workloads.potts_lattice_3d(side, q, seed=side + q)
    rep, ex, _ = gh.run_parity(prog, C, 4, mode=mode, init=_init(prog, C))
    assert [g.kernel_artifact.kind for g in ex.compiled.sampling_groups] == ["potts3d", "potts3d"]
    _assert_parity(rep)


def test_potts_non_cubic_lattice_matches_oracle(cuda_device):
    prog = workloads.PottsLattice3D((8, 4, 6), *_random_params((8, 4, 6), 5, seed=3))
    rep, _, _ = gh.run_parity(prog, 64, 6, mode="philox", init=_init(prog, 64))
    _assert_parity(rep)


def _random_params(dims, q, seed):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((3, q, q)).astype(np.float32)
    J = ((A + A.transpose(0, 2, 1)) * np.float32(0.5)).astype(np.float32)
    bias = (0.7 * rng.standard_normal((int(np.prod(dims)), q))).astype(np.float32)
    return J, bias


@pytest.mark.parametrize("mode", ["variates", "philox"])
def test_potts_stencil_equals_generic_kernel(cuda_device, mode):
    prog = workloads.potts_lattice_3d(8, 8, seed=4)
    C = 32
    states = []
    for force_generic in (False, True):
        cfg = make_cuda_config(rng_mode="parity" if mode == "variates" else "philox", n_chains=C, cuda_graphs=False)
        compiled = compile_program(None, 0, prog, cfg, n_sweeps=6, n_chains=C, force_generic=force_generic)
        kinds = {g.kernel_artifact.kind for g in compiled.sampling_groups}
        assert kinds == ({"generic"} if force_generic else {"potts3d"})
        ex = Executor(None, 0, prog, cfg, compiled, n_sweeps=6, n_chains=C)
        ex.load_state(_init(prog, C, 2), [])
        if mode == "variates":
            buffers, _ = gh.make_variates(ex, 6, seed=9)
            ex._install_rng(buffers, 6)
        else:
            ex.prepare_rng(17)
        ex.run_sweeps(6)
        states.append(ex.raw_state())
    np.testing.assert_array_equal(states[0], states[1])


def test_potts_graph_replay_equals_eager(cuda_device):
    prog = workloads.potts_lattice_3d(8, 8, seed=5)
    C = 64
    states = []
    for graphs in (False, True):
        ex = Executor(None, 0, prog, make_cuda_config(n_chains=C, cuda_graphs=graphs), n_sweeps=20, n_chains=C)
        ex.load_state(_init(prog, C, 3), [])
        ex.prepare_rng(5)
        ex.run_sweeps(8)
        ex.run_sweeps(8)
        states.append(ex.raw_state())
    np.testing.assert_array_equal(states[0], states[1])


def _exact_potts_distribution(prog):
    """Exact joint of a tiny lattice: log p(s) = sum_i b_i[s_i] + 1/2 sum_i sum_(j in N(i)) J_a[s_i][s_j]."""
    n, q = prog.n_sites, prog.q
    X, Y, Z = prog.dims
    states = np.array(list(itertools.product(range(q), repeat=n)), dtype=np.int64)  # [S, n] by linear site
    logw = np.zeros(len(states))
    for i in range(n):
        logw += prog.site_bias[i][states[:, i]]
        x, y, z = i % X, (i // X) % Y, i // (X * Y)
        for a, (dx, dy, dz) in enumerate(((1, 0, 0), (0, 1, 0), (0, 0, 1))):
            for sgn in (-1, 1):
                j = (((z + sgn * dz) % Z) * Y + (y + sgn * dy) % Y) * X + (x + sgn * dx) % X
                logw += 0.5 * prog.J[a][states[:, i], states[:, j]]
    p = np.exp(logw - logw.max())
    return states, p / p.sum()


@pytest.mark.parametrize("q", [2, 3])
def test_potts_samples_exact_boltzmann_distribution(cuda_device, q):
    """2x2x2 periodic lattice: q=2 compares the full joint (256 states, total variation below
    twice the iid sampling noise sqrt(K/N)); q=3 (6561 states) compares every site marginal."""
    dims = (2, 2, 2)
    J, bias = _random_params(dims, q, seed=10 + q)
    J *= np.float32(0.25)  # every bond of a side-2 lattice is doubled: keep the chain fast-mixing
    prog = workloads.PottsLattice3D(dims, J, bias)
    C = 4096
    n_burn, n_keep, thin = 40, 60, 3
    ex = Executor(None, 0, prog, make_cuda_config(n_chains=C), n_sweeps=n_burn + n_keep * thin + 4, n_chains=C)
    ex.load_state(_init(prog, C, 7), [])
    ex.prepare_rng(23)
    ex.run_sweeps(n_burn)
    sites = [prog.sites_of_block(0), prog.sites_of_block(1)]
    half = prog.n_sites // 2
    samples = []
    for _ in range(n_keep):
        ex.run_sweeps(thin)
        raw = ex.raw_state().astype(np.int64)  # [rows, C]
        full = np.empty((C, prog.n_sites), dtype=np.int64)
        full[:, sites[0]] = raw[:half].T
        full[:, sites[1]] = raw[half:].T
        samples.append(full)
    samples = np.concatenate(samples)
    n_eff = len(samples)
    states, p = _exact_potts_distribution(prog)
    if q == 2:
        w = q ** np.arange(prog.n_sites)
        emp = np.bincount(samples @ w, minlength=len(p)).astype(np.float64)
        emp = emp[states @ w] / n_eff
        tv = 0.5 * np.abs(emp - p).sum()
        assert tv < 2.0 * np.sqrt(len(p) / n_eff), tv
    else:
        for i in range(prog.n_sites):
            exact = np.array([p[states[:, i] == k].sum() for k in range(q)])
            emp = np.bincount(samples[:, i], minlength=q) / n_eff
            sd = np.sqrt(exact * (1 - exact) / n_eff)
            assert np.all(np.abs(emp - exact) < 6.0 * sd + 1e-4), (i, emp, exact)


@pytest.mark.parametrize("q", [3, 8])
def test_potts_conditional_frequencies(cuda_device, q):
    """Only colour 0 is resampled, from fixed colour-1 neighbours: each colour-0 site's
    category frequencies must follow softmax(theta) of its (fixed) field."""
    prog = workloads.potts_lattice_3d(4, q, seed=30 + q, j_std=0.5)
    C = 4096
    ex = Executor(None, 0, prog, make_cuda_config(n_chains=C), n_sweeps=64, n_chains=C)
    rng = np.random.default_rng(31)
    half = prog.n_sites // 2
    other = rng.integers(0, q, half).astype(np.int32)
    ex.load_state([np.zeros((C, half), np.int32), np.broadcast_to(other, (C, half)).copy()], [])
    ex.prepare_rng(41)
    group0 = ex.compiled.sampling_groups[0]
    assert group0.block_indices == (0,)
    counts = np.zeros((half, q))
    n_rep = 12
    for s in range(n_rep):
        ex._run_sampling_group(group0, s)
        raw = ex.raw_state()[:half].astype(np.int64)  # [rows, C]
        for k in range(q):
            counts[:, k] += (raw == k).sum(1)
    freq = counts / (n_rep * C)
    # exact conditional in float64 from the fixed neighbours
    nb = prog.neighbour_rows(0) - half
    theta = prog.site_bias[prog.sites_of_block(0)].astype(np.float64)
    for a in range(3):
        for t in range(2):
            theta += prog.J[a][:, other[nb[:, 2 * a + t]]].T
    p = np.exp(theta - theta.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    sd = np.sqrt(p * (1 - p) / (n_rep * C))
    assert np.all(np.abs(freq - p) < 5.5 * sd + 2e-4), np.max(np.abs(freq - p) / (sd + 1e-9))
