"""A lattice written with thrml factors (IsingEBM over a periodic grid) runs on the stencil kernels.

The compiler recognises the lowered tables as a 2-D lattice: with many chains the shared-memory resident
kernel, with one chain the single-chain stencil kernel.  Checked against the oracle's lowering of the thrml
program (table path), and against the native lattice program of the same model: the same kernels and
draws give bit-identical samples.
"""

from __future__ import annotations

import numpy as np
import pytest

import gpu_harness as gh
import thrml_shim as th
from tt_thrml_b200 import Executor, make_cuda_config, workloads

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("C,kind", [(64, "ising2d_resident"), (1, "ising2d")])
def test_thrml_ising_grid_runs_on_the_stencil_kernels(cuda_device, C, kind):
    prog, _ = th.ising_grid_program(16, 32, J=1.0, h=0.1, beta=0.4407)
    rep, ex, o = gh.run_parity(prog, C, 4, mode="philox")
    assert {g.kernel_artifact.kind for g in ex.compiled.sampling_groups} == {kind}
    assert o.prog.model is None  # the oracle lowers the thrml program itself (per-term tables)
    assert rep.hard_mismatches == 0, rep
    assert rep.band_fraction < 1e-4, rep


def test_thrml_grid_equals_the_native_lattice(cuda_device):
    H, W, C = 16, 32, 128
    grid, _ = th.ising_grid_program(H, W, J=1.0, h=0.0, beta=0.44)
    native = workloads.IsingLattice2D(H, W, J=1.0, h=0.0, beta=0.44)
    rng = np.random.default_rng(4)
    init = [rng.integers(0, 2, (C, H * W // 2)).astype(bool) for _ in range(2)]
    sched = th.SamplingSchedule(n_warmup=5, n_samples=4, steps_per_sample=3)
    out = []
    for prog in (grid, native):
        ex = Executor(None, 0, prog, make_cuda_config(n_chains=C), n_sweeps=32, n_chains=C)
        assert {g.kernel_artifact.kind for g in ex.compiled.sampling_groups} == {"ising2d_resident"}
        out.append(ex.sample_states(9, sched, prog.gibbs_spec.free_blocks, init_state_free=init))
    for a, b in zip(*out):
        np.testing.assert_array_equal(np.asarray(a), np.asarray(b))


def _potts_params(dims, q, seed):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((3, q, q)).astype(np.float32)
    J = ((A + A.transpose(0, 2, 1)) * np.float32(0.5)).astype(np.float32)
    bias = (0.7 * rng.standard_normal((int(np.prod(dims)), q))).astype(np.float32)
    return J, bias


@pytest.mark.parametrize("mode", ["philox", "variates"])
def test_thrml_potts_grid_runs_on_the_stencil_kernel(cuda_device, mode):
    dims, q, C = (8, 4, 6), 5, 32
    J, bias = _potts_params(dims, q, 1)
    prog, _ = th.potts_grid_program(dims, J, bias)
    rng = np.random.default_rng(2)
    init = [rng.integers(0, q, (C, 96)).astype(np.uint8) for _ in range(2)]
    rep, ex, o = gh.run_parity(prog, C, 4, mode=mode, init=init)
    assert {g.kernel_artifact.kind for g in ex.compiled.sampling_groups} == {"potts3d"}
    assert o.prog.model is None  # the oracle lowers the thrml program itself
    assert rep.hard_mismatches == 0, rep
    assert rep.band_fraction < 1e-4, rep


def test_thrml_potts_grid_equals_the_native_lattice(cuda_device):
    dims, q, C = (8, 8, 8), 8, 64
    J, bias = _potts_params(dims, q, 3)
    grid, _ = th.potts_grid_program(dims, J, bias)
    native = workloads.PottsLattice3D(dims, J, bias)
    rng = np.random.default_rng(4)
    init = [rng.integers(0, q, (C, 256)).astype(np.uint8) for _ in range(2)]
    sched = th.SamplingSchedule(n_warmup=3, n_samples=3, steps_per_sample=2)
    out = []
    for prog in (grid, native):
        ex = Executor(None, 0, prog, make_cuda_config(n_chains=C), n_sweeps=16, n_chains=C)
        assert {g.kernel_artifact.kind for g in ex.compiled.sampling_groups} == {"potts3d"}
        out.append(ex.sample_states(11, sched, prog.gibbs_spec.free_blocks, init_state_free=init))
    for a, b in zip(*out):
        np.testing.assert_array_equal(np.asarray(a), np.asarray(b))
