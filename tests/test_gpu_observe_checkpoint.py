"""Device-side moment observer and executor checkpoint / restore on the GPU.

DeviceMomentObserver must return exactly the carry of the host
MomentAccumulatorObserver (same run, same seed); a checkpoint taken mid-run
and restored into a fresh executor must continue bit for bit, for every state
layout (bit-packed, int8 stencil, bf16 dense, float32 generic).
"""

from __future__ import annotations

import numpy as np
import pytest

import thrml_shim as th
from tt_thrml_b200 import Executor, make_cuda_config, workloads
from tt_thrml_b200.observers import DeviceMomentObserver, MomentAccumulatorObserver

pytestmark = pytest.mark.gpu


def _moment_spec(prog, rng, n=12):
    blocks = prog.gibbs_spec.blocks
    nodes = [(bi, k) for bi, b in enumerate(blocks) for k in range(len(b.nodes))]
    pick = rng.choice(len(nodes), size=(n, 2), replace=False)
    node = lambda i: blocks[nodes[i][0]].nodes[nodes[i][1]]  # noqa: E731
    return [[(node(i),) for i in pick[:, 0]], [(node(i), node(j)) for i, j in pick]]


@pytest.mark.parametrize("spin_as_bool", [True, False])
def test_device_moments_equal_host_moments(cuda_device, spin_as_bool):
    prog = workloads.erdos_renyi_ising(4096, 6.0, seed=3)
    C = 256
    rng = np.random.default_rng(0)
    spec = _moment_spec(prog, rng)
    init = [rng.integers(0, 2, (C, len(b.nodes))).astype(bool) for b in prog.gibbs_spec.free_blocks]
    sched = th.SamplingSchedule(n_warmup=4, n_samples=10, steps_per_sample=2)

    def transform(states, blocks):
        return [np.where(np.asarray(s), 1.0, 0.0) if spin_as_bool else np.where(np.asarray(s), 1.0, -1.0)
                for s in states]

    out = []
    for obs in (MomentAccumulatorObserver(spec, transform), DeviceMomentObserver(spec, spin_as_bool=spin_as_bool)):
        ex = Executor(None, 0, prog, make_cuda_config(n_chains=C), n_sweeps=64, n_chains=C)
        carry, _ = ex.sample_with_observation(7, sched, obs, init_state_free=init)
        out.append(carry)
    for host, dev in zip(*out):
        np.testing.assert_array_equal(np.asarray(host, np.float32), dev)


def _continue_check(prog, C, n_first, n_second, **cfg):
    init_rng = np.random.default_rng(1)

    def init():
        out = []
        for b in prog.gibbs_spec.free_blocks:
            fam = getattr(b, "family", None)
            n = len(b.nodes)
            if getattr(fam, "value", fam) == "gaussian":
                out.append(init_rng.standard_normal((C, n)).astype(np.float32))
            elif getattr(fam, "value", fam) == "categorical":
                out.append(init_rng.integers(0, b.n_categories, (C, n)).astype(np.int32))
            else:
                out.append(init_rng.integers(0, 2, (C, n)).astype(bool))
        return out

    state0 = init()
    n = n_first + n_second
    a = Executor(None, 0, prog, make_cuda_config(n_chains=C, **cfg), n_sweeps=n, n_chains=C)
    a.load_state(state0, [])
    a.prepare_rng(11)
    a.run_sweeps(n)
    b = Executor(None, 0, prog, make_cuda_config(n_chains=C, **cfg), n_sweeps=n, n_chains=C)
    b.load_state(state0, [])
    b.prepare_rng(11)
    b.run_sweeps(n_first)
    ck = b.checkpoint()
    c = Executor(None, 0, prog, make_cuda_config(n_chains=C, **cfg), n_sweeps=n, n_chains=C)
    c.restore(ck, key=11)
    c.run_sweeps(n_second)
    np.testing.assert_array_equal(c.raw_state(), a.raw_state())
    return c


@pytest.mark.parametrize(
    "name",
    ["er_bits", "er_int8", "potts", "rbm", "ising_one_chain", "gaussian_generic"],
)
def test_checkpoint_continues_bit_for_bit(cuda_device, name, tmp_path):
    if name == "er_bits":
        c = _continue_check(workloads.erdos_renyi_ising(8192, 8.0, seed=1), 256, 5, 7)
        assert c.compiled.state_dtype == "bits"
    elif name == "er_int8":
        _continue_check(workloads.erdos_renyi_ising(8192, 8.0, seed=1), 64, 4, 4)
    elif name == "potts":
        _continue_check(workloads.potts_lattice_3d(8, 8, seed=2), 64, 3, 5)
    elif name == "rbm":
        _continue_check(workloads.gaussian_bernoulli_rbm(256, 512, seed=3, w_std=0.05), 128, 4, 4)
    elif name == "ising_one_chain":
        _continue_check(workloads.IsingLattice2D(64, 128, beta=0.44), 1, 6, 6)
    else:
        case = th.make_gaussian_case()
        _continue_check(case.program, 32, 3, 3)
    if name == "er_bits":  # file round trip
        prog = workloads.erdos_renyi_ising(8192, 8.0, seed=1)
        ex = Executor(None, 0, prog, make_cuda_config(n_chains=256), n_sweeps=8, n_chains=256)
        ex.load_state([np.ones((256, len(b.nodes)), bool) for b in prog.gibbs_spec.free_blocks], [])
        ex.prepare_rng(3)
        ex.run_sweeps(3)
        ex.save_checkpoint(tmp_path / "ck.npz")
        ex2 = Executor(None, 0, prog, make_cuda_config(n_chains=256), n_sweeps=8, n_chains=256)
        ex2.load_checkpoint(tmp_path / "ck.npz")
        np.testing.assert_array_equal(ex2.raw_state(), ex.raw_state())
        ex.run_sweeps(2)
        ex2.run_sweeps(2)
        np.testing.assert_array_equal(ex2.raw_state(), ex.raw_state())


def test_checkpoint_rejects_a_different_executor(cuda_device):
    prog = workloads.erdos_renyi_ising(2048, 6.0, seed=1)
    a = Executor(None, 0, prog, make_cuda_config(n_chains=64), n_sweeps=4, n_chains=64)
    a.load_state([np.ones((64, len(b.nodes)), bool) for b in prog.gibbs_spec.free_blocks], [])
    a.prepare_rng(1)
    ck = a.checkpoint()
    b = Executor(None, 0, prog, make_cuda_config(n_chains=32), n_sweeps=4, n_chains=32)
    with pytest.raises(ValueError):
        b.restore(ck)


@pytest.mark.parametrize("graphs", [True, False])
def test_magnetisation_schedule_equals_state_samples(cuda_device, graphs):
    """The device-side magnetisation of a whole schedule (one CUDA graph when graphs are on) equals the
    per-chain sums of the states that sample_states returns for the same key."""
    from tt_thrml_b200.observers import MagnetizationObserver

    prog = workloads.ising_lattice_2d(32, 32, beta=0.44)
    C = 256
    rng = np.random.default_rng(4)
    init = [rng.integers(0, 2, (C, len(b.nodes))).astype(bool) for b in prog.gibbs_spec.free_blocks]
    sched = th.SamplingSchedule(n_warmup=6, n_samples=9, steps_per_sample=3)
    ex = Executor(None, 0, prog, make_cuda_config(n_chains=C, cuda_graphs=graphs), n_sweeps=64, n_chains=C)
    blocks = prog.gibbs_spec.free_blocks
    _, mags = ex.sample_with_observation(5, sched, MagnetizationObserver(blocks), init_state_free=init)
    _, mags2 = ex.sample_with_observation(5, sched, MagnetizationObserver(blocks), init_state_free=init)
    states = ex.sample_states(5, sched, blocks, init_state_free=init)
    want = sum(np.where(s, 1.0, -1.0).sum(-1) for s in states)  # [n_samples, C]
    assert mags.shape == (9, C)
    np.testing.assert_array_equal(mags, want)
    np.testing.assert_array_equal(mags2, want)
