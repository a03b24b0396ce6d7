"""GPU parity: CUDA kernels (through the C ABI) against the CPU oracle.

Criteria (per sampled site): spin / categorical states bit-exact except where
the decision margin is within 1e-5 of the threshold (such ties are counted and
must stay below 1e-4 of all sites); gaussian states within 1e-4 relative.
Comparisons run group by group from the same input state and variates.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import gpu_harness as gh
import thrml_shim as th
from oracle import oracle as orc
from tt_thrml_b200 import Executor, make_cuda_config, workloads
from tt_thrml_b200.compiler import compile_program

pytestmark = pytest.mark.gpu

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())


def _assert_parity(rep: gh.ParityReport):
    assert rep.hard_mismatches == 0, rep
    assert rep.band_fraction < 1e-4, rep
    assert rep.gauss_max_rel <= gh.GAUSS_RTOL, rep


def _case_init(case, C):
    return [np.broadcast_to(np.asarray(s), (C,) + np.asarray(s).shape).copy() for s in case.init_state_free]


SCENARIOS = {
    "spin": th.make_spin_case,
    "categorical": th.make_categorical_case,
    "gaussian": th.make_gaussian_case,
    "mixed": th.make_mixed_case,
}


@pytest.mark.parametrize("mode", ["variates", "philox"])
@pytest.mark.parametrize("name", sorted(SCENARIOS))
def test_reference_scenarios_match_oracle(cuda_device, name, mode):
    case = SCENARIOS[name]()
    C = 64
    rep, ex, _ = gh.run_parity(case.program, C, 12, mode=mode, init=_case_init(case, C))
    _assert_parity(rep)
    if name == "spin":  # the IsingEBM-style program: two pair interactions per block, merged into one CSR
        assert ex.compiled.sampling_groups[0].kernel_artifact.kind == "spin_csr"


@pytest.mark.parametrize("mode", ["variates", "philox"])
def test_clamped_program_matches_oracle(cuda_device, mode):
    prog, sched, init, clamp, _ = th.make_clamp_case()
    C = 32
    rep, ex, _ = gh.run_parity(prog, C, 10, mode=mode, init=[np.repeat(s[None], C, 0) for s in init], clamp=clamp)
    _assert_parity(rep)
    # the clamped row never changes
    assert (gh.gpu_state(ex)[2] == 1.0).all()


@pytest.mark.parametrize("C", [32, 64, 256])
@pytest.mark.parametrize("mode", ["variates", "philox"])
def test_spin_csr_kernel_matches_oracle_on_random_graph(cuda_device, mode, C):
    prog = workloads.erdos_renyi_ising(3000, 8.0, seed=3)
    rep, ex, _ = gh.run_parity(prog, C, 4, mode=mode)
    kind = "spin_bits" if C % 256 == 0 else "spin_csr"
    assert all(g.kernel_artifact.kind == kind for g in ex.compiled.sampling_groups)
    _assert_parity(rep)


@pytest.mark.parametrize("mode", ["variates", "philox"])
def test_lattice_runs_on_spin_csr_and_matches_oracle(cuda_device, mode):
    prog = workloads.ising_lattice_2d(16, 24, beta=0.44)
    rep, ex, _ = gh.run_parity(prog, 128, 6, mode=mode, stencil=False)  # the lattice's tables, not its stencil
    assert [g.kernel_artifact.kind for g in ex.compiled.sampling_groups] == ["spin_csr", "spin_csr"]
    _assert_parity(rep)


def test_generic_and_spin_csr_paths_agree_bit_for_bit(cuda_device):
    prog = workloads.erdos_renyi_ising(2000, 6.0, seed=5)
    C = 64
    outs = []
    for force in (False, True):
        cfg = make_cuda_config(n_chains=C, cuda_graphs=False)
        comp = compile_program(None, 0, prog, cfg, n_sweeps=8, n_chains=C, force_generic=force)
        assert (comp.sampling_groups[0].kernel_artifact.kind == "generic") == force
        ex = Executor(None, 0, prog, cfg, comp, n_sweeps=8, n_chains=C)
        ex.load_state(gh.random_init(prog, C, 1), [])
        ex.prepare_rng(99)
        for _ in range(8):
            ex.run_sweep()
        outs.append(gh.gpu_state(ex))
    np.testing.assert_array_equal(outs[0], outs[1])


def test_degree_ordered_rows_give_the_same_samples(cuda_device):
    """The bit-packed kernel runs each colour block's rows sorted by degree; the order changes no sample."""
    prog = workloads.erdos_renyi_ising(5000, 8.0, seed=4)
    C = 256
    outs = []
    cfg = make_cuda_config(n_chains=C)
    for ordered in (True, False):
        # an uncached compile: the plan objects changed below are this executor's alone
        comp = compile_program(None, 0, prog, cfg, n_sweeps=6, n_chains=C, cache=False)
        ex = Executor(None, 0, prog, cfg, comp, n_sweeps=6, n_chains=C)
        plans = [g.kernel_artifact for g in ex.compiled.sampling_groups]
        assert {p.kind for p in plans} == {"spin_bits"}
        for plan in plans:
            for blk in plan.blocks:
                order = blk.row_order.cpu().numpy()
                deg = np.diff(blk.row_ptr.cpu().numpy())
                assert sorted(order.tolist()) == list(range(blk.n_rows))
                assert np.all(np.diff(deg[order]) >= 0)
                if not ordered:
                    blk.row_order = None  # natural order through tthrml_spin_bits_step
        ex.load_state(gh.random_init(prog, C, 7), [])
        ex.prepare_rng(13)
        ex.run_sweeps(6)
        outs.append(gh.gpu_state(ex))
    np.testing.assert_array_equal(outs[0], outs[1])


@pytest.mark.parametrize("C", [256, 512])
def test_bit_packed_and_int8_layouts_agree_bit_for_bit(cuda_device, C):
    prog = workloads.erdos_renyi_ising(3000, 9.0, seed=8)
    outs = []
    for layout in ("int8", "bits"):
        cfg = make_cuda_config(n_chains=C, cuda_graphs=True, spin_layout=layout)
        ex = Executor(None, 0, prog, cfg, n_sweeps=12, n_chains=C)
        assert ex.compiled.state_dtype == layout
        ex.load_state(gh.random_init(prog, C, 2), [])
        ex.prepare_rng(31)
        ex.run_sweeps(12)
        outs.append(gh.gpu_state(ex))
        sums = ex.block_sums(prog.gibbs_spec.free_blocks)
        np.testing.assert_array_equal(sums, outs[-1].sum(0))
    np.testing.assert_array_equal(outs[0], outs[1])


def test_cuda_graph_replay_equals_eager_sweeps(cuda_device):
    prog = workloads.erdos_renyi_ising(4000, 8.0, seed=2)
    C = 128
    res = []
    for graphs in (False, True):
        cfg = make_cuda_config(n_chains=C, cuda_graphs=graphs)
        ex = Executor(None, 0, prog, cfg, n_sweeps=40, n_chains=C)
        ex.load_state(gh.random_init(prog, C, 4), [])
        ex.prepare_rng(5)
        ex.run_sweeps(7)
        ex.run_sweep()
        ex.run_sweeps(7)  # replays the cached 7-sweep graph at a new position
        ex.run_sweeps(16)
        assert ex._sweep_counter == 31
        res.append(gh.gpu_state(ex))
    np.testing.assert_array_equal(res[0], res[1])


def test_parity_mode_graph_replay_reads_the_right_sweep(cuda_device):
    prog = workloads.ising_lattice_2d(8, 8)
    C = 32
    res = []
    for graphs in (False, True):
        cfg = make_cuda_config(n_chains=C, cuda_graphs=graphs, rng_mode="parity")
        ex = Executor(None, 0, prog, cfg, n_sweeps=20, n_chains=C)
        ex.load_state(gh.random_init(prog, C, 4), [])
        buffers, _ = gh.make_variates(ex, 20, seed=3)
        ex._install_rng(buffers, 20)
        ex.run_sweeps(5)
        ex.run_sweeps(5)
        ex.run_sweeps(10)
        res.append(gh.gpu_state(ex))
    np.testing.assert_array_equal(res[0], res[1])


def test_reference_kats_on_gpu(cuda_device):
    """KAT 2 and KAT 3 of the reference through the executor and the C ABI."""
    k2 = GOLD["kat2_categorical_source"]
    prog = th.make_mixed_case().program
    cfg = make_cuda_config(rng_mode="parity", n_chains=1, cuda_graphs=False)
    for c in k2["cases"]:
        ex = Executor(None, 0, prog, cfg, n_sweeps=1)
        st = np.asarray(c["state"], np.float32)
        init = [st[i : i + 1] for i in range(6)]
        init[0] = init[0] > 0
        init[3] = init[3] > 0
        ex.load_state(init, [])
        buffers, _ = gh.make_variates(ex, 1)
        buffers.spin_threshold_logits[0].zero_()
        ex._install_rng(buffers, 1)
        ex._run_sampling_group(ex.compiled.sampling_groups[0], 0)
        assert gh.gpu_state(ex)[0, 0] == c["expected_out0"]
    k3 = GOLD["kat3_superblock"]
    prog = th.two_spin_superblock_program()
    ex = Executor(None, 0, prog, cfg, n_sweeps=1)
    ex.load_state([np.array([k3["state"][0] > 0]), np.array([k3["state"][1] > 0])], [])
    buffers, _ = gh.make_variates(ex, 1)
    for bi in (0, 1):
        buffers.spin_threshold_logits[bi].zero_()
    ex._install_rng(buffers, 1)
    ex.run_sweep()
    np.testing.assert_array_equal(gh.gpu_state(ex)[:, 0], np.asarray(k3["expected"], np.float32))


def test_spin_distribution_matches_exact_boltzmann(cuda_device):
    """The reference's spin scenario thresholds (state hist L-inf <= 0.05, mean <= 0.02) against the exact law."""
    case = th.make_spin_case()
    C = 2048
    ex = Executor(None, 0, case.program, make_cuda_config(n_chains=C), n_sweeps=200, n_chains=C)
    samples = ex.sample_states(123, th.SamplingSchedule(32, 20, 4), case.nodes_to_sample,
                               init_state_free=_case_init(case, C))
    s = np.asarray(samples[0]).reshape(-1, 4)  # (samples*chains, 4) bool
    code = (s.astype(np.int64) << np.arange(4)).sum(1)
    hist = np.bincount(code, minlength=16) / code.size
    p = gh.exact_spin_distribution([0.35, -0.25, 0.2, -0.15], {(0, 1): 0.75, (1, 2): -0.45, (2, 3): 0.3}, 4)
    assert np.max(np.abs(hist - p)) <= 0.05 * 0.2
    mean = (2 * s - 1).mean(0)
    pm = (((np.arange(16)[:, None] >> np.arange(4)) & 1) * 2 - 1).T @ p
    assert np.max(np.abs(mean - pm)) <= 0.02


def test_gaussian_moments_match_exact(cuda_device):
    """Gaussian scenario: exact mean/covariance of the joint normal (reference thresholds 5e-3 / 1e-2)."""
    case = th.make_gaussian_case()
    C = 4096
    ex = Executor(None, 0, case.program, make_cuda_config(n_chains=C), n_sweeps=400, n_chains=C)
    out = ex.sample_states(7, th.SamplingSchedule(40, 30, 3), case.nodes_to_sample,
                           init_state_free=_case_init(case, C))
    x = np.asarray(out[0], np.float64).reshape(-1, 3)
    # p(x) ~ exp(b.x - 0.5 x^T P x) with P_ii = 1/iw_i (+1e-6 in the kernel) and P_ij = -J
    iw = np.array([0.7, 0.9, 0.8])
    P = np.diag(1.0 / iw + 1e-6)
    P[0, 1] = P[1, 0] = -0.12
    P[1, 2] = P[2, 1] = 0.08
    cov = np.linalg.inv(P)
    mean = cov @ np.array([0.15, -0.35, 0.2])
    assert np.max(np.abs(x.mean(0) - mean)) <= 5e-3
    assert np.max(np.abs(np.cov(x.T, bias=True) - cov)) <= 1e-2


def test_observe_and_state_roundtrip(cuda_device):
    prog = workloads.erdos_renyi_ising(500, 4.0, seed=1)
    C = 64
    ex = Executor(None, 0, prog, make_cuda_config(n_chains=C), n_sweeps=4, n_chains=C)
    init = gh.random_init(prog, C, 3)
    ex.load_state(init, [])
    obs = ex.observe(prog.gibbs_spec.free_blocks)
    for b, s in zip(prog.gibbs_spec.free_blocks, init):
        np.testing.assert_array_equal(obs[b], s)
    sums = ex.block_sums(prog.gibbs_spec.free_blocks)
    expect = sum((2 * s.astype(np.int64) - 1).sum(1) for s in init)
    np.testing.assert_array_equal(sums, expect.astype(np.float64))


@pytest.mark.slow
def test_full_size_random_graph_group_step_matches_oracle(cuda_device):
    """Full configuration size (2^20 nodes, 256 chains): one sweep group by group against the oracle."""
    prog = workloads.erdos_renyi_ising(1 << 20, 8.0, seed=0)
    rep, ex, _ = gh.run_parity(prog, 256, 1, mode="philox", seed=2024)
    assert rep.sites == (1 << 20) * 256
    _assert_parity(rep)


@pytest.mark.slow
def test_full_size_chain_sharding_is_invariant(cuda_device):
    """Running 256 chains at once or as two 128-chain shards (chain_offset 0 / 128) gives identical chains."""
    prog = workloads.erdos_renyi_ising(1 << 20, 8.0, seed=0)
    init = gh.random_init(prog, 256, 9)
    cfg = make_cuda_config(n_chains=256)
    full = Executor(None, 0, prog, cfg, n_sweeps=3, n_chains=256)
    full.load_state(init, [])
    full.prepare_rng(1)
    full.run_sweeps(3)
    whole = gh.gpu_state(full)
    del full
    parts = []
    for off in (0, 128):
        ex = Executor(None, 0, prog, make_cuda_config(n_chains=128), n_sweeps=3, n_chains=128, chain_offset=off)
        ex.load_state([s[off : off + 128] for s in init], [])
        ex.prepare_rng(1)
        ex.run_sweeps(3)
        parts.append(gh.gpu_state(ex))
    np.testing.assert_array_equal(whole, np.concatenate(parts, axis=1))
