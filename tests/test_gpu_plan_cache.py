"""The plan cache on a GPU: a second executor, or a second top-level `sample_states` call, over the same
program reuses the first one's device tables (no lowering, no upload) and samples identically; a different
chain count or configuration compiles anew; the cache stays bounded."""

from __future__ import annotations

import numpy as np
import pytest

import gpu_harness as gh
import thrml_shim as th
import tt_thrml_b200 as tt
from tt_thrml_b200 import Executor, compiler, make_cuda_config, workloads

pytestmark = pytest.mark.gpu


def test_second_executor_reuses_the_tables(cuda_device):
    compiler.clear_plan_cache()
    prog = workloads.erdos_renyi_ising(5000, 8.0, seed=7)
    cfg = make_cuda_config(n_chains=256)
    a = Executor(None, 0, prog, cfg, n_sweeps=8, n_chains=256)
    assert compiler.plan_cache_size() == 1
    b = Executor(None, 0, workloads.erdos_renyi_ising(5000, 8.0, seed=7), cfg, n_sweeps=8, n_chains=256)
    assert compiler.plan_cache_size() == 1  # equal contents: the same entry
    pa, pb = a.compiled.sampling_groups[0].kernel_artifact, b.compiled.sampling_groups[0].kernel_artifact
    assert pa is not pb and pa.blocks[0].cols is pb.blocks[0].cols  # own plan objects, shared tables
    init = gh.random_init(prog, 256, 1)
    out = []
    for ex in (a, b):
        ex.load_state(init, [])
        ex.prepare_rng(3)
        ex.run_sweeps(5)
        out.append(ex.raw_state())
    np.testing.assert_array_equal(out[0], out[1])
    Executor(None, 0, prog, make_cuda_config(n_chains=512), n_sweeps=8, n_chains=512)
    assert compiler.plan_cache_size() == 2  # another chain count: another plan


def test_top_level_sample_states_does_not_lower_again(cuda_device, monkeypatch):
    compiler.clear_plan_cache()
    case = th.make_mixed_case()
    calls = []
    real = compiler.lower_program

    def counting(program):
        calls.append(1)
        return real(program)

    monkeypatch.setattr(compiler, "lower_program", counting)
    cfg = make_cuda_config(n_chains=1)
    res = [tt.sample_states(5, case.program, case.schedule, case.init_state_free, [], case.nodes_to_sample,
                            config=cfg) for _ in range(3)]
    assert len(calls) == 1
    for r in res[1:]:
        for x, y in zip(r, res[0]):
            np.testing.assert_array_equal(np.asarray(x), np.asarray(y))


def test_generic_plans_keep_private_descriptors(cuda_device):
    """Two executors of one program in parity mode upload different variates; each plan copy keeps its own
    block descriptor, so they do not overwrite each other's."""
    compiler.clear_plan_cache()
    case = th.make_mixed_case()
    C = 32
    exs = []
    for seed in (1, 2):
        rep, ex, _ = gh.run_parity(case.program, C, 2, mode="variates", seed=seed)
        assert rep.hard_mismatches == 0, rep
        exs.append(ex)
    p0, p1 = (e.compiled.sampling_groups[0].kernel_artifact for e in exs)
    assert p0._desc is not None and p1._desc is not None and p0._desc.data_ptr() != p1._desc.data_ptr()


def test_cache_is_bounded(cuda_device):
    compiler.clear_plan_cache()
    for k in range(compiler.PLAN_CACHE_SIZE + 3):
        Executor(None, 0, workloads.IsingLattice2D(8, 8 + 2 * k, beta=0.4), make_cuda_config(n_chains=32),
                 n_sweeps=2, n_chains=32)
    assert compiler.plan_cache_size() == compiler.PLAN_CACHE_SIZE
    compiler.clear_plan_cache()
    assert compiler.plan_cache_size() == 0
