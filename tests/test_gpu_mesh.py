"""MeshExecutor on a GPU: chain shards reproduce one executor over all chains bit for bit.

Two shards of one CudaMeshDevice may sit on the same GPU (each with its own
stream), which runs the multi-device driver of MeshExecutor on a one-GPU box.
Philox counters are keyed by the global chain index, so the chains do not
depend on how they are sharded.
"""

from __future__ import annotations

import numpy as np
import pytest

import gpu_harness as gh
import thrml_shim as th
from tt_thrml_b200 import Executor, make_cuda_config, make_mesh_executor, workloads
from tt_thrml_b200.backend import CudaDevice, CudaMeshDevice

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["er", "lattice"])
def test_two_shards_equal_one_executor(cuda_device, name):
    if name == "er":
        prog, C = workloads.erdos_renyi_ising(4096, 8.0, seed=3), 512
    else:
        prog, C = workloads.ising_lattice_2d(64, 64, beta=0.44), 2048
    init = gh.random_init(prog, C, 4)
    cfg = make_cuda_config(n_chains=C)
    blocks = prog.gibbs_spec.free_blocks

    one = Executor(None, 0, prog, cfg, n_sweeps=16, n_chains=C)
    one.load_state(init, [])
    one.prepare_rng(5)
    one.run_sweeps(6)
    want = one.observe(blocks)

    dev = CudaMeshDevice((2,), [CudaDevice(0), CudaDevice(0)])
    mesh = make_mesh_executor(None, dev, prog, cfg, n_sweeps=16, n_chains=C)
    assert mesh._mode == "devices" and [s.chain_offset for s in mesh.shards] == [0, C // 2]
    assert {g.kernel_artifact.kind for g in mesh.compiled.sampling_groups} == \
        {g.kernel_artifact.kind for g in one.compiled.sampling_groups}
    mesh.load_state(init, [])
    mesh.prepare_rng(5)
    mesh.run_sweeps(6)
    got = mesh.observe(blocks)
    for b in blocks:
        np.testing.assert_array_equal(got[b], want[b])
    np.testing.assert_array_equal(mesh.block_sums(blocks), one.block_sums(blocks))

    sched = th.SamplingSchedule(n_warmup=3, n_samples=4, steps_per_sample=2)
    a = one.sample_states(9, sched, blocks, init_state_free=init)
    b = mesh.sample_states(9, sched, blocks, init_state_free=init)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(np.asarray(x), np.asarray(y))
