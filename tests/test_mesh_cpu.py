"""MeshExecutor's shard bookkeeping on two gloo ranks (CPU, no GPU).

The shard executor is replaced by a host fake that keeps its block states in
numpy, so the test checks what MeshExecutor itself does with one process per
GPU (tt_thrml/mesh.py:29-57 is the interface it keeps): which chains each
rank owns, how full and rank-local initial states are split, that sweeps
reach every shard, and that read-backs (observe, sample_states, block_sums)
are all-gathered in chain order -- or stay rank-local with gather=False.
"""

from __future__ import annotations

import os
import socket
from types import SimpleNamespace

import numpy as np
import pytest

import thrml_shim as th

C_TOTAL = 8


class _FakeShard:
    """Stands in for the CUDA Executor: state per block as (chains, n) numpy arrays, a sweep flips signs."""

    def __init__(self, ttnn, device, program, config, compiled=None, *, n_sweeps=100, profile=False, n_chains=None,
                 chain_offset=0):
        self.program = program
        self.n_chains, self.chain_offset = int(n_chains), int(chain_offset)
        blocks = list(program.gibbs_spec.blocks)
        self.compiled = SimpleNamespace(
            blocks=[SimpleNamespace(spec=SimpleNamespace(n_nodes=len(b.nodes))) for b in blocks],
            n_free_blocks=len(program.gibbs_spec.free_blocks))
        self.states = None
        self.sweeps = 0
        self.stream = SimpleNamespace(synchronize=lambda: None)

    @property
    def state_is_loaded(self):
        return self.states is not None

    def load_state(self, free, clamp):
        self.states = [np.asarray(s).reshape(self.n_chains, -1).astype(np.int8) for s in list(free) + list(clamp)]

    def prepare_rng(self, key):
        self.key = key

    def _prepare_rng_thrml_compat(self, key, schedule, n_total):
        self.key = key

    def run_sweep(self):
        self.run_sweeps(1)

    def run_sweeps(self, n):
        self.sweeps += n
        if n % 2:
            self.states = [1 - s for s in self.states]

    def _block_states_host(self, blocks):
        return [self.states[b].astype(bool) for b in blocks]

    def block_sums(self, blocks):
        return np.stack([s.sum(1) for s in self.states[: len(blocks)]], axis=0).sum(0).astype(np.float64)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import tt_thrml_b200.mesh as mesh
        from tt_thrml_b200 import make_cuda_config

        mesh.Executor = _FakeShard
        case = th.make_spin_case()
        cfg = make_cuda_config(n_chains=C_TOTAL)
        rng = np.random.default_rng(0)  # the same full initial state on every rank
        full = [rng.integers(0, 2, (C_TOTAL, len(b.nodes))).astype(bool) for b in case.program.gibbs_spec.free_blocks]
        res = {}

        ex = mesh.make_mesh_executor(None, "gpu", case.program, cfg, n_sweeps=8)
        assert ex._mode == "ranks" and len(ex.shards) == 1
        sh = ex.shards[0]
        res["offset"], res["local"] = sh.chain_offset, sh.n_chains
        ex.load_state(full, [])
        res["loaded"] = [s.copy() for s in sh.states]
        ex.run_sweeps(3)
        res["sweeps"] = sh.sweeps
        obs = ex.observe(case.program.gibbs_spec.free_blocks)
        res["observed"] = [obs[b] for b in case.program.gibbs_spec.free_blocks]
        res["sums"] = ex.block_sums(case.program.gibbs_spec.free_blocks)
        samples = ex.sample_states(1, th.SamplingSchedule(2, 3, 1), case.program.gibbs_spec.free_blocks,
                                   init_state_free=full)
        res["samples_shape"] = [np.asarray(x).shape for x in samples]

        # rank-local initial states and read-backs
        loc = mesh.make_mesh_executor(None, "gpu", case.program, cfg, n_sweeps=8, gather=False)
        mine = [s[rank * 4 : rank * 4 + 4] for s in full]
        loc.load_state(mine, [])
        obs = loc.observe(case.program.gibbs_spec.free_blocks)
        res["local_observed"] = [obs[b] for b in case.program.gibbs_spec.free_blocks]
        with pytest.raises(ValueError):
            loc.load_state([s[:3] for s in full], [])
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.array(res, dtype=object), allow_pickle=True)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_mesh_executor_shards_chains_over_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    case = th.make_spin_case()
    rng = np.random.default_rng(0)
    full = [rng.integers(0, 2, (C_TOTAL, len(b.nodes))).astype(bool) for b in case.program.gibbs_spec.free_blocks]
    for rank in range(2):
        res = np.load(tmp_path / f"rank{rank}.npy", allow_pickle=True).item()
        assert (res["offset"], res["local"]) == (4 * rank, 4)
        for got, want in zip(res["loaded"], full):
            np.testing.assert_array_equal(got.astype(bool), want[4 * rank : 4 * rank + 4])
        assert res["sweeps"] == 3
        # three sweeps of the fake flip every spin; the read-back holds all 8 chains in chain order on every rank
        for got, want in zip(res["observed"], full):
            np.testing.assert_array_equal(got, ~want)
        np.testing.assert_array_equal(res["sums"], sum((~w).sum(1) for w in full).astype(np.float64))
        assert res["samples_shape"] == [(3, C_TOTAL, len(b.nodes)) for b in case.program.gibbs_spec.free_blocks]
        for got, want in zip(res["local_observed"], full):
            np.testing.assert_array_equal(got, want[4 * rank : 4 * rank + 4])
