"""Single-chain 2-D Ising stencil kernel (tthrml_ising2d_halfsweep) and the strip decomposition on GPUs.

The kernel is checked against the oracle on the lattice's per-edge tables
(spins bit-exact outside the 1e-5 band, counters in the row4 layout); the
strip decomposition (LatticeStrips) against the executor's whole-lattice run,
and its energy/magnetisation trace against the lattice it leaves.  With two
or more GPUs visible, a 2-rank NCCL run must reproduce the 1-GPU run bit for
bit.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import gpu_harness as gh
import ising_ref
from tt_thrml_b200 import Executor, make_cuda_config, workloads
from tt_thrml_b200.domain import LatticeStrips

pytestmark = pytest.mark.gpu


def _assert_parity(rep):
    assert rep.hard_mismatches == 0, rep
    assert rep.band_fraction < 1e-4, rep


@pytest.mark.parametrize("mode", ["variates", "philox"])
@pytest.mark.parametrize("H,W", [(64, 64), (32, 96)])
def test_ising2d_stencil_matches_oracle(cuda_device, mode, H, W):
    prog = workloads.IsingLattice2D(H, W, beta=0.4407)
    rep, ex, _ = gh.run_parity(prog, 1, 6, mode=mode)
    assert [g.kernel_artifact.kind for g in ex.compiled.sampling_groups] == ["ising2d", "ising2d"]
    _assert_parity(rep)


def test_ising2d_with_field_matches_oracle(cuda_device):
    prog = workloads.IsingLattice2D(32, 64, J=-0.7, h=0.3, beta=0.9)
    rep, _, _ = gh.run_parity(prog, 1, 6, mode="philox")
    _assert_parity(rep)


def _split(lattice, c):
    H, W = lattice.shape
    rows = np.arange(H)
    cols = (np.arange(W // 2)[None, :] * 2) + ((rows[:, None] + c) & 1)
    return np.take_along_axis(lattice, cols, axis=1)


@pytest.mark.parametrize("graphs", [False, True])
def test_strips_reproduce_the_executor(cuda_device, graphs):
    H, W, n = 128, 256, 12
    prog = workloads.IsingLattice2D(H, W, beta=0.4407)
    st = LatticeStrips(prog, device=cuda_device, halo=4, cuda_graphs=graphs)
    st.load_random(9)
    lat0 = st.gather_lattice()
    st.prepare_rng(33, n)
    st.run_sweeps(n)
    lat = st.gather_lattice()

    ex = Executor(None, 0, prog, make_cuda_config(n_chains=1, cuda_graphs=graphs), n_sweeps=n, n_chains=1)
    ex.load_state([_split(lat0, 0).reshape(-1) > 0, _split(lat0, 1).reshape(-1) > 0], [])
    ex.prepare_rng(33)
    ex.run_sweeps(n)
    raw = ex.raw_state()[:, 0]
    half = H * W // 2
    np.testing.assert_array_equal(_split(lat, 0).reshape(-1).astype(np.float32), raw[:half])
    np.testing.assert_array_equal(_split(lat, 1).reshape(-1).astype(np.float32), raw[half:])


def test_strip_trace_matches_the_lattice(cuda_device):
    H, W = 64, 128
    prog = workloads.IsingLattice2D(H, W, beta=0.4407)
    st = LatticeStrips(prog, device=cuda_device, halo=2)
    st.load_random(4)
    st.prepare_rng(8, 10)
    for _ in range(10):
        st.run_sweeps(1)
        bonds, mag = ising_ref.lattice_energy_magnetisation(st.gather_lattice())
        tr = st.trace()
        assert tr[-1, 0] == mag and tr[-1, 1] == bonds
    em = st.energy_magnetisation()
    assert em.shape == (10, 2) and np.all(np.abs(em) <= 2.0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, H, W, halo, n, out):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        prog = workloads.IsingLattice2D(H, W, beta=0.4407)
        st = LatticeStrips(prog, device=torch.device("cuda", rank), halo=halo)
        st.load_random(9)
        st.prepare_rng(33, n)
        st.run_sweeps(n)
        lat = st.gather_lattice()
        tr = st.trace()
        if rank == 0:
            np.savez(out, lattice=lat, trace=tr)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpu_strips_reproduce_one_gpu(cuda_device, tmp_path):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    H, W, halo, n = 256, 512, 8, 16
    prog = workloads.IsingLattice2D(H, W, beta=0.4407)
    st = LatticeStrips(prog, device=cuda_device, halo=halo)
    st.load_random(9)
    st.prepare_rng(33, n)
    st.run_sweeps(n)
    lat1, tr1 = st.gather_lattice(), st.trace()
    out = tmp_path / "nccl.npz"
    mp.start_processes(_nccl_worker, args=(2, _free_port(), H, W, halo, n, str(out)), nprocs=2, join=True,
                       start_method="spawn")
    res = np.load(out)
    np.testing.assert_array_equal(res["lattice"], lat1)
    np.testing.assert_array_equal(res["trace"], tr1)
