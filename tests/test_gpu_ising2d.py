"""Single-chain 2-D Ising stencil kernel (tthrml_ising2d_halfsweep) and the strip decomposition on GPUs.

The kernel is checked against the oracle on the lattice's per-edge tables
(spins bit-exact outside the 1e-5 band, counters in the row4 layout); the
strip decomposition (LatticeStrips, peer-memory and NCCL exchanges) against
the executor's whole-lattice run, and its energy/magnetisation trace against
the lattice it leaves.  With two or more GPUs visible, a 2-rank run must
reproduce the 1-GPU run bit for bit, and resume from a mid-run checkpoint.
The halo import's wait is bounded: a flag nobody sets ends it with an error.
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


@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
@pytest.mark.parametrize("graphs", [False, True])
def test_strips_reproduce_the_executor(cuda_device, graphs, exchange):
    H, W, n = 128, 256, 12
    prog = workloads.IsingLattice2D(H, W, beta=0.4407)
    st = LatticeStrips(prog, device=cuda_device, halo=4, cuda_graphs=graphs, exchange=exchange)
    st.load_random(9)
    lat0 = st.gather_lattice()
    st.prepare_rng(33, n)
    st.run_sweeps(n // 2)
    st.run_sweeps(n // 2)
    st.check_errors()
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


def _nccl_worker(rank, world, port, H, W, halo, n, out, exchange):
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
        st = LatticeStrips(prog, device=torch.device("cuda", rank), halo=halo, exchange=exchange)
        st.load_random(9)
        st.prepare_rng(33, n)
        st.run_sweeps(n // 2)
        ck = st.checkpoint()
        st.run_sweeps(n // 2)
        st.check_errors()
        lat = st.gather_lattice()
        tr = st.trace()
        # resume from the mid-run checkpoint: the same lattice again
        st.restore(ck)
        st.run_sweeps(n // 2)
        st.check_errors()
        assert np.array_equal(st.gather_lattice(), lat)
        st.close()
        if rank == 0:
            np.savez(out, lattice=lat, trace=tr)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
def test_two_gpu_strips_reproduce_one_gpu(cuda_device, tmp_path, exchange):
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
    mp.start_processes(_nccl_worker, args=(2, _free_port(), H, W, halo, n, str(out), exchange), nprocs=2,
                       join=True, start_method="spawn")
    res = np.load(out)
    np.testing.assert_array_equal(res["lattice"], lat1)
    np.testing.assert_array_equal(res["trace"], tr1)


@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
def test_bit_packed_strips_equal_int8_strips(cuda_device, exchange):
    """The bit-packed strips (k_ising2d_bits) and the int8 strips (k_ising2d_planes) evolve the same
    lattice and trace, through a checkpoint and resume of the bit-packed ones."""
    H, W, n = 128, 512, 12
    prog = workloads.IsingLattice2D(H, W, beta=0.4407)
    out = []
    for storage in ("int8", "bits"):
        st = LatticeStrips(prog, device=cuda_device, halo=4, exchange=exchange, storage=storage)
        assert st.storage == storage and st.colours[0].dtype == (torch_dtype("int8") if storage == "int8"
                                                                   else torch_dtype("int32"))
        st.load_random(5)
        st.prepare_rng(7, n)
        st.run_sweeps(n // 2)
        ck = st.checkpoint()
        st.run_sweeps(n // 2)
        st.check_errors()
        out.append((st.gather_lattice(), st.trace()))
        if storage == "bits":
            st.restore(ck)
            st.run_sweeps(n // 2)
            st.check_errors()
            np.testing.assert_array_equal(st.gather_lattice(), out[-1][0])
        st.close()
    np.testing.assert_array_equal(out[0][0], out[1][0])
    np.testing.assert_array_equal(out[0][1], out[1][1])


def torch_dtype(name):
    import torch

    return getattr(torch, name)


def test_strip_checkpoint_continues_on_one_gpu(cuda_device):
    prog = workloads.IsingLattice2D(64, 128, beta=0.4407)
    a = LatticeStrips(prog, device=cuda_device, halo=4)
    a.load_random(1)
    a.prepare_rng(2, 12)
    a.run_sweeps(12)
    b = LatticeStrips(prog, device=cuda_device, halo=4)
    b.load_random(1)
    b.prepare_rng(2, 12)
    b.run_sweeps(6)
    ck = b.checkpoint()
    c = LatticeStrips(prog, device=cuda_device, halo=4)
    c.restore(ck)
    c.run_sweeps(6)
    c.check_errors()
    np.testing.assert_array_equal(c.gather_lattice(), a.gather_lattice())
    np.testing.assert_array_equal(c.trace(), a.trace())


def test_halo_import_wait_is_bounded(cuda_device):
    """A neighbour that never publishes its period: the import gives up after its wait budget, reports
    the error and leaves the halo rows untouched; the context stays usable."""
    import time

    import torch

    from tt_thrml_b200 import _native as nat

    W, D, rows = 64, 2, 8
    hw = W // 2
    c0 = torch.ones((rows, hw), dtype=torch.int8, device=cuda_device)
    c1 = torch.ones((rows, hw), dtype=torch.int8, device=cuda_device)
    mailbox = torch.full((8 * D * hw,), -1, dtype=torch.int8, device=cuda_device)
    flags = torch.zeros(2, dtype=torch.int32, device=cuda_device)  # nobody sets them
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    nat.bind_device(0)
    t0 = time.perf_counter()
    rc = nat.lib().tthrml_halo_import(c0.data_ptr(), c1.data_ptr(), W, D, 0, rows - D, mailbox.data_ptr(),
                                      flags.data_ptr(), 1, 1, None, err.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream)  # sweep 1, 1 sweep/period: p = 2
    assert rc == 0
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 30.0
    assert int(err.item()) == 1
    assert bool((c0 == 1).all()) and bool((c1 == 1).all())
    # the same call with the flag published imports the mailbox
    flags.fill_(1)
    err.zero_()
    rc = nat.lib().tthrml_halo_import(c0.data_ptr(), c1.data_ptr(), W, D, 0, rows - D, mailbox.data_ptr(),
                                      flags.data_ptr(), 1, 1, None, err.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0 and int(err.item()) == 0
    assert bool((c0[:D] == -1).all()) and bool((c0[rows - D :] == -1).all()) and bool((c0[D : rows - D] == 1).all())


@pytest.mark.parametrize("H,W,C,layout", [(32, 64, 64, "planes8"), (16, 32, 256, "planes8"), (16, 20, 64, "chain8s")])
def test_resident_lattice_matches_oracle(cuda_device, H, W, C, layout):
    prog = workloads.IsingLattice2D(H, W, beta=0.4407)
    rep, ex, _ = gh.run_parity(prog, C, 4, mode="philox")
    assert [g.kernel_artifact.kind for g in ex.compiled.sampling_groups] == ["ising2d_resident"] * 2
    assert {g.kernel_artifact.rng_layout for g in ex.compiled.sampling_groups} == {layout}
    _assert_parity(rep)


@pytest.mark.parametrize("H,W,layout", [(64, 64, "planes"), (32, 96, "row8s")])
def test_single_chain_lattice_layout_choice(cuda_device, H, W, layout):
    prog = workloads.IsingLattice2D(H, W, beta=0.4407)
    rep, ex, _ = gh.run_parity(prog, 1, 3, mode="philox")
    assert {g.kernel_artifact.rng_layout for g in ex.compiled.sampling_groups} == {layout}
    _assert_parity(rep)


def test_resident_fused_sweeps_equal_group_launches(cuda_device):
    prog = workloads.IsingLattice2D(64, 64, J=0.8, h=0.1, beta=0.5)
    C = 128
    rng = np.random.default_rng(2)
    init = [rng.integers(0, 2, (C, len(b.nodes))).astype(bool) for b in prog.gibbs_spec.free_blocks]
    out = []
    for fused in (True, False):
        ex = Executor(None, 0, prog, make_cuda_config(n_chains=C), n_sweeps=12, n_chains=C)
        ex.load_state(init, [])
        ex.prepare_rng(9)
        if fused:
            ex.run_sweeps(5)
            ex.run_sweeps(7)
        else:
            for _ in range(12):
                ex.run_sweep()
        out.append(ex.raw_state())
    np.testing.assert_array_equal(out[0], out[1])


def test_resident_lattice_samples_the_same_law_as_the_table_kernel(cuda_device):
    """The resident kernel (exact threshold table) and the bit-packed table kernel (heat bath with ex2)
    agree on the mean |magnetisation| per site of a 16x32 lattice near criticality."""
    from tt_thrml_b200.observers import MagnetizationObserver
    import thrml_shim as th

    prog = workloads.IsingLattice2D(16, 32, beta=0.44)
    C = 1024
    rng = np.random.default_rng(3)
    init = [rng.integers(0, 2, (C, len(b.nodes))).astype(bool) for b in prog.gibbs_spec.free_blocks]
    sched = th.SamplingSchedule(n_warmup=200, n_samples=50, steps_per_sample=4)
    res = []
    for stencil in (True, False):
        ex = Executor(None, 0, prog, make_cuda_config(n_chains=C, stencil=stencil), n_sweeps=500, n_chains=C)
        kinds = {g.kernel_artifact.kind for g in ex.compiled.sampling_groups}
        assert kinds == ({"ising2d_resident"} if stencil else {"spin_bits"})
        _, m = ex.sample_with_observation(13, sched, MagnetizationObserver(prog.gibbs_spec.free_blocks),
                                          init_state_free=init)
        res.append(np.abs(m).mean() / 512.0)
    assert abs(res[0] - res[1]) < 0.02, res


@pytest.mark.parametrize("W,offset", [(64, 0), (128, 0), (192, 0), (256, 0), (384, 0), (512, 1), (512, 2)])
def test_bit_packed_halfsweep_any_word_count(cuda_device, W, offset):
    """tthrml_ising2d_halfsweep_bits takes 4, 2 or 1 words per thread by the row's word count and the
    other colour's alignment (offset: words before the buffer's start); every choice evolves the same
    lattice as the int8 kernel tthrml_ising2d_halfsweep_planes on the same draws, whole lattice, wrapped."""
    import torch

    from tt_thrml_b200 import _native as nat
    from tt_thrml_b200.compiler import ising_pattern_tables

    H, seed, n_sweeps = 16, 0x1234_5678_9ABC, 3
    prog = workloads.IsingLattice2D(H, W, beta=0.4407)
    st = prog.tt_stencil()
    _, thr = ising_pattern_tables(st["edge_weight"], st["site_bias"])
    thresholds = torch.from_numpy(thr.view(np.int32)).to(cuda_device)
    lib, stream = nat.lib(), nat.stream_handle(torch.cuda.current_stream(cuda_device))
    rng = np.random.default_rng(W + offset)
    int8 = [torch.from_numpy(rng.choice(np.array([-1, 1], np.int8), (H, W // 2))).to(cuda_device) for _ in range(2)]
    words = W // 64
    bits = []
    for c in range(2):
        buf = torch.zeros(offset + H * words, dtype=torch.int32, device=cuda_device)
        view = buf[offset:].view(H, words)
        view.copy_(LatticeStrips.pack_rows(int8[c]))
        bits.append((buf, view))
    for sweep in range(n_sweeps):
        for c in range(2):
            args = (W, H, 1, 0, H, 0, H, c, int(st["block_rows"][c]), thresholds.data_ptr(), 0, seed, sweep, None,
                    0, H, None, 0, None, stream)
            nat.check(lib.tthrml_ising2d_halfsweep_planes(int8[c].data_ptr(), int8[1 - c].data_ptr(), *args),
                      "tthrml_ising2d_halfsweep_planes")
            nat.check(lib.tthrml_ising2d_halfsweep_bits(bits[c][1].data_ptr(), bits[1 - c][1].data_ptr(), *args),
                      "tthrml_ising2d_halfsweep_bits")
            torch.cuda.synchronize(cuda_device)
            assert torch.equal(LatticeStrips.unpack_rows(bits[c][1]), int8[c]), (sweep, c)
    assert all(int(b[0][:offset].abs().sum()) == 0 for b in bits)  # nothing written before the rows
