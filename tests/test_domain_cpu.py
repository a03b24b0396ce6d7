"""Strip domain decomposition of a single-chain 2-D Ising lattice, on CPU ranks.

LatticeStrips is driven with the host restatement of the half-sweep kernel
(tests/ising_ref.py) on CPU tensors, over gloo process groups of 2 and 4
ranks: the decomposed run must reproduce the single-domain run bit for bit
(state and energy/magnetisation trace), and the single-domain run must
reproduce the oracle on the lattice's per-edge tables.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import ising_ref
from oracle import oracle as orc
from tt_thrml_b200 import workloads
from tt_thrml_b200.domain import LatticeStrips


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_single(prog, halo, seed, n_sweeps, init_seed=5):
    st = LatticeStrips(prog, device="cpu", halo=halo, halfsweep=lambda *a: None)
    st._halfsweep = ising_ref.make_halfsweep(st)
    st.load_random(init_seed)
    st.prepare_rng(seed, n_sweeps)
    st.run_sweeps(n_sweeps)
    return st.gather_lattice(), st.trace()


def test_numpy_philox_matches_oracle():
    rng = np.random.default_rng(0)
    ctr = rng.integers(0, 2**32, (5, 4), dtype=np.uint64)
    key = (0x1234ABCD, 0x0BADF00D)
    got = ising_ref.philox4x32_10(ctr[:, 0], ctr[:, 1], ctr[:, 2], ctr[:, 3], *key)
    for i in range(5):
        want = orc.philox4x32_10(ctr[i].astype(np.uint32), np.array(key, np.uint32))
        assert [int(g[i]) for g in got] == [int(w) for w in want]


@pytest.mark.parametrize("H,W", [(8, 32), (6, 64)])
def test_single_domain_matches_oracle(H, W):
    prog = workloads.IsingLattice2D(H, W, beta=0.4407)
    st = LatticeStrips(prog, device="cpu", halo=2, halfsweep=lambda *a: None)
    st._halfsweep = ising_ref.make_halfsweep(st)
    st.load_random(3)
    st.prepare_rng(11, 6)
    o = orc.OracleSampler(prog, n_chains=1, rng_layout=st.rng_layout)
    lat = st.gather_lattice()
    half = H * W // 2
    # oracle state rows: block c = colour-c sites in linear order = split-colour rows
    blocks = []
    for c in range(2):
        rows = np.arange(H)
        cols = (np.arange(W // 2)[None, :] * 2) + ((rows[:, None] + c) & 1)
        blocks.append(np.take_along_axis(lat, cols, axis=1).reshape(-1))
    o.load_state([(b > 0) for b in blocks])
    from tt_thrml_b200.rng import seed_from_key

    for s in range(3):
        o.sweep(s, seed=seed_from_key(11))
    st.run_sweeps(3)
    lat = st.gather_lattice()
    for c in range(2):
        rows = np.arange(H)
        cols = (np.arange(W // 2)[None, :] * 2) + ((rows[:, None] + c) & 1)
        mine = np.take_along_axis(lat, cols, axis=1).reshape(-1)
        np.testing.assert_array_equal(mine.astype(np.float32), o.state[c * half : (c + 1) * half, 0])
    bonds, mag = ising_ref.lattice_energy_magnetisation(lat)
    tr = st.trace()
    assert tr.shape == (3, 2) and tr[-1, 0] == mag and tr[-1, 1] == bonds


def _worker(rank, world, port, H, W, halo, n_sweeps, out_path):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        prog = workloads.IsingLattice2D(H, W, beta=0.4407)
        st = LatticeStrips(prog, device="cpu", halo=halo, halfsweep=lambda *a: None)
        st._halfsweep = ising_ref.make_halfsweep(st)
        st.load_random(5)
        st.prepare_rng(21, n_sweeps)
        st.run_sweeps(n_sweeps)
        lat = st.gather_lattice()
        tr = st.trace()
        if rank == 0:
            np.savez(out_path, lattice=lat, trace=tr)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,halo", [(2, 2), (2, 4), (4, 2)])
def test_strip_decomposition_reproduces_single_domain(tmp_path, world, halo):
    import torch.multiprocessing as mp

    H, W, n_sweeps = 16, 32, 8
    prog = workloads.IsingLattice2D(H, W, beta=0.4407)
    lat1, tr1 = _run_single(prog, halo, 21, n_sweeps)
    out = tmp_path / "res.npz"
    mp.start_processes(_worker, args=(world, _free_port(), H, W, halo, n_sweeps, str(out)), nprocs=world,
                       join=True, start_method="spawn")
    res = np.load(out)
    np.testing.assert_array_equal(res["lattice"], lat1)
    np.testing.assert_array_equal(res["trace"], tr1)
    bonds, mag = ising_ref.lattice_energy_magnetisation(lat1)
    assert tr1[-1, 0] == mag and tr1[-1, 1] == bonds


def test_strip_arguments_are_checked():
    prog = workloads.IsingLattice2D(16, 32)
    with pytest.raises(ValueError):
        LatticeStrips(prog, device="cpu", halo=3, halfsweep=lambda *a: None)  # odd halo
    with pytest.raises(ValueError):
        LatticeStrips(prog, device="cpu", halo=18, halfsweep=lambda *a: None)  # deeper than the strip
    with pytest.raises(ValueError):
        LatticeStrips(workloads.IsingLattice2D(16, 48), device="cpu", halo=2, halfsweep=lambda *a: None)
    st = LatticeStrips(prog, device="cpu", halo=4, halfsweep=lambda *a: None)
    st.prepare_rng(0, 4)
    with pytest.raises(ValueError):
        st.run_sweeps(3)  # not a multiple of halo/2


def test_strip_checkpoint_continues_bit_for_bit():
    prog = workloads.IsingLattice2D(16, 32, beta=0.4407)

    def fresh():
        st = LatticeStrips(prog, device="cpu", halo=2, halfsweep=lambda *a: None)
        st._halfsweep = ising_ref.make_halfsweep(st)
        return st

    a = fresh()
    a.load_random(2)
    a.prepare_rng(5, 10)
    a.run_sweeps(10)
    b = fresh()
    b.load_random(2)
    b.prepare_rng(5, 10)
    b.run_sweeps(4)
    ck = b.checkpoint()
    c = fresh()
    c.restore(ck)
    c.run_sweeps(6)
    np.testing.assert_array_equal(c.gather_lattice(), a.gather_lattice())
    np.testing.assert_array_equal(c.trace(), a.trace())
    with pytest.raises(ValueError):
        LatticeStrips(prog, device="cpu", halo=4, halfsweep=lambda *a: None).restore(ck)


def _dropout_worker(rank, world, port, out_path):
    """Rank 1 leaves before the run (between steps, with nothing in flight); rank 0's next exchange must
    end with an error from the process group's timeout instead of waiting forever."""
    import datetime
    import time

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    prog = workloads.IsingLattice2D(16, 32, beta=0.4407)
    st = LatticeStrips(prog, device="cpu", halo=2, halfsweep=lambda *a: None)
    st._halfsweep = ising_ref.make_halfsweep(st)
    st.load_random(1)
    st.prepare_rng(2, 8)
    st.run_sweeps(2)  # both ranks exchange normally
    if rank == 1:
        return  # leaves without a word to its neighbour
    t0 = time.perf_counter()
    try:
        st.run_sweeps(2)
        outcome = "no error"
    except Exception as e:  # noqa: BLE001 - the process group reports the missing peer
        outcome = f"error: {type(e).__name__}"
    with open(out_path, "w") as f:
        f.write(f"{outcome} after {time.perf_counter() - t0:.1f}s")


def test_a_rank_that_leaves_ends_the_exchange_with_an_error(tmp_path):
    import torch.multiprocessing as mp

    out = tmp_path / "dropout.txt"
    ctx = mp.start_processes(_dropout_worker, args=(2, _free_port(), str(out)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    text = out.read_text()
    assert text.startswith("error"), text
    assert float(text.split(" after ")[1].rstrip("s")) < 60.0


def test_bit_packed_rows_round_trip_and_load():
    """Bit-packed strip storage: pack/unpack invert each other (site s of a word at bit 8 (s % 4) + s / 4),
    and loading a lattice then gathering it returns it unchanged."""
    import torch

    rng = np.random.default_rng(4)
    rows = torch.from_numpy(rng.choice(np.array([-1, 1], np.int8), size=(5, 128)))
    words = LatticeStrips.pack_rows(rows)
    assert words.dtype == torch.int32 and tuple(words.shape) == (5, 4)
    np.testing.assert_array_equal(LatticeStrips.unpack_rows(words).numpy(), rows.numpy())
    # bit 8 (s % 4) + s / 4 of word w is site 32 w + s
    w = words.numpy().astype(np.int64) & 0xFFFFFFFF
    for s_ in (0, 1, 5, 31):
        bit = (w[:, 1] >> (8 * (s_ % 4) + s_ // 4)) & 1
        np.testing.assert_array_equal(bit, (rows.numpy()[:, 32 + s_] < 0).astype(np.int64))
    prog = workloads.IsingLattice2D(16, 256, beta=0.4407)
    st = LatticeStrips(prog, device="cpu", halo=2, halfsweep=lambda *a: None, storage="bits")
    lat = rng.choice(np.array([-1, 1], np.int8), size=(16, 256))
    st.load_lattice(lat)
    np.testing.assert_array_equal(st.gather_lattice(), lat)
    ref = LatticeStrips(prog, device="cpu", halo=2, halfsweep=lambda *a: None, storage="int8")
    st.load_random(3)
    ref.load_random(3)
    np.testing.assert_array_equal(st.gather_lattice(), ref.gather_lattice())
    with pytest.raises(ValueError):
        LatticeStrips(workloads.IsingLattice2D(16, 64, beta=0.4407), device="cpu", halo=2,
                      halfsweep=lambda *a: None, storage="bits")
