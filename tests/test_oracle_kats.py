"""Pins the CPU oracle to the reference's own known-answer tests (CPU only).

Golden values come from tests/golden/reference_kats.json, extracted from the
reference's tests/test_compiler_lowering.py and scripts/probe_gather_pipeline.py
by tests/golden/make_golden.py.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import thrml_shim as th
from oracle import oracle as orc
from tt_thrml_b200.core import Family, FusedBlockSpec, FusedInteractionSpec
from tt_thrml_b200.workloads import IndexBlock, TableGibbsSpec, TableProgram

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())


def _flat_sources(block, k, src):
    it = block.interactions[k]
    n, T = block.n_nodes, it.n_terms
    return it.sources[src].reshape(n, T).tolist()


def test_kat1_mixed_program_flat_gather_offsets():
    prog = th.make_mixed_case().program
    op = orc.lower_program(prog)
    assert len(GOLD["kat1_flat_offsets"]) == 6
    for case in GOLD["kat1_flat_offsets"]:
        got = _flat_sources(op.blocks[case["block"]], case["interaction"], case["source"])
        assert got == case["expected"], case["expr"]


def _variates_zero(op, group, C=1, value=0.0):
    out = {}
    for bi in group:
        b = op.blocks[bi]
        out[bi] = np.full((b.n_nodes, b.q if b.family == "categorical" else 1, C), value, dtype=np.float32)
    return out


def test_kat2_spin_target_selects_categorical_source():
    case = GOLD["kat2_categorical_source"]
    prog = th.make_mixed_case().program
    sampler = orc.OracleSampler(prog, n_chains=1, n_threads=1)
    group = sampler.prog.sampling_order[0]
    assert case["block"] in group
    for c in case["cases"]:
        sampler.state[:, 0] = np.asarray(c["state"], dtype=np.float32)
        v = _variates_zero(sampler.prog, group)
        v[case["block"]][:] = np.asarray(case["rng"], dtype=np.float32).reshape(-1, 1, 1)
        sampler.group_step(0, 0, variates=v)
        assert sampler.state[0, 0] == c["expected_out0"]


def test_kat3_superblock_blocks_sample_from_the_same_state():
    case = GOLD["kat3_superblock"]
    prog = th.two_spin_superblock_program()
    assert case["coupling"] == [-1.0]
    sampler = orc.OracleSampler(prog, n_chains=1, n_threads=1)
    sampler.state[:, 0] = np.asarray(case["state"], dtype=np.float32)
    v = {bi: np.asarray(r, dtype=np.float32).reshape(1, 1, 1) for bi, r in zip((0, 1), case["rng"])}
    sampler.group_step(0, 0, variates=v)
    np.testing.assert_array_equal(sampler.state[:, 0], np.asarray(case["expected"], dtype=np.float32))


def probe_program(family: Family, global_state, indices, wm, extra_gaussian_rows: int = 0):
    """Table program: one free block of len(indices) targets reading a clamped block holding global_state."""
    idx = np.asarray(indices, dtype=np.int32)
    n, T = idx.shape
    gs = np.asarray(global_state, dtype=np.float32)
    total = n + gs.size
    inter = FusedInteractionSpec(
        weighted_mask=np.asarray(wm, dtype=np.float32).reshape(n, T),
        gather_indices=(idx + n,),
        n_spin=1,
        n_categorical=0,
        n_terms=T,
        contribution_kind="default" if family == Family.SPIN else "linear",
    )
    free = FusedBlockSpec(0, family, n, None, 0, total, (inter,))
    clamped = FusedBlockSpec(1, Family.GAUSSIAN, gs.size, None, n, total, ())
    blocks = [IndexBlock(n, family), IndexBlock(gs.size, Family.GAUSSIAN)]
    spec = TableGibbsSpec(free_blocks=blocks[:1], clamped_blocks=blocks[1:], sampling_order=[[0]])
    return TableProgram(spec, [free, clamped]), gs


def test_kat4_kat5_gather_and_field():
    k4, k5 = GOLD["kat4_gather"], GOLD["kat5_gamma"]
    # KAT 4: pure gather, read through a unit-weight one-term field per gathered element
    idx = np.asarray(k4["indices"])
    prog, gs = probe_program(Family.GAUSSIAN, k4["global_state"], idx.reshape(-1, 1), np.ones((idx.size, 1)))
    s = orc.OracleSampler(prog, n_chains=1, n_threads=1)
    s.load_state([np.zeros(idx.size, np.float32)], [gs])
    s.group_step(0, 0, variates={0: np.zeros((idx.size, 1, 1), np.float32)})
    expected = np.asarray(k4["global_state"], np.float32)[idx].reshape(-1)
    np.testing.assert_allclose(s.state[: idx.size, 0], expected / np.float32(1.0 + 1e-6), rtol=1e-6)
    # KAT 5: gamma = sum(w * m * state[idx])
    w, m = np.asarray(k5["weights"], np.float32), np.asarray(k5["mask"], np.float32)
    prog, gs = probe_program(Family.GAUSSIAN, k5["global_state"], k5["indices"], w * m)
    s = orc.OracleSampler(prog, n_chains=1, n_threads=1)
    s.load_state([np.zeros(3, np.float32)], [gs])
    s.group_step(0, 0, variates={0: np.zeros((3, 1, 1), np.float32)})
    gamma = np.sum(w * m * np.asarray(k5["global_state"], np.float32)[np.asarray(k5["indices"])], axis=-1)
    np.testing.assert_allclose(s.state[:3, 0], gamma / np.float32(1.0 + 1e-6), rtol=1e-6)


def test_kat6_threshold():
    k6 = GOLD["kat6_threshold"]
    w, m = np.asarray(k6["weights"], np.float32), np.asarray(k6["mask"], np.float32)
    rng = np.asarray(k6["rng"], np.float32)
    prog, gs = probe_program(Family.SPIN, k6["global_state"], k6["indices"], w * m)
    s = orc.OracleSampler(prog, n_chains=1, n_threads=1)
    s.load_state([np.ones(3, bool)], [gs])
    # the probe compares gamma > rng; the sweep kernels compare 2*gamma > l, so l = 2*rng (exact)
    s.group_step(0, 0, variates={0: (2.0 * rng).reshape(3, 1, 1)})
    gamma = np.sum(w * m * np.asarray(k6["global_state"], np.float32)[np.asarray(k6["indices"])], axis=-1, keepdims=True)
    expected = np.where(gamma > rng, 1.0, -1.0).reshape(-1)
    np.testing.assert_array_equal(s.state[:3, 0], expected)


# Published Philox4x32-10 known-answer vectors (Salmon et al., Random123 distribution).
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    (
        (0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344),
        (0xA4093822, 0x299F31D0),
        (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1),
    ),
]


@pytest.mark.parametrize("ctr,key,expected", PHILOX_KAT)
def test_oracle_philox_known_answers(ctr, key, expected):
    assert tuple(int(x) for x in orc.philox4x32_10(ctr, key)) == expected


def test_oracle_runs_multichain_philox_deterministically():
    prog = th.make_spin_case().program
    a = orc.OracleSampler(prog, n_chains=8, n_threads=2)
    b = orc.OracleSampler(prog, n_chains=8, n_threads=1)
    init = [np.random.default_rng(0).integers(0, 2, (8, 2)).astype(bool) for _ in range(2)]
    for s in (a, b):
        s.load_state(init)
        for sweep in range(5):
            s.sweep(sweep, seed=1234)
    np.testing.assert_array_equal(a.state, b.state)


def test_oracle_dense_rng_layout_differs_from_site_layout():
    """The dense (unit-axis) Philox counter layout gives different draws from the site layout."""
    import numpy as np

    from tt_thrml_b200 import workloads

    prog = workloads.gaussian_bernoulli_rbm(256, 256, seed=0, w_std=0.05)
    rng = np.random.default_rng(13)
    init = [rng.standard_normal((8, 256)).astype(np.float32), rng.integers(0, 2, (8, 256)).astype(bool)]
    res = []
    for layout in ("chain4", "row4"):
        o = orc.OracleSampler(prog, n_chains=8, rng_layout=layout)
        o.load_state(init)
        o.group_step(0, 0, seed=99)
        res.append(o.state.copy())
    assert not np.array_equal(res[0], res[1])
    with pytest.raises(ValueError):
        orc.OracleSampler(prog, n_chains=8, rng_layout="tiles")


def test_oracle_split_uniform_lattice_layouts():
    """The oracle's lattice draws ("row8s", "chain8s" split uniforms, "planes" bit-planes) follow their counters:
    a numpy restatement of one colour half-sweep (neighbour-sign pattern, exact threshold,
    23-bit draw = 16 shared bits << 7 | 7 refill bits) gives the same states."""
    import numpy as np

    import ising_ref
    from tt_thrml_b200 import workloads
    from tt_thrml_b200.compiler import ising_pattern_tables

    H, W, C, seed, sweep = 8, 16, 16, 0x0123456789ABCDEF, 5
    prog = workloads.IsingLattice2D(H, W, beta=0.4407)
    st = prog.tt_stencil()
    _, thr = ising_pattern_tables(st["edge_weight"], st["site_bias"])
    rng = np.random.default_rng(5)
    lat = rng.choice(np.array([-1, 1], np.int8), size=(C, H, W))
    blocks = []
    for c in range(2):
        ys, xs = np.nonzero(((np.arange(H)[:, None] + np.arange(W)[None, :]) & 1) == c)
        blocks.append(lat[:, ys, xs] > 0)
    k0, k1 = seed & 0xFFFFFFFF, seed >> 32
    for layout in ("row8s", "chain8s", "planes", "planes8"):
        o = orc.OracleSampler(prog, n_chains=C, rng_layout=layout)
        o.load_state(blocks)
        o.group_step(0, sweep, seed=seed)
        got = o.state[: H * W // 2].T > 0  # [C][rows] of colour 0
        ys, xs = np.nonzero(((np.arange(H)[:, None] + np.arange(W)[None, :]) & 1) == 0)
        s = lat.astype(np.int64)
        idx = ((s[:, ys, (xs - 1) % W] < 0) * 1 + (s[:, ys, (xs + 1) % W] < 0) * 2
               + (s[:, (ys - 1) % H, xs] < 0) * 4 + (s[:, (ys + 1) % H, xs] < 0) * 8)
        row = np.broadcast_to(np.arange(len(ys))[None, :], (C, len(ys))).astype(np.uint64)
        gc = np.broadcast_to(np.arange(C)[:, None], (C, len(ys))).astype(np.uint64)
        sw = np.full(row.shape, sweep, np.uint64)
        if layout == "planes8":  # bit 8 (row % 4) + chain % 8 of counter (chain / 8, row / 4, sweep, "LPL0" + b / 4)
            pos = np.uint64(8) * (row & np.uint64(3)) + (gc & np.uint64(7))
            m = np.zeros(row.shape, np.int64)
            for b in range(23):
                wb = ising_ref.philox4x32_10(gc >> np.uint64(3), row >> np.uint64(2), sw,
                                             np.full(row.shape, 0x4C504C30 + b // 4), k0, k1)[b % 4]
                m |= ((wb >> pos) & np.uint64(1)).astype(np.int64) << (22 - b)
            np.testing.assert_array_equal(got, m < thr.astype(np.int64)[idx])
            continue
        if layout in ("row8s", "planes"):  # one chain per counter: the numpy restatement, chain by chain
            m = np.stack([ising_ref.lattice_draws(layout, row[c].astype(np.int64), c, sweep, seed) for c in range(C)])
            np.testing.assert_array_equal(got, m < thr.astype(np.int64)[idx])
            continue
        else:
            words = ising_ref.philox4x32_10(gc >> np.uint64(3), row, sw, np.full(row.shape, 0x4C535049), k0, k1)
            pos = gc
        w = np.choose(((pos >> np.uint64(1)) & np.uint64(3)).astype(np.int64), words)
        h = (w >> (np.uint64(16) * (pos & np.uint64(1)))) & np.uint64(0xFFFF)
        f = ising_ref.philox4x32_10(gc, row, sw, np.full(row.shape, 0x4C524546), k0, k1)[0] >> np.uint64(25)
        m = ((h << np.uint64(7)) | f).astype(np.int64)
        want = m < thr.astype(np.int64)[idx]
        np.testing.assert_array_equal(got, want)
