"""CPU tests of the oracle's own model construction (oracle/models.py).

The stencil paths (2-D Ising, 3-D Potts) and the dense path (RBM) of
oracle.c must reproduce the table path on the same model built as per-term
tables; the random-graph generator and greedy colouring must reproduce the
configuration's inputs; the oracle's tables built from raw parameters must
equal the product's lowering of the same models.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import models
from oracle import oracle as orc
from tt_thrml_b200 import workloads


def _run_both(build, C, sweeps, init, *, layout="chain4", variates=None, **kw):
    """Runs the stencil / dense path and the table path side by side, group by group."""
    out = []
    for tables in (False, True):
        prog = build(tables)
        o = orc.OracleSampler(prog, n_chains=C, rng_layout=layout, n_threads=3, **kw)
        o.load_state(init)
        margins = []
        for s in range(sweeps):
            for gi in range(len(prog.sampling_order)):
                v = None
                if variates is not None:
                    v = {bi: variates(bi, s) for bi in prog.sampling_order[gi]}
                margins.append(o.group_step(gi, s, seed=0x1234_5678_9ABC, variates=v, return_margin=True))
        out.append((o.state.copy(), margins))
    return out


@pytest.mark.parametrize("layout", ["chain4", "row8s", "chain8s", "planes", "planes8"])
@pytest.mark.parametrize("J,h,beta", [(1.0, 0.0, 0.4407), (-0.7, 0.3, 0.9)])
def test_ising2d_stencil_path_equals_table_path(layout, J, h, beta):
    H, W, C = 8, 12, 16
    rng = np.random.default_rng(1)
    init = [rng.integers(0, 2, (C, H * W // 2)).astype(bool) for _ in range(2)]
    (s0, m0), (s1, m1) = _run_both(lambda t: models.ising2d(H, W, J=J, h=h, beta=beta, tables=t), C, 3, init,
                                   layout=layout)
    np.testing.assert_array_equal(s0, s1)
    for a, b in zip(m0, m1):
        np.testing.assert_array_equal(a, b)


def test_ising2d_stencil_path_equals_table_path_with_variates():
    H, W, C = 6, 10, 8
    rng = np.random.default_rng(2)
    init = [rng.integers(0, 2, (C, H * W // 2)).astype(bool) for _ in range(2)]
    logits = rng.logistic(size=(3, 2, H * W // 2, 1, C)).astype(np.float32)
    (s0, _), (s1, _) = _run_both(lambda t: models.ising2d(H, W, J=0.8, h=-0.2, beta=0.6, tables=t), C, 3, init,
                                 variates=lambda bi, s: logits[s, bi])
    np.testing.assert_array_equal(s0, s1)


@pytest.mark.parametrize("dims,q", [((4, 4, 4), 8), ((6, 4, 2), 3), ((2, 6, 4), 5)])
@pytest.mark.parametrize("mode", ["philox", "variates"])
def test_potts3d_stencil_path_equals_table_path(dims, q, mode):
    rng = np.random.default_rng(3)
    A = rng.standard_normal((3, q, q)).astype(np.float32)
    J = ((A + A.transpose(0, 2, 1)) * np.float32(0.5)).astype(np.float32)
    n = int(np.prod(dims))
    bias = (0.7 * rng.standard_normal((n, q))).astype(np.float32)
    C = 8
    init = [rng.integers(0, q, (C, n // 2)) for _ in range(2)]
    gum = (-np.log(-np.log(rng.uniform(1e-7, 1.0, (3, 2, n // 2, q, C))))).astype(np.float32)
    (s0, m0), (s1, m1) = _run_both(lambda t: models.potts3d(dims, J, bias, tables=t), C, 3, init,
                                   variates=(lambda bi, s: gum[s, bi]) if mode == "variates" else None)
    np.testing.assert_array_equal(s0, s1)
    for a, b in zip(m0, m1):
        np.testing.assert_array_equal(a, b)


def test_potts3d_out_of_range_neighbour_selects_zero():
    """A neighbour category outside [0, q) contributes weight 0 in both paths."""
    dims, q, C = (2, 2, 2), 3, 4
    rng = np.random.default_rng(4)
    J = rng.standard_normal((3, q, q)).astype(np.float32)
    bias = rng.standard_normal((8, q)).astype(np.float32)
    init = [np.full((C, 4), 7), rng.integers(0, q, (C, 4))]
    (s0, _), (s1, _) = _run_both(lambda t: models.potts3d(dims, J, bias, tables=t), C, 1, init)
    np.testing.assert_array_equal(s0, s1)


@pytest.mark.parametrize("visible", ["gaussian", "spin"])
@pytest.mark.parametrize("mode", ["philox", "variates"])
def test_dense_path_equals_table_path(visible, mode):
    V, H, C = 48, 80, 8
    rng = np.random.default_rng(5)
    W = (0.08 * rng.standard_normal((V, H))).astype(np.float32)
    b_v = (0.3 * rng.standard_normal(V)).astype(np.float32)
    b_h = (0.2 * rng.standard_normal(H)).astype(np.float32)
    init = [rng.standard_normal((C, V)).astype(np.float32) if visible == "gaussian"
            else rng.integers(0, 2, (C, V)).astype(bool), rng.integers(0, 2, (C, H)).astype(bool)]
    var = {0: rng.standard_normal((3, V, 1, C)).astype(np.float32) if visible == "gaussian"
           else rng.logistic(size=(3, V, 1, C)).astype(np.float32),
           1: rng.logistic(size=(3, H, 1, C)).astype(np.float32)}
    (s0, m0), (s1, m1) = _run_both(
        lambda t: models.dense_bipartite(W, b_v, b_h, visible_family=visible, tables=t), C, 3, init,
        layout="row4", variates=(lambda bi, s: var[bi][s]) if mode == "variates" else None)
    # the dense path sums in double, the table path in float32: spins agree outside the band, values within 1e-5
    for a, b in zip(m0, m1):
        assert np.all((np.abs(a) < 1e-5) | (np.sign(a) == np.sign(b)) | (a == 0))
    np.testing.assert_array_equal(s0[V:], s1[V:])
    if visible == "gaussian":
        np.testing.assert_allclose(s0[:V], s1[:V], rtol=1e-5, atol=1e-6)
    else:
        np.testing.assert_array_equal(s0[:V], s1[:V])


def test_dense_path_bf16_storage_rounds_gaussians():
    V, H, C = 32, 64, 4
    rng = np.random.default_rng(6)
    W = workloads.bf16_representable((0.05 * rng.standard_normal((V, H))).astype(np.float32))
    prog = models.dense_bipartite(W, np.zeros(V, np.float32), np.zeros(H, np.float32))
    o = orc.OracleSampler(prog, n_chains=C, rng_layout="row4", gaussian_storage="bf16")
    o.load_state([rng.standard_normal((C, V)).astype(np.float32), rng.integers(0, 2, (C, H)).astype(bool)])
    o.group_step(1, 0, seed=3)  # visible block (sampling order: hidden, visible)
    vis = o.state[:V]
    np.testing.assert_array_equal(vis, workloads.bf16_representable(vis))
    with pytest.raises(ValueError):
        orc.OracleSampler(prog, n_chains=C, gaussian_storage="fp16")


def test_er_generator_and_colouring_reproduce_the_configuration_inputs():
    """The oracle's seeded G(n, p) graph, couplings, biases and greedy colouring equal the workload's."""
    n, deg, seed = 3000, 8.0, 5
    raw = models.er_ising_raw(n, deg, seed=seed)
    prog = workloads.erdos_renyi_ising(n, deg, seed=seed)
    g = prog.meta["graph"]
    np.testing.assert_array_equal(raw["row_ptr"], g["row_ptr"])
    np.testing.assert_array_equal(raw["cols"], g["cols"])
    np.testing.assert_array_equal(raw["J"], g["J"])
    np.testing.assert_array_equal(raw["h"], g["h"])
    np.testing.assert_array_equal(raw["colours"], np.asarray(g["colours"]))
    # the colouring is proper and greedy: each node takes the smallest colour its lower neighbours leave free
    rp, cols, col = raw["row_ptr"], raw["cols"], raw["colours"]
    for v in range(0, n, 37):
        nb = cols[rp[v] : rp[v + 1]]
        assert col[v] not in set(col[nb])
        lower = set(col[nb[nb < v]])
        assert all(k in lower for k in range(col[v]))


def _same_tables(op, specs):
    for ob, spec in zip(op.blocks, specs):
        assert ob.start == spec.block_global_start and ob.n_nodes == spec.n_nodes
        ref = orc._from_spec(spec)
        assert len(ob.interactions) == len(ref.interactions)
        for a, b in zip(ob.interactions, ref.interactions):
            np.testing.assert_array_equal(a.row_ptr, b.row_ptr)
            np.testing.assert_array_equal(a.weights, b.weights)
            np.testing.assert_array_equal(a.sources, b.sources)
            assert a.n_categorical == b.n_categorical


@pytest.mark.parametrize("name", ["er", "ising", "potts", "rbm"])
def test_oracle_tables_from_raw_parameters_equal_the_product_lowering(name):
    """Two independent constructions of each synthetic model's tables agree entry for entry."""
    if name == "er":
        prog = workloads.erdos_renyi_ising(2000, 6.0, seed=1)
        op = orc.lower_program(prog)
        assert op.model is None
    elif name == "ising":
        prog = workloads.IsingLattice2D(8, 12, J=0.6, h=0.1, beta=0.7)
        op = orc.lower_program(prog, tables=True)
    elif name == "potts":
        prog = workloads.potts_lattice_3d(4, 5, seed=2)
        op = orc.lower_program(prog, tables=True)
    else:
        prog = workloads.gaussian_bernoulli_rbm(16, 24, seed=3)
        op = orc.lower_program(prog, tables=True)
    _same_tables(op, prog.tt_lower_blocks())
    assert [list(g) for g in prog.gibbs_spec.sampling_order] == op.sampling_order


def test_lattice_programs_use_the_model_paths_by_default():
    assert isinstance(orc.lower_program(workloads.IsingLattice2D(4, 4)).model, models.Ising2DModel)
    assert isinstance(orc.lower_program(workloads.potts_lattice_3d(4, 3)).model, models.Potts3DModel)
    assert isinstance(orc.lower_program(workloads.gaussian_bernoulli_rbm(8, 8)).model, models.DenseModel)


def test_rbm_and_potts_generators_reproduce_the_configuration_inputs():
    raw = models.rbm_raw(64, 96, seed=3)
    prog = workloads.gaussian_bernoulli_rbm(64, 96, seed=3)
    np.testing.assert_array_equal(raw["W"], prog.W)
    np.testing.assert_array_equal(raw["b_v"], prog.b_v)
    np.testing.assert_array_equal(raw["b_h"], prog.b_h)
    raw = models.potts_raw(6, 5, seed=4)
    prog = workloads.potts_lattice_3d(6, 5, seed=4)
    np.testing.assert_array_equal(raw["J"], prog.J)
    np.testing.assert_array_equal(raw["bias"], prog.site_bias)
    assert raw["dims"] == prog.dims


def test_dense_gaussian_draws_follow_the_paired_box_muller_layout():
    """The dense path's Philox gaussians, restated independently: counter (chain, row / 4, sweep, "DGAU"), words
    2p, 2p + 1 give rows 4j + 2p (r cos theta) and 4j + 2p + 1 (r sin theta); value = field / (1 + 1e-6) +
    sqrt(1 / (1 + 1e-6)) * normal, field = b_v + W h in double."""
    from ising_ref import philox4x32_10

    V, H, C, seed, sweep = 12, 16, 5, 0x0123_4567_89AB_CDEF, 3
    rng = np.random.default_rng(8)
    W = (0.05 * rng.standard_normal((V, H))).astype(np.float32)
    b_v = (0.2 * rng.standard_normal(V)).astype(np.float32)
    prog = models.dense_bipartite(W, b_v, np.zeros(H, np.float32))
    o = orc.OracleSampler(prog, n_chains=C, rng_layout="row4")
    h = rng.integers(0, 2, (C, H)).astype(bool)
    o.load_state([rng.standard_normal((C, V)).astype(np.float32), h])
    o.group_step(1, sweep, seed=seed)  # the visible (gaussian) block; sampling order: hidden, visible
    got = o.state[:V].astype(np.float64)  # [V][C]

    field = b_v.astype(np.float64)[:, None] + W.astype(np.float64) @ np.where(h, 1.0, -1.0).T  # [V][C]
    rows = np.arange(V)[:, None] + np.zeros((1, C), dtype=np.int64)  # the visible block starts at row 0
    chains = np.zeros((V, 1), dtype=np.int64) + np.arange(C)[None, :]
    words = np.stack(philox4x32_10(chains, rows >> 2, np.full_like(rows, sweep), np.full_like(rows, 0x44474155),
                                   seed & 0xFFFFFFFF, seed >> 32), axis=0)  # [4][V][C]
    p = (rows >> 1) & 1
    w0 = np.take_along_axis(words, (2 * p)[None], 0)[0]
    w1 = np.take_along_axis(words, (2 * p + 1)[None], 0)[0]
    uniform = lambda w: ((w >> 9) * 2 + 1).astype(np.float64) * 2.0**-24  # noqa: E731
    rad, theta = np.sqrt(-2.0 * np.log(uniform(w0))), 2.0 * np.pi * uniform(w1)
    xi = np.where(rows & 1, rad * np.sin(theta), rad * np.cos(theta))
    inv = 1.0 / (1.0 + 1e-6)
    want = field * inv + np.sqrt(inv) * xi
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)


def test_dense_spin_draws_follow_the_row4_layout():
    """The dense path's Philox spins, restated independently: word row % 4 of counter (chain, row / 4, sweep,
    "DSPI"); +1 where 2 field > logit(u), field = b_h + W^T v in double (row = V + unit for the hidden block)."""
    from ising_ref import philox4x32_10

    V, H, C, seed, sweep = 8, 20, 6, 0x00FE_DCBA_9876_5432, 5
    rng = np.random.default_rng(9)
    W = (0.3 * rng.standard_normal((V, H))).astype(np.float32)
    b_h = (0.2 * rng.standard_normal(H)).astype(np.float32)
    prog = models.dense_bipartite(W, np.zeros(V, np.float32), b_h)
    o = orc.OracleSampler(prog, n_chains=C, rng_layout="row4")
    v = rng.standard_normal((C, V)).astype(np.float32)
    o.load_state([v, rng.integers(0, 2, (C, H)).astype(bool)])
    margins = o.group_step(0, sweep, seed=seed, return_margin=True)  # the hidden (spin) block
    got = o.state[V:]  # [H][C], +-1

    field = b_h.astype(np.float64)[:, None] + W.astype(np.float64).T @ v.astype(np.float64).T  # [H][C]
    rows = V + np.arange(H)[:, None] + np.zeros((1, C), dtype=np.int64)
    chains = np.zeros((H, 1), dtype=np.int64) + np.arange(C)[None, :]
    words = np.stack(philox4x32_10(chains, rows >> 2, np.full_like(rows, sweep), np.full_like(rows, 0x44535049),
                                   seed & 0xFFFFFFFF, seed >> 32), axis=0)
    u = ((np.take_along_axis(words, (rows & 3)[None], 0)[0] >> 9) * 2 + 1).astype(np.float64) * 2.0**-24
    margin = 2.0 * field - (np.log(u) - np.log1p(-u))
    want = np.where(margin > 0, 1.0, -1.0)
    tie = np.abs(margin) < 1e-5
    assert np.all((got == want) | tie)
    np.testing.assert_allclose(np.abs(np.asarray(margins)).reshape(H, C), np.abs(margin), rtol=1e-9, atol=1e-9)


def test_sparse_spin_draws_follow_the_chain4_layout():
    """The sparse (table) path's Philox spins, restated independently: field = beta h + (sequential float32 sum of
    beta J s over the node's CSR entries); word chain % 4 of counter (chain / 4, flat row, sweep, "SPIN");
    +1 where 2 field > logit(u)."""
    from ising_ref import philox4x32_10

    raw = models.er_ising_raw(400, 6.0, seed=11)
    prog = models.graph_ising(raw["row_ptr"], raw["cols"], raw["J"], raw["h"], raw["colours"], raw["beta"])
    C, seed, sweep, chain_offset = 12, 0x0BAD_CAFE_1234_5678, 7, 8
    o = orc.OracleSampler(prog, n_chains=C, rng_layout="chain4", chain_offset=chain_offset)
    rng = np.random.default_rng(12)
    o.load_state([rng.integers(0, 2, (C, b.n_nodes)).astype(bool) for b in prog.blocks])
    before = o.state.copy()  # [flat rows][C], +-1
    margins = np.asarray(o.group_step(0, sweep, seed=seed, return_margin=True))
    after = o.state

    colours, rp, cols = np.asarray(raw["colours"]), raw["row_ptr"], raw["cols"]
    order = np.concatenate([np.flatnonzero(colours == k) for k in range(int(colours.max()) + 1)])
    flat = np.empty_like(order)
    flat[order] = np.arange(order.size)
    b32 = np.float32(raw["beta"])
    wJ = (b32 * raw["J"].astype(np.float32)).astype(np.float32)
    wh = (b32 * raw["h"].astype(np.float32)).astype(np.float32)
    members = np.flatnonzero(colours == 0)
    for c in range(C):
        gc = chain_offset + c
        for idx, node in enumerate(members):
            acc = None
            for e in range(rp[node], rp[node + 1]):
                term = np.float32(wJ[e] * np.float32(before[flat[cols[e]], c]))
                acc = term if acc is None else np.float32(acc + term)
            field = wh[node] if acc is None else np.float32(wh[node] + acc)
            row = flat[node]
            words = philox4x32_10(gc >> 2, row, sweep, 0x5350494E, seed & 0xFFFFFFFF, seed >> 32)
            u = ((int(words[gc & 3]) >> 9) * 2 + 1) * 2.0**-24
            margin = 2.0 * float(field) - (np.log(u) - np.log1p(-u))
            assert after[row, c] == (1.0 if margin > 0 else -1.0)
            assert abs(abs(margins.reshape(-1, C)[idx, c]) - abs(margin)) < 1e-9
