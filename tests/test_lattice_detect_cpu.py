"""Lattice detection in lowered thrml programs (CPU): an IsingEBM written over a periodic grid lowers to
per-term tables (tt_thrml/compiler.py:156-271) that the compiler recognises as a 2-D lattice, so it runs on
the stencil kernels; anything else is left to the table kernels."""

from __future__ import annotations

import numpy as np
import pytest

import thrml_shim as th
from tt_thrml_b200.compiler import detect_ising_lattice, ising_pattern_tables, lower_program


@pytest.mark.parametrize("H,W", [(4, 4), (8, 12), (6, 32), (16, 8)])
def test_periodic_ising_grid_is_detected(H, W):
    prog, _ = th.ising_grid_program(H, W, J=0.8, h=0.1, beta=0.5)
    st = detect_ising_lattice(lower_program(prog))
    assert st is not None
    assert st["dims"] == (H, W) and st["block_rows"] == (0, H * W // 2)
    assert st["edge_weight"] == np.float32(0.5) * np.float32(0.8)
    assert st["site_bias"] == np.float32(0.5) * np.float32(0.1)
    ising_pattern_tables(st["edge_weight"], st["site_bias"])  # a usable stencil description


@pytest.mark.parametrize("kind", ["open", "rows", "nonuniform"])
def test_other_programs_are_not_lattices(kind):
    if kind == "open":
        prog, _ = th.ising_grid_program(8, 8, periodic=False)
    elif kind == "rows":
        prog, _ = th.ising_grid_program(8, 8, colour_blocks=False)
    else:
        J = np.ones(128, np.float32)
        J[3] = 2.0  # one coupling differs
        prog, _ = th.ising_grid_program(8, 8, J=J)
    assert detect_ising_lattice(lower_program(prog)) is None


def test_small_non_lattice_cases_are_not_detected():
    assert detect_ising_lattice(lower_program(th.make_spin_case().program)) is None
    assert detect_ising_lattice(lower_program(th.make_mixed_case().program)) is None


def _sym(q, seed):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((3, q, q)).astype(np.float32)
    return ((A + A.transpose(0, 2, 1)) * np.float32(0.5)).astype(np.float32)


@pytest.mark.parametrize("dims,q", [((4, 4, 4), 8), ((6, 4, 8), 3), ((4, 6, 4), 5)])
def test_potts_grid_is_detected(dims, q):
    from tt_thrml_b200.compiler import detect_potts_lattice
    from tt_thrml_b200 import workloads

    J = _sym(q, 1)
    bias = np.random.default_rng(2).standard_normal((int(np.prod(dims)), q)).astype(np.float32)
    prog, _ = th.potts_grid_program(dims, J, bias)
    st = detect_potts_lattice(lower_program(prog))
    assert st is not None and st["dims"] == dims and st["q"] == q
    np.testing.assert_array_equal(st["J"], J)
    native = workloads.PottsLattice3D(dims, J, bias).tt_stencil()
    for c in range(2):
        np.testing.assert_array_equal(st["bias"][c], native["bias"][c])


def test_potts_grid_with_asymmetric_or_varying_couplings_is_not_detected():
    from tt_thrml_b200.compiler import detect_potts_lattice

    q = 3
    J = _sym(q, 3)
    J[1, 0, 2] += 0.5  # axis-y matrix no longer symmetric: the two directions differ
    prog, _ = th.potts_grid_program((4, 4, 4), J, np.zeros((64, q), np.float32))
    assert detect_potts_lattice(lower_program(prog)) is None
    assert detect_potts_lattice(lower_program(th.make_categorical_case().program)) is None
