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
