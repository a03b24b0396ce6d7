"""Program signatures of the plan cache (CPU): the counterpart of the reference's kernel signature keys
(tt_thrml/compiler.py:398-433).  Equal contents give equal signatures, any change of a weight, a gather
index, a size or the block order gives a new one, and a program object is lowered once however often it
is compiled."""

from __future__ import annotations

import threading

import numpy as np

import thrml_shim as th
from tt_thrml_b200 import compiler, workloads


def test_equal_contents_give_equal_signatures():
    a = workloads.erdos_renyi_ising(600, 5.0, seed=1)
    b = workloads.erdos_renyi_ising(600, 5.0, seed=1)
    c = workloads.erdos_renyi_ising(600, 5.0, seed=2)
    sa, sb, sc = (compiler.program_signature(p)[0] for p in (a, b, c))
    assert sa == sb and sa != sc
    assert compiler.program_signature(th.make_spin_case().program)[0] == \
        compiler.program_signature(th.make_spin_case().program)[0]
    assert compiler.program_signature(th.make_spin_case().program)[0] != \
        compiler.program_signature(th.make_categorical_case().program)[0]


def test_any_content_change_changes_the_signature():
    base = workloads.IsingLattice2D(8, 8, J=1.0, beta=0.5)
    sigs = {compiler.program_signature(p)[0] for p in (
        base, workloads.IsingLattice2D(8, 8, J=1.0, beta=0.6), workloads.IsingLattice2D(8, 10, J=1.0, beta=0.5),
        workloads.IsingLattice2D(8, 8, J=1.0, h=0.1, beta=0.5))}
    assert len(sigs) == 4
    rbm = workloads.gaussian_bernoulli_rbm(16, 24, seed=0)
    rbm2 = workloads.gaussian_bernoulli_rbm(16, 24, seed=0)
    rbm2.W[3, 4] = workloads.bf16_representable(np.array([rbm2.W[3, 4] + 0.5], np.float32))[0]
    assert compiler.program_signature(rbm)[0] != compiler.program_signature(rbm2)[0]
    p1 = workloads.potts_lattice_3d(4, 3, seed=0)
    p2 = workloads.potts_lattice_3d(4, 3, seed=0)
    assert compiler.program_signature(p1)[0] == compiler.program_signature(p2)[0]
    p2.site_bias[0, 0] += 1.0
    assert compiler.program_signature(p1)[0] != compiler.program_signature(p2)[0]


def test_a_program_object_is_lowered_once(monkeypatch):
    compiler.clear_plan_cache()
    calls = []
    real = compiler.lower_program

    def counting(program):
        calls.append(program)
        return real(program)

    monkeypatch.setattr(compiler, "lower_program", counting)
    prog = th.make_mixed_case().program
    s1, low1 = compiler._signature_of(prog)
    s2, low2 = compiler._signature_of(prog)
    assert s1 == s2 and low1 is low2 and len(calls) == 1
    other = th.make_mixed_case().program  # equal contents, another object: lowered for its signature
    assert compiler._signature_of(other)[0] == s1 and len(calls) == 2


def test_signatures_are_thread_safe():
    compiler.clear_plan_cache()
    progs = [th.make_spin_case().program for _ in range(4)]
    out = [None] * 16

    def work(i):
        out[i] = compiler._signature_of(progs[i % 4])[0]

    threads = [threading.Thread(target=work, args=(i,)) for i in range(16)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert len(set(out)) == 1
