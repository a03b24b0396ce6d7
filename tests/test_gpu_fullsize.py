"""Parity at the benchmark configurations' full sizes, group by group, against the oracle.

The oracle builds each model from its raw parameters (oracle/models.py:
lattice dimensions with J, h and beta; q x q matrices with site biases; the
weight matrix with unit biases) and runs its stencil and dense paths, so it
shares no table with the product.  Criteria: spins and categories bit-exact
outside the 1e-5 threshold band with the band below 1e-4 of the sites;
gaussians within 1e-4 relative (fp32 mode) or one bf16 unit in the last place (2^-7 relative; bf16 mode,
the oracle storing its gaussian block as bf16 too).

* 64 x 64 Ising lattice, 1024 chains, on the shared-memory resident kernel;
* 4096 x 8192 Gauss-Bernoulli RBM on the tensor-core kernel (128 chains), fp32
  and bf16 modes;
* 128^3 q = 8 Potts lattice, 64 chains, on the Potts stencil kernel;
* a 256 x 32768 single-chain Ising lattice on the bit-packed strip kernel
  (the 32768-wide rows of the 32768^2 configuration), half-sweep by half-sweep.
"""

from __future__ import annotations

import numpy as np
import pytest

import gpu_harness as gh
from oracle import oracle as orc
from tt_thrml_b200 import workloads
from tt_thrml_b200.rng import seed_from_key

pytestmark = pytest.mark.gpu

# a value the GPU and the oracle round to neighbouring bf16 numbers differs by one unit in the last place:
# 2^-7 relative just above a power of two
BF16_ULP = 2.0**-7


def _assert_parity(rep, gauss_rtol=gh.GAUSS_RTOL):
    assert rep.hard_mismatches == 0, rep
    assert rep.band_fraction < 1e-4, rep
    assert rep.gauss_max_rel <= gauss_rtol, rep


def test_lattice_64x64_1024_chains_resident_kernel(cuda_device):
    prog = workloads.ising_lattice_2d(64, 64, J=1.0, h=0.0, beta=0.44)
    C = 1024
    rep, ex, o = gh.run_parity(prog, C, 3, mode="philox", seed=0)
    assert [g.kernel_artifact.kind for g in ex.compiled.sampling_groups] == ["ising2d_resident"] * 2
    assert {g.kernel_artifact.rng_layout for g in ex.compiled.sampling_groups} == {"planes8"}
    assert o.prog.model is not None  # the oracle's stencil path, built from (H, W, J, h, beta)
    assert rep.sites == 3 * 4096 * C
    _assert_parity(rep)


def _rbm_init(C, seed):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal((C, 4096)).astype(np.float32), rng.integers(0, 2, (C, 8192)).astype(bool)]


@pytest.mark.parametrize("mode", ["philox", "variates"])
def test_rbm_4096x8192_fp32_mode(cuda_device, mode):
    prog = workloads.gaussian_bernoulli_rbm(4096, 8192, seed=0)
    C = 128
    rep, ex, o = gh.run_parity(prog, C, 2 if mode == "philox" else 1, mode=mode, init=_rbm_init(C, 1),
                               dense_precision="fp32")
    assert [g.kernel_artifact.kind for g in ex.compiled.sampling_groups] == ["dense", "dense"]
    assert o.gaussian_storage == "f32" and o.prog.model is not None
    _assert_parity(rep)


def test_rbm_4096x8192_bf16_mode(cuda_device):
    """The throughput mode: gaussian visible units stored as bf16 operands, in the GPU and in the oracle."""
    prog = workloads.gaussian_bernoulli_rbm(4096, 8192, seed=0)
    C = 128
    rep, ex, o = gh.run_parity(prog, C, 2, mode="philox", init=_rbm_init(C, 2), dense_precision="bf16",
                               gauss_rtol=BF16_ULP)
    assert all(g.kernel_artifact.source_pieces == 1 for g in ex.compiled.sampling_groups)
    assert o.gaussian_storage == "bf16"
    _assert_parity(rep, gauss_rtol=BF16_ULP)


def test_potts_128cube_q8_64_chains(cuda_device):
    prog = workloads.potts_lattice_3d(128, 8, seed=0)
    C = 64
    rng = np.random.default_rng(3)
    init = [rng.integers(0, 8, (C, prog.n_sites // 2)).astype(np.int8) for _ in range(2)]
    rep, ex, o = gh.run_parity(prog, C, 1, mode="philox", init=init, seed=5)
    assert [g.kernel_artifact.kind for g in ex.compiled.sampling_groups] == ["potts3d", "potts3d"]
    assert o.prog.model is not None
    assert rep.sites == 128**3 * C
    _assert_parity(rep)


def _split(lattice, c):
    H, W = lattice.shape
    rows = np.arange(H)
    cols = (np.arange(W // 2)[None, :] * 2) + ((rows[:, None] + c) & 1)
    return np.take_along_axis(lattice, cols, axis=1).reshape(-1)


def test_bit_packed_strip_32768_wide(cuda_device):
    """k_ising2d_bits on 256 rows of 32768 sites: each half-sweep against the oracle's stencil path."""
    from tt_thrml_b200.domain import LatticeStrips

    H, W, n_sweeps, key = 256, 32768, 3, 21
    prog = workloads.IsingLattice2D(H, W, beta=0.4407)
    st = LatticeStrips(prog, device=cuda_device, halo=2)
    assert st.storage == "bits" and st.rng_layout == "planes"
    st.load_random(4)
    st.prepare_rng(key, n_sweeps)
    o = orc.OracleSampler(prog, n_chains=1, rng_layout="planes")
    assert o.prog.model is not None
    half = H * W // 2
    rep = gh.ParityReport()
    lat = st.gather_lattice()
    for sweep in range(n_sweeps):
        st.run_sweeps(1)
        st.check_errors()
        new = st.gather_lattice()
        o.state[:half, 0] = _split(lat, 0)
        o.state[half:, 0] = _split(lat, 1)
        for c in range(2):
            m = o.group_step(c, sweep, seed=seed_from_key(key), return_margin=True)[:, 0]
            got = _split(new, c).astype(np.float32)
            want = o.state[c * half : (c + 1) * half, 0]
            tie = np.abs(m) < gh.BAND
            rep.sites += half
            rep.band += int(tie.sum())
            rep.hard_mismatches += int(((got != want) & ~tie).sum())
            o.state[c * half : (c + 1) * half, 0] = got  # the next colour reads the GPU's result (ties included)
        lat = new
    tr = st.trace()
    assert tr.shape == (n_sweeps, 2) and tr[-1, 0] == int(lat.astype(np.int64).sum())
    st.close()
    _assert_parity(rep)
