"""The CTA-pair tensor-core kernel (tcgen05 cta_group::2), used for chain counts that are multiples of 256.

Checked against the oracle like the single-CTA kernel (spins bit-exact outside the 1e-5 band; gaussians
within 1e-5 + 1e-4 relative in fp32 mode, one bf16 ulp in bf16 mode), at a small size and at the full
4096 x 8192 size; and chain-sharded runs of 128 chains (single-CTA kernel) against one run of 256 chains
(pair kernel) must give the same chains.
"""

from __future__ import annotations

import numpy as np
import pytest

import gpu_harness as gh
from tt_thrml_b200 import Executor, make_cuda_config, workloads

pytestmark = pytest.mark.gpu

BF16_ULP = 2.0**-7


def _init(V, H, C, seed):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal((C, V)).astype(np.float32), rng.integers(0, 2, (C, H)).astype(bool)]


def _assert_parity(rep, gauss_rtol=gh.GAUSS_RTOL):
    assert rep.hard_mismatches == 0, rep
    assert rep.band_fraction < 1e-4, rep
    assert rep.gauss_max_rel <= gauss_rtol, rep


@pytest.mark.parametrize("mode,precision", [("philox", "fp32"), ("variates", "fp32"), ("philox", "bf16")])
def test_pair_kernel_small_rbm_matches_oracle(cuda_device, mode, precision):
    V, H, C = 256, 512, 256
    prog = workloads.gaussian_bernoulli_rbm(V, H, seed=1, w_std=0.05)
    rtol = BF16_ULP if precision == "bf16" else gh.GAUSS_RTOL
    rep, ex, _ = gh.run_parity(prog, C, 3, mode=mode, init=_init(V, H, C, 2), dense_precision=precision,
                               gauss_rtol=rtol)
    assert [g.kernel_artifact.kind for g in ex.compiled.sampling_groups] == ["dense", "dense"]
    ex.check_device_errors()
    _assert_parity(rep, rtol)


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_pair_kernel_full_size_rbm_matches_oracle(cuda_device, precision):
    V, H, C = 4096, 8192, 256
    prog = workloads.gaussian_bernoulli_rbm(V, H, seed=0)
    rtol = BF16_ULP if precision == "bf16" else gh.GAUSS_RTOL
    rep, ex, _ = gh.run_parity(prog, C, 1, mode="philox", init=_init(V, H, C, 3), dense_precision=precision,
                               gauss_rtol=rtol)
    ex.check_device_errors()
    _assert_parity(rep, rtol)


def test_pair_kernel_equals_single_cta_kernel_on_chain_shards(cuda_device):
    V, H = 512, 1024
    prog = workloads.gaussian_bernoulli_rbm(V, H, seed=5, w_std=0.03)
    init = _init(V, H, 256, 6)
    whole = Executor(None, 0, prog, make_cuda_config(n_chains=256), n_sweeps=6, n_chains=256)
    whole.load_state(init, [])
    whole.prepare_rng(7)
    whole.run_sweeps(4)
    whole.check_device_errors()
    parts = []
    for off in (0, 128):
        ex = Executor(None, 0, prog, make_cuda_config(n_chains=128), n_sweeps=6, n_chains=128, chain_offset=off)
        ex.load_state([s[off : off + 128] for s in init], [])
        ex.prepare_rng(7)
        ex.run_sweeps(4)
        ex.check_device_errors()
        parts.append(ex.raw_state())
    np.testing.assert_array_equal(whole.raw_state(), np.concatenate(parts, axis=1))
