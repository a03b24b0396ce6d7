"""Dense bipartite (RBM) programs on the tensor-core path against the oracle.

dense_precision "fp32" (gaussian blocks held as three bf16 pieces, the weights
repeated along K) meets the float32 criteria: spins bit-exact outside the
1e-5 threshold band, gaussians within 1e-4 relative.  dense_precision "bf16"
(gaussian blocks stored as bf16, the throughput configuration) meets them for
spins against an oracle that stores its gaussian block as bf16 as well, and
stays within bf16 rounding (one bf16 unit in the last place: 2^-7 relative at most) for gaussians.
"""

from __future__ import annotations

import numpy as np
import pytest

import gpu_harness as gh
from tt_thrml_b200 import Executor, make_cuda_config, workloads
from tt_thrml_b200.compiler import compile_program

pytestmark = pytest.mark.gpu

# a value the GPU and the oracle round to neighbouring bf16 numbers differs by one unit in the last place:
# 2^-7 relative just above a power of two
BF16_ULP = 2.0**-7

V, H, C = 256, 512, 128


def _rbm(seed=0):
    return workloads.gaussian_bernoulli_rbm(V, H, seed=seed, w_std=0.05)


def _init(seed=1, n_chains=C):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal((n_chains, V)).astype(np.float32), rng.integers(0, 2, (n_chains, H)).astype(bool)]


def _assert_parity(rep: gh.ParityReport, gauss_rtol=gh.GAUSS_RTOL):
    assert rep.hard_mismatches == 0, rep
    assert rep.band_fraction < 1e-4, rep
    assert rep.gauss_max_rel <= gauss_rtol, rep


@pytest.mark.parametrize("mode", ["variates", "philox"])
def test_rbm_fp32_dense_matches_oracle(cuda_device, mode):
    prog = _rbm()
    rep, ex, _ = gh.run_parity(prog, C, 4, mode=mode, init=_init(), dense_precision="fp32")
    plans = [g.kernel_artifact for g in ex.compiled.sampling_groups]
    assert [p.kind for p in plans] == ["dense", "dense"]
    assert plans[0].source_pieces == 3 and plans[1].out_pieces == 3  # hidden reads, visible writes 3 pieces
    _assert_parity(rep)


@pytest.mark.parametrize("mode", ["variates", "philox"])
def test_rbm_bf16_dense_matches_oracle_within_bf16(cuda_device, mode):
    prog = _rbm(seed=2)
    rtol = BF16_ULP
    rep, ex, o = gh.run_parity(prog, C, 4, mode=mode, init=_init(3), dense_precision="bf16", gauss_rtol=rtol)
    assert all(g.kernel_artifact.source_pieces == 1 for g in ex.compiled.sampling_groups)
    assert o.gaussian_storage == "bf16"  # the oracle stores its gaussian block as bf16 too
    _assert_parity(rep, gauss_rtol=rtol)


def test_rbm_generic_path_matches_oracle(cuda_device):
    prog = _rbm(seed=4)
    rep, ex, _ = gh.run_parity(prog, 32, 3, mode="variates", init=_init(5, 32))
    assert ex.compiled.state_dtype != "dense_bf16"  # 32 chains: not a multiple of 128
    _assert_parity(rep)


def test_dense_parity_mode_defaults_to_fp32(cuda_device):
    prog = _rbm()
    par = compile_program(None, 0, prog, make_cuda_config(rng_mode="parity", n_chains=C), n_chains=C)
    phi = compile_program(None, 0, prog, make_cuda_config(rng_mode="philox", n_chains=C), n_chains=C)
    assert par.sampling_groups[0].kernel_artifact.source_pieces == 3
    assert phi.sampling_groups[0].kernel_artifact.source_pieces == 1


def test_rbm_graph_replay_equals_eager(cuda_device):
    prog = _rbm(seed=6)
    states = []
    for graphs in (False, True):
        cfg = make_cuda_config(n_chains=C, cuda_graphs=graphs)
        ex = Executor(None, 0, prog, cfg, n_sweeps=24, n_chains=C)
        ex.load_state(_init(7), [])
        ex.prepare_rng(123)
        ex.run_sweeps(8)
        ex.run_sweeps(8)  # second replay continues the counter stream
        ex.check_device_errors()
        states.append(ex.raw_state())
    np.testing.assert_array_equal(states[0], states[1])


def test_rbm_sample_states_api(cuda_device):
    import thrml_shim as th

    prog = _rbm(seed=8)
    cfg = make_cuda_config(n_chains=C)
    ex = Executor(None, 0, prog, cfg, n_sweeps=16, n_chains=C)
    vis, hid = prog.gibbs_spec.blocks
    sched = th.SamplingSchedule(n_warmup=2, n_samples=3, steps_per_sample=2)
    out = ex.sample_states(5, sched, [vis, hid], init_state_free=_init(9))
    assert out[0].shape == (3, C, V) and out[0].dtype == np.float32
    assert out[1].shape == (3, C, H) and out[1].dtype == bool
    assert np.isfinite(out[0]).all()


def test_rbm_hidden_conditional_frequencies(cuda_device):
    """With the visible block clamped by the initial state (hidden-only sweeps),
    hidden spins follow sigmoid(2 * (W^T v + b_h)) for every chain."""
    prog = _rbm(seed=10)
    n_chains = 1024
    cfg = make_cuda_config(n_chains=n_chains)
    compiled = compile_program(None, 0, prog, cfg, n_sweeps=64, n_chains=n_chains)
    ex = Executor(None, 0, prog, cfg, compiled, n_sweeps=64, n_chains=n_chains)
    v0 = np.random.default_rng(11).standard_normal(V).astype(np.float32)
    ex.load_state([np.broadcast_to(v0, (n_chains, V)).copy(), np.zeros((n_chains, H), bool)], [])
    ex.prepare_rng(77)
    hidden_group = ex.compiled.sampling_groups[0]
    assert hidden_group.block_indices == (1,)
    freq = np.zeros(H)
    n_rep = 8
    for s in range(n_rep):
        ex._run_sampling_group(hidden_group, s)
        freq += ex.observe([prog.gibbs_spec.blocks[1]])[prog.gibbs_spec.blocks[1]].mean(0)
    freq /= n_rep
    vb = v0.astype(np.float32)
    import torch

    vb = torch.from_numpy(vb).to(torch.bfloat16).double().numpy()  # bf16 state operand
    field = vb @ prog.W.astype(np.float64) + prog.b_h
    p = 1.0 / (1.0 + np.exp(-2.0 * field))
    n = n_rep * n_chains
    assert np.max(np.abs(freq - p)) < 5.0 * np.sqrt(0.25 / n)


def test_dense_pieces_reconstruct_float32(cuda_device):
    import ctypes

    import torch

    from tt_thrml_b200 import _native as nat

    M, N, K = 128, 256, 128
    g = torch.Generator().manual_seed(12)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    Bt = (0.05 * torch.randn(N, K, generator=g)).to(torch.bfloat16).cuda()
    bias = (0.3 * torch.randn(N, generator=g)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for pieces in (2, 3):
        out = torch.empty(M, pieces * N, dtype=torch.bfloat16, device="cuda")
        out32 = torch.empty(M, N, dtype=torch.float32, device="cuda")
        nat.bind_device(0)
        rc = nat.lib().tthrml_dense_field_sample(
            A.data_ptr(), Bt.data_ptr(), M, N, K, bias.data_ptr(), nat.GAUSSIAN, ctypes.c_float(1.0),
            out.data_ptr(), out32.data_ptr(), pieces, 0, 0, None, 0, 5, 1, None, err.data_ptr(),
            torch.cuda.current_stream().cuda_stream,
        )
        assert rc == 0, nat.lib().tthrml_last_error()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        parts = out.double().reshape(M, pieces, N)
        recon = parts.sum(1)
        if pieces == 3:
            assert torch.equal(recon, out32.double())
        else:
            rel = ((recon - out32.double()).abs() / out32.double().abs().clamp_min(1e-30)).max().item()
            assert rel <= 2.0**-16
        # the first piece is the bf16 rounding of the value
        assert torch.equal(out[:, :N], out32.to(torch.bfloat16))



@pytest.mark.parametrize("mode", ["variates", "philox"])
def test_plain_table_rbm_runs_on_the_tensor_cores(cuda_device, mode):
    """The same RBM handed over only as per-term tables (what a thrml-factor program lowers to):
    the compiler detects the dense structure, and the tensor-core run matches the oracle."""
    from tt_thrml_b200.workloads import TableProgram

    rbm = _rbm(seed=12)
    plain = TableProgram(rbm.gibbs_spec, rbm.tt_lower_blocks(), {})
    rep, ex, _ = gh.run_parity(plain, C, 3, mode=mode, init=_init(13), dense_precision="fp32")
    assert [g.kernel_artifact.kind for g in ex.compiled.sampling_groups] == ["dense", "dense"]
    _assert_parity(rep)
