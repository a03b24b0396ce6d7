"""tcgen05 dense block kernel (tthrml_dense_field_sample) through the C ABI.

The field is checked against a plain PyTorch float32 (float64 here) matmul of
the same bf16 operands; spin decisions against the threshold rule on that
field (ties within the accumulation-order rounding are allowed); Philox-mode
spin frequencies against sigmoid(2 * bias).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from tt_thrml_b200 import _native as nat

pytestmark = pytest.mark.gpu


def _call(A, Bt, bias, family, precision, out, out32, *, pieces=1, row0=0, variates=None, seed=1, sweep=0, chain_offset=0):
    import torch

    lib = nat.lib()
    nat.bind_device(A.device.index or 0)
    err = torch.zeros(1, dtype=torch.int32, device=A.device)
    M, K = A.shape
    N = Bt.shape[0]
    rc = lib.tthrml_dense_field_sample(
        A.data_ptr(), Bt.data_ptr(), M, N, K, None if bias is None else bias.data_ptr(), family, ctypes.c_float(precision),
        out.data_ptr(), None if out32 is None else out32.data_ptr(), pieces, row0, chain_offset,
        None if variates is None else variates.data_ptr(), 0 if variates is None else variates.shape[0],
        seed, sweep, None, err.data_ptr(), torch.cuda.current_stream().cuda_stream,
    )
    assert rc == 0, lib.tthrml_last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0, f"in-kernel wait expired (code {int(err.item())})"


def _operands(M, N, K, seed=0, scale=0.05):
    import torch

    g = torch.Generator().manual_seed(seed)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16)
    Bt = (scale * torch.randn(N, K, generator=g)).to(torch.bfloat16)
    bias = 0.1 * torch.randn(N, generator=g)
    return A.cuda(), Bt.cuda(), bias.float().cuda()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 384), (384, 768, 1024)])
def test_dense_gaussian_field_matches_fp64_matmul(cuda_device, M, N, K):
    import torch

    A, Bt, bias = _operands(M, N, K)
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    out32 = torch.empty(M, N, dtype=torch.float32, device="cuda")
    zeros = torch.zeros(1, N, M, dtype=torch.float32, device="cuda")  # xi = 0: the draw is the conditional mean
    _call(A, Bt, bias, nat.GAUSSIAN, 1.0, out, out32, variates=zeros)
    inv = np.float32(1.0) / (np.float32(1.0) + np.float32(1e-6))
    ref = (A.double().cpu() @ Bt.double().cpu().T + bias.double().cpu()).numpy() * float(inv)
    scale = (A.double().abs().cpu() @ Bt.double().abs().cpu().T).numpy() + 1.0
    np.testing.assert_array_less(np.abs(out32.cpu().numpy() - ref) / scale, 2e-6)
    np.testing.assert_array_equal(out.float().cpu().numpy(), out32.to(torch.bfloat16).float().cpu().numpy())


def test_dense_spin_decisions_follow_the_threshold(cuda_device):
    import torch

    M, N, K = 256, 512, 512
    A, Bt, bias = _operands(M, N, K, seed=3)
    g = torch.Generator().manual_seed(5)
    logits = torch.logit(torch.rand(1, N, M, generator=g).clamp(1e-6, 1 - 1e-6)).float().cuda()
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    _call(A, Bt, bias, nat.SPIN, 1.0, out, None, variates=logits)
    field = (A.double().cpu() @ Bt.double().cpu().T + bias.double().cpu()).numpy()
    lt = logits[0].T.cpu().numpy().astype(np.float64)  # [M][N]
    margin = 2 * field - lt
    got = out.float().cpu().numpy()
    want = np.where(margin > 0, 1.0, -1.0)
    tie = np.abs(margin) < 1e-4
    assert set(np.unique(got)) <= {-1.0, 1.0}
    assert int(((got != want) & ~tie).sum()) == 0
    assert tie.mean() < 1e-3


def test_dense_philox_spin_frequency_matches_sigmoid(cuda_device):
    import torch

    M, N, K = 2048, 256, 64
    A = torch.zeros(M, K, dtype=torch.bfloat16, device="cuda")  # field = bias
    Bt = torch.zeros(N, K, dtype=torch.bfloat16, device="cuda")
    bias = torch.linspace(-1.5, 1.5, N, device="cuda")
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    _call(A, Bt, bias, nat.SPIN, 1.0, out, None, seed=11, sweep=3)
    freq = (out.float() > 0).float().mean(0).cpu().numpy()
    p = 1.0 / (1.0 + np.exp(-2.0 * bias.cpu().numpy()))
    assert np.max(np.abs(freq - p)) < 5.0 * np.sqrt(0.25 / M)
    out2 = torch.empty_like(out)
    _call(A, Bt, bias, nat.SPIN, 1.0, out2, None, seed=11, sweep=3)
    assert torch.equal(out, out2)  # counter-based: same (seed, sweep) gives the same draw
