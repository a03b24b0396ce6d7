"""Near-threshold settling of the dense kernel (tthrml_dense_field_sample_ties) through the C ABI.

Uploaded logits are set within a few 1e-7 of 2 * field, so every spin
decision of the launch is a near tie that the tensor cores' float32 field
can get wrong: with the tie list each one must equal the decision from the
exact (float64) field, the list must be empty again after the call, and a
list too small for the launch must count what it dropped.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from tt_thrml_b200 import _native as nat

pytestmark = pytest.mark.gpu


def _call(A, Bt, bias, out, out32, logits, *, pieces, ties=None, cap=0):
    import torch

    lib = nat.lib()
    nat.bind_device(A.device.index or 0)
    err = torch.zeros(1, dtype=torch.int32, device=A.device)
    M, K = A.shape
    N = Bt.shape[0]
    args = [A.data_ptr(), Bt.data_ptr(), M, N, K, bias.data_ptr(), nat.SPIN, ctypes.c_float(1.0), out.data_ptr(),
            None if out32 is None else out32.data_ptr(), pieces, 0, 0, logits.data_ptr(), logits.shape[0], 1, 0,
            None, err.data_ptr()]
    if ties is None:
        rc = lib.tthrml_dense_field_sample(*args, torch.cuda.current_stream().cuda_stream)
    else:
        rc = lib.tthrml_dense_field_sample_ties(*args, ties.data_ptr(), cap, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.tthrml_last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0


def _near_case(M, N, K, seed):
    """bf16 operands of RBM scale and logits float32(2 * exact field + noise of a few 1e-7)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16)
    Bt = (0.01 * torch.randn(N, K, generator=g)).to(torch.bfloat16)
    bias = (0.1 * torch.randn(N, generator=g)).float()
    field = A.double() @ Bt.double().T + bias.double()  # float64: bf16 products are exact, sums within 1e-15
    noise = 3e-7 * (2 * torch.rand(M, N, generator=g, dtype=torch.float64) - 1)
    logits = (2 * field + noise).float()  # [M][N]
    want = np.where((2 * field).numpy() > logits.double().numpy(), 1.0, -1.0)
    lt = logits.T.contiguous().reshape(1, N, M)  # [sweeps][N][M]
    return A.cuda(), Bt.cuda(), bias.cuda(), lt.cuda(), want


@pytest.mark.parametrize("M", [128, 256])  # single-CTA and CTA-pair kernels
def test_near_threshold_spins_are_settled_from_the_exact_field(cuda_device, M):
    import torch

    N, K, pieces = 512, 512, 3
    A, Bt, bias, lt, want = _near_case(M, N, K, seed=M)
    out = torch.empty(M, pieces * N, dtype=torch.bfloat16, device="cuda")
    out32 = torch.empty(M, N, dtype=torch.float32, device="cuda")
    ties = torch.zeros(4 + 2 * M * N, dtype=torch.int32, device="cuda")
    _call(A, Bt, bias, out, out32, lt, pieces=pieces, ties=ties, cap=M * N)
    got = out32.cpu().numpy()
    np.testing.assert_array_equal(got, want)
    o = out.float().cpu().numpy()
    np.testing.assert_array_equal(o[:, :N], want)
    assert not o[:, N:].any()  # remainder pieces of +-1 are zero
    assert ties[:3].tolist() == [0, 0, 0]  # list empty again, nothing dropped

    # the float32 field alone gets some of these decisions wrong
    plain = torch.empty_like(out32)
    _call(A, Bt, bias, torch.empty_like(out), plain, lt, pieces=pieces)
    assert int((plain.cpu().numpy() != want).sum()) > 0

    # a second launch on the same list settles the same way (the list was cleared)
    _call(A, Bt, bias, out, out32, lt, pieces=pieces, ties=ties, cap=M * N)
    np.testing.assert_array_equal(out32.cpu().numpy(), want)


def test_tie_list_overflow_keeps_float32_decisions_and_counts_them(cuda_device):
    import torch

    M, N, K, cap = 256, 256, 512, 1000
    A, Bt, bias, lt, want = _near_case(M, N, K, seed=9)
    plain = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    _call(A, Bt, bias, plain, None, lt, pieces=1)
    plain = plain.float().cpu().numpy()
    ties = torch.zeros(4 + 2 * cap, dtype=torch.int32, device="cuda")
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    for call in (1, 2):
        _call(A, Bt, bias, out, None, lt, pieces=1, ties=ties, cap=cap)
        assert ties[:2].tolist() == [0, 0]
        assert int(ties[2].item()) == call * (M * N - cap)
        got = out.float().cpu().numpy()
        changed = got != plain
        assert np.all(got[changed] == want[changed])  # only settled decisions differ from the float32 ones
        assert int(changed.sum()) <= cap


def test_tie_list_arguments_are_checked(cuda_device):
    import torch

    lib = nat.lib()
    A, Bt, bias, lt, _ = _near_case(128, 256, 64, seed=1)
    out = torch.empty(128, 256, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ties = torch.zeros(64, dtype=torch.int32, device="cuda")
    base = [A.data_ptr(), Bt.data_ptr(), 128, 256, 64, bias.data_ptr(), nat.SPIN, ctypes.c_float(1.0),
            out.data_ptr(), None, 1, 0, 0, lt.data_ptr(), 1, 1, 0, None, err.data_ptr()]
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.tthrml_dense_field_sample_ties(*base, None, 8, stream) != 0
    assert lib.tthrml_dense_field_sample_ties(*base, ties.data_ptr(), 0, stream) != 0
    assert lib.tthrml_dense_field_sample_ties(*base, ties.data_ptr() + 4, 8, stream) != 0
    assert lib.tthrml_dense_field_sample_ties(*base, ties.data_ptr(), 30, stream) == 0
    torch.cuda.synchronize()
