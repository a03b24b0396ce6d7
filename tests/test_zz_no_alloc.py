"""GPU test of the allocation-free group step (this file is collected last on purpose).

`tthrml_group_step_static_scratch` is for callers that cannot allocate device
memory, such as a plugin or FFI host that passes only buffers it owns, or a
running control loop that must not call cudaMalloc: it stages a superblock's
new values in the library's own device array instead of a caller buffer.  The
test calls it through the C ABI twice in a row and checks each result against
`tthrml_group_step` given a caller-provided scratch buffer, then checks that a
group too large for the array is refused before anything is launched.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import thrml_shim as th
from tt_thrml_b200 import Executor, make_cuda_config
from tt_thrml_b200 import _native as nat

pytestmark = pytest.mark.gpu

C = 64
N_CALLS = 2


def _descriptor(ex, plan, desc, sweep, scratch_ptr):
    g = nat.GroupDesc()
    g.blocks = desc.data_ptr()
    g.n_blocks = len(plan.block_indices)
    g.state_dtype = nat.STATE_F32
    g.group_rows = plan.group_rows
    g.n_chains = ex.n_chains
    g.chain_offset = 0
    g.state = ex.global_state.data_ptr()
    g.scratch = scratch_ptr
    g.in_place = 0
    g.use_variates = 0
    g.seed = ex._rng_buffers.seed
    g.sweep = sweep
    g.ctl = None
    return g


def _mixed_executor():
    case = th.make_mixed_case()
    ex = Executor(None, 0, case.program, make_cuda_config(n_chains=C, cuda_graphs=False), n_sweeps=N_CALLS, n_chains=C)
    rng = np.random.default_rng(12)
    init = []
    for s in case.init_state_free:
        a = np.asarray(s)
        if a.dtype == bool:
            init.append(rng.integers(0, 2, (C, 1)).astype(bool))
        elif a.dtype == np.uint8:
            init.append(rng.integers(0, 3, (C, 1)).astype(np.uint8))
        else:
            init.append((0.3 * rng.standard_normal((C, 1))).astype(np.float32))
    ex.load_state(init, [])
    ex.prepare_rng(77)
    plan = ex.compiled.sampling_groups[0].kernel_artifact
    # the group's spin block reads its categorical block: values are staged in scratch before commit
    assert plan.kind == "generic" and not plan.in_place
    return ex, plan


def test_static_scratch_step_matches_caller_scratch_step(cuda_device):
    import torch

    ex, plan = _mixed_executor()
    lib = nat.lib()
    nat.bind_device(cuda_device.index or 0)
    desc = plan.descriptor(None, N_CALLS)
    caller_scratch = torch.empty((plan.group_rows, C), dtype=torch.float32, device=cuda_device)
    stream = nat.stream_handle(ex.stream)
    for sweep in range(N_CALLS):  # two calls in a row, the second continuing from the first
        ex.stream.synchronize()
        before = ex.global_state.clone()
        ref = _descriptor(ex, plan, desc, sweep, caller_scratch.data_ptr())
        assert lib.tthrml_group_step(ctypes.byref(ref), stream) == 0, lib.tthrml_last_error()
        ex.stream.synchronize()
        expected = ex.global_state.clone()
        assert not torch.equal(expected, before)  # the step changed the state

        ex.global_state.copy_(before)
        torch.cuda.synchronize()
        mine = _descriptor(ex, plan, desc, sweep, None)
        assert lib.tthrml_group_step_static_scratch(ctypes.byref(mine), stream) == 0, lib.tthrml_last_error()
        ex.stream.synchronize()
        got = ex.global_state.clone()
        np.testing.assert_allclose(got.cpu().numpy(), expected.cpu().numpy(), rtol=1e-4, atol=1e-6)
        assert torch.equal(got, expected)


def test_static_scratch_step_refuses_groups_beyond_its_array(cuda_device):
    ex, plan = _mixed_executor()
    lib = nat.lib()
    nat.bind_device(cuda_device.index or 0)
    desc = plan.descriptor(None, N_CALLS)
    g = _descriptor(ex, plan, desc, 0, None)
    g.group_rows = (16 << 20) // (4 * C) + 1  # one row more than 16 MiB of float32 scratch holds
    rc = lib.tthrml_group_step_static_scratch(ctypes.byref(g), nat.stream_handle(ex.stream))
    assert rc == -1
    assert b"static scratch holds" in lib.tthrml_last_error()
