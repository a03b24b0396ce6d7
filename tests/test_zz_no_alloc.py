"""GPU test of the allocation-free group step (this file is collected last on purpose).

`tthrml_group_step_static_scratch` is for callers that cannot allocate device
memory, such as a plugin or FFI host that passes only buffers it owns, or a
running control loop that must not call cudaMalloc: it stages a superblock's
new values in the library's own device array instead of a caller buffer.  For
a float32 state (spin + categorical + gaussian superblocks) and an int8 state
(spin + categorical superblocks) the test calls it through the C ABI twice in
a row and checks each result against `tthrml_group_step` given a
caller-provided scratch buffer, and the first result against the CPU oracle.
It checks that the two calls change neither torch's allocated bytes nor the
device's free memory, that a group too large for the array is refused before
anything is launched, and that an in-place group (no staging) is not refused
whatever its size.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import gpu_harness as gh
import thrml_shim as th
from oracle import oracle as orc
from tt_thrml_b200 import Executor, make_cuda_config
from tt_thrml_b200 import _native as nat
from tt_thrml_b200.rng import seed_from_key

pytestmark = pytest.mark.gpu

C = 64
N_CALLS = 2
SEED = 77


def _descriptor(ex, plan, desc, sweep, scratch_ptr):
    g = nat.GroupDesc()
    g.blocks = desc.data_ptr()
    g.n_blocks = len(plan.block_indices)
    g.state_dtype = ex._state_code
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


def _spin_categorical_program(n_categories: int = 3):
    """Spin + categorical superblocks whose spins read their own superblock's category (int8 state)."""
    spin = [th.SpinNode() for _ in range(2)]
    cat = [th.CategoricalNode() for _ in range(2)]
    free = [(th.Block([spin[0]]), th.Block([cat[0]])), (th.Block([spin[1]]), th.Block([cat[1]]))]
    sds = {th.SpinNode: th.sd(np.bool_), th.CategoricalNode: th.sd(np.uint8)}
    return th.FactorSamplingProgram(
        th.BlockGibbsSpec(free, [], sds),
        [th.SpinGibbsConditional(), th.CategoricalGibbsConditional(n_categories)] * 2,
        [
            th.SpinEBMFactor([th.Block(spin)], [0.25, -0.2]),
            th.CategoricalEBMFactor([th.Block(cat)], [[0.2, -0.1, 0.0], [-0.15, 0.3, -0.05]]),
            th.DiscreteEBMFactor([th.Block(spin)], [th.Block(cat)], [[0.55, -0.25, 0.15], [-0.2, 0.4, 0.1]]),
        ],
        [],
    )


def _executor(kind):
    program = th.make_mixed_case().program if kind == "f32" else _spin_categorical_program()
    ex = Executor(None, 0, program, make_cuda_config(n_chains=C, cuda_graphs=False), n_sweeps=N_CALLS, n_chains=C)
    rng = np.random.default_rng(12)
    init = []
    for b in program.gibbs_spec.free_blocks:
        name = type(b.nodes[0]).__name__
        if name == "SpinNode":
            init.append(rng.integers(0, 2, (C, 1)).astype(bool))
        elif name == "CategoricalNode":
            init.append(rng.integers(0, 3, (C, 1)).astype(np.uint8))
        else:
            init.append((0.3 * rng.standard_normal((C, 1))).astype(np.float32))
    ex.load_state(init, [])
    ex.prepare_rng(SEED)
    plan = ex.compiled.sampling_groups[0].kernel_artifact
    # the group's spin block reads its categorical block: values are staged in scratch before commit
    assert plan.kind == "generic" and not plan.in_place
    assert ex._state_code == (nat.STATE_F32 if kind == "f32" else nat.STATE_I8)
    return program, ex, plan


def _check_against_oracle(program, before, after, plan):
    """The static-scratch step's first result equals the oracle's group step outside the threshold band."""
    o = orc.OracleSampler(program, n_chains=C)
    o.state[...] = before
    margin = o.group_step(0, 0, seed=seed_from_key(SEED), return_margin=True)
    off = 0
    for bi in o.prog.sampling_order[0]:
        b = o.prog.blocks[bi]
        rows = slice(b.start, b.start + b.n_nodes)
        got, want = after[rows], o.state[rows]
        m = margin[off : off + b.n_nodes]
        off += b.n_nodes
        if b.family == "gaussian":
            np.testing.assert_allclose(got, want, rtol=gh.GAUSS_RTOL, atol=gh.GAUSS_ATOL)
        else:
            assert not np.any((got != want) & (np.abs(m) >= gh.BAND))


@pytest.mark.parametrize("kind", ["f32", "i8"])
def test_static_scratch_step_matches_caller_scratch_step(cuda_device, kind):
    import torch

    program, ex, plan = _executor(kind)
    lib = nat.lib()
    nat.bind_device(cuda_device.index or 0)
    desc = plan.descriptor(None, N_CALLS)
    caller_scratch = torch.empty((plan.group_rows, C), dtype=ex.global_state.dtype, device=cuda_device)
    stream = nat.stream_handle(ex.stream)
    start = ex.global_state.clone()

    # reference results: tthrml_group_step with a caller buffer, two calls in a row
    expected = []
    for sweep in range(N_CALLS):
        ref = _descriptor(ex, plan, desc, sweep, caller_scratch.data_ptr())
        assert lib.tthrml_group_step(ctypes.byref(ref), stream) == 0, lib.tthrml_last_error()
        ex.stream.synchronize()
        expected.append(ex.global_state.clone())
    assert not torch.equal(expected[0], start)  # the step changed the state

    # the allocation-free entry point from the same start, two calls in a row, with no allocation
    ex.global_state.copy_(start)
    torch.cuda.synchronize()
    descs = [_descriptor(ex, plan, desc, sweep, None) for sweep in range(N_CALLS)]
    got = []
    for sweep in range(N_CALLS):
        torch.cuda.synchronize()
        allocated, (free_before, _) = torch.cuda.memory_allocated(), torch.cuda.mem_get_info()
        rc = lib.tthrml_group_step_static_scratch(ctypes.byref(descs[sweep]), stream)
        assert rc == 0, lib.tthrml_last_error()
        ex.stream.synchronize()
        free_after, _ = torch.cuda.mem_get_info()
        assert torch.cuda.memory_allocated() == allocated
        if sweep > 0:  # the first call on a device may load the library's module there
            assert free_after == free_before
        got.append(ex.global_state.clone())
    for g, e in zip(got, expected):
        np.testing.assert_allclose(g.cpu().double().numpy(), e.cpu().double().numpy(), rtol=gh.GAUSS_RTOL,
                                   atol=gh.GAUSS_ATOL)
    _check_against_oracle(program, start.cpu().float().numpy(), got[0].cpu().float().numpy(), plan)


def test_static_scratch_step_refuses_groups_beyond_its_array(cuda_device):
    _, ex, plan = _executor("f32")
    lib = nat.lib()
    nat.bind_device(cuda_device.index or 0)
    desc = plan.descriptor(None, N_CALLS)
    g = _descriptor(ex, plan, desc, 0, None)
    g.group_rows = (16 << 20) // (4 * C) + 1  # one row more than 16 MiB of float32 scratch holds
    rc = lib.tthrml_group_step_static_scratch(ctypes.byref(g), nat.stream_handle(ex.stream))
    assert rc == -1
    assert b"static scratch holds" in lib.tthrml_last_error()
    g.group_rows = 1 << 62  # would overflow a byte count: refused by the row test, not wrapped
    assert lib.tthrml_group_step_static_scratch(ctypes.byref(g), nat.stream_handle(ex.stream)) == -1


def test_static_scratch_step_runs_in_place_groups_of_any_size(cuda_device):
    """An in-place group stages nothing, so the array's size does not limit it."""
    import torch

    from tt_thrml_b200 import workloads
    from tt_thrml_b200.compiler import compile_program

    side, chains = 256, 1024  # a colour block is 32768 rows x 1024 chains: 32 MiB if it were staged
    prog = workloads.ising_lattice_2d(side, side, beta=0.44)
    cfg = make_cuda_config(n_chains=chains, cuda_graphs=False, stencil=False)
    compiled = compile_program(None, 0, prog, cfg, n_sweeps=1, n_chains=chains, force_generic=True)
    ex = Executor(None, 0, prog, cfg, compiled, n_sweeps=1, n_chains=chains)
    ex.load_state(gh.random_init(prog, chains, 3), [])
    ex.prepare_rng(SEED)
    plan = ex.compiled.sampling_groups[0].kernel_artifact
    assert plan.kind == "generic" and plan.in_place
    assert plan.group_rows * chains * ex.global_state.element_size() > (16 << 20)
    lib = nat.lib()
    nat.bind_device(cuda_device.index or 0)
    desc = plan.descriptor(None, 1)
    stream = nat.stream_handle(ex.stream)
    start = ex.global_state.clone()
    g = _descriptor(ex, plan, desc, 0, None)
    g.in_place = 1
    assert lib.tthrml_group_step_static_scratch(ctypes.byref(g), stream) == 0, lib.tthrml_last_error()
    ex.stream.synchronize()
    mine = ex.global_state.clone()
    assert not torch.equal(mine, start)
    ex.global_state.copy_(start)
    torch.cuda.synchronize()
    assert lib.tthrml_group_step(ctypes.byref(g), stream) == 0, lib.tthrml_last_error()
    ex.stream.synchronize()
    assert torch.equal(mine, ex.global_state)
