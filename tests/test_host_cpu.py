"""Host-side logic on CPU: lowering, planning, API contracts, library exports, PRNG restatement."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

import thrml_shim as th
import tt_thrml
import tt_thrml_b200 as tb
from oracle import oracle as orc
from tt_thrml_b200 import _native as nat
from tt_thrml_b200 import jax_prng, workloads
from tt_thrml_b200.compiler import lower_program
from tt_thrml_b200.core import Family

ROOT = Path(__file__).resolve().parents[1]


# --------------------------------------------------------------- library ABI


def _header_symbols():
    text = (ROOT / "include" / "tthrml.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tthrml_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_header_symbol():
    lib = nat.lib()
    syms = _header_symbols()
    assert "tthrml_group_step" in syms and "tthrml_spin_csr_step" in syms
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) <= set(nat.exported_symbols())
    assert lib.tthrml_abi_version() == 1


def test_struct_layouts_match_header_sizes():
    assert ctypes.sizeof(nat.Interaction) == 64
    assert ctypes.sizeof(nat.BlockDesc) == 56
    assert ctypes.sizeof(nat.GroupDesc) == 88


def test_library_rejects_bad_arguments_without_a_gpu():
    lib = nat.lib()
    rc = lib.tthrml_spin_csr_step(1, 1, 1, None, 0, 10, 16, 33, 0, None, 0, 0, 0, None, None)
    assert rc == -1
    assert b"multiple of 32" in lib.tthrml_last_error()
    g = nat.GroupDesc()
    assert lib.tthrml_group_step(ctypes.byref(g), None) == -1



_A, _M = 4096, 4100  # a 16-byte aligned and a misaligned stand-in address: rejected calls never dereference them
_BAD_CALLS = [
    ("tthrml_spin_bits_step", (_A, _A, _A, None, 0, 10, _A, 100, 0, None, 0, 0, 0, None, None), b"multiple of 256"),
    ("tthrml_spin_bits_step", (_A, _A, _A, None, 0, 10, _M, 256, 0, None, 0, 0, 0, None, None), b"16-byte aligned"),
    ("tthrml_spin_bits_step_ordered", (_A, _A, _A, None, 0, 10, _A, 256, 0, None, 0, 0, 0, None, None, None),
     b"NULL row order"),
    ("tthrml_dense_field_sample", (_A, _A, 100, 256, 64, None, 0, 1.0, _A, None, 1, 0, 0, None, 0, 0, 0, None, _A,
                                   None), b"chains must be a multiple of 128"),
    ("tthrml_dense_field_sample", (_A, _A, 128, 256, 64, None, 1, 1.0, _A, None, 1, 0, 0, None, 0, 0, 0, None, _A,
                                   None), b"family must be spin or gaussian"),
    ("tthrml_dense_field_sample", (_A, _A, 128, 256, 64, None, 0, 1.0, _A, None, 4, 0, 0, None, 0, 0, 0, None, _A,
                                   None), b"out_pieces must be 1, 2 or 3"),
    ("tthrml_dense_field_sample_ties", (_A, _A, 128, 256, 64, None, 0, 1.0, _A, None, 1, 0, 0, None, 0, 0, 0, None,
                                        _A, _M, 10, None), b"ties must be 16-byte aligned"),
    ("tthrml_dense_field_sample_ties", (_A, _A, 128, 256, 64, None, 0, 1.0, _A, None, 1, 0, 0, None, 0, 0, 0, None,
                                        _A, None, 10, None), b"NULL tie list"),
    ("tthrml_potts3d_step", (_A, 64, 5, 4, 4, 0, 0, 40, _A, _A, 8, 0, None, 0, 0, 0, None, None),
     b"positive and even"),
    ("tthrml_potts3d_step", (_A, 64, 4, 4, 4, 0, 0, 40, _A, _A, 9, 0, None, 0, 0, 0, None, None), b"q must be in [1, 8]"),
    ("tthrml_potts3d_step", (_A, 64, 4, 4, 4, 0, 0, 16, _A, _A, 8, 0, None, 0, 0, 0, None, None),
     b"disjoint row ranges"),
    ("tthrml_potts3d_step_weights", (_A, 64, 4, 4, 4, 0, 0, 40, _A, _A, 8, 0, None, 0, 0, 0, None, _M, None),
     b"16-byte aligned device array"),
    ("tthrml_potts3d_bias_weights", (_A, 64, 4, _A, None), b"q must be 8"),
    ("tthrml_ising2d_halfsweep_bits", (_A, _A, 96, 8, 1, 0, 8, 0, 8, 0, 0, _A, 0, 0, 0, None, 0, 8, None, 0, None,
                                       None), b"positive multiple of 64"),
    ("tthrml_ising2d_halfsweep_bits", (_A, _A, 128, 8, 1, 0, 10, 0, 8, 0, 0, _A, 0, 0, 0, None, 0, 8, None, 0, None,
                                       None), b"row range [0, 10) outside the 8 local rows"),
    ("tthrml_ising2d_halfsweep_bits", (_A, _A, 128, 12, 1, 0, 8, 0, 8, 0, 0, _A, 0, 0, 0, None, 0, 8, None, 0, None,
                                       None), b"rows_local == height"),
    ("tthrml_ising2d_halfsweep_bits", (_A, _A, 128, 8, 0, 0, 8, 0, 8, 0, 0, _A, 0, 0, 0, None, 0, 8, None, 0, None,
                                       None), b"halo row on both sides"),
    ("tthrml_ising2d_halfsweep_bits", (_A + 2, _A, 128, 8, 1, 0, 8, 0, 8, 0, 0, _A, 0, 0, 0, None, 0, 8, None, 0,
                                       None, None), b"4-byte aligned"),
    ("tthrml_ising2d_halfsweep_planes", (_A, _A, 96, 8, 1, 0, 8, 0, 8, 0, 0, _A, 0, 0, 0, None, 0, 8, None, 0, None,
                                         None), b"width % 64 == 0"),
    ("tthrml_ising2d_resident", (_A, 48, 8, 8, 0, 32, _A, 0, 0, 0, 4, None, 0, 0, 0, 0, 0, None, _A, None),
     b"n_chains % 32 == 0"),
    ("tthrml_ising2d_resident_planes", (_A, 64, 8, 8, 0, 32, _A, 0, 0, 0, 4, _A, 1, 5, 2, 3, 0, None, _A, None),
     b"observation schedule outside the run"),
    ("tthrml_decode_rows", (_A, 0, 64, 0, 4, 3, _A, None), b"invalid arguments"),
    ("tthrml_encode_rows", (_A, 5, 1, 4, 0, 64, 0, _A, None), b"unknown input dtype 5"),
    ("tthrml_encode_rows", (_A, 0, 1, 4, 2, 48, 0, _A, None), b"n_chains % 32 == 0"),
    ("tthrml_sum_rows", (_A, 0, 64, 0, 4, None, None), b"invalid arguments"),
    ("tthrml_moments_accumulate", (_A, 2, 64, _A, None, 0, 3, 0, _A, None), b"invalid arguments"),
    ("tthrml_halo_import", (_A, _A, 48, 2, 0, 10, _A, _A, 1, 0, None, _A, None), b"invalid arguments"),
    ("tthrml_ctl_advance", (None, 1, None), b"ctl is NULL"),
]


@pytest.mark.parametrize("name,args,message", _BAD_CALLS, ids=[f"{c[0]}-{i}" for i, c in enumerate(_BAD_CALLS)])
def test_entry_points_reject_bad_arguments_before_any_cuda_call(name, args, message):
    """Argument checks come first in every entry point: a rejected call returns TTHRML_ERR_ARG with the reason
    in tthrml_last_error() and touches neither the device nor the (stand-in) pointers, so it runs without a GPU."""
    lib = nat.lib()
    assert getattr(lib, name)(*args) == -1
    err = lib.tthrml_last_error()
    assert name.encode() in err or name.rsplit("_", 1)[0].encode() in err, err
    assert message in err, err


def test_static_scratch_step_rejects_an_empty_descriptor_without_a_gpu():
    lib = nat.lib()
    g = nat.GroupDesc()
    assert lib.tthrml_group_step_static_scratch(ctypes.byref(g), None) == -1
    assert b"invalid group descriptor" in lib.tthrml_last_error()


@pytest.mark.parametrize("call", [
    ("tthrml_spin_bits_step", (None, None, None, None, 0, 0, None, 0, 0, None, 0, 0, 0, None, None)),
    ("tthrml_decode_rows", (None, 0, 64, 0, 0, 0, None, None)),
    ("tthrml_encode_rows", (None, 0, 1, 0, 0, 64, 0, None, None)),
    ("tthrml_sum_rows", (None, 0, 64, 0, 0, None, None)),
    ("tthrml_moments_accumulate", (None, 0, 64, None, None, 1, 0, 0, None, None)),
], ids=lambda c: c[0])
def test_empty_inputs_are_no_ops_without_a_gpu(call):
    """Zero rows (or zero moments) launch nothing and succeed, whatever the pointers."""
    name, args = call
    assert getattr(nat.lib(), name)(*args) == 0

def test_greedy_colouring_is_proper():
    rp, cols = workloads.lattice_2d_csr(6, 8)
    col = workloads.greedy_colouring(rp, cols)
    for v in range(rp.shape[0] - 1):
        for e in range(rp[v], rp[v + 1]):
            assert col[v] != col[cols[e]]


# ------------------------------------------------------------------ lowering


def _ragged(it, n):
    return it.ragged(n)


@pytest.mark.parametrize(
    "make", [th.make_spin_case, th.make_categorical_case, th.make_gaussian_case, th.make_mixed_case]
)
def test_product_lowering_matches_oracle_lowering(make):
    prog = make().program
    lp = lower_program(prog)
    op = orc.lower_program(prog)
    assert [list(g) for g in lp.sampling_order] == op.sampling_order
    assert lp.total_nodes == op.total
    for spec, ob in zip(lp.specs[: lp.n_free_blocks], op.blocks):
        assert spec.family.value == ob.family
        assert spec.block_global_start == ob.start
        assert len(spec.interactions) == len(ob.interactions)
        for it, oit in zip(spec.interactions, ob.interactions):
            rp, w, src = _ragged(it, spec.n_nodes)
            np.testing.assert_array_equal(rp, oit.row_ptr)
            np.testing.assert_array_equal(w, oit.weights)
            np.testing.assert_array_equal(src, oit.sources)
            assert it.n_categorical == oit.n_categorical


def test_clamped_program_layout_puts_clamped_blocks_last():
    prog, *_ = th.make_clamp_case()
    lp = lower_program(prog)
    assert lp.block_global_starts == (0, 1, 2)
    assert lp.n_free_blocks == 2


def test_global_map_must_be_dense():
    prog = th.make_spin_case().program
    gs = prog.gibbs_spec
    node = gs.free_blocks[0].nodes[0]
    gi, off = gs.node_global_location_map[node]
    gs.node_global_location_map[node] = (gi, off + 100)
    with pytest.raises(ValueError, match="not dense"):
        lower_program(prog)


def test_unknown_interaction_raises_type_error():
    from tt_thrml_b200.compiler import _lower_interaction

    with pytest.raises(TypeError):
        _lower_interaction(object(), Family.SPIN)


# ------------------------------------------------------------------ planning


def test_plans_pick_the_spin_csr_kernel_for_ising_programs():
    pytest.importorskip("torch")
    from tt_thrml_b200.compiler import plan_program

    prog = workloads.ising_lattice_2d(8, 8)
    lp = lower_program(prog)
    dtype, plans = plan_program(lp, 64, "cpu")
    assert dtype == "int8" and all(p.kind == "spin_csr" for p in plans)
    dtype, plans = plan_program(lp, 8, "cpu")  # chains not a multiple of 32
    assert all(p.kind == "generic" for p in plans)


def test_plans_use_scratch_for_self_reading_superblocks():
    from tt_thrml_b200.compiler import plan_program

    lp = lower_program(th.two_spin_superblock_program())
    _, plans = plan_program(lp, 64, "cpu")
    assert plans[0].kind == "generic" and not plans[0].in_place
    lp = lower_program(th.make_mixed_case().program)
    dtype, plans = plan_program(lp, 4, "cpu")
    assert dtype == "float32"
    assert [p.kind for p in plans] == ["generic", "generic"]


def test_spin_csr_drops_masked_terms_exactly():
    from tt_thrml_b200.compiler import plan_program

    n = [th.SpinNode() for _ in range(4)]
    # one interaction group in which node 0 is head twice and node 2 once: node 2's second slot is padding
    group = th.InteractionGroup(
        th.DiscreteEBMInteraction(1, [0.5, -0.25, 0.75]), th.Block([n[0], n[0], n[2]]), [th.Block([n[1], n[3], n[1]])]
    )
    free = [th.Block([n[0], n[2]]), th.Block([n[1], n[3]])]
    prog = th.FactorSamplingProgram(
        th.BlockGibbsSpec(free, []), [th.SpinGibbsConditional()] * 2, [th.SpinEBMFactor([th.Block(n)], [0.1] * 4)],
        [group],
    )
    lp = lower_program(prog)
    assert lp.specs[0].interactions[1].n_terms == 2
    _, plans = plan_program(lp, 32, "cpu")
    assert [p.kind for p in plans] == ["spin_csr", "spin_csr"]
    blk = plans[0].blocks[0]
    assert blk.row_ptr.tolist() == [0, 2, 3]
    assert blk.cols.tolist() == [2, 3, 2]
    np.testing.assert_array_equal(blk.vals.numpy(), np.float32([0.5, -0.25, 0.75]))


# ------------------------------------------------------------------ API surface


class _FakeTTNN:
    class MeshShape:
        def __init__(self, *dims):
            self.dims = dims

    def __init__(self):
        self.open_device_calls, self.close_device_calls = [], []
        self.open_mesh_calls, self.close_mesh_calls = [], []

    def open_device(self, *, device_id):
        self.open_device_calls.append(device_id)
        return f"device:{device_id}"

    def close_device(self, device):
        self.close_device_calls.append(device)

    def open_mesh_device(self, **kwargs):
        self.open_mesh_calls.append(kwargs)
        return f"mesh:{kwargs['mesh_shape'].dims}"

    def close_mesh_device(self, device):
        self.close_mesh_calls.append(device)


def test_device_helpers_delegate_like_the_reference():
    """tests/test_device_open.py of the reference, through the tt_thrml alias."""
    t = _FakeTTNN()
    assert tt_thrml.open_device(t, device_id=3) == "device:3"
    tt_thrml.open_device(t)
    assert t.open_device_calls == [3, 0]
    assert tt_thrml.open_devices(t, device_ids=(0, 1, 2)) == ("device:0", "device:1", "device:2")
    with pytest.raises(ValueError):
        tt_thrml.open_devices(t, device_ids=())
    tt_thrml.open_mesh_device(t, mesh_shape=(2, 4), device_ids=range(8), num_command_queues=2)
    call = t.open_mesh_calls[-1]
    assert call["mesh_shape"].dims == (2, 4) and call["physical_device_ids"] == list(range(8))
    assert call["num_command_queues"] == 2
    tt_thrml.open_mesh_device(t, mesh_shape=(1, 4))
    assert "physical_device_ids" not in t.open_mesh_calls[-1]
    tt_thrml.close_device(t, "d")
    tt_thrml.close_mesh_device(t, "m")
    tt_thrml.close_devices(t, ["a", "b"])
    assert t.close_device_calls == ["d", "a", "b"] and t.close_mesh_calls == ["m"]


class _FakeObserver:
    def init(self):
        return "observer-init"

    def __call__(self, program, state_free, state_clamped, carry, sample_index):
        return f"{carry}:{int(sample_index)}", np.asarray(int(sample_index))


class _ExecutorShell:
    program = object()

    def load_state(self, state_free, state_clamp):
        self.loaded = (state_free, state_clamp)

    def _prepare_rng_thrml_compat(self, key, schedule, n_total):
        self.rng = (key, schedule, n_total)

    def run_warmup(self, n_warmup):
        self.warmup = n_warmup

    def _read_state_lists(self):
        return [], []


def test_sample_with_observation_uses_supplied_initial_carry():
    """tests/test_executor_api.py of the reference."""
    shell = _ExecutorShell()
    carry, obs = tb.Executor.sample_with_observation(
        shell,
        key=object(),
        schedule=th.SamplingSchedule(n_warmup=0, n_samples=1, steps_per_sample=1),
        f_observe=_FakeObserver(),
        init_state_free=[],
        state_clamp=[],
        observation_carry_init="caller-init",
    )
    assert carry == "caller-init:0"
    assert obs.tolist() == [0]
    assert shell.rng[2] == 0


def test_schedule_sweep_count_matches_reference():
    shell = _ExecutorShell()
    shell.run_sweeps = lambda n: None
    sched = th.SamplingSchedule(n_warmup=32, n_samples=64, steps_per_sample=2)
    tb.Executor.sample_with_observation(
        shell, key=0, schedule=sched, f_observe=_FakeObserver(), init_state_free=[], state_clamp=[]
    )
    assert shell.rng[2] == 32 + 63 * 2


def test_make_ttmlir_config_keeps_reference_argument_checks():
    with pytest.raises(ValueError):
        tb.make_ttmlir_config(system_desc_path="x", build_dir="b", ttmlir_opt="o", ttmlir_translate="t")
    with pytest.raises(ValueError):
        tb.make_ttmlir_config(system_desc_path="x", ttmlir_opt="o")
    cfg = tb.make_ttmlir_config(system_desc_path="x", build_dir="b")
    assert isinstance(cfg, tb.CUDAConfig) and cfg.rng_mode == "philox"
    with pytest.raises(ValueError):
        tb.make_cuda_config(rng_mode="bogus")


def test_public_surface_matches_reference():
    ref_all = {
        "TTMLIRConfig", "make_ttmlir_config", "open_device", "open_devices", "open_mesh_device", "close_device",
        "close_mesh_device", "close_devices", "Executor", "make_executor", "MeshExecutor", "make_mesh_executor",
        "sample_states", "sample_with_observation", "GaussianConditional",
    }
    assert ref_all <= set(tt_thrml.__all__)
    import tt_thrml.compiler as c
    import tt_thrml.executor as e

    assert c.compile_program is tb.compile_program and e.Executor is tb.Executor


def test_executor_requires_cuda():
    import torch

    if torch.cuda.is_available():
        pytest.skip("CUDA present")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        tb.make_executor(None, None, workloads.ising_lattice_2d(4, 4), tb.make_cuda_config())


# ------------------------------------------------------------------ PRNG restatement

# Published Threefry-2x32-20 known-answer vectors (Salmon et al., Random123 distribution).
THREEFRY_KAT = [
    ((0, 0), (0, 0), (0x6B200159, 0x99BA4EFE)),
    ((0xFFFFFFFF, 0xFFFFFFFF), (0xFFFFFFFF, 0xFFFFFFFF), (0x1CB996FC, 0xBB002BE7)),
    ((0x13198A2E, 0x03707344), (0x243F6A88, 0x85A308D3), (0xC4923A9C, 0x483DF7A0)),
]


@pytest.mark.parametrize("key,ctr,expected", THREEFRY_KAT)
def test_threefry_known_answers(key, ctr, expected):
    a, b = jax_prng.threefry2x32(key[0], key[1], ctr[0], ctr[1])
    assert (int(a), int(b)) == expected


def test_prng_restatement_shapes_and_ranges():
    k = jax_prng.key_from_seed(42)
    assert k.tolist() == [0, 42]
    ks = jax_prng.split(k, 5)
    assert ks.shape == (5, 2) and len({tuple(x) for x in ks.tolist()}) == 5
    u = jax_prng.uniform(k, (1000,))
    assert u.dtype == np.float32 and (u >= 0).all() and (u < 1).all()
    g = jax_prng.gumbel(k, (10, 3))
    assert np.isfinite(g).all()
    z = jax_prng.normal(jax_prng.split(k, 3), (4000,))
    assert z.shape == (3, 4000) and abs(float(z.mean())) < 0.1 and abs(float(z.std()) - 1) < 0.1


def test_parity_variates_follow_schedule_key_tree():
    torch = pytest.importorskip("torch")
    from tt_thrml_b200.rng import _NumpySource, generate_bulk_rng_for_schedule, make_rng_spec
    from tt_thrml_b200.core import CompiledFusedBlock

    prog = th.make_mixed_case().program
    lp = lower_program(prog)
    blocks = tuple(CompiledFusedBlock(s, None) for s in lp.specs)
    sched = th.SamplingSchedule(3, 4, 2)
    n_total = 3 + 3 * 2
    spec = make_rng_spec(blocks, n_total)
    buf = generate_bulk_rng_for_schedule(0, spec, sched, 6, "cpu", n_chains=2, source=_NumpySource())
    assert buf.spin_threshold_logits[0].shape == (n_total, 1, 1, 2)
    assert buf.categorical_gumbel[1].shape == (n_total, 1, 3, 2)
    assert buf.gaussian_noise[2].shape == (n_total, 1, 1, 2)
    assert isinstance(buf.spin_threshold_logits[0], torch.Tensor)


def test_ising_pattern_tables_are_the_exact_threshold_of_the_float32_field():
    import numpy as np

    from tt_thrml_b200.compiler import ising_pattern_tables

    w, b = np.float32(0.4407), np.float32(0.0)
    fields, thr = ising_pattern_tables(w, b)
    for idx in range(16):
        signs = [-1 if (idx >> k) & 1 else 1 for k in range(4)]
        acc = np.float32(signs[0] * w)
        for sgn in signs[1:]:
            acc = np.float32(acc + np.float32(sgn * w))
        assert fields[idx] == np.float32(b + acc)
        p = 1.0 / (1.0 + np.exp(-2.0 * float(fields[idx])))
        T = int(thr[idx])
        # m < T  <=>  u = (2m + 1) / 2^24 < p, checked at the boundary
        if T > 0:
            assert (2 * (T - 1) + 1) / 2.0**24 < p
        if T < 2**23:
            assert (2 * T + 1) / 2.0**24 >= p
    assert thr[0] > thr[15]  # all neighbours up favours up


def test_stencil_and_dense_eligibility():
    from tt_thrml_b200 import workloads
    from tt_thrml_b200.compiler import dense_eligible, stencil_eligible

    potts = workloads.potts_lattice_3d(4, 8, seed=0)
    assert stencil_eligible(potts, 64) and not stencil_eligible(potts, 6)
    lat = workloads.IsingLattice2D(8, 64)
    assert stencil_eligible(lat, 1) and not stencil_eligible(lat, 2)
    assert stencil_eligible(lat, 64) and not stencil_eligible(lat, 64, "parity")  # shared-memory resident
    assert not stencil_eligible(workloads.IsingLattice2D(8, 48), 1)  # width not a multiple of 32
    rbm = workloads.gaussian_bernoulli_rbm(256, 512, seed=0)
    assert dense_eligible(rbm, 128) and not dense_eligible(rbm, 64)
    assert not dense_eligible(workloads.gaussian_bernoulli_rbm(128, 512, seed=0), 128)  # 128 units
    assert not stencil_eligible(rbm, 128) and not dense_eligible(potts, 128)


def test_dense_structure_is_detected_in_plain_tables():
    """An RBM handed over as plain per-term tables (as a thrml-factor program lowers) is recognised."""
    import numpy as np

    from tt_thrml_b200 import workloads
    from tt_thrml_b200.compiler import detect_dense_couplings, lower_program
    from tt_thrml_b200.workloads import TableProgram

    rbm = workloads.gaussian_bernoulli_rbm(256, 512, seed=1, w_std=0.05)
    plain = TableProgram(rbm.gibbs_spec, rbm.tt_lower_blocks(), {})
    lowered = lower_program(plain)
    got = detect_dense_couplings(lowered, 128)
    assert got is not None
    np.testing.assert_array_equal(got[0]["weights_nk"], rbm.W)
    np.testing.assert_array_equal(got[1]["weights_nk"], rbm.W.T)
    np.testing.assert_array_equal(got[0]["bias"], rbm.b_v)
    assert got[0]["family"] == tb.core.Family.GAUSSIAN and got[0]["precision"] == 1.0
    assert detect_dense_couplings(lowered, 64) is None  # chains not a multiple of 128
    # weights that bf16 cannot hold: only with rounding allowed
    W = rbm.W.copy()
    W[0, 0] = np.float32(0.1234567)
    rough = workloads.DenseBipartiteProgram(W, rbm.b_v, rbm.b_h)
    lowered2 = lower_program(TableProgram(rough.gibbs_spec, rough.tt_lower_blocks(), {}))
    assert detect_dense_couplings(lowered2, 128) is None
    assert detect_dense_couplings(lowered2, 128, round_weights=True) is not None
    # a sparse program is not dense
    assert detect_dense_couplings(lower_program(workloads.erdos_renyi_ising(512, 4.0, seed=0)), 128) is None


def test_merge_rows_concatenates_terms_row_by_row():
    from tt_thrml_b200.compiler import _merge_rows

    a = (np.array([0, 2, 2, 3], np.int64), np.array([1.0, 2.0, 3.0], np.float32), np.array([10, 11, 12], np.int32))
    b = (np.array([0, 1, 3, 3], np.int64), np.array([4.0, 5.0, 6.0], np.float32), np.array([20, 21, 22], np.int32))
    rp, vals, cols = _merge_rows([a, b], 3)
    assert rp.tolist() == [0, 3, 5, 6]
    assert vals.tolist() == [1.0, 2.0, 4.0, 5.0, 6.0, 3.0]
    assert cols.tolist() == [10, 11, 20, 21, 22, 12]


def _device_categorical_rule(theta, q, qmax, u, ref):
    """float32 restatement of the kernels' inverse-CDF draw (csrc/common.cuh): weights relative to `ref`
    (the maximum of theta), categories reversed for u >= 1/2 over qmax slots (zeros past q), one running
    sum, one compare per boundary, mirrored count; None if the sum overflows."""
    f32 = np.float32
    c = f32(1.44269502162933349609375)
    ml = f32(f32(ref) * c)
    with np.errstate(over="ignore"):  # ex2 of a large argument is +inf, as on the device
        # fma(theta, c, -ml): one rounding of the exact product minus ml
        e = [f32(np.exp2(np.float64(f32(np.float64(theta[k]) * np.float64(c) - np.float64(ml)))))
             if k < q else f32(0.0) for k in range(qmax)]
    low = u < 0.5
    order = e if low else e[::-1]
    s, h = f32(0.0), []
    for j, x in enumerate(order):
        s = x if j == 0 else f32(s + x)
        h.append(s)
    if not s <= f32(3.0e38):
        return None
    t = f32(f32(u if low else f32(1.0) - f32(u)) * s)
    cnt = sum(1 for j in range(qmax - 1) if h[j] <= t)
    return cnt if low else qmax - 1 - cnt


def test_categorical_draw_rule_matches_exact_decision():
    """The kernels' categorical rule (weights relative to max theta) agrees with the exact decision
    (double precision inverse CDF) wherever the draw is more than 1e-5 from a boundary in logit
    units, for q <= qmax, both halves of u and wide fields."""
    rng = np.random.default_rng(12)
    checked = 0
    for trial in range(4000):
        q = int(rng.integers(1, 9))
        qmax = 8 if trial % 2 else q
        scale = 3.0 if trial % 5 else 60.0
        theta = (rng.standard_normal(q) * scale).astype(np.float32)
        theta[0] = theta[0] if trial % 7 else np.float32(-80.0)  # one category far below the others
        u = float((2 * int(rng.integers(0, 2**23)) + 1) * 2.0**-24)
        got = _device_categorical_rule(theta, q, qmax, u, theta.max())
        ex = np.exp(theta.astype(np.float64) - theta.max())
        head = np.cumsum(ex)
        tail = np.cumsum(ex[::-1])[::-1]
        want = int(np.sum(head[:-1] <= u * head[-1]))
        lu = np.log(u) - np.log1p(-u)
        margin = min((abs(lu - (np.log(head[k]) - np.log(tail[k + 1]))) for k in range(q - 1)), default=np.inf)
        if margin > 1e-5:
            assert got == want, (trial, q, qmax, theta, u, got, want)
            checked += 1
    assert checked > 3900


def test_lattice_layout_selection():
    """Uniform lattices take the bit-sliced kernels ("planes" from width % 64 == 0, bit-packed strips from
    width % 256 == 0); a table that is not count-symmetric keeps the per-site kernels."""
    from tt_thrml_b200 import workloads
    from tt_thrml_b200.compiler import ising_count_symmetric, ising_pattern_tables, ising_stencil_layout
    from tt_thrml_b200.domain import LatticeStrips

    _, thr = ising_pattern_tables(np.float32(0.4407), np.float32(0.0))
    assert ising_count_symmetric(thr)
    assert ising_stencil_layout(thr, 64) == "planes" and ising_stencil_layout(thr, 96) == "row8s"
    skew = thr.copy()
    skew[1] += 1  # left neighbour at -1 no longer equals right neighbour at -1
    assert not ising_count_symmetric(skew) and ising_stencil_layout(skew, 64) == "row8s"
    none = lambda *a: None  # noqa: E731
    for W, storage in ((64, "int8"), (256, "int8")):  # a host half-sweep keeps int8 rows by default
        st = LatticeStrips(workloads.IsingLattice2D(8, W, beta=0.4407), device="cpu", halo=2, halfsweep=none)
        assert st.storage == storage and st.row_bytes == W // 2
    st = LatticeStrips(workloads.IsingLattice2D(8, 256, beta=0.4407), device="cpu", halo=2, halfsweep=none,
                       storage="bits")
    assert st.row_bytes == 256 // 16 and tuple(st.colours[0].shape) == (8 + 4, 256 // 64)
