"""Executor with device-resident state: one CUDA kernel per sampling group per sweep.

Mirrors tt_thrml/executor.py: the same methods, guards, error messages and
schedule semantics (load_state, prepare_rng, run_sweep, run_warmup, observe,
sample_states, sample_with_observation, timing_summary, state_is_loaded,
make_executor; executor.py:66-450).  What changes underneath:

* the state is one torch CUDA tensor per executor, chain innermost, that
  never leaves the GPU mid-sweep: bit-packed uint32 words [total_nodes,
  n_chains/32] for all-spin programs with a multiple of 256 chains, int8
  [total_nodes, n_chains] for other spin / categorical programs, float32 for
  programs with gaussian blocks;
* each group runs through libtthrml_b200 (`tthrml_spin_bits_step`,
  `tthrml_spin_csr_step` or `tthrml_group_step`) on the executor's stream;
  there is no host dispatch layer, no per-call tensor wrapping and no CPU
  fallback;
* Philox-mode variates are drawn inside the kernels; parity-mode variates are
  uploaded once per run like the reference's bulk buffers;
* `run_sweeps(n)` replays the sweep loop from a captured CUDA graph.
"""

from __future__ import annotations

import ctypes
import time
from typing import Any, Sequence

import numpy as np

from . import _native as nat
from .compiler import compile_program, resolve_torch_device
from .core import BulkRNGBuffers, CompiledProgram, CUDAConfig, Family
from .observers import StateObserver, tree_expand, tree_stack
from .rng import (
    block_variates,
    generate_bulk_rng,
    generate_bulk_rng_for_schedule,
    make_rng_spec,
    philox_buffers,
)

_OUT_KIND = {Family.SPIN: 0, Family.CATEGORICAL: 1, Family.GAUSSIAN: 2}


def _torch():
    import torch

    return torch


class Executor:
    def __init__(
        self,
        ttnn,
        device,
        program,
        config: CUDAConfig,
        compiled: CompiledProgram | None = None,
        *,
        n_sweeps: int = 100,
        profile: bool = False,
        n_chains: int | None = None,
        chain_offset: int = 0,
    ):
        torch = _torch()
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA is not available: the B200 executor has no CPU fallback")
        self.ttnn = ttnn
        self.device = device
        self.program = program
        self.config = config
        self.n_sweeps = n_sweeps
        self.profile = profile
        if compiled is not None and n_chains is None:
            n_chains = compiled.n_chains
        self.n_chains = int(n_chains if n_chains is not None else config.n_chains)
        if chain_offset % 4:
            raise ValueError("chain_offset must be a multiple of 4")
        self.chain_offset = int(chain_offset)
        self.compiled = (
            compiled
            if compiled is not None
            else compile_program(ttnn, device, program, config, n_sweeps=n_sweeps, n_chains=self.n_chains)
        )
        if self.compiled.n_chains != self.n_chains:
            raise ValueError(f"compiled for {self.compiled.n_chains} chains, executor has {self.n_chains}")
        self._tdev = self.compiled.device or resolve_torch_device(device)
        self._lib = nat.lib()
        # a stream of its own (CUDA graphs cannot be captured on the default stream)
        stream = getattr(device, "stream", None)
        self._stream = stream if stream is not None else torch.cuda.Stream(device=self._tdev)
        self._state_code = {"int8": nat.STATE_I8, "bits": nat.STATE_BITS}.get(self.compiled.state_dtype, nat.STATE_F32)
        self._torch_state_dtype = {nat.STATE_I8: torch.int8, nat.STATE_BITS: torch.int32}.get(
            self._state_code, torch.float32
        )
        # elements per state row: chains, or 32-chain words when bit-packed
        self._row_len = self.n_chains // 32 if self._state_code == nat.STATE_BITS else self.n_chains
        # dense (tensor-core) programs keep one bf16 [n_chains, n_units] tensor per block
        self._dense = self.compiled.state_dtype == "dense_bf16"
        self._block_states: list | None = None
        self._error_word = None
        self._ties = None

        self._global_state = None
        self._state_loaded = False
        self._rng_buffers: BulkRNGBuffers | None = None
        self._sweep_counter = 0
        self._rng_n_sweeps = 0
        self._timing_log: list[tuple[str, float, float]] = []
        self._scratch: dict[int, Any] = {}
        self._graphs: dict[int, Any] = {}
        self._ctl = None  # device tthrml_run_ctl read by graph-captured kernels
        self._ctl_value = None

    # ------------------------------------------------------------------ state

    @property
    def state_is_loaded(self) -> bool:
        return self._state_loaded

    @property
    def stream(self):
        return self._stream

    @property
    def global_state(self):
        """The device state tensor [total_nodes, n_chains] (chain innermost)."""
        return self._global_state

    def _ensure_state(self):
        torch = _torch()
        if self._dense:
            if self._block_states is None:
                pieces = {plan.block_indices[0]: plan.out_pieces for plan in self._plans()}
                self._dense_pieces = [pieces.get(bi, 1) for bi in range(len(self.compiled.blocks))]
                self._block_states = [
                    torch.empty((self.n_chains, p * cb.spec.n_nodes), dtype=torch.bfloat16, device=self._tdev)
                    for p, cb in zip(self._dense_pieces, self.compiled.blocks)
                ]
                # float32 copies of the blocks held in several pieces (the readable state)
                self._block_f32 = [
                    torch.empty((self.n_chains, cb.spec.n_nodes), dtype=torch.float32, device=self._tdev)
                    if p > 1
                    else None
                    for p, cb in zip(self._dense_pieces, self.compiled.blocks)
                ]
                self._error_word = torch.zeros(1, dtype=torch.int32, device=self._tdev)
                # near-threshold spin decisions of one dense launch, settled from the exact field
                # (4 header words, then (chain, unit) pairs; a few in 10^5 decisions are near)
                sizes = [self.n_chains * plan.n_units for plan in self._plans()
                         if plan.kind == "dense" and plan.family == Family.SPIN]
                self._ties_cap = min(2**31 - 1, max([min(n, max(4096, n // 256)) for n in sizes], default=1))
                self._ties = torch.zeros(4 + 2 * self._ties_cap, dtype=torch.int32, device=self._tdev)
            return self._block_states
        if self._global_state is None:
            self._global_state = torch.empty(
                (self.compiled.total_nodes, self._row_len), dtype=self._torch_state_dtype, device=self._tdev
            )
            if any(plan.kind == "ising2d_resident" for plan in self._plans()):
                # set by the resident lattice kernel if its half-sweep barrier wait expired
                self._error_word = torch.zeros(1, dtype=torch.int32, device=self._tdev)
            for plan in self._plans():
                if plan.kind == "potts3d" and plan.q == 8 and plan.bias_w is None:
                    # e^(b - max b) per site, once: the q = 8 sweep kernel reads it instead of recomputing
                    with torch.cuda.stream(self._stream):
                        plan.bias_w = torch.empty_like(plan.bias)
                    nat.bind_device(self._tdev.index)
                    nat.check(
                        self._lib.tthrml_potts3d_bias_weights(
                            plan.bias.data_ptr(), plan.bias.shape[0], plan.q, plan.bias_w.data_ptr(),
                            nat.stream_handle(self._stream),
                        ),
                        "tthrml_potts3d_bias_weights",
                    )
        return self._global_state

    def _plans(self):
        return [g.kernel_artifact for g in self.compiled.sampling_groups]

    def _dense_write_block(self, block_index: int, values) -> None:
        """Stores float32 values [C or 1, n] into a dense block (bf16 pieces + float32 copy)."""
        torch = _torch()
        n = self.compiled.blocks[block_index].spec.n_nodes
        rem = values.to(torch.float32).expand(self.n_chains, n)
        if self._block_f32[block_index] is not None:
            self._block_f32[block_index].copy_(rem)
        dst = self._block_states[block_index]
        for p in range(self._dense_pieces[block_index]):
            piece = rem.to(torch.bfloat16)
            dst[:, p * n : (p + 1) * n].copy_(piece)
            rem = rem - piece.float()

    def _dense_block_values(self, block_index: int):
        """A dense block's float32 values [C, n] (device)."""
        f32 = self._block_f32[block_index]
        if f32 is not None:
            return f32
        return self._block_states[block_index].float()

    def _block_source(self, block_index: int, state):
        """One block's states as a contiguous device tensor [C or 1, n] of int8 or float32.

        Host data (numpy arrays, or torch CPU tensors, ideally pinned) is
        copied to the device as is; the spin sign mapping and the transpose to
        the chain-innermost layout happen in tthrml_encode_rows.
        """
        torch = _torch()
        spec = self.compiled.blocks[block_index].spec
        n, C = spec.n_nodes, self.n_chains
        t = state if isinstance(state, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(np.asarray(state)))
        if t.numel() not in (n, C * n):
            raise ValueError(
                f"block {block_index}: expected state of shape ({n},) or ({C}, {n}), got {tuple(t.shape)}"
            )
        t = t.reshape(-1, n)
        if t.dtype in (torch.bool, torch.uint8):
            t = t.view(torch.int8) if t.dtype == torch.uint8 else t.view(torch.uint8).view(torch.int8)
        elif t.dtype != torch.int8:
            if spec.family == Family.GAUSSIAN or self._state_code == nat.STATE_F32 or t.is_floating_point():
                t = t.to(torch.float32)
            else:
                t = t.to(torch.int8)
        t = t.contiguous().to(self._tdev, non_blocking=True)
        return t

    def load_state(self, state_free, state_clamp) -> None:
        """Encode the block states and upload them into the device state (tt_thrml/executor.py:104-127)."""
        torch = _torch()
        n_free = self.compiled.n_free_blocks
        states = list(state_free) + list(state_clamp)
        if len(state_free) > n_free or len(states) != len(self.compiled.blocks):
            raise ValueError(f"Expected {len(self.compiled.blocks)} block states, got {len(states)}")
        self._ensure_state()
        nat.bind_device(self._tdev.index)
        if self._dense:
            with torch.cuda.stream(self._stream):
                for bi, st in enumerate(states):
                    spec = self.compiled.blocks[bi].spec
                    src = self._block_source(bi, st)
                    if spec.family == Family.SPIN:
                        src = torch.where(src > 0, 1.0, -1.0)
                    self._dense_write_block(bi, src)
            self._state_loaded = True
            return
        with torch.cuda.stream(self._stream):
            for bi, st in enumerate(states):
                spec = self.compiled.blocks[bi].spec
                src = self._block_source(bi, st)
                if src.shape[0] == 1 and self.n_chains > 1:  # one state for every chain
                    src = src.expand(self.n_chains, spec.n_nodes).contiguous()
                in_code = nat.STATE_I8 if src.dtype == torch.int8 else nat.STATE_F32
                nat.check(
                    self._lib.tthrml_encode_rows(
                        src.data_ptr(),
                        in_code,
                        1 if spec.family == Family.SPIN else 0,
                        spec.n_nodes,
                        self._state_code,
                        self.n_chains,
                        spec.block_global_start,
                        self._global_state.data_ptr(),
                        nat.stream_handle(self._stream),
                    ),
                    "tthrml_encode_rows",
                )
                src.record_stream(self._stream)
        self._state_loaded = True

    # -------------------------------------------------------------------- rng

    def _install_rng(self, buffers: BulkRNGBuffers, n_sweeps: int) -> None:
        # Philox-mode graphs read seed and sweep from the device run control and
        # stay valid; parity-mode graphs hold variate pointers and are rebuilt.
        if buffers.seed is None or (self._rng_buffers is not None and self._rng_buffers.seed is None):
            self._graphs.clear()
        self._rng_buffers = buffers
        self._sweep_counter = 0
        self._rng_n_sweeps = n_sweeps

    def prepare_rng(self, key) -> None:
        """Prepare variates for `n_sweeps` sweeps (tt_thrml/executor.py:138-148)."""
        n = self.compiled.rng_spec.n_sweeps
        if self.config.rng_mode == "philox":
            self._install_rng(philox_buffers(key, n), n)
        else:
            buffers = generate_bulk_rng(key, self.compiled.rng_spec, self._tdev, n_chains=self.n_chains)
            self._install_rng(buffers, n)

    def _prepare_rng_for_n_sweeps(self, key, n_sweeps: int) -> None:
        if self.config.rng_mode == "philox":
            self._install_rng(philox_buffers(key, n_sweeps), n_sweeps)
            return
        spec = make_rng_spec(self.compiled.blocks[: self.compiled.n_free_blocks], n_sweeps)
        self._install_rng(generate_bulk_rng(key, spec, self._tdev, n_chains=self.n_chains), n_sweeps)

    def _prepare_rng_thrml_compat(self, key, schedule, n_total: int) -> None:
        if self.config.rng_mode == "philox":
            self._install_rng(philox_buffers(key, n_total), n_total)
            return
        spec = make_rng_spec(self.compiled.blocks[: self.compiled.n_free_blocks], n_total)
        buffers = generate_bulk_rng_for_schedule(
            key, spec, schedule, self.compiled.n_free_blocks, self._tdev, n_chains=self.n_chains
        )
        self._install_rng(buffers, n_total)

    # ------------------------------------------------------------------ sweeps

    def _check_ready(self, n: int = 1) -> None:
        if not self._state_loaded:
            raise RuntimeError("State must be loaded before running sweep")
        if self._rng_buffers is None:
            raise RuntimeError("RNG must be prepared before running sweep")
        if self._sweep_counter + n > self._rng_n_sweeps:
            raise RuntimeError("RNG buffer exhausted - call prepare_rng again")

    def run_sweep(self) -> None:
        """One sweep: every sampling group in order (tt_thrml/executor.py:150-163)."""
        self._check_ready()
        sweep_idx = self._sweep_counter
        for group in self.compiled.sampling_groups:
            self._run_sampling_group(group, sweep_idx)
        self._sweep_counter += 1

    def run_warmup(self, n_warmup: int) -> None:
        self.run_sweeps(n_warmup)

    def _resident_plans(self):
        """The resident lattice plans when the whole program is one (colour 0 sampled first), else None."""
        plans = [g.kernel_artifact for g in self.compiled.sampling_groups]
        if plans and all(p.kind == "ising2d_resident" for p in plans) and [p.colour for p in plans] == [0, 1]:
            return plans
        return None

    def _run_resident(self, n_sweeps: int, obs=None, obs_first=0, obs_every=0, n_obs=0, obs_colours=0) -> None:
        """n sweeps (and scheduled magnetisation samples) of a resident lattice in one launch."""
        plan = self._resident_plans()[0]
        H, W = plan.dims
        nat.bind_device(self._tdev.index)
        fn = "tthrml_ising2d_resident_planes" if plan.rng_layout == "planes8" else "tthrml_ising2d_resident"
        nat.check(
            getattr(self._lib, fn)(
                self._global_state.data_ptr(), self.n_chains, H, W, plan.block_rows[0], plan.block_rows[1],
                plan.thresholds.data_ptr(), self._rng_buffers.seed, self._sweep_counter, 0, 2 * n_sweeps,
                None if obs is None else obs.data_ptr(), obs_first, obs_every, n_obs, obs_colours,
                self.chain_offset, None, self._error_word.data_ptr(), nat.stream_handle(self._stream),
            ),
            fn,
        )
        self._sweep_counter += n_sweeps

    def run_sweeps(self, n: int) -> None:
        """n sweeps; replayed from a CUDA graph when config.cuda_graphs is set (one launch for a
        shared-memory-resident lattice)."""
        if n <= 0:
            return
        self._check_ready(n)
        if self._resident_plans() is not None and self._rng_buffers.seed is not None and not self.profile:
            self._run_resident(n)
            return
        if not self.config.cuda_graphs or self.profile or n < 2:
            for _ in range(n):
                self.run_sweep()
            return
        self._run_sweeps_graph(n)

    def _run_sweeps_graph(self, n: int) -> None:
        """Replays a captured graph of n sweeps.

        Captured kernels read the sweep index as `k + ctl.sweep` (k = 0..n-1
        baked into the graph) and the Philox seed from `ctl.seed`; the graph's
        last node adds n to ctl.sweep.  One graph per n therefore serves every
        position of every run; the host only rewrites ctl when it drifts.
        """
        torch = _torch()
        self._ensure_ctl()
        g = self._graphs.get(n)
        if g is None:
            self._prepare_launch_state()
            nat.bind_device(self._tdev.index)
            g = torch.cuda.CUDAGraph()
            self._stream.synchronize()
            with torch.cuda.graph(g, stream=self._stream):
                for k in range(n):
                    for group in self.compiled.sampling_groups:
                        self._run_sampling_group(group, k, capturing=True)
                nat.check(
                    self._lib.tthrml_ctl_advance(
                        self._ctl.data_ptr(), n, nat.stream_handle(torch.cuda.current_stream(self._tdev))
                    ),
                    "tthrml_ctl_advance",
                )
            self._graphs[n] = g
        self._replay_with_ctl(g, n)

    def _resident_observation(self, f_observe, schedule) -> int:
        """Colour mask for the fused resident schedule when it applies (magnetisation of lattice blocks)."""
        from .observers import MagnetizationObserver

        if (type(f_observe) is not MagnetizationObserver or self._resident_plans() is None or self.profile
                or self._rng_buffers is None or self._rng_buffers.seed is None or schedule.n_warmup < 1
                or schedule.n_samples < 1 or schedule.steps_per_sample < 1):
            return 0
        lookup = {id(b): i for i, b in enumerate(self.program.gibbs_spec.blocks)}
        mask = 0
        for b in f_observe.blocks:
            bi = lookup.get(id(b)) if not isinstance(b, int) else b
            if bi not in (0, 1):
                return 0
            mask |= 1 << bi
        return mask

    def _ensure_ctl(self) -> None:
        torch = _torch()
        if self._ctl is None:
            self._ctl = torch.zeros(2, dtype=torch.int64, device=self._tdev)  # tthrml_run_ctl
            self._ctl_host = torch.zeros(2, dtype=torch.int64, pin_memory=True)
            self._ctl_value = None

    def _replay_with_ctl(self, g, n: int) -> None:
        """Sets the device run control to (sweep counter, seed) if it drifted, replays g, advances n sweeps."""
        torch = _torch()
        seed = self._rng_buffers.seed if self._rng_buffers.seed is not None else 0
        want = (self._sweep_counter, seed)
        with torch.cuda.stream(self._stream):
            if self._ctl_value != want:
                self._stream.synchronize()  # the pinned staging word may still be in flight
                lo = seed & 0xFFFFFFFFFFFFFFFF
                self._ctl_host[0] = self._sweep_counter
                self._ctl_host[1] = lo - (1 << 64) if lo >= (1 << 63) else lo
                self._ctl.copy_(self._ctl_host, non_blocking=True)
            g.replay()
        self._sweep_counter += n
        self._ctl_value = (self._sweep_counter, seed)

    def _run_schedule_graph(self, schedule, f_observe, carry):
        """Warm-up, every sample's sweeps and every observation as one CUDA graph (captured once per
        schedule and observer); returns the device tensor of observations [n_samples, ...]."""
        torch = _torch()
        n_w, n_s, steps = int(schedule.n_warmup), int(schedule.n_samples), int(schedule.steps_per_sample)
        n_total = n_w + max(0, n_s - 1) * steps
        self._check_ready(n_total)
        self._ensure_ctl()
        key = ("schedule", n_w, n_s, steps, id(f_observe))
        entry = self._graphs.get(key)
        if entry is None or entry[2] is not carry:
            self._prepare_launch_state()
            obs = f_observe.capture_buffer(self, n_s)
            nat.bind_device(self._tdev.index)
            g = torch.cuda.CUDAGraph()
            self._stream.synchronize()
            with torch.cuda.graph(g, stream=self._stream):
                s = torch.cuda.current_stream(self._tdev)
                k = 0
                for _ in range(n_w):
                    for group in self.compiled.sampling_groups:
                        self._run_sampling_group(group, k, capturing=True)
                    k += 1
                f_observe.observe_capture(self, carry, obs, 0, s)
                for i in range(1, n_s):
                    for _ in range(steps):
                        for group in self.compiled.sampling_groups:
                            self._run_sampling_group(group, k, capturing=True)
                        k += 1
                    f_observe.observe_capture(self, carry, obs, i, s)
                nat.check(self._lib.tthrml_ctl_advance(self._ctl.data_ptr(), n_total, nat.stream_handle(s)),
                          "tthrml_ctl_advance")
            entry = (g, obs, carry)
            self._graphs[key] = entry
        g, obs, _ = entry
        self._replay_with_ctl(g, n_total)
        return obs

    def _prepare_launch_state(self) -> None:
        """Uploads descriptors and allocates scratch ahead of a graph capture."""
        rng = self._rng_buffers
        for group in self.compiled.sampling_groups:
            plan = group.kernel_artifact
            if plan.kind != "generic":
                continue
            variates = None if rng.seed is not None else {bi: self._variates(bi) for bi in plan.block_indices}
            plan.descriptor(variates, self._rng_n_sweeps)
            if not plan.in_place:
                self._scratch_for(id(plan), plan.group_rows)
        self._stream.synchronize()

    def _scratch_for(self, gi: int, rows: int):
        torch = _torch()
        buf = self._scratch.get(gi)
        if buf is None:
            buf = torch.empty((max(1, rows), self.n_chains), dtype=self._torch_state_dtype, device=self._tdev)
            self._scratch[gi] = buf
        return buf

    def _variates(self, block_index: int):
        spec = self.compiled.blocks[block_index].spec
        return block_variates(self._rng_buffers, block_index, spec.family)

    def _run_sampling_group(self, group, sweep_idx: int, capturing: bool = False) -> None:
        rng = self._rng_buffers
        if rng is None:
            raise RuntimeError("RNG must be prepared before running sweep")
        plan = group.kernel_artifact
        torch = _torch()
        stream = nat.stream_handle(torch.cuda.current_stream(self._tdev) if capturing else self._stream)
        seed = rng.seed if rng.seed is not None else 0
        ctl = self._ctl.data_ptr() if capturing else None
        nat.bind_device(self._tdev.index)
        t0 = time.perf_counter()
        if self.profile:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record(self._stream)
        if plan.kind == "dense":
            bi = plan.block_indices[0]
            v = self._variates(bi)
            nat.check(
                self._lib.tthrml_dense_field_sample_ties(
                    self._block_states[plan.source].data_ptr(),
                    plan.weights_nk.data_ptr(),
                    self.n_chains,
                    plan.n_units,
                    plan.n_sources,
                    plan.bias.data_ptr(),
                    nat.SPIN if plan.family == Family.SPIN else nat.GAUSSIAN,
                    ctypes.c_float(plan.precision),
                    self._block_states[bi].data_ptr(),
                    None if self._block_f32[bi] is None else self._block_f32[bi].data_ptr(),
                    plan.out_pieces,
                    plan.row0,
                    self.chain_offset,
                    None if v is None else v.data_ptr(),
                    self._rng_n_sweeps if v is not None else 0,
                    seed,
                    sweep_idx,
                    ctl,
                    self._error_word.data_ptr(),
                    self._ties.data_ptr(),
                    self._ties_cap,
                    stream,
                ),
                "tthrml_dense_field_sample_ties",
            )
        elif plan.kind == "ising2d":
            bi = plan.block_indices[0]
            v = self._variates(bi)
            H, W = plan.dims
            base = self._global_state.data_ptr()  # one chain: flat row r is byte r
            if v is None and plan.rng_layout == "planes":
                nat.check(
                    self._lib.tthrml_ising2d_halfsweep_planes(
                        base + plan.target_row0, base + plan.source_row0, W, H, 1, 0, H, 0, H, plan.colour,
                        plan.target_row0, plan.thresholds.data_ptr(), self.chain_offset, seed, sweep_idx, ctl, 0, 0,
                        None, 0, None, stream,
                    ),
                    "tthrml_ising2d_halfsweep_planes",
                )
            else:
                nat.check(
                    self._lib.tthrml_ising2d_halfsweep(
                        base + plan.target_row0, base + plan.source_row0, W, H, 1, 0, H, 0, H, plan.colour,
                        plan.target_row0, plan.thresholds.data_ptr(), plan.fields.data_ptr(),
                        None if v is None else v.data_ptr(), self._rng_n_sweeps if v is not None else 0,
                        self.chain_offset, seed, sweep_idx, ctl, 0, 0, None, 0, stream,
                    ),
                    "tthrml_ising2d_halfsweep",
                )
        elif plan.kind == "ising2d_resident":
            H, W = plan.dims
            fn = "tthrml_ising2d_resident_planes" if plan.rng_layout == "planes8" else "tthrml_ising2d_resident"
            nat.check(
                getattr(self._lib, fn)(
                    self._global_state.data_ptr(), self.n_chains, H, W, plan.block_rows[0], plan.block_rows[1],
                    plan.thresholds.data_ptr(), seed, sweep_idx, plan.colour, 1, None, 0, 0, 0, 0, self.chain_offset,
                    ctl, self._error_word.data_ptr(), stream,
                ),
                fn,
            )
        elif plan.kind == "potts3d":
            bi = plan.block_indices[0]
            v = self._variates(bi)
            X, Y, Z = plan.dims
            args = [
                self._global_state.data_ptr(), self.n_chains, X, Y, Z, plan.colour, plan.target_row0,
                plan.source_row0, plan.J.data_ptr(), plan.bias.data_ptr(), plan.q, self.chain_offset,
                None if v is None else v.data_ptr(), self._rng_n_sweeps if v is not None else 0, seed, sweep_idx,
                ctl,
            ]
            if plan.bias_w is not None:
                nat.check(self._lib.tthrml_potts3d_step_weights(*args, plan.bias_w.data_ptr(), stream),
                          "tthrml_potts3d_step_weights")
            else:
                nat.check(self._lib.tthrml_potts3d_step(*args, stream), "tthrml_potts3d_step")
        elif plan.kind in ("spin_csr", "spin_bits"):
            bits = plan.kind == "spin_bits"
            for blk in plan.blocks:
                v = self._variates(blk.block_index)
                vptr = None if v is None else v.data_ptr()
                args = [
                    blk.row_ptr.data_ptr(),
                    blk.cols.data_ptr(),
                    blk.vals.data_ptr(),
                    None if blk.bias is None else blk.bias.data_ptr(),
                    blk.row_start,
                    blk.n_rows,
                    self._global_state.data_ptr(),
                    self.n_chains,
                    self.chain_offset,
                    vptr,
                    self._rng_n_sweeps if v is not None else 0,
                    seed,
                    sweep_idx,
                    ctl,
                ]
                if bits and blk.row_order is not None:
                    step, args = self._lib.tthrml_spin_bits_step_ordered, args + [blk.row_order.data_ptr()]
                else:
                    step = self._lib.tthrml_spin_bits_step if bits else self._lib.tthrml_spin_csr_step
                nat.check(
                    step(
                        *args,
                        stream,
                    ),
                    plan.kind,
                )
        else:
            variates = None
            if rng.seed is None:
                variates = {bi: self._variates(bi) for bi in plan.block_indices}
                missing = [bi for bi, v in variates.items() if v is None]
                if missing:
                    raise RuntimeError(f"RNG buffers hold no variates for blocks {missing}")
            desc = plan.descriptor(variates, self._rng_n_sweeps)
            gi = id(plan)
            g = nat.GroupDesc()
            g.blocks = desc.data_ptr()
            g.n_blocks = len(plan.block_indices)
            g.state_dtype = self._state_code
            g.group_rows = plan.group_rows
            g.n_chains = self.n_chains
            g.chain_offset = self.chain_offset
            g.state = self._global_state.data_ptr()
            g.scratch = None if plan.in_place else self._scratch_for(gi, plan.group_rows).data_ptr()
            g.in_place = 1 if plan.in_place else 0
            g.use_variates = 0 if rng.seed is not None else 1
            g.seed = seed
            g.sweep = sweep_idx
            g.ctl = ctl
            nat.check(self._lib.tthrml_group_step(ctypes.byref(g), stream), "tthrml_group_step")
        if self.profile:
            t1 = time.perf_counter()
            ev1.record(self._stream)
            ev1.synchronize()
            self._timing_log.append((plan.family_label, (t1 - t0) * 1000.0, ev0.elapsed_time(ev1)))

    # ------------------------------------------------------------- read-back

    # ------------------------------------------------------------ checkpoint

    CHECKPOINT_FORMAT = "tt_thrml_b200.checkpoint/1"

    def _device_buffers(self) -> list:
        if self._dense:
            return list(self._block_states) + [b for b in self._block_f32 if b is not None]
        return [self._global_state]

    def checkpoint(self) -> dict:
        """What a later run needs to continue these chains bit for bit: the raw device state (in its own
        layout), the sweep counter and the Philox seed.  Parity-mode variates are not stored: restore()
        rebuilds them from the same key."""
        torch = _torch()
        if not self._state_loaded:
            raise RuntimeError("State must be loaded before a checkpoint")
        self._stream.synchronize()
        rng = self._rng_buffers
        return {
            "format": self.CHECKPOINT_FORMAT,
            "state_dtype": self.compiled.state_dtype,
            "n_chains": self.n_chains,
            "chain_offset": self.chain_offset,
            "total_nodes": self.compiled.total_nodes,
            "buffers": [(b.view(torch.int16) if b.dtype == torch.bfloat16 else b).cpu().numpy()
                        for b in self._device_buffers()],
            "sweep": int(self._sweep_counter),
            "seed": None if rng is None or rng.seed is None else int(rng.seed),
            "rng_sweeps": int(self._rng_n_sweeps),
            "rng_mode": self.config.rng_mode,
        }

    def restore(self, ckpt: dict, key=None) -> None:
        """Continues from checkpoint(): state, sweep counter and RNG position (parity mode: pass the key)."""
        torch = _torch()
        if ckpt.get("format") != self.CHECKPOINT_FORMAT:
            raise ValueError(f"not a {self.CHECKPOINT_FORMAT} checkpoint")
        mine = (self.compiled.state_dtype, self.n_chains, self.chain_offset, self.compiled.total_nodes)
        theirs = (ckpt["state_dtype"], int(ckpt["n_chains"]), int(ckpt["chain_offset"]), int(ckpt["total_nodes"]))
        if mine != theirs:
            raise ValueError(f"checkpoint of a different executor: {theirs} (state layout, chains, chain offset, "
                             f"nodes), this one is {mine}")
        self._ensure_state()
        bufs = self._device_buffers()
        if len(bufs) != len(ckpt["buffers"]):
            raise ValueError("checkpoint buffers do not match this program")
        for dst, src in zip(bufs, ckpt["buffers"]):
            src = np.asarray(src)
            if tuple(src.shape) != tuple(dst.shape):
                raise ValueError(f"checkpoint buffer of shape {src.shape}, expected {tuple(dst.shape)}")
            dst.copy_(torch.from_numpy(np.ascontiguousarray(src)).view(dst.dtype).reshape(dst.shape))
        torch.cuda.synchronize(self._tdev)
        self._state_loaded = True
        if ckpt["seed"] is not None:
            n = int(ckpt["rng_sweeps"])
            self._install_rng(BulkRNGBuffers(None, None, None, seed=int(ckpt["seed"]), n_sweeps=n), n)
        else:
            if key is None:
                raise ValueError("a parity-mode checkpoint needs the RNG key to rebuild its variates")
            self.prepare_rng(key)
        self._sweep_counter = int(ckpt["sweep"])

    def save_checkpoint(self, path) -> None:
        ck = self.checkpoint()
        meta = {k: v for k, v in ck.items() if k != "buffers"}
        arrays = {f"buffer{i}": b for i, b in enumerate(ck["buffers"])}
        np.savez(path, meta=np.array(repr(meta)), **arrays)

    def load_checkpoint(self, path, key=None) -> None:
        import ast

        with np.load(path, allow_pickle=False) as f:
            meta = ast.literal_eval(str(f["meta"]))
            meta["buffers"] = [f[f"buffer{i}"] for i in range(sum(1 for k in f.files if k.startswith("buffer")))]
        self.restore(meta, key=key)

    def near_ties_dropped(self) -> int:
        """Near-threshold dense spin decisions that did not fit the tie list (they kept their float32 decision)."""
        if self._ties is None:
            return 0
        self._stream.synchronize()
        return int(self._ties[2].item())

    def check_device_errors(self) -> None:
        """Raises if a kernel recorded an expired in-kernel wait (dense and resident lattice programs)."""
        if self._error_word is not None:
            self._stream.synchronize()
            self._raise_error_code(int(self._error_word.item()))

    @staticmethod
    def _raise_error_code(code: int) -> None:
        if code:
            raise RuntimeError(f"a device kernel reported an expired wait (code {code})")

    def _error_copy(self):
        """A pinned host copy of the device error word, queued on the executor's stream (None without one)."""
        if self._error_word is None:
            return None
        torch = _torch()
        host = torch.empty(1, dtype=torch.int32, pin_memory=True)
        with torch.cuda.stream(self._stream):
            host.copy_(self._error_word, non_blocking=True)
        return host

    def raw_state(self) -> np.ndarray:
        """The whole state as host float32 [total_nodes, n_chains] values (spins +-1)."""
        torch = _torch()
        if self._dense:
            self._stream.synchronize()
            vals = [self._dense_block_values(bi) for bi in range(len(self._block_states))]
            return torch.cat(vals, dim=1).cpu().numpy().T.copy()
        out = torch.empty((self.n_chains, self.compiled.total_nodes), dtype=torch.float32, device=self._tdev)
        nat.bind_device(self._tdev.index)
        nat.check(
            self._lib.tthrml_decode_rows(
                self._global_state.data_ptr(), self._state_code, self.n_chains, 0, self.compiled.total_nodes, 2,
                out.data_ptr(), nat.stream_handle(self._stream),
            ),
            "tthrml_decode_rows",
        )
        self._stream.synchronize()
        return out.cpu().numpy().T.copy()

    def set_raw_state(self, values: np.ndarray) -> None:
        """Overwrites the whole state from host float32 [total_nodes, n_chains] values."""
        torch = _torch()
        if self._dense:
            self._ensure_state()
            vals = torch.from_numpy(np.ascontiguousarray(np.asarray(values, np.float32).T)).to(self._tdev)
            pos = 0
            for bi, cb in enumerate(self.compiled.blocks):
                self._dense_write_block(bi, vals[:, pos : pos + cb.spec.n_nodes])
                pos += cb.spec.n_nodes
            torch.cuda.synchronize(self._tdev)
            self._state_loaded = True
            return
        src = torch.from_numpy(np.ascontiguousarray(np.asarray(values, np.float32).T)).to(self._tdev)
        self._ensure_state()
        nat.bind_device(self._tdev.index)
        with torch.cuda.stream(self._stream):
            pos = 0
            for cb in self.compiled.blocks:
                s = cb.spec
                part = src[:, pos : pos + s.n_nodes].contiguous()
                nat.check(
                    self._lib.tthrml_encode_rows(
                        part.data_ptr(), nat.STATE_F32, 1 if s.family == Family.SPIN else 0, s.n_nodes,
                        self._state_code, self.n_chains, s.block_global_start, self._global_state.data_ptr(),
                        nat.stream_handle(self._stream),
                    ),
                    "tthrml_encode_rows",
                )
                part.record_stream(self._stream)
                pos += s.n_nodes
        self._stream.synchronize()
        self._state_loaded = True

    def _decode_block(self, block_index: int, *, to_host: bool = True):
        """One block as chain-major (C, n) bool / int32 / float32 (tt_thrml/executor.py:433-438)."""
        torch = _torch()
        spec = self.compiled.blocks[block_index].spec
        kind = _OUT_KIND[spec.family]
        dtype = (torch.uint8, torch.int32, torch.float32)[kind]
        if self._dense:
            self.check_device_errors()
            with torch.cuda.stream(self._stream):
                b = self._dense_block_values(block_index)
                dev = (b > 0).to(torch.uint8) if spec.family == Family.SPIN else b.contiguous()
            if not to_host:
                return dev
            host = torch.empty(dev.shape, dtype=dtype, pin_memory=True)
            with torch.cuda.stream(self._stream):
                host.copy_(dev, non_blocking=True)
            return host
        with torch.cuda.stream(self._stream):
            dev = torch.empty((self.n_chains, spec.n_nodes), dtype=dtype, device=self._tdev)
        nat.bind_device(self._tdev.index)
        nat.check(
            self._lib.tthrml_decode_rows(
                self._global_state.data_ptr(),
                self._state_code,
                self.n_chains,
                spec.block_global_start,
                spec.n_nodes,
                kind,
                dev.data_ptr(),
                nat.stream_handle(self._stream),
            ),
            "tthrml_decode_rows",
        )
        if not to_host:
            return dev
        # a fresh pinned buffer from torch's caching host allocator: the caller
        # receives it as is (no host-side copy) and it returns to the cache
        # when the caller drops the array
        host = torch.empty(dev.shape, dtype=dtype, pin_memory=True)
        with torch.cuda.stream(self._stream):
            host.copy_(dev, non_blocking=True)
        dev.record_stream(self._stream)
        return host

    def _to_host(self, dev) -> np.ndarray:
        """A device tensor as a numpy array, copied on the executor's stream into a pinned buffer from torch's
        caching host allocator (the array keeps the buffer alive); raises if a kernel recorded an expired
        wait (the error word travels with the same synchronisation)."""
        torch = _torch()
        host = torch.empty(dev.shape, dtype=dev.dtype, pin_memory=True)
        with torch.cuda.stream(self._stream):
            host.copy_(dev, non_blocking=True)
        err = self._error_copy()
        self._stream.synchronize()
        if err is not None:
            self._raise_error_code(int(err[0]))
        return host.numpy()

    def _block_states_host(self, block_indices) -> list[np.ndarray]:
        hosts = [self._decode_block(bi) for bi in block_indices]
        err = None if self._dense else self._error_copy()
        self._stream.synchronize()
        if err is not None:
            self._raise_error_code(int(err[0]))
        out = []
        for bi, h in zip(block_indices, hosts):
            spec = self.compiled.blocks[bi].spec
            a = h.numpy()  # shares the pinned buffer, which the array keeps alive
            if spec.family == Family.SPIN:
                a = a.view(np.bool_)  # decoded spins are 0 / 1 bytes
            out.append(a.reshape(spec.n_nodes) if self.n_chains == 1 else a)
        return out

    def observe(self, blocks: Sequence) -> dict:
        """Block states keyed by block (tt_thrml/executor.py:277-292)."""
        if self._global_state is None and self._block_states is None:
            return {}
        lookup = {id(b): i for i, b in enumerate(self.program.gibbs_spec.blocks)}
        wanted = [(b, lookup.get(id(b))) for b in blocks]
        idx = [bi for _, bi in wanted if bi is not None]
        states = dict(zip(idx, self._block_states_host(idx)))
        return {b: states[bi] for b, bi in wanted if bi is not None}

    def _read_state_lists(self) -> tuple[list, list]:
        """(state_free, state_clamped) as host arrays (tt_thrml/executor.py:297-312)."""
        n_free = self.compiled.n_free_blocks
        all_states = self._block_states_host(range(len(self.compiled.blocks)))
        return all_states[:n_free], all_states[n_free:]

    def block_sums(self, blocks: Sequence, *, to_host: bool = True):
        """Per-chain sum over the listed blocks' rows, on device.

        Returns a (n_chains,) float64 numpy array, or the device tensor when
        to_host is False (no synchronisation).
        """
        torch = _torch()
        lookup = {id(b): i for i, b in enumerate(self.program.gibbs_spec.blocks)}
        with torch.cuda.stream(self._stream):
            out = torch.zeros(self.n_chains, dtype=torch.float64, device=self._tdev)
        nat.bind_device(self._tdev.index)
        if self._dense:
            lookup = {id(b): i for i, b in enumerate(self.program.gibbs_spec.blocks)}
            with torch.cuda.stream(self._stream):
                for b in blocks:
                    bi = lookup[id(b)] if not isinstance(b, int) else b
                    out += self._dense_block_values(bi).double().sum(1)
                if not to_host:
                    return out
                host = out.cpu()
            return host.numpy()
        for b in blocks:
            bi = lookup[id(b)] if not isinstance(b, int) else b
            spec = self.compiled.blocks[bi].spec
            nat.check(
                self._lib.tthrml_sum_rows(
                    self._global_state.data_ptr(),
                    self._state_code,
                    self.n_chains,
                    spec.block_global_start,
                    spec.n_nodes,
                    out.data_ptr(),
                    nat.stream_handle(self._stream),
                ),
                "tthrml_sum_rows",
            )
        if not to_host:
            return out
        with torch.cuda.stream(self._stream):
            host = out.cpu()
        return host.numpy()

    def accumulate_moments(self, rows, spin_rows, order: int, acc, spin_as_bool: bool = True, stream=None) -> None:
        """acc[m][chain] += product of the values at rows[m][:order] (device tensors; DeviceMomentObserver)."""
        if self._dense:
            raise NotImplementedError("device-side moments need a row-major state (not a dense program)")
        nat.bind_device(self._tdev.index)
        nat.check(
            self._lib.tthrml_moments_accumulate(
                self._global_state.data_ptr(), self._state_code, self.n_chains, rows.data_ptr(), spin_rows.data_ptr(),
                int(order), int(rows.shape[0]), 1 if spin_as_bool else 0, acc.data_ptr(),
                nat.stream_handle(stream if stream is not None else self._stream),
            ),
            "tthrml_moments_accumulate",
        )

    def block_sums_into(self, blocks: Sequence, out, stream) -> None:
        """Per-chain sums of the listed blocks written into the device tensor `out` on `stream`
        (no allocation, no synchronisation: usable inside a CUDA-graph capture)."""
        torch = _torch()
        lookup = {id(b): i for i, b in enumerate(self.program.gibbs_spec.blocks)}
        with torch.cuda.stream(stream):
            out.zero_()
            if self._dense:
                for b in blocks:
                    bi = lookup[id(b)] if not isinstance(b, int) else b
                    out += self._dense_block_values(bi).double().sum(1)
                return
        nat.bind_device(self._tdev.index)
        for b in blocks:
            bi = lookup[id(b)] if not isinstance(b, int) else b
            spec = self.compiled.blocks[bi].spec
            nat.check(
                self._lib.tthrml_sum_rows(
                    self._global_state.data_ptr(), self._state_code, self.n_chains, spec.block_global_start,
                    spec.n_nodes, out.data_ptr(), nat.stream_handle(stream),
                ),
                "tthrml_sum_rows",
            )

    # --------------------------------------------------------------- schedule

    def sample_states(self, key, schedule, nodes_to_sample: Sequence, *, init_state_free, state_clamp=()):
        """thrml.sample_states over the schedule (tt_thrml/executor.py:342-365)."""
        try:
            from thrml.observers import StateObserver as _ThrmlStateObserver  # type: ignore

            f_observe = _ThrmlStateObserver(list(nodes_to_sample))
        except ImportError:
            f_observe = StateObserver(list(nodes_to_sample))
        _, results = self.sample_with_observation(
            key, schedule, f_observe, init_state_free=init_state_free, state_clamp=state_clamp
        )
        return results

    def sample_with_observation(
        self, key, schedule, f_observe, *, init_state_free, state_clamp=(), observation_carry_init=None
    ):
        """thrml.sample_with_observation semantics (tt_thrml/executor.py:367-409).

        Sample 0 is taken after warmup, samples 1..n_samples-1 after each
        group of steps_per_sample sweeps.  Returns (carry, stacked observations).
        """
        n_total = schedule.n_warmup + max(0, schedule.n_samples - 1) * schedule.steps_per_sample
        self.load_state(list(init_state_free), list(state_clamp))
        self._prepare_rng_thrml_compat(key, schedule, n_total)

        carry = f_observe.init() if observation_carry_init is None else observation_carry_init
        device_side = getattr(f_observe, "device_side", False)
        colours = self._resident_observation(f_observe, schedule) if device_side else 0
        if colours:
            # a resident lattice with its magnetisation observable: the whole schedule is one launch
            torch = _torch()
            n_s = int(schedule.n_samples)
            self._check_ready(n_total)
            with torch.cuda.stream(self._stream):
                obs = torch.empty((n_s, self.n_chains), dtype=torch.float64, device=self._tdev)
            self._run_resident(n_total, obs, 2 * int(schedule.n_warmup), 2 * int(schedule.steps_per_sample), n_s,
                               colours)
            host = self._to_host(obs)
            return carry, (tree_expand(host[0]) if n_s <= 1 else host)
        if (device_side and self.config.cuda_graphs and not self.profile and schedule.n_samples >= 1
                and callable(getattr(f_observe, "observe_capture", None))):
            # the whole schedule is one graph replay; observations stay on the device until the end
            carry = f_observe.prepare(self, carry)
            obs = self._run_schedule_graph(schedule, f_observe, carry)
            host = self._to_host(obs) if obs is not None else None
            finalize = getattr(f_observe, "finalize", None)
            if callable(finalize):
                self._stream.synchronize()
                carry = finalize(carry)
            if host is None:
                return carry, None
            return carry, (tree_expand(host[0]) if schedule.n_samples <= 1 else host)
        self.run_warmup(schedule.n_warmup)

        def observe(carry, i):
            if device_side:
                return f_observe.observe_device(self, carry, i)
            state_free, state_clamped = self._read_state_lists()
            return f_observe(self.program, state_free, state_clamped, carry, np.asarray(i))

        carry, obs = observe(carry, 0)
        all_obs = [obs]
        for i in range(1, schedule.n_samples):
            self.run_sweeps(schedule.steps_per_sample)
            carry, obs = observe(carry, i)
            all_obs.append(obs)
        if device_side:  # observations are device tensors: one read-back for the whole run
            all_obs = _device_obs_to_host(all_obs, self._stream)
            finalize = getattr(f_observe, "finalize", None)
            if callable(finalize):
                self._stream.synchronize()
                carry = finalize(carry)
        if schedule.n_samples <= 1:
            return carry, tree_expand(all_obs[0])
        if all(o is None for o in all_obs):
            return carry, None
        return carry, tree_stack(all_obs)

    def timing_summary(self) -> dict:
        """Per-family dispatch and kernel ms of profiled runs (tt_thrml/executor.py:411-431)."""
        groups: dict[str, list[tuple[float, float]]] = {}
        for label, d, k in self._timing_log:
            groups.setdefault(label, []).append((d, k))
        summary = {}
        for label, entries in sorted(groups.items()):
            ds = [d for d, _ in entries]
            ks = [k for _, k in entries]
            summary[label] = {
                "n": len(entries),
                "dispatch_mean_ms": sum(ds) / len(ds),
                "dispatch_total_ms": sum(ds),
                "kernel_mean_ms": sum(ks) / len(ks),
                "kernel_total_ms": sum(ks),
            }
        return summary


def torch_stream(stream):
    return _torch().cuda.stream(stream)


def _device_obs_to_host(all_obs: list, stream) -> list:
    """Stacks per-sample device tensors (or lists/tuples of them) and copies them to the host once."""
    torch = _torch()
    first = all_obs[0]
    if first is None:
        return all_obs
    if isinstance(first, (list, tuple)):
        cols = [_device_obs_to_host([o[k] for o in all_obs], stream) for k in range(len(first))]
        return [type(first)(c[i] for c in cols) for i in range(len(all_obs))]
    if not isinstance(first, torch.Tensor):
        return all_obs
    with torch.cuda.stream(stream):
        host = torch.stack(all_obs).cpu().numpy()
    return list(host)


def make_executor(
    ttnn,
    device,
    program,
    config: CUDAConfig,
    *,
    n_sweeps: int = 100,
    profile: bool = False,
    n_chains: int | None = None,
) -> Executor:
    return Executor(ttnn, device, program, config, n_sweeps=n_sweeps, profile=profile, n_chains=n_chains)
