"""Multi-GPU execution: chains sharded across GPUs.

The reference's MeshExecutor replicates one state over a Tenstorrent mesh and
synchronises the mesh after every group (tt_thrml/mesh.py:29-46); it has no
data exchange.  Here independent chains are split across GPUs, which needs no
exchange either: each GPU runs the whole program on its own chain shard, with
Philox counters keyed by the global chain index so the samples of a chain do
not depend on how many GPUs share the run.  Two drivers:

* one process per GPU (torch.distributed initialised, world size > 1): this
  process owns chains [rank*C/W, (rank+1)*C/W); initial states are given for
  all C chains or for this rank's chains only; host read-backs are
  all-gathered so every rank sees all chains (or, with gather=False, each
  rank gets its own chains);
* one process driving a `CudaMeshDevice` of G GPUs: one shard executor per
  GPU, all launched from this thread on per-GPU streams.

No collective runs inside a sweep; `mesh_barrier` synchronises the devices
when the caller wants a fence.
"""

from __future__ import annotations

from typing import Any, Iterable, Sequence, cast

import numpy as np

from . import jax_prng
from .backend import CudaMeshDevice
from .core import CUDAConfig
from .executor import Executor
from .observers import StateObserver, tree_expand, tree_stack


def mesh_device_ids(device) -> tuple[int, ...]:
    get_ids = getattr(device, "get_device_ids", None)
    if callable(get_ids):
        return tuple(int(d) for d in cast(Iterable[Any], get_ids()))
    return ()


def mesh_size(device) -> int:
    ids = mesh_device_ids(device)
    return len(ids) if ids else 1


def mesh_barrier(ttnn, device) -> None:
    if ttnn is None:
        from .backend import cuda as ttnn
    ttnn.synchronize_device(device)


def _dist():
    try:
        import torch.distributed as dist
    except ImportError:
        return None
    if dist.is_available() and dist.is_initialized():
        return dist
    return None


class MeshExecutor(Executor):
    """Executor whose chains are sharded across GPUs (same public methods as Executor)."""

    def __init__(
        self,
        ttnn,
        device,
        program,
        config: CUDAConfig,
        compiled=None,
        *,
        n_sweeps: int = 100,
        profile: bool = False,
        n_chains: int | None = None,
        process_group=None,
        gather: bool = True,
    ):
        """gather: with one process per GPU, host read-backs (observe, sample_states, block_sums) return
        every chain on every rank (all-gathered, like the reference's replicated state); False returns
        this rank's own chains only (no collective: for outputs too large to replicate)."""
        total = int(n_chains if n_chains is not None else config.n_chains)
        self.gather = bool(gather)
        self.ttnn, self.device, self.program, self.config = ttnn, device, program, config
        self.n_sweeps, self.profile = n_sweeps, profile
        self.total_chains = total
        self.process_group = process_group
        dist = _dist()
        if dist is not None and dist.get_world_size(process_group) > 1:
            world, rank = dist.get_world_size(process_group), dist.get_rank(process_group)
            self._mode = "ranks"
            self._world, self._rank = world, rank
            devs = [device]
        elif isinstance(device, CudaMeshDevice) and len(device.devices) > 1:
            self._mode = "devices"
            world, rank = len(device.devices), 0
            devs = list(device.devices)
        else:
            self._mode = "single"
            world, rank = 1, 0
            devs = [device.devices[0] if isinstance(device, CudaMeshDevice) else device]
        if total % world:
            raise ValueError(f"{total} chains do not split evenly over {world} GPUs")
        local = total // world
        if world > 1 and local % 4:
            raise ValueError("chains per GPU must be a multiple of 4")
        first = rank * local if self._mode == "ranks" else 0
        self.shards = [
            Executor(
                ttnn,
                d,
                program,
                config,
                compiled if (k == 0 and compiled is not None) else None,
                n_sweeps=n_sweeps,
                profile=profile,
                n_chains=local,
                chain_offset=first + k * local,
            )
            for k, d in enumerate(devs)
        ]
        self.compiled = self.shards[0].compiled
        self.n_chains = local * len(self.shards)
        self.chain_offset = first

    # -------------------------------------------------------------- helpers
    def _split_state(self, states):
        """Per-shard lists of block states (chain axis split when present)."""
        out = [[] for _ in self.shards]
        for bi, st in enumerate(states):
            a = np.asarray(st)
            n = self.compiled.blocks[bi].spec.n_nodes
            if a.size == n:
                for k in range(len(self.shards)):
                    out[k].append(a)
                continue
            a = a.reshape(-1, n)
            if self._mode == "ranks" and a.shape[0] == self.n_chains != self.total_chains:
                out[0].append(a)  # this rank's own chains only
                continue
            if a.shape[0] != self.total_chains:
                raise ValueError(f"block {bi}: expected ({n},) or ({self.total_chains}, {n}) states, got {a.shape}")
            for k, sh in enumerate(self.shards):
                lo = sh.chain_offset
                out[k].append(a[lo : lo + sh.n_chains])
        return out

    def _chain_keys(self, key):
        kd = jax_prng.as_key_data(key)
        if kd.ndim == 2:
            return kd
        from .rng import variate_source

        return variate_source().split(kd, self.total_chains) if self.total_chains > 1 else kd.reshape(1, 2)

    def _gather_chains(self, arrays: list[np.ndarray]) -> np.ndarray:
        """Concatenates per-shard (C_local, ...) arrays along the chain axis, across ranks too."""
        local = np.concatenate(arrays, axis=0)
        if self._mode != "ranks" or not self.gather:
            return local
        dist = _dist()
        parts: list = [None] * self._world
        dist.all_gather_object(parts, local, group=self.process_group)
        return np.concatenate(parts, axis=0)

    # --------------------------------------------------------------- state
    @property
    def state_is_loaded(self) -> bool:
        return all(s.state_is_loaded for s in self.shards)

    def load_state(self, state_free, state_clamp) -> None:
        states = list(state_free) + list(state_clamp)
        n_free = len(list(state_free))
        for sh, part in zip(self.shards, self._split_state(states)):
            sh.load_state(part[:n_free], part[n_free:])

    def prepare_rng(self, key) -> None:
        if self.config.rng_mode == "philox":
            for sh in self.shards:
                sh.prepare_rng(key)
            return
        keys = self._chain_keys(key)
        for sh in self.shards:
            sh.prepare_rng(keys[sh.chain_offset : sh.chain_offset + sh.n_chains])

    def _prepare_rng_thrml_compat(self, key, schedule, n_total: int) -> None:
        keys = key if self.config.rng_mode == "philox" else self._chain_keys(key)
        for sh in self.shards:
            k = keys if self.config.rng_mode == "philox" else keys[sh.chain_offset : sh.chain_offset + sh.n_chains]
            sh._prepare_rng_thrml_compat(k, schedule, n_total)

    # --------------------------------------------------------------- sweeps
    def run_sweep(self) -> None:
        """One sweep on every shard (tt_thrml/mesh.py:32-46; no exchange is needed)."""
        for sh in self.shards:
            sh.run_sweep()

    def run_sweeps(self, n: int) -> None:
        for sh in self.shards:
            sh.run_sweeps(n)

    def run_warmup(self, n_warmup: int) -> None:
        self.run_sweeps(n_warmup)

    def synchronize(self) -> None:
        for sh in self.shards:
            sh.stream.synchronize()

    # ------------------------------------------------------------ read-back
    def _state_lists(self, blocks=None):
        per = [sh._block_states_host(range(len(self.compiled.blocks))) for sh in self.shards]
        merged = []
        for bi in range(len(self.compiled.blocks)):
            parts = [p[bi].reshape(sh.n_chains, -1) for p, sh in zip(per, self.shards)]
            full = self._gather_chains(parts)
            merged.append(full.reshape(-1) if self.total_chains == 1 else full)
        return merged

    def _read_state_lists(self):
        merged = self._state_lists()
        n_free = self.compiled.n_free_blocks
        return merged[:n_free], merged[n_free:]

    def observe(self, blocks: Sequence) -> dict:
        lookup = {id(b): i for i, b in enumerate(self.program.gibbs_spec.blocks)}
        merged = self._state_lists()
        return {b: merged[lookup[id(b)]] for b in blocks if id(b) in lookup}

    def block_sums(self, blocks: Sequence, *, to_host: bool = True) -> np.ndarray:
        """Per-chain sums over all shards; always a host array (the shards live on several devices)."""
        del to_host
        return self._gather_chains([sh.block_sums(blocks) for sh in self.shards])

    def sample_states(self, key, schedule, nodes_to_sample, *, init_state_free, state_clamp=()):
        f_observe = StateObserver(list(nodes_to_sample))
        _, results = self.sample_with_observation(
            key, schedule, f_observe, init_state_free=init_state_free, state_clamp=state_clamp
        )
        return results

    def sample_with_observation(
        self, key, schedule, f_observe, *, init_state_free, state_clamp=(), observation_carry_init=None
    ):
        if len(self.shards) == 1 and (self._mode == "single" or not self.gather):
            # this process's chains only: the shard's own schedule (one CUDA graph, fused device observers)
            sh = self.shards[0]
            n_free = len(list(init_state_free))
            part = self._split_state(list(init_state_free) + list(state_clamp))[0]
            k = key if self.config.rng_mode == "philox" else \
                self._chain_keys(key)[sh.chain_offset : sh.chain_offset + sh.n_chains]
            return sh.sample_with_observation(k, schedule, f_observe, init_state_free=part[:n_free],
                                              state_clamp=part[n_free:], observation_carry_init=observation_carry_init)
        n_total = schedule.n_warmup + max(0, schedule.n_samples - 1) * schedule.steps_per_sample
        self.load_state(list(init_state_free), list(state_clamp))
        self._prepare_rng_thrml_compat(key, schedule, n_total)
        self.run_warmup(schedule.n_warmup)
        carry = f_observe.init() if observation_carry_init is None else observation_carry_init
        device_side = getattr(f_observe, "device_side", False)

        def observe(carry, i):
            if device_side:
                return f_observe.observe_device(self, carry, i)
            sf, sc = self._read_state_lists()
            return f_observe(self.program, sf, sc, carry, np.asarray(i))

        carry, obs = observe(carry, 0)
        if schedule.n_samples <= 1:
            return carry, tree_expand(obs)
        all_obs = [obs]
        for i in range(1, schedule.n_samples):
            self.run_sweeps(schedule.steps_per_sample)
            carry, obs = observe(carry, i)
            all_obs.append(obs)
        if all(o is None for o in all_obs):
            return carry, None
        return carry, tree_stack(all_obs)

    def timing_summary(self) -> dict:
        return self.shards[0].timing_summary()


def make_mesh_executor(ttnn, device, program, config: CUDAConfig, *, n_sweeps: int = 100, n_chains: int | None = None,
                       gather: bool = True):
    return MeshExecutor(ttnn, device, program, config, n_sweeps=n_sweeps, n_chains=n_chains, gather=gather)
