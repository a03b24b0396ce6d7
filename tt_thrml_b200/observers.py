"""Observers for `Executor.sample_with_observation`.

The executor calls observers with the signature thrml uses,
`f_observe(program, state_free, state_clamped, carry, sample_index) ->
(carry, observation)` with an `init()` method (tt_thrml/executor.py:389-403),
so thrml's own observers work unchanged when thrml is installed.  The classes
here give the same two observers without thrml/JAX (NumPy arrays in and out):

* `StateObserver(blocks)`: records the state of each listed block
  (thrml.observers.StateObserver, used by tt_thrml/executor.py:355);
* `MomentAccumulatorObserver(moment_spec, f_transform)`: accumulates
  products of node values over the samples (thrml.observers.
  MomentAccumulatorObserver; used by the reference's parity scenarios).

Device-side observers never copy the state to the host per sample:
`MagnetizationObserver` sums spin blocks per chain, `DeviceMomentObserver`
accumulates MomentAccumulatorObserver's products on the GPU.
"""

from __future__ import annotations

from typing import Sequence

import numpy as np


def _block_lookup(program):
    blocks = program.gibbs_spec.blocks
    return {id(b): i for i, b in enumerate(blocks)}


def _node_positions(program):
    """node -> (block index, position in block)."""
    pos = {}
    for bi, block in enumerate(program.gibbs_spec.blocks):
        for k, node in enumerate(block.nodes):
            pos[node] = (bi, k)
    return pos


def _full_states(program, state_free, state_clamped):
    n_free = len(program.gibbs_spec.free_blocks)
    return list(state_free) + list(state_clamped), n_free


class StateObserver:
    """Records the state of `blocks` at every sample."""

    def __init__(self, blocks: Sequence):
        self.blocks = list(blocks)

    def init(self):
        return None

    def __call__(self, program, state_free, state_clamped, carry, sample_index):
        states, _ = _full_states(program, state_free, state_clamped)
        lookup = _block_lookup(program)
        out = []
        for block in self.blocks:
            bi = lookup.get(id(block))
            if bi is not None:
                out.append(np.asarray(states[bi]))
                continue
            # a block made of nodes of several program blocks: gather node by node
            pos = _node_positions(program)
            out.append(np.stack([np.asarray(states[pos[n][0]])[..., pos[n][1]] for n in block.nodes], axis=-1))
        return carry, out


def _default_transform(state, blocks):
    return state


class MomentAccumulatorObserver:
    """Sums products of node values per moment over the samples.

    moment_spec: a sequence of moment groups; each group is a sequence of
    node tuples, e.g. ([(a,), (b,)], [(a, b)]) for first and second moments.
    f_transform(state_list, blocks) maps raw block states to the values that
    are multiplied (default: the raw states; spins are then booleans).
    The carry is one float array per group with one entry per node tuple; the
    observation is None.
    """

    def __init__(self, moment_spec, f_transform=_default_transform):
        self.moment_spec = [list(group) for group in moment_spec]
        self.f_transform = f_transform

    def init(self):
        return [np.zeros(len(group), dtype=np.float32) for group in self.moment_spec]

    def __call__(self, program, state_free, state_clamped, carry, sample_index):
        states, _ = _full_states(program, state_free, state_clamped)
        values = self.f_transform([np.asarray(s) for s in states], program.gibbs_spec.blocks)
        pos = _node_positions(program)
        new = []
        for acc, group in zip(carry, self.moment_spec):
            contrib = []
            for nodes in group:
                prod = None
                for node in nodes:
                    bi, k = pos[node]
                    v = np.asarray(values[bi], dtype=np.float32)[..., k]
                    prod = v if prod is None else prod * v
                contrib.append(prod)
            new.append(np.asarray(acc) + np.stack(contrib, axis=-1).astype(np.float32))
        return new, None


class DeviceMomentObserver:
    """MomentAccumulatorObserver with the products accumulated on the GPU.

    Same moment_spec (groups of node tuples) and the same final carry -- one
    float32 array per group, [n_chains, len(group)] ([len(group)] with one
    chain) -- but each sample is one launch of tthrml_moments_accumulate on
    the device state instead of a full state read-back (the reference reads
    the whole state back per sample, tt_thrml/executor.py:294-295, 389-409).
    spin_as_bool: spins enter the products as 1 / 0 (the reference's boolean
    spin state, what the default transform of MomentAccumulatorObserver
    multiplies) or, when False, as +-1.
    """

    device_side = True

    def __init__(self, moment_spec, spin_as_bool: bool = True):
        self.moment_spec = [list(group) for group in moment_spec]
        self.spin_as_bool = bool(spin_as_bool)

    def init(self):
        return None

    def _tables(self, executor):
        import torch

        program = executor.program
        pos = _node_positions(program)
        specs = [cb.spec for cb in executor.compiled.blocks]
        tuples = [nodes for group in self.moment_spec for nodes in group]
        order = max((len(t) for t in tuples), default=1)
        rows = np.full((len(tuples), order), -1, dtype=np.int64)
        spin = np.zeros((len(tuples), order), dtype=np.uint8)
        for m, nodes in enumerate(tuples):
            for k, node in enumerate(nodes):
                bi, j = pos[node]
                rows[m, k] = specs[bi].block_global_start + j
                spin[m, k] = 1 if getattr(specs[bi].family, "value", specs[bi].family) == "spin" else 0
        dev = executor.compiled.device
        acc = torch.zeros((len(tuples), executor.n_chains), dtype=torch.float64, device=dev)
        return {"rows": torch.from_numpy(rows).to(dev), "spin": torch.from_numpy(spin).to(dev), "order": order,
                "acc": acc}

    def observe_device(self, executor, carry, sample_index):
        if carry is None:
            carry = self._tables(executor)
        executor.accumulate_moments(carry["rows"], carry["spin"], carry["order"], carry["acc"], self.spin_as_bool)
        return carry, None

    # graph capture of a whole schedule (Executor.sample_with_observation)
    def prepare(self, executor, carry):
        if carry is None:  # tables are kept per executor, so a captured schedule graph is reused
            cache = self.__dict__.setdefault("_carry_cache", {})
            carry = cache.get(id(executor))
            if carry is None:
                carry = cache[id(executor)] = self._tables(executor)
        carry["acc"].zero_()
        return carry

    def capture_buffer(self, executor, n_samples):
        return None

    def observe_capture(self, executor, carry, obs, sample_index, stream):
        executor.accumulate_moments(carry["rows"], carry["spin"], carry["order"], carry["acc"], self.spin_as_bool,
                                    stream=stream)

    def finalize(self, carry, stream=None):
        if carry is None:
            return [np.zeros(len(group), dtype=np.float32) for group in self.moment_spec]
        acc = carry["acc"].cpu().numpy()  # [n_moments][C]
        out, m = [], 0
        for group in self.moment_spec:
            part = acc[m : m + len(group)].T.astype(np.float32)  # [C][len(group)]
            out.append(part[0] if part.shape[0] == 1 else part)
            m += len(group)
        return out


class MagnetizationObserver:
    """Per-chain sum of the listed spin blocks, computed on the GPU.

    The observation of each sample is a float64 array of shape (n_chains,)
    (the magnetisation observable of the lattice workloads).  Used through
    `Executor.sample_with_observation` it never copies the state to the host.
    """

    device_side = True

    def __init__(self, blocks: Sequence):
        self.blocks = list(blocks)

    def init(self):
        return None

    def observe_device(self, executor, carry, sample_index):
        # a device tensor; the executor reads every sample back in one copy at the end
        return carry, executor.block_sums(self.blocks, to_host=False)

    # graph capture of a whole schedule (Executor.sample_with_observation)
    def prepare(self, executor, carry):
        return carry

    def capture_buffer(self, executor, n_samples):
        import torch

        return torch.empty((n_samples, executor.n_chains), dtype=torch.float64, device=executor.compiled.device)

    def observe_capture(self, executor, carry, obs, sample_index, stream):
        executor.block_sums_into(self.blocks, obs[sample_index], stream)


def tree_stack(observations):
    """Stacks a list of observation pytrees (lists/tuples/dicts of arrays)."""
    first = observations[0]
    if first is None:
        return None
    if isinstance(first, dict):
        return {k: tree_stack([o[k] for o in observations]) for k in first}
    if isinstance(first, (list, tuple)):
        return type(first)(tree_stack([o[i] for o in observations]) for i in range(len(first)))
    return np.stack([np.asarray(o) for o in observations])


def tree_expand(obs):
    if obs is None:
        return None
    if isinstance(obs, dict):
        return {k: tree_expand(v) for k, v in obs.items()}
    if isinstance(obs, (list, tuple)):
        return type(obs)(tree_expand(v) for v in obs)
    return np.asarray(obs)[None]
