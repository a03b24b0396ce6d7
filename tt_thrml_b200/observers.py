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

A device-side observer, `MagnetizationObserver`, sums spin blocks per chain on
the GPU so no state crosses to the host per sample.
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
