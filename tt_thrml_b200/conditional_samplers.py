"""GaussianConditional: the scalar gaussian conditional of the reference.

Restates tt_thrml/conditional_samplers.py:10-71 without JAX so it can be used
by the host-side program description and by observers.  Interactions are
duck-typed exactly like the reference:

* `interaction.weights` -> linear contribution
* `interaction.inverse_weights` -> precision contribution, precision =
  reciprocal(inverse_weights)

`compute_parameters` returns (linear, precision); `sample_given_parameters`
returns mean + sqrt(variance) * N(0, 1) with variance = 1 / precision (no
epsilon; the device kernels add 1e-6 to the precision like
tt_thrml/compiler.py:362, a relative difference of about 1e-6 at unit
precision).  The CUDA kernels never call this class: the sweep path lowers the
interactions to tables instead.
"""

from __future__ import annotations

import numpy as np

from . import jax_prng
from .core import Family


class GaussianConditional:
    family = Family.GAUSSIAN

    def init(self) -> None:
        return None

    def compute_parameters(self, key, interactions, active_flags, states, sampler_state, output_sd):
        del key
        shape = tuple(getattr(output_sd, "shape", output_sd))
        dtype = np.dtype(getattr(output_sd, "dtype", np.float32))
        linear = np.zeros(shape, dtype=dtype)
        precision = np.zeros(shape, dtype=dtype)
        for interaction, active, state_slots in zip(interactions, active_flags, states, strict=True):
            scale = np.asarray(active).astype(dtype)
            mult = [np.asarray(s).astype(dtype) for s in state_slots if not np.issubdtype(np.asarray(s).dtype, np.integer)]
            if mult:
                scale = scale * np.prod(np.stack(mult, axis=-1), axis=-1)
            if hasattr(interaction, "weights"):
                w = np.asarray(interaction.weights, dtype=dtype)
                weighted = w * scale
                linear = linear + np.sum(weighted, axis=tuple(range(1, weighted.ndim)))
            elif hasattr(interaction, "inverse_weights"):
                w = np.reciprocal(np.asarray(interaction.inverse_weights, dtype=dtype))
                weighted = w * scale
                precision = precision + np.sum(weighted, axis=tuple(range(1, weighted.ndim)))
        return (linear, precision), sampler_state

    def sample_given_parameters(self, key, parameters, sampler_state, output_sd):
        linear, precision = parameters
        shape = tuple(getattr(output_sd, "shape", np.shape(linear)))
        variance = np.reciprocal(np.asarray(precision, dtype=np.float32))
        mean = np.asarray(linear, dtype=np.float32) * variance
        noise = jax_prng.normal(jax_prng.as_key_data(key), shape)
        return (np.sqrt(variance) * noise + mean).astype(np.float32), sampler_state


__all__ = ["GaussianConditional"]
