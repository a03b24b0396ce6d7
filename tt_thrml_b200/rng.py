"""Random variates for the sweep kernels.

Two modes:

* "philox" (default): nothing is generated on the host.  Every kernel draws
  its variates on device from Philox4x32-10 keyed by a 64-bit seed derived
  from the caller's key, with counter (chain/4, row, sweep, salt), so a
  (sweep, block) slice is addressed by index exactly like the reference's
  bulk buffers (tt_thrml/rng.py:203-222) but costs no memory or upload.
* "parity": the reference's bulk upload (tt_thrml/rng.py:50-200): per
  (block, sweep) spin threshold logits, categorical Gumbel noise and gaussian
  normals derived from the caller's key with thrml's key tree, uploaded once
  as one device buffer per block [n_sweeps, n_nodes, qv, n_chains].  With
  several chains, chain c uses key split(key, n_chains)[c].  Variates come
  from `jax.random` when JAX is importable, else from the NumPy restatement
  in tt_thrml_b200.jax_prng.
"""

from __future__ import annotations

import numpy as np

from . import jax_prng
from .core import BulkRNGBuffers, Family, RNGSpec


def make_rng_spec(blocks: tuple, n_sweeps: int) -> RNGSpec:
    """tt_thrml/rng.py:19-40."""
    spin, cat, gauss, nodes, cats = [], [], [], [], []
    for block in blocks:
        spec = block.spec
        nodes.append(spec.n_nodes)
        cats.append(spec.n_categories)
        if spec.family == Family.SPIN:
            spin.append(spec.block_index)
        elif spec.family == Family.CATEGORICAL:
            cat.append(spec.block_index)
        elif spec.family == Family.GAUSSIAN:
            gauss.append(spec.block_index)
    return RNGSpec(
        n_sweeps=n_sweeps,
        spin_blocks=tuple(spin),
        categorical_blocks=tuple(cat),
        gaussian_blocks=tuple(gauss),
        nodes_per_block=tuple(nodes),
        categories_per_block=tuple(cats),
    )


def seed_from_key(key) -> int:
    """64-bit Philox seed of a key (int seed, raw uint32[2] key data or JAX key)."""
    kd = jax_prng.as_key_data(key).reshape(-1, 2)[0]
    return (int(kd[0]) << 32) | int(kd[1])


def philox_buffers(key, n_sweeps: int) -> BulkRNGBuffers:
    return BulkRNGBuffers(None, None, None, seed=seed_from_key(key), n_sweeps=n_sweeps)


# ----------------------------------------------------------------------------
# Variate sources: jax.random when importable, else the NumPy restatement.
# ----------------------------------------------------------------------------


class _NumpySource:
    name = "numpy-threefry"

    @staticmethod
    def split(keys, n):
        return jax_prng.split(keys, n)

    @staticmethod
    def uniform(keys, shape, minval=0.0, maxval=1.0):
        return jax_prng.uniform(keys, shape, minval, maxval)

    @staticmethod
    def gumbel(keys, shape):
        return jax_prng.gumbel(keys, shape)

    @staticmethod
    def normal(keys, shape):
        return jax_prng.normal(keys, shape)


class _JaxSource:
    name = "jax"

    def __init__(self, jax):
        self.jax = jax

    def _vmap(self, fn, keys):
        jax = self.jax
        flat = np.asarray(keys, dtype=np.uint32).reshape(-1, 2)
        ks = jax.random.wrap_key_data(flat)
        out = np.asarray(jax.vmap(fn)(ks))
        return out.reshape(np.asarray(keys).shape[:-1] + out.shape[1:])

    def split(self, keys, n):
        jax = self.jax
        return self._vmap(lambda k: jax.random.key_data(jax.random.split(k, n)), keys)

    def uniform(self, keys, shape, minval=0.0, maxval=1.0):
        jax = self.jax
        return self._vmap(lambda k: jax.random.uniform(k, shape=shape, minval=minval, maxval=maxval), keys)

    def gumbel(self, keys, shape):
        jax = self.jax
        return self._vmap(lambda k: jax.random.gumbel(k, shape=shape), keys)

    def normal(self, keys, shape):
        jax = self.jax
        return self._vmap(lambda k: jax.random.normal(k, shape=shape), keys)


def variate_source(prefer_jax: bool = True):
    if prefer_jax:
        try:
            import jax  # noqa: F401

            return _JaxSource(jax)
        except ImportError:
            pass
    return _NumpySource()


def _chain_keys(key, n_chains: int, src) -> np.ndarray:
    kd = jax_prng.as_key_data(key)
    if kd.ndim == 2:  # one key per chain given explicitly
        if kd.shape[0] != n_chains:
            raise ValueError(f"{kd.shape[0]} chain keys for {n_chains} chains")
        return kd
    if n_chains == 1:
        return kd.reshape(1, 2)
    return src.split(kd, n_chains)


def _logit(u):
    return jax_prng.logit(np.asarray(u, dtype=np.float32))


def _to_device(arr: np.ndarray, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32)).to(device)


def _layout(per_chain: np.ndarray) -> np.ndarray:
    """(chains, sweeps, n, qv) -> (sweeps, n, qv, chains)."""
    return np.ascontiguousarray(np.moveaxis(per_chain, 0, -1))


def generate_bulk_rng(key, rng_spec: RNGSpec, device, *, n_chains: int = 1, source=None) -> BulkRNGBuffers:
    """Non-schedule bulk variates (tt_thrml/rng.py:50-129) for prepare_rng()."""
    src = source or variate_source()
    ck = _chain_keys(key, n_chains, src)  # (C, 2)
    fam_keys = src.split(ck, 4)  # (C, 4, 2): key, spin, cat, gauss
    out: dict[str, dict[int, object] | None] = {"spin": None, "cat": None, "gauss": None}
    S = rng_spec.n_sweeps
    for slot, fam_blocks, name in ((1, rng_spec.spin_blocks, "spin"), (2, rng_spec.categorical_blocks, "cat"),
                                   (3, rng_spec.gaussian_blocks, "gauss")):
        if not fam_blocks:
            continue
        keys = src.split(fam_keys[:, slot], len(fam_blocks) * S)  # (C, nb*S, 2)
        res = {}
        for j, bi in enumerate(fam_blocks):
            n = rng_spec.nodes_per_block[bi]
            ks = keys[:, j * S : (j + 1) * S]
            if name == "spin":
                u = src.uniform(ks, (n,), 1e-7, 1.0 - 1e-7)
                v = _logit(u)[..., None]
            elif name == "cat":
                q = rng_spec.categories_per_block[bi] or 2
                v = src.gumbel(ks, (n, q))
            else:
                v = src.normal(ks, (n,))[..., None]
            res[bi] = _to_device(_layout(np.asarray(v, dtype=np.float32)), device)
        out[name] = res
    return BulkRNGBuffers(out["spin"], out["cat"], out["gauss"], seed=None, n_sweeps=S)


def schedule_sweep_keys(key_chains: np.ndarray, schedule, src) -> np.ndarray:
    """Per-sweep keys of thrml.sample_with_observation (tt_thrml/rng.py:151-160): (C, n_total, 2)."""
    pair = src.split(key_chains, 2)
    sample_key, warmup_key = pair[:, 0], pair[:, 1]
    parts = []
    if schedule.n_warmup > 0:
        parts.append(src.split(warmup_key, schedule.n_warmup))
    if schedule.n_samples > 1:
        outer = src.split(sample_key, schedule.n_samples - 1)  # (C, n_s-1, 2)
        inner = src.split(outer, schedule.steps_per_sample)  # (C, n_s-1, steps, 2)
        parts.append(inner.reshape(inner.shape[0], -1, 2))
    if not parts:
        return np.zeros((key_chains.shape[0], 0, 2), dtype=np.uint32)
    return np.concatenate(parts, axis=1)


def generate_bulk_rng_for_schedule(
    key, rng_spec: RNGSpec, schedule, n_free_blocks: int, device, *, n_chains: int = 1, source=None
) -> BulkRNGBuffers:
    """Variates following thrml's sample_with_observation key tree (tt_thrml/rng.py:132-200)."""
    src = source or variate_source()
    ck = _chain_keys(key, n_chains, src)
    sweep_keys = schedule_sweep_keys(ck, schedule, src)  # (C, T, 2)
    T = sweep_keys.shape[1]
    per_block = src.split(sweep_keys, n_free_blocks)  # (C, T, nb, 2)
    out: dict[str, dict[int, object]] = {"spin": {}, "cat": {}, "gauss": {}}
    for bi in range(n_free_blocks):
        bk = src.split(per_block[:, :, bi], 2)[:, :, 0]  # (C, T, 2)
        n = rng_spec.nodes_per_block[bi]
        if bi in rng_spec.spin_blocks:
            v = _logit(src.uniform(bk, (n,)))[..., None]
            out["spin"][bi] = _to_device(_layout(v), device)
        elif bi in rng_spec.categorical_blocks:
            q = rng_spec.categories_per_block[bi] or 2
            out["cat"][bi] = _to_device(_layout(np.asarray(src.gumbel(bk, (n, q)))), device)
        elif bi in rng_spec.gaussian_blocks:
            v = np.asarray(src.normal(bk, (n,)))[..., None]
            out["gauss"][bi] = _to_device(_layout(v), device)
    return BulkRNGBuffers(out["spin"] or None, out["cat"] or None, out["gauss"] or None, seed=None, n_sweeps=T)


def block_variates(rng_buffers: BulkRNGBuffers, block_index: int, family: Family):
    """The device buffer [n_sweeps, n, qv, C] of one block, or None in Philox mode."""
    table = {
        Family.SPIN: rng_buffers.spin_threshold_logits,
        Family.CATEGORICAL: rng_buffers.categorical_gumbel,
        Family.GAUSSIAN: rng_buffers.gaussian_noise,
    }[family]
    if table is None:
        return None
    return table.get(block_index)


def slice_rng_for_sweep(ttnn, rng_buffers: BulkRNGBuffers, sweep_index: int, block_index: int, family: Family):
    """One (sweep, block) slice, shaped [n, qv, C] (tt_thrml/rng.py:203-222)."""
    del ttnn
    if rng_buffers.seed is not None:
        raise RuntimeError("Philox-mode RNG has no host-visible slices; variates are drawn on device.")
    buf = block_variates(rng_buffers, block_index, family)
    if buf is None:
        raise RuntimeError(f"{family.value.capitalize()} RNG buffer is not available.")
    return buf[sweep_index]
