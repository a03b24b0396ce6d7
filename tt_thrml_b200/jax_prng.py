"""NumPy restatement of JAX's default PRNG, used to make parity-mode variates.

The reference's parity RNG (tt_thrml/rng.py:132-200) derives every
(sweep, block) key from the caller's key with `jax.random.split` and draws
`uniform` / `gumbel` / `normal` from it.  When `jax` is importable the
executor calls it directly; this module restates the same algorithms for
hosts without JAX:

* Threefry-2x32 with 20 rounds (Salmon et al., "Parallel random numbers: as
  easy as 1, 2, 3", SC'11), the hash behind `jax.random`;
* the "partitionable" key derivation that is JAX's default from 0.5.0 on
  (thrml 0.1.3 pins jax 0.6.2 / 0.9.2): split(key, n)[i] = threefry(key,
  (hi(i), lo(i))) and 32-bit random bits = b0 ^ b1 of threefry(key, (hi(i),
  lo(i))) over the row-major position i;
* `uniform`: mantissa fill (bits >> 9 | 0x3f800000) - 1, scaled and clamped;
  `gumbel`: -log(-log(uniform(tiny, 1))); `normal`: sqrt(2)*erfinv(uniform(
  nextafter(-1, 0), 1)) with erfinv from Giles' single-precision polynomial
  ("Approximating the erfinv function", GPU Computing Gems, 2010).

Keys are uint32 arrays of shape (..., 2); every function is vectorised over
the leading key dimensions (one key per chain).  The transcendental steps use
NumPy float32 math, which may differ from XLA's by an ulp; no JAX exists in
this build's environment to pin the restatement bit for bit.
"""

from __future__ import annotations

import numpy as np

_ROT = ((13, 15, 26, 6), (17, 29, 16, 24))
U32 = np.uint32


def _rotl(x: np.ndarray, r: int) -> np.ndarray:
    return (x << U32(r)) | (x >> U32(32 - r))


def threefry2x32(k0, k1, x0, x1) -> tuple[np.ndarray, np.ndarray]:
    """Threefry-2x32-20 of counters (x0, x1) under key (k0, k1); broadcasting."""
    with np.errstate(over="ignore"):
        k0 = np.asarray(k0, dtype=U32)
        k1 = np.asarray(k1, dtype=U32)
        ks = (k0, k1, k0 ^ k1 ^ U32(0x1BD11BDA))
        x0 = np.asarray(x0, dtype=U32) + ks[0]
        x1 = np.asarray(x1, dtype=U32) + ks[1]
        for i in range(5):
            for r in _ROT[i % 2]:
                x0 = x0 + x1
                x1 = _rotl(x1, r)
                x1 = x1 ^ x0
            x0 = x0 + ks[(i + 1) % 3]
            x1 = x1 + ks[(i + 2) % 3] + U32(i + 1)
        return x0, x1


def key_from_seed(seed: int) -> np.ndarray:
    """jax.random.key(seed) data: (seed >> 32, seed & 0xffffffff) of an int32/64 seed."""
    s = int(seed)
    if -(2**31) <= s < 2**31:
        return np.array([0, s & 0xFFFFFFFF], dtype=U32)
    s &= (1 << 64) - 1
    return np.array([s >> 32, s & 0xFFFFFFFF], dtype=U32)


def as_key_data(key) -> np.ndarray:
    """Raw uint32 key data from an int seed, a raw key array or a JAX key."""
    if isinstance(key, (int, np.integer)):
        return key_from_seed(int(key))
    dtype = getattr(key, "dtype", None)
    if dtype is not None and "key" in str(dtype):
        import jax  # only reachable when the caller already uses JAX keys

        key = jax.random.key_data(key)
    arr = np.asarray(key)
    if arr.shape[-1:] != (2,):
        raise ValueError(f"expected key data of shape (..., 2), got {arr.shape}")
    return arr.astype(U32)


def _iota_hi_lo(n: int) -> tuple[np.ndarray, np.ndarray]:
    i = np.arange(n, dtype=np.uint64)
    return (i >> np.uint64(32)).astype(U32), (i & np.uint64(0xFFFFFFFF)).astype(U32)


def split(key: np.ndarray, n: int) -> np.ndarray:
    """jax.random.split(key, n): (..., 2) -> (..., n, 2)."""
    key = np.asarray(key, dtype=U32)
    hi, lo = _iota_hi_lo(n)
    k0 = key[..., 0:1]
    k1 = key[..., 1:2]
    b0, b1 = threefry2x32(k0, k1, hi, lo)
    return np.stack([b0, b1], axis=-1)


def random_bits(key: np.ndarray, shape: tuple[int, ...]) -> np.ndarray:
    """32-bit random bits of the given shape: (..., 2) -> (..., *shape)."""
    key = np.asarray(key, dtype=U32)
    n = int(np.prod(shape, dtype=np.int64))
    hi, lo = _iota_hi_lo(n)
    b0, b1 = threefry2x32(key[..., 0:1], key[..., 1:2], hi, lo)
    return (b0 ^ b1).reshape(key.shape[:-1] + tuple(shape))


def uniform(key, shape, minval=0.0, maxval=1.0) -> np.ndarray:
    bits = random_bits(key, shape)
    f = ((bits >> U32(9)) | U32(0x3F800000)).view(np.float32) - np.float32(1.0)
    lo = np.float32(minval)
    hi = np.float32(maxval)
    out = (f * (hi - lo) + lo).astype(np.float32)
    return np.maximum(lo, out)


def gumbel(key, shape) -> np.ndarray:
    tiny = np.finfo(np.float32).tiny
    u = uniform(key, shape, tiny, 1.0)
    with np.errstate(divide="ignore"):
        return (-np.log(-np.log(u))).astype(np.float32)


def _erfinv_f32(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        w = (-np.log1p(-x * x)).astype(np.float32)
        small = w < np.float32(5.0)
        ws = (w - np.float32(2.5)).astype(np.float32)
        p = np.float32(2.81022636e-08)
        for c in (3.43273939e-07, -3.5233877e-06, -4.39150654e-06, 0.00021858087, -0.00125372503,
                  -0.00417768164, 0.246640727, 1.50140941):
            p = (np.float32(c) + p * ws).astype(np.float32)
        wl = (np.sqrt(w) - np.float32(3.0)).astype(np.float32)
        pl = np.float32(-0.000200214257)
        for c in (0.000100950558, 0.00134934322, -0.00367342844, 0.00573950773, -0.0076224613,
                  0.00943887047, 1.00167406, 2.83297682):
            pl = (np.float32(c) + pl * wl).astype(np.float32)
        out = np.where(small, p, pl) * x
        out = np.where(np.abs(x) == np.float32(1.0), np.copysign(np.float32(np.inf), x), out)
    return out.astype(np.float32)


def normal(key, shape) -> np.ndarray:
    lo = np.nextafter(np.float32(-1.0), np.float32(0.0), dtype=np.float32)
    u = uniform(key, shape, lo, 1.0)
    return (np.float32(np.sqrt(2.0)) * _erfinv_f32(u)).astype(np.float32)


def logit(u: np.ndarray) -> np.ndarray:
    """log(u / (1 - u)) in float32, the reference's spin threshold transform."""
    u = u.astype(np.float32)
    with np.errstate(divide="ignore"):
        return np.log(u / (np.float32(1.0) - u)).astype(np.float32)
