"""GaussianConditional against the formulas of tt_thrml/conditional_samplers.py:23-71 (CPU).

compute_parameters: linear = sum over `weights` interactions of sum_terms w * active * prod(float sources);
precision = the same over `inverse_weights` interactions with w = 1 / inverse_weights; integer (categorical)
sources never multiply.  sample_given_parameters: mean = linear / precision, value = mean +
sqrt(1 / precision) * N(0, 1) with the noise of the key (no epsilon).
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest

from tt_thrml_b200 import GaussianConditional, jax_prng


def _sd(shape):
    return SimpleNamespace(shape=shape, dtype=np.float32)


def _case(rng, n=5, T=3):
    lin_a = SimpleNamespace(weights=rng.standard_normal((n, T)).astype(np.float32))
    lin_b = SimpleNamespace(weights=rng.standard_normal((n, 2)).astype(np.float32))
    prec = SimpleNamespace(inverse_weights=rng.uniform(0.5, 2.0, (n, 1)).astype(np.float32))
    act_a = rng.integers(0, 2, (n, T)).astype(bool)
    act_b = np.ones((n, 2), bool)
    act_p = np.ones((n, 1), bool)
    src_a = [rng.standard_normal((n, T)).astype(np.float32), rng.standard_normal((n, T)).astype(np.float32),
             rng.integers(0, 3, (n, T)).astype(np.int32)]  # two gaussian sources multiply, one categorical does not
    src_b = [rng.standard_normal((n, 2)).astype(np.float32)]
    return [lin_a, lin_b, prec], [act_a, act_b, act_p], [src_a, src_b, []]


def test_compute_parameters_matches_the_formulas():
    rng = np.random.default_rng(0)
    inters, active, states = _case(rng)
    (lin, prec), st = GaussianConditional().compute_parameters(None, inters, active, states, None, _sd((5,)))
    assert st is None and lin.dtype == np.float32 and prec.dtype == np.float32
    want_lin = np.zeros(5)
    want_prec = np.zeros(5)
    for i in range(5):
        for t in range(3):
            want_lin[i] += float(inters[0].weights[i, t]) * active[0][i, t] * states[0][0][i, t] * states[0][1][i, t]
        for t in range(2):
            want_lin[i] += float(inters[1].weights[i, t]) * states[1][0][i, t]
        want_prec[i] += 1.0 / float(inters[2].inverse_weights[i, 0])
    np.testing.assert_allclose(lin, want_lin, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(prec, want_prec, rtol=1e-6)


def test_compute_parameters_without_contributions_is_zero():
    (lin, prec), _ = GaussianConditional().compute_parameters(None, [], [], [], None, _sd((4,)))
    assert not lin.any() and not prec.any()


def test_sample_given_parameters_uses_the_keys_normal_noise():
    lin = np.array([0.3, -1.2, 0.0, 2.0], np.float32)
    prec = np.array([1.0, 2.5, 0.8, 4.0], np.float32)
    key = jax_prng.as_key_data(17)
    out, st = GaussianConditional().sample_given_parameters(key, (lin, prec), None, _sd((4,)))
    noise = jax_prng.normal(key, (4,))
    want = np.sqrt(1.0 / prec) * noise + lin / prec
    assert st is None and out.dtype == np.float32
    np.testing.assert_allclose(out, want.astype(np.float32), rtol=1e-6, atol=1e-7)


def test_samples_follow_the_conditional_law():
    lin = np.full(20000, 0.6, np.float32)
    prec = np.full(20000, 2.0, np.float32)
    out, _ = GaussianConditional().sample_given_parameters(jax_prng.as_key_data(3), (lin, prec), None,
                                                           _sd((20000,)))
    assert abs(out.mean() - 0.3) < 4 * np.sqrt(0.5 / 20000)
    assert abs(out.var() - 0.5) < 0.03


@pytest.mark.parametrize("family", ["gaussian"])
def test_family_is_gaussian(family):
    assert GaussianConditional.family.value == family
