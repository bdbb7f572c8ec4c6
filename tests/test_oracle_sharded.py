"""The oracle's restatement of the long-axis sharded Gram chain (CPU only).

``gram_iterations`` is one restart-free segment of the reference's Gram loop
(newton_schulz.py:177-212); chaining segments at the reset iterations must give
``gram_newton_schulz`` bit for bit, and the sharded restatement over a single
shard must too. Over several shards only the summation order of the norm and
the Gram matrix changes, so the result stays within the parity bar.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import gns_oracle as G

PARITY_TOL = 2e-2


def _matrices(shape, seed):
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32)


@pytest.mark.parametrize("shape", [(2, 24, 40), (2, 40, 24)])
@pytest.mark.parametrize("resets", [(), (2,), (1, 3), (2, 4)])
def test_segments_compose_to_gram_newton_schulz(shape, resets):
    x = _matrices(shape, 7)
    coeffs = G.polar_express_coefficients()
    expected = G.gram_newton_schulz(x, coeffs, resets, 1e-7)
    tall = shape[-2] > shape[-1]
    xh = G.normalize(x, 1e-7)
    xt = np.swapaxes(xh, -1, -2)
    gram = G.baddbmm(None, xt, xh) if tall else G.baddbmm(None, xh, xt)
    n = len(coeffs)
    begin = 0
    for end in sorted({i for i in resets if 0 < i < n}) + [n]:
        q = G.gram_iterations(gram, coeffs, begin, end)
        xh = G.baddbmm(None, xh, q) if tall else G.baddbmm(None, q, xh)
        if end < n:
            xt = np.swapaxes(xh, -1, -2)
            gram = G.baddbmm(None, xt, xh) if tall else G.baddbmm(None, xh, xt)
        begin = end
    np.testing.assert_array_equal(xh, expected)


@pytest.mark.parametrize("tall", [False, True])
def test_single_shard_is_gram_newton_schulz(tall):
    shape = (3, 48, 20) if tall else (3, 20, 48)
    x = _matrices(shape, 11)
    got = G.long_axis_sharded_gram_newton_schulz([x], tall)
    np.testing.assert_array_equal(got[0], G.gram_newton_schulz(x))


@pytest.mark.parametrize("tall", [False, True])
@pytest.mark.parametrize("splits", [(16, 16), (20, 7, 5), (1, 31)])
def test_sharded_matches_whole_matrix(tall, splits):
    long = sum(splits)
    shape = (2, long, 12) if tall else (2, 12, long)
    x = _matrices(shape, 5)
    axis = -2 if tall else -1
    shards = np.split(x, np.cumsum(splits)[:-1], axis=axis)
    got = np.concatenate(G.long_axis_sharded_gram_newton_schulz(shards, tall), axis=axis)
    assert G.relative_error(got, G.gram_newton_schulz(x)) < PARITY_TOL


def test_empty_iteration_range_rejected():
    with pytest.raises(ValueError):
        G.gram_iterations(np.eye(4, dtype=np.float32), G.polar_express_coefficients(), 2, 2)
