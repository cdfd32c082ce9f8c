"""The speculative acceptance step's oracle (oracle/gdn_oracle.py:
spec_residual, spec_verify) on the CPU: pinned to the reference's own
``residual`` (python/speculative.py:100-106, golden vectors made by running
it), and the property the reference's selftest proves
(python/speculative.py:256-283): summed over every draft token, accept-or-
resample reproduces the target distribution exactly."""
import numpy as np
import pytest

import gdn_oracle as O
from conftest import golden


def test_residual_matches_reference_golden():
    g = golden("spec_residual.npz")
    n = len([k for k in g if k.startswith("p")])
    assert n >= 18
    for i in range(n):
        r = O.spec_residual(g[f"p{i}"], g[f"q{i}"])
        assert np.max(np.abs(r - g[f"r{i}"])) < 1e-6, i


def test_rejection_marginal_equals_target():
    """speculative.py:256-283: for 200 random 6-way (p, q) pairs, the
    marginal of accept-else-residual over d ~ q equals p to 1e-5."""
    rng = np.random.default_rng(0)
    for _ in range(200):
        V = 6
        p = np.exp(rng.standard_normal(V) * 2)
        p /= p.sum()
        q = np.exp(rng.standard_normal(V) * 2)
        q /= q.sum()
        marg = np.zeros(V)
        for d in range(V):
            a = min(1.0, p[d] / q[d]) if q[d] > 0 else 1.0
            marg[d] += q[d] * a
            if a < 1.0:
                marg += q[d] * (1 - a) * O.spec_residual(p, q)
        assert np.max(np.abs(marg - p)) < 1e-5


def test_spec_verify_accept_length_and_inverse_cdf():
    p = np.array([[0.1, 0.6, 0.3], [0.2, 0.2, 0.6], [0.5, 0.25, 0.25]], np.float32)
    q = np.array([[0.2, 0.5, 0.3], [0.6, 0.2, 0.2]], np.float32)
    # draft 1 accepted (q<p), draft 0 of row 1: p/q = 1/3, accepted iff u <= 1/3
    assert O.spec_verify(p, q, [1, 0], [0.9, 0.2], 0.5)[:2] == (2, 3)
    j, n, v = O.spec_verify(p, q, [1, 0], [0.9, 0.5], 0.1)
    assert (j, n) == (1, 2)
    # residual of row 1: max(p - q, 0) = [0, 0, 0.4] -> token 2 whatever the uniform
    assert v == 2
    # all accepted: draw from p_2 by inverse CDF: 0.5 | 0.25 | 0.25
    assert O.spec_verify(p, q, [1, 2], [0.1, 0.1], 0.49)[2] == 0
    assert O.spec_verify(p, q, [1, 2], [0.1, 0.1], 0.51)[2] == 1
    assert O.spec_verify(p, q, [1, 2], [0.1, 0.1], 0.99)[2] == 2
    # q == 0 at the draft: accepted iff p > 0
    q0 = np.array([[0.5, 0.0, 0.5], [0.6, 0.2, 0.2]], np.float32)
    assert O.spec_verify(p, q0, [1, 0], [0.99, 0.0], 0.5)[0] == 2


@pytest.mark.parametrize("seed", range(5))
def test_empty_residual_falls_back_to_p(seed):
    rng = np.random.default_rng(seed)
    p = rng.dirichlet(np.ones(8)).astype(np.float32)
    P = np.stack([p, p]).astype(np.float32)
    Q = P[:1].copy()
    d = int(np.argmin(p))
    j, _, v = O.spec_verify(P, Q, [d], [2.0], 0.3)       # u * q > p: rejected
    assert j == 0
    assert v == int(np.searchsorted(np.cumsum(p.astype(np.float64)), 0.3 * p.sum(dtype=np.float64), side="right"))
