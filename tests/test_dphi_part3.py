"""The O(NB^2) evaluation of the strictly-between part of dphi that dphi_part3_kernel performs for long contexts,
restated in float64 NumPy and checked against the O(NB^3) sum it replaces (kernel.py:352-364): for every tile U,
    S_U = sum_{j < U < i} 2^{c_U - M(j, i)} TB[i][j],   M(j, i) = max_{j < n < i} c_n.
The restatement follows the kernel's passes: per key tile j, the suffix sums over query tiles i at each pair's scale,
then per tile U the sum over key tiles j < U, all kept as (m, v) = v 2^m with a running maximum."""
import numpy as np
import pytest


def part3_cubic(c, tb):
    nb = len(c)
    out = np.zeros(nb)
    for u in range(1, nb - 1):
        out[u] = sum(2.0 ** (c[u] - c[j + 1:i].max()) * tb[i, j] for i in range(u + 1, nb) for j in range(u))
    return out


def join(m, v, m2, v2):
    mm = max(m, m2)
    if mm == -np.inf:
        return mm, 0.0
    return mm, v * 2.0 ** (m - mm) + v2 * 2.0 ** (m2 - mm)


def part3_quadratic(c, tb):
    nb = len(c)
    pair = np.zeros((nb, nb, 2))  # the kernel reuses the first two floats of each pair's TB slot
    for j in range(nb - 2):
        for i in range(j + 2, nb):  # pass 1: the pair's value and -M(j, i)
            pair[i, j] = (tb[i, j], -c[j + 1:i].max())
        m, v = -np.inf, 0.0
        for i in range(nb - 1, j + 1, -1):  # pass 2: suffix sums C_j(i - 1) = sum_{i' >= i} X[i'][j]
            m, v = join(m, v, pair[i, j, 1], pair[i, j, 0])
            pair[i, j] = (v, m)
    out = np.zeros(nb)
    for u in range(1, nb - 1):  # pass 3: sum_{j < U} C_j(U), C_j(U) at pair (U + 1, j)
        m, v = -np.inf, 0.0
        for j in range(u):
            m, v = join(m, v, pair[u + 1, j, 1], pair[u + 1, j, 0])
        out[u] = 0.0 if v == 0.0 else v * 2.0 ** (m + c[u])
    return out


@pytest.mark.parametrize("nb", [1, 2, 3, 4, 9, 24])
@pytest.mark.parametrize("spread", [1.0, 60.0])
def test_quadratic_part3_matches_the_cubic_sum(nb, spread):
    rng = np.random.default_rng(nb * 7 + int(spread))
    c = np.cumsum(rng.standard_normal(nb)) * spread  # per-tile maxima of a2 over a random-walk field
    tb = rng.standard_normal((nb, nb))
    want, got = part3_cubic(c, tb), part3_quadratic(c, tb)
    assert np.allclose(got, want, rtol=1e-12, atol=1e-12 * max(np.abs(want).max(), 1e-300))
