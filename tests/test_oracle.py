"""The oracle pinned against the reference: golden vectors made by the reference itself and the reference's own
known-answer tests (test.py:33-105), restated. CPU only."""
import glob
import math
import os

import numpy as np
import pytest
import torch

from oracle import fpa_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
NAMES = ("o", "dq", "dk", "dv", "dphi", "dpsi", "dbeta")
CASE_FILES = sorted(glob.glob(os.path.join(GOLDEN, "t*.npz"))) + [os.path.join(GOLDEN, "config1_t256_d32_fp32.npz")]


def random_field(B, H, T, seed, ties=False):
    """test.py:23-30."""
    g = torch.Generator().manual_seed(seed)
    phi = torch.randn(B, H, T, generator=g, dtype=torch.float64).cumsum(-1)
    if ties:
        phi = torch.round(phi)
    psi = phi + 0.5 * torch.randn(B, H, T, generator=g, dtype=torch.float64)
    beta = torch.rand(H, generator=g, dtype=torch.float64) + 0.5
    return phi.numpy(), psi.numpy(), beta.numpy()


def bias_by_loops(phi, psi, beta):
    """The definition as a scalar loop (test.py:33-42)."""
    B, H, T = phi.shape
    out = np.zeros((B, H, T, T))
    for b in range(B):
        for h in range(H):
            for t in range(T):
                for s in range(t):
                    m = min(phi[b, h, u] for u in range(s + 1, t + 1))
                    out[b, h, t, s] = beta[h] * min(0.0, m - psi[b, h, s])
    return out


@pytest.mark.parametrize("path", CASE_FILES, ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_matches_reference_golden(path):
    z = np.load(path)
    o, _ = O.forward(z["q"], z["k"], z["v"], z["phi"], z["psi"], z["beta"])
    grads = O.backward(z["q"], z["k"], z["v"], z["phi"], z["psi"], z["beta"], z["do"], float(z["tau"]))
    for name, x in zip(NAMES, (o,) + tuple(grads)):
        assert O.rel_err(x, z[name]) < 1e-12, (name, O.rel_err(x, z[name]))


def test_bias_is_the_definition():
    z = np.load(os.path.join(GOLDEN, "bias_kat.npz"))
    for ties in (0, 1):
        phi, psi, beta = z[f"phi{ties}"], z[f"psi{ties}"], z[f"beta{ties}"]
        loops = bias_by_loops(phi, psi, beta)
        assert np.array_equal(O.bias(phi, psi, beta), loops)
        assert np.array_equal(z[f"bias{ties}"], loops)          # the golden made by the reference itself


def test_attention_is_softmax_with_the_bias():
    """test.py:51-63."""
    B, H, T, D = 2, 3, 10, 8
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(B, H, T, D, generator=g, dtype=torch.float64).numpy() for _ in range(3))
    phi, psi, beta = random_field(B, H, T, seed=4)
    bias = bias_by_loops(phi, psi, beta)
    o = np.zeros((B, H, T, D))
    for t in range(T):
        logits = (q[:, :, t:t + 1] @ np.swapaxes(k[:, :, :t + 1], -1, -2))[:, :, 0] / math.sqrt(D)
        logits = logits + bias[:, :, t, :t + 1]
        w = np.exp(logits - logits.max(-1, keepdims=True))
        w /= w.sum(-1, keepdims=True)
        o[:, :, t] = (w[:, :, None, :] @ v[:, :, :t + 1])[:, :, 0]
    got, _ = O.forward(q, k, v, phi, psi, beta)
    assert np.allclose(got, o, rtol=1e-12, atol=1e-12)


def test_gradient_of_the_bias():
    """test.py:66-84: the explicit soft-min gradient through the attention's dS at tau = 0.7.

    The oracle's backward takes dS from the attention; here a bias-only objective sum(bias * G) is recovered by
    choosing v, do so that the loop below is the whole gradient: the oracle's internal formula is exercised
    through _softmin_grad_phi directly."""
    B, H, T, tau = 1, 2, 9, 0.7
    phi, psi, beta = random_field(B, H, T, seed=5)
    G = torch.randn(B, H, T, T, generator=torch.Generator().manual_seed(6), dtype=torch.float64).numpy()
    e_phi = np.zeros_like(phi)
    for h in range(H):
        for t in range(T):
            for s in range(t):
                rng = phi[0, h, s + 1:t + 1]
                x = rng.min() - psi[0, h, s]
                if x <= 0:
                    w = np.exp(-rng / tau - (-rng / tau).max())
                    e_phi[0, h, s + 1:t + 1] += beta[h] * G[0, h, t, s] * w / w.sum()
    x = O.range_min(phi) - psi[..., None, :]
    strict = np.tril(np.ones((T, T), dtype=bool), -1)
    for h in range(H):
        g = np.where(strict & (x[0, h] <= 0), G[0, h], 0.0)
        got = beta[h] * O._softmin_grad_phi(g, phi[0, h], tau)
        assert np.allclose(got, e_phi[0, h], rtol=1e-10, atol=1e-12)


def test_causal():
    """test.py:87-97: outputs up to t0 do not depend on later positions."""
    B, H, T, D, t0 = 1, 2, 16, 8, 9
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(B, H, T, D, generator=g, dtype=torch.float64).numpy() for _ in range(3))
    phi, psi, beta = random_field(B, H, T, seed=8)
    o, _ = O.forward(q, k, v, phi, psi, beta)
    later = [x.copy() for x in (q, k, v, phi, psi)]
    for x in later:
        x[:, :, t0 + 1:] = np.random.default_rng(0).standard_normal(x[:, :, t0 + 1:].shape) * 10
    o2, _ = O.forward(*later, beta)
    assert np.array_equal(o[:, :, :t0 + 1], o2[:, :, :t0 + 1])


def test_bias_never_rises():
    """test.py:100-105: for a fixed key, the bias is non-increasing in the query position."""
    phi, psi, beta = random_field(2, 3, 24, seed=10)
    b = O.bias(phi, psi, beta)
    T = phi.shape[-1]
    keys = np.tril(np.ones((T, T), dtype=bool))[:-1]
    assert (b[:, :, 1:][..., keys] <= b[:, :, :-1][..., keys]).all()


def test_oracle_stable_for_extreme_fields():
    """A field scaled by 1e3 (exp(-phi) far outside float64) still gives finite soft-min gradients."""
    B, H, T, D = 1, 1, 48, 8
    g = torch.Generator().manual_seed(21)
    q, k, v, do = (torch.randn(B, H, T, D, generator=g, dtype=torch.float64).numpy() for _ in range(4))
    phi = torch.randn(B, H, T, generator=g, dtype=torch.float64).cumsum(-1).numpy() * 1e3
    psi = phi + 300 * torch.randn(B, H, T, generator=g, dtype=torch.float64).numpy()
    grads = O.backward(q, k, v, phi, psi, np.ones(H), do)
    assert all(np.isfinite(x).all() for x in grads)


@pytest.mark.parametrize("path", CASE_FILES[:3])
def test_single_row_forward_matches_the_golden_rows(path):
    """forward_row (the O(T*D) one-row evaluation the long-context GPU test uses) reproduces the reference's own
    outputs row by row, including the first and last rows."""
    z = np.load(path)
    q, k, v, phi, psi, beta = (z[n] for n in ("q", "k", "v", "phi", "psi", "beta"))
    B, H, T, D = q.shape
    beta = np.broadcast_to(np.asarray(beta, dtype=np.float64).reshape(-1), (H,))
    for b in range(B):
        for h in range(H):
            for t in sorted({0, 1, T // 2, T - 1}):
                row = O.forward_row(q[b, h], k[b, h], v[b, h], phi[b, h], psi[b, h], beta[h], t)
                assert np.allclose(row, z["o"][b, h, t], rtol=0, atol=1e-10 * max(1.0, np.abs(z["o"]).max()))
