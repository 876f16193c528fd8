"""CPU oracle for First Passage Attention: a float64 NumPy restatement of the reference path.

TEST INFRASTRUCTURE ONLY. This module is the checker that the CUDA kernels are compared against. Only the tests, the
smoke check in ``__graft_entry__`` and the CPU-baseline leg of ``bench.py`` may import it; the library never does.

It restates the math of the reference implementation (yliu-fort/first-passage-attention, ``kernel.py``):

* ``range_min``        -- ``kernel.py:31-34``: m[t, s] = min_{s<u<=t} phi_u, +inf for the empty range (s >= t).
* ``bias``             -- ``kernel.py:44-54``: b[t, s] = beta * min(0, m[t, s] - psi_s); the hard minimum in value.
* ``forward``          -- ``kernel.py:57-64``: causal softmax of q k^T / sqrt(D) + b, times v.
* ``backward``         -- the gradients that autograd takes through ``kernel.py:44-64``: the exact gradients for
                          q, k, v, psi and beta, and for phi the soft-minimum gradient of ``kernel.py:37-41,53``
                          (``README.md:13``): dphi_u = beta * sum_{s<u<=t, x_ts<=0} dS_ts * softmax_{u'in(s,t]}(-phi/tau)_u.

The gradient for phi is evaluated with a reverse recurrence over t for each key s, in which every factor is a ratio
of partial sums Z_{s,t} = sum_{s<u<=t} exp(-phi_u/tau) that lies in [0, 1]; it never forms exp(-phi/tau) itself and
so stays finite for any field (the reference tests use fields scaled by 40, ``test.py:138,142``).

Everything is float64 and per head; memory is O(T^2) per head, so the oracle is meant for T up to a few thousand.
"""
import math

import numpy as np

LOG2E = 1.4426950408889634


def _f64(x):
    return np.asarray(x, dtype=np.float64)


def range_min(phi):
    """m[..., t, s] = min_{s<u<=t} phi_u (inf where s >= t). ``kernel.py:31-34``."""
    phi = _f64(phi)
    T = phi.shape[-1]
    s_idx = np.arange(T)[:, None]
    u_idx = np.arange(T)[None, :]
    y = np.where(u_idx > s_idx, phi[..., None, :], np.inf)        # [..., s, u]
    m = np.minimum.accumulate(y, axis=-1)                           # [..., s, t] = min over s<u<=t
    return np.swapaxes(m, -1, -2)                                   # [..., t, s]


def _beta_hw(beta, H):
    beta = _f64(beta).reshape(-1)
    if beta.size == 1:
        beta = np.full(H, beta.item())
    assert beta.shape == (H,)
    return beta


def bias(phi, psi, beta):
    """b[b, h, t, s] = beta_h * min(0, min_{s<u<=t} phi_u - psi_s); 0 on the diagonal. ``kernel.py:44-54``."""
    phi, psi = _f64(phi), _f64(psi)
    H = phi.shape[1]
    x = range_min(phi) - psi[..., None, :]
    return _beta_hw(beta, H)[None, :, None, None] * np.minimum(x, 0.0)


def forward(q, k, v, phi, psi, beta):
    """(o, lse) with o [B,H,T,D] and lse [B,H,T] (natural log) of the causal FPA softmax. ``kernel.py:57-64``."""
    q, k, v = _f64(q), _f64(k), _f64(v)
    T, D = q.shape[-2], q.shape[-1]
    s = q @ np.swapaxes(k, -1, -2) * D ** -0.5 + bias(phi, psi, beta)
    causal = np.tril(np.ones((T, T), dtype=bool))
    s = np.where(causal, s, -np.inf)
    m = s.max(-1, keepdims=True)
    e = np.exp(s - m)
    l = e.sum(-1, keepdims=True)
    p = e / l
    return p @ v, (m + np.log(l))[..., 0]


def forward_row(q, k, v, phi, psi, beta, t):
    """o[t] of one head (q, k, v [T, D]; phi, psi [T]; beta a scalar) in O(T*D): the same definition as ``forward``
    (``kernel.py:44-64``) for one query row. For a fixed t, min_{s<u<=t} phi_u as a function of s is the running
    minimum of phi taken backwards from t, so the row's bias needs no [T, T] table. Lets long contexts (T = 16383)
    be checked at late rows at full size."""
    q, k, v, phi, psi = _f64(q), _f64(k), _f64(v), _f64(phi), _f64(psi)
    D = q.shape[-1]
    m = np.empty(t + 1)
    m[t] = np.inf                                                   # empty range on the diagonal
    if t > 0:
        m[:t] = np.minimum.accumulate(phi[1:t + 1][::-1])[::-1]     # m[s] = min(phi[s+1 .. t])
    s = k[:t + 1] @ q[t] * D ** -0.5 + float(beta) * np.minimum(m - psi[:t + 1], 0.0)
    e = np.exp(s - s.max())
    return (e / e.sum()) @ v[:t + 1]


def _softmin_grad_phi(g, phi, tau):
    """R[u] = sum_{s<u<=t} g[t, s] * exp(a_u) / Z_{s,t}, a = -phi/tau, for one head (g: [T, T] indexed [t, s]).

    Reverse recurrence per key s: H_s(u) = g[u, s] + (Z_{s,u} / Z_{s,u+1}) H_s(u+1), and
    R[u] = sum_{s<u} (exp(a_u) / Z_{s,u}) H_s(u). All ratios are in [0, 1]."""
    T = phi.shape[-1]
    a = -_f64(phi) / tau
    s_idx = np.arange(T)[:, None]
    u_idx = np.arange(T)[None, :]
    y = np.where(u_idx > s_idx, a[None, :], -np.inf)               # [s, u]
    L = np.logaddexp.accumulate(y, axis=-1)                         # L[s, t] = log Z_{s,t} (-inf for t <= s)
    R = np.zeros(T)
    Hs = np.zeros(T)
    with np.errstate(invalid="ignore"):
        _reverse_scan(T, L, a, g, Hs, R)
    return R


def _reverse_scan(T, L, a, g, Hs, R):
    for t in range(T - 1, 0, -1):
        valid = np.arange(T) < t                                    # keys s < t
        if t < T - 1:
            rho = np.where(valid, np.exp(np.where(valid, L[:, t] - L[:, t + 1], 0.0)), 0.0)
            Hs = rho * Hs
        Hs = Hs + np.where(valid, g[t, :], 0.0)
        w = np.where(valid, np.exp(np.where(valid, a[t] - L[:, t], 0.0)), 0.0)
        R[t] = np.dot(w, Hs)


def backward(q, k, v, phi, psi, beta, do, tau=1.0):
    """(dq, dk, dv, dphi, dpsi, dbeta) of sum(o * do), as autograd gives them through ``kernel.py:44-64``.

    dbeta is summed over the batch, shape (H,), as ``kernel.py:450`` returns it."""
    if not tau > 0:
        raise ValueError("tau must be positive")
    q, k, v, do = _f64(q), _f64(k), _f64(v), _f64(do)
    phi, psi = _f64(phi), _f64(psi)
    B, H, T, D = q.shape
    betah = _beta_hw(beta, H)
    scale = D ** -0.5
    m = range_min(phi)
    x = m - psi[..., None, :]                                       # [B,H,t,s]
    b = betah[None, :, None, None] * np.minimum(x, 0.0)
    s = q @ np.swapaxes(k, -1, -2) * scale + b
    causal = np.tril(np.ones((T, T), dtype=bool))
    strict = np.tril(np.ones((T, T), dtype=bool), -1)
    s = np.where(causal, s, -np.inf)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    o = p @ v
    dv = np.swapaxes(p, -1, -2) @ do
    dp = do @ np.swapaxes(v, -1, -2)
    delta = (do * o).sum(-1, keepdims=True)
    ds = p * (dp - delta)
    dq = ds @ k * scale
    dk = np.swapaxes(ds, -1, -2) @ q * scale
    gate = strict & (x <= 0.0)
    g = np.where(gate, ds, 0.0)                                     # gradient reaching min(x, 0), per unit beta
    dpsi = -betah[None, :, None] * g.sum(-2)
    dbeta = np.where(strict, ds * np.minimum(x, 0.0), 0.0).sum((0, 2, 3))
    dphi = np.zeros((B, H, T))
    for bi in range(B):
        for h in range(H):
            dphi[bi, h] = betah[h] * _softmin_grad_phi(g[bi, h], phi[bi, h], tau)
    return dq, dk, dv, dphi, dpsi, dbeta


def make_inputs(B, H, T, D, phi_scale=1.0, ties=False, seed=0):
    """Inputs drawn exactly as ``test.py:108-117`` draws them (torch CPU generator), returned as float64 NumPy
    arrays of the values the kernels see (q, k, v, do already rounded to fp16 where the case is fp16 is up to the
    caller). Requires torch only for the generator."""
    import torch
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, H, T, D, generator=g) for _ in range(3))
    phi = torch.randn(B, H, T, generator=g).cumsum(-1) * phi_scale
    if ties:
        phi = torch.round(phi)
    psi = phi + 0.5 * torch.randn(B, H, T, generator=g)
    beta = torch.rand(H, generator=g) + 0.5
    do = torch.randn(B, H, T, D, generator=g)
    return [t.numpy() for t in (q, k, v, phi, psi, beta, do)]


def rel_err(x, ref):
    """max|x - ref| / max|ref|, the normwise metric of ``test.py:120-121``."""
    x, ref = _f64(x), _f64(ref)
    return float(np.abs(x - ref).max() / max(np.abs(ref).max(), 1e-30))


def flops(B, H, T, D, which="fwd"):
    """Algorithmic FLOPs in the causal FlashAttention convention: fwd 2*B*H*T^2*D, fwd+bwd 3.5x that."""
    f = 2.0 * B * H * T * T * D
    return f if which == "fwd" else 3.5 * f


if __name__ == "__main__":
    args = make_inputs(1, 2, 64, 16, seed=0)
    o, lse = forward(*args[:6])
    print("o", o.shape, float(np.abs(o).max()), "lse", float(lse.mean()), math.isfinite(float(lse.sum())))
