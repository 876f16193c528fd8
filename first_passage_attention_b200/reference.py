"""The PyTorch definition of FPA: ``impl="reference"`` of the operator and the public ``first_passage_bias``.

It evaluates the definition densely ([B, H, T, T] tensors) with PyTorch autograd, in float64 when any input is
float64 and float32 otherwise, on any device (kernel.py:23-64 defines the same function):

* the value of the bias uses the hard range minimum min_{s<u<=t} phi_u (a masked running minimum, ``cummin``);
* its gradient for phi is that of the soft minimum -tau * log sum_{s<u<=t} exp(-phi_u / tau) (``logcumsumexp``),
  joined to the hard value by a straight-through term (soft - soft.detach()).
"""
import torch

_MASKED = 1e30  # stands for -inf in the log-sum-exp so the masked entries get exactly zero weight and no NaN


def _compute_dtype(*xs):
    return torch.float64 if any(x.dtype == torch.float64 for x in xs) else torch.float32


def _strictly_after(T, device):
    """after[s, u] = u > s."""
    idx = torch.arange(T, device=device)
    return idx[None, :] > idx[:, None]


def range_min(phi):
    """m[..., t, s] = min_{s<u<=t} phi_u, +inf where the range is empty (s >= t)."""
    T = phi.shape[-1]
    rows = phi.unsqueeze(-2).expand(*phi.shape[:-1], T, T)
    rows = rows.masked_fill(~_strictly_after(T, phi.device), float("inf"))
    return torch.cummin(rows, dim=-1).values.transpose(-1, -2)


def range_softmin(phi, tau):
    """-tau * log sum_{s<u<=t} exp(-phi_u / tau), indexed [..., t, s] (a huge value where the range is empty)."""
    T = phi.shape[-1]
    rows = (-phi / tau).unsqueeze(-2).expand(*phi.shape[:-1], T, T)
    rows = rows.masked_fill(~_strictly_after(T, phi.device), -_MASKED)
    return (-tau * torch.logcumsumexp(rows, dim=-1)).transpose(-1, -2)


def first_passage_bias(phi, psi, beta, tau=1.0):
    """The bias (B, H, T, T), indexed [t, s], of phi and psi (B, H, T) and beta (H,); tau enters only the gradient."""
    if not tau > 0:
        raise ValueError("tau must be positive")
    dt = _compute_dtype(phi, psi)
    phi, psi = phi.to(dt), psi.to(dt)
    if torch.is_tensor(beta):
        beta = beta.reshape(-1, 1, 1)
    soft = range_softmin(phi, tau)
    x = range_min(phi).detach() + (soft - soft.detach()) - psi.unsqueeze(-2)
    return beta * torch.clamp(x, max=0.0)


def causal_attention(q, k, v, bias):
    """softmax(q k^T / sqrt(D) + bias, causal) v, computed with autocast off; returned in q's dtype."""
    dt = _compute_dtype(q, bias)
    T = q.shape[-2]
    with torch.autocast(device_type=q.device.type, enabled=False):
        s = (q.to(dt) @ k.to(dt).transpose(-1, -2)) * q.shape[-1] ** -0.5 + bias.to(dt)
        causal = torch.ones(T, T, dtype=torch.bool, device=q.device).tril()
        s = s.masked_fill(~causal, float("-inf"))
        return (s.softmax(-1) @ v.to(dt)).to(q.dtype)


def first_passage_attention_reference(q, k, v, phi, psi, beta, tau=1.0):
    return causal_attention(q, k, v, first_passage_bias(phi, psi, beta, tau))
