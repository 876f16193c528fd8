"""Generate the golden fixtures in this folder from the reference implementation itself.

Run where the reference checkout is available, with its path in FPA_REFERENCE:

    FPA_REFERENCE=<reference checkout> python tests/golden/make_golden.py

It imports the reference ``kernel.py`` and evaluates its float64 PyTorch path (``impl="reference"``,
``kernel.py:44-64``) with torch autograd on seeded inputs drawn as the reference tests draw them (``test.py:108-117``)
and as the benchmark configurations describe them. The results are written as ``*.npz`` next to this script. The
tests read only the ``.npz`` files; nothing at test time needs the reference checkout.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("FPA_REFERENCE")


def _reference():
    if not REF:
        raise SystemExit("set FPA_REFERENCE to the reference checkout (the folder holding its kernel.py)")
    sys.path.insert(0, REF)
    import kernel  # noqa: E402  (the reference module)
    return kernel


def test_inputs(B, H, T, D, phi_scale=1.0, ties=False, seed=0, dtype=torch.float16):
    """``test.py:108-117``: q, k, v, do are rounded to the kernel dtype; phi, psi, beta stay fp32."""
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, H, T, D, generator=g).to(dtype) for _ in range(3))
    phi = torch.randn(B, H, T, generator=g).cumsum(-1) * phi_scale
    if ties:
        phi = torch.round(phi)
    psi = phi + 0.5 * torch.randn(B, H, T, generator=g)
    beta = torch.rand(H, generator=g) + 0.5
    do = torch.randn(B, H, T, D, generator=g).to(dtype)
    return q, k, v, phi, psi, beta, do


def config1_inputs():
    """Benchmark configuration 1: B1 H2 T256 D32 fp32; phi = cumsum N(0,1); psi = phi + N(0,1); beta = 1;
    backward of o.sum() (do = ones)."""
    g = torch.Generator().manual_seed(0)
    B, H, T, D = 1, 2, 256, 32
    q, k, v = (torch.randn(B, H, T, D, generator=g) for _ in range(3))
    phi = torch.randn(B, H, T, generator=g).cumsum(-1)
    psi = phi + torch.randn(B, H, T, generator=g)
    beta = torch.ones(H)
    do = torch.ones(B, H, T, D)
    return q, k, v, phi, psi, beta, do


def run_reference(kernel, q, k, v, phi, psi, beta, do, tau):
    r = [t.detach().double().requires_grad_() for t in (q, k, v, phi, psi, beta)]
    o = kernel.first_passage_attention(*r, tau=tau, impl="reference")
    grads = torch.autograd.grad(o, r, do.double())
    return [o.detach()] + list(grads)


CASES = {
    # name: (inputs, tau, dtype of q/k/v/do as the kernels see them)
    "t64_d16_fp16_s100": (lambda: test_inputs(1, 2, 64, 16, seed=100), 1.0, "f16"),
    "t100_d32_fp16_s101": (lambda: test_inputs(2, 3, 100, 32, seed=101), 1.0, "f16"),
    "t96_d16_scale40_s103": (lambda: test_inputs(1, 2, 96, 16, 40.0, seed=103), 1.0, "f16"),
    "t96_d16_ties_s104": (lambda: test_inputs(1, 2, 96, 16, ties=True, seed=104), 1.0, "f16"),
    "t72_d32_fp32_tau025_s11": (lambda: test_inputs(1, 2, 72, 32, seed=11, dtype=torch.float32), 0.25, "f32"),
    "t130_d16_fp32_scale40_s112": (lambda: test_inputs(1, 2, 130, 16, 40.0, seed=112, dtype=torch.float32), 1.0, "f32"),
    "config1_t256_d32_fp32": (config1_inputs, 1.0, "f32"),
}


def make_cases(kernel):
    for name, (mk, tau, dt) in CASES.items():
        q, k, v, phi, psi, beta, do = mk()
        o, dq, dk, dv, dphi, dpsi, dbeta = run_reference(kernel, q, k, v, phi, psi, beta, do, tau)
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            q=q.float().numpy(), k=k.float().numpy(), v=v.float().numpy(), do=do.float().numpy(),
            phi=phi.numpy(), psi=psi.numpy(), beta=beta.numpy(), tau=np.float64(tau), dtype=np.array(dt),
            o=o.numpy(), dq=dq.numpy(), dk=dk.numpy(), dv=dv.numpy(),
            dphi=dphi.numpy(), dpsi=dpsi.numpy(), dbeta=dbeta.numpy())
        print(name, tuple(q.shape))


def make_bias_kat(kernel):
    """``test.py:45-48``: the bias of small fields, with and without ties."""
    out = {}
    for ties in (False, True):
        g = torch.Generator().manual_seed(1 + ties)
        phi = torch.randn(2, 3, 12, generator=g, dtype=torch.float64).cumsum(-1)
        if ties:
            phi = torch.round(phi)
        psi = phi + 0.5 * torch.randn(2, 3, 12, generator=g, dtype=torch.float64)
        beta = torch.rand(3, generator=g, dtype=torch.float64) + 0.5
        b = kernel.first_passage_bias(phi, psi, beta)
        out.update({f"phi{int(ties)}": phi.numpy(), f"psi{int(ties)}": psi.numpy(),
                    f"beta{int(ties)}": beta.numpy(), f"bias{int(ties)}": b.numpy()})
    np.savez_compressed(os.path.join(HERE, "bias_kat.npz"), **out)
    print("bias_kat")


def make_layer(kernel):
    """``test.py:177-197``: the reference layer (impl="reference", fp32) at d_model 64, 4 heads, T 50."""
    torch.manual_seed(0)
    layer = kernel.FirstPassageAttention(64, 4, impl="reference")
    x = torch.randn(2, 50, 64, generator=torch.Generator().manual_seed(1))
    y = layer(x)
    loss = y.float().square().mean()
    grads = torch.autograd.grad(loss, list(layer.parameters()))
    names = [n for n, _ in layer.named_parameters()]
    state = {f"param:{n}": p.detach().numpy() for n, p in layer.named_parameters()}
    np.savez_compressed(os.path.join(HERE, "layer_d64_h4_t50.npz"), x=x.numpy(), y=y.detach().numpy(),
                        names=np.array(names), **state,
                        **{f"grad:{n}": g.numpy() for n, g in zip(names, grads)})
    print("layer", names)


if __name__ == "__main__":
    ref = _reference()
    make_cases(ref)
    make_bias_kat(ref)
    make_layer(ref)
