"""The forward's key-range split: on grids too small to fill the GPU (few heads per call, as a GPU holds under the
strong split of configuration 2 over 4 or 8 ranks), each query tile's key tiles are cut into chunks of L tiles that
run on separate CTAs; the chunk that finishes last joins their partial outputs (row maximum, row sum, unnormalised
O) in chunk order, whichever chunk that is. The reference walks all key tiles of a query tile in one program
(kernel.py:104-162). The split changes only the order of the additions, so the checks are: o and lse against the
float64 oracle at the reference's fp16 tolerance, against the unsplit kernel (FPA_B200_FWD_SPLIT=0) to rounding,
the gradients through the split forward, repeat runs bit for bit, and the workspace rule of the C ABI (a workspace
sized without the split's room runs the unsplit kernel, bit for bit as FPA_B200_FWD_SPLIT=0 does)."""
import ctypes
import os

import numpy as np
import pytest
import torch

from first_passage_attention_b200 import LaunchStats, _lib, first_passage_attention
from first_passage_attention_b200.ops import fpa_forward
from oracle import fpa_oracle as O

pytestmark = pytest.mark.gpu

LOG2E = 1.4426950408889634


def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")


def inputs(B, H, T, D, seed, beta_sign=1.0):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, H, T, D, generator=g).half() for _ in range(3))
    phi = torch.randn(B, H, T, generator=g).cumsum(-1)
    psi = phi + 0.5 * torch.randn(B, H, T, generator=g)
    beta = beta_sign * (torch.rand(H, generator=g) + 0.5)
    do = torch.randn(B, H, T, D, generator=g).half()
    return q, k, v, phi, psi, beta, do


def forward(q, k, v, phi, psi, beta, split=True):
    """(o, lse, kernels launched) of the native forward on the GPU."""
    old = os.environ.get("FPA_B200_FWD_SPLIT")
    if not split:
        os.environ["FPA_B200_FWD_SPLIT"] = "0"
    try:
        LaunchStats.reset()
        o, lse = fpa_forward(*(x.cuda().contiguous() for x in (q, k, v)), phi.cuda().float().contiguous(),
                             psi.cuda().float().contiguous(), beta.cuda().float().contiguous(), 1.0)
        torch.cuda.synchronize()
        return o.cpu(), lse.cpu(), LaunchStats.kernels
    finally:
        if old is None:
            os.environ.pop("FPA_B200_FWD_SPLIT", None)
        else:
            os.environ["FPA_B200_FWD_SPLIT"] = old


# (B, H, T, D, beta sign): few heads, so the grid leaves SM slots idle and the split runs; ragged tails and every
# head dimension of the one-tile kernel; beta < 0 turns the field's minima into maxima.
SPLIT_CASES = [
    (1, 6, 2048, 64, 1.0),
    (1, 2, 1000, 32, 1.0),
    (1, 3, 777, 16, 1.0),
    (2, 1, 1500, 64, -1.0),
    (1, 1, 4100, 64, 1.0),
]


@pytest.mark.parametrize("B,H,T,D,sign", SPLIT_CASES)
def test_split_forward_matches_the_oracle_and_the_unsplit_kernels(B, H, T, D, sign):
    need_gpu()
    q, k, v, phi, psi, beta, _ = inputs(B, H, T, D, seed=T + D, beta_sign=sign)
    o, lse, n_split = forward(q, k, v, phi, psi, beta)
    o1, lse1, n_one = forward(q, k, v, phi, psi, beta, split=False)
    assert n_split == n_one              # the chunks join inside the kernel: no extra launch
    ref_o, ref_lse = O.forward(*(x.double().numpy() for x in (q, k, v, phi, psi, beta)))
    assert O.rel_err(o.double().numpy(), ref_o) <= 2e-3
    assert np.abs(lse.double().numpy() - ref_lse * LOG2E).max() <= 2e-3
    # Against the unsplit kernels: the same sums in another order, so fp16 rounding of o and float32 of lse.
    assert (o.float() - o1.float()).abs().max() <= 2e-3 * o1.float().abs().max()
    assert (lse - lse1).abs().max() <= 1e-4


def test_split_forward_gradients_match_the_oracle():
    need_gpu()
    q, k, v, phi, psi, beta, do = inputs(1, 2, 1200, 64, seed=5)
    a = [t.cuda().clone().requires_grad_() for t in (q, k, v, phi, psi, beta)]
    LaunchStats.reset()
    o = first_passage_attention(*a, impl="cuda")
    grads = torch.autograd.grad(o, a, do.cuda())
    n = [t.double().numpy() for t in (q, k, v, phi, psi, beta, do)]
    ref = [O.forward(*n[:6])[0]] + list(O.backward(*n))
    names = ("o", "dq", "dk", "dv", "dphi", "dpsi", "dbeta")
    for name, x, r in zip(names, [o.detach()] + list(grads), ref):
        tol = 1e-2 if name == "dbeta" else 2e-3
        assert O.rel_err(x.double().cpu().numpy(), r) <= tol, name


def _args(q, k, v, phi, psi, beta, o, lse, ws, nbytes):
    B, H, T, D = q.shape
    s = lambda t: (ctypes.c_int64 * 4)(*t.stride())  # noqa: E731
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    return _lib.FpaFwdArgs(dtype=_lib.DTYPE_F16, path=_lib.PATH_AUTO, B=B, H=H, T=T, D=D, tau=1.0,
                           q=p(q), q_stride=s(q), k=p(k), k_stride=s(k), v=p(v), v_stride=s(v),
                           phi=p(phi), psi=p(psi), beta=p(beta), o=p(o), o_stride=s(o), lse=p(lse),
                           workspace=p(ws), workspace_bytes=nbytes)


def test_workspace_without_the_split_room_runs_unsplit():
    """fpa_fwd_workspace_bytes includes the split's room on a small grid; a workspace of the size without it (what
    the query reports with FPA_B200_FWD_SPLIT=0) is accepted and runs the unsplit kernels."""
    need_gpu()
    lib = _lib.load()
    B, H, T, D = 1, 4, 2048, 64
    q, k, v, phi, psi, beta, _ = (x.cuda() for x in inputs(B, H, T, D, seed=11))
    phi, psi, beta = phi.float(), psi.float(), beta.float()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    full = lib.fpa_fwd_workspace_bytes(_lib.DTYPE_F16, B, H, T, D, _lib.PATH_AUTO)
    os.environ["FPA_B200_FWD_SPLIT"] = "0"
    try:
        small = lib.fpa_fwd_workspace_bytes(_lib.DTYPE_F16, B, H, T, D, _lib.PATH_AUTO)
        o_off, lse_off = torch.empty_like(q), torch.empty(B, H, T, device="cuda")
        ws_off = torch.empty(small, dtype=torch.uint8, device="cuda")
        a = _args(q, k, v, phi, psi, beta, o_off, lse_off, ws_off, small)
        _lib.check(lib.fpa_fwd(ctypes.byref(a), stream))
        n_off = a.kernels_launched
    finally:
        os.environ.pop("FPA_B200_FWD_SPLIT", None)
    assert full > small
    o_min, lse_min = torch.empty_like(q), torch.empty(B, H, T, device="cuda")
    ws_min = torch.empty(small, dtype=torch.uint8, device="cuda")
    b = _args(q, k, v, phi, psi, beta, o_min, lse_min, ws_min, small)
    _lib.check(lib.fpa_fwd(ctypes.byref(b), stream))
    o_full, lse_full = torch.empty_like(q), torch.empty(B, H, T, device="cuda")
    ws_full = torch.empty(full, dtype=torch.uint8, device="cuda")
    c = _args(q, k, v, phi, psi, beta, o_full, lse_full, ws_full, full)
    _lib.check(lib.fpa_fwd(ctypes.byref(c), stream))
    torch.cuda.synchronize()
    assert b.kernels_launched == n_off == c.kernels_launched
    assert torch.equal(o_min, o_off) and torch.equal(lse_min, lse_off)
    assert (o_full.float() - o_off.float()).abs().max() <= 2e-3 * o_off.float().abs().max()
    # Too small even for the unsplit kernels: refused.
    d = _args(q, k, v, phi, psi, beta, o_min, lse_min, ws_min, small - 256)
    assert lib.fpa_fwd(ctypes.byref(d), stream) == _lib.ERR_WORKSPACE



def test_split_forward_is_deterministic():
    need_gpu()
    q, k, v, phi, psi, beta, _ = inputs(1, 3, 2048, 64, seed=77)
    o1, l1, _ = forward(q, k, v, phi, psi, beta)
    o2, l2, _ = forward(q, k, v, phi, psi, beta)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
