"""The failure path of the bounded device-side waits, driven to expiry on the GPU without faulting or hanging it.

Every mbarrier wait of the tensor-core kernels is bounded: when its limit passes, the wait records FPA_ERR_TIMEOUT
and its call-site id in the workspace status word and returns, the kernel unwinds, and the host learns of it through
fpa_workspace_status. fpa_selftest_wait_timeout runs that same wait on an mbarrier nothing arrives on, with a short
limit. The test checks that the kernel returns, that the status word carries FPA_ERR_TIMEOUT with the self-test's
site id, that reading the status clears it, and that the next ordinary forward + backward on the same device still
matches the oracle (the context stays usable)."""
import ctypes

import pytest
import torch

from first_passage_attention_b200 import _lib, first_passage_attention
from oracle import fpa_oracle as O

pytestmark = pytest.mark.gpu

SELFTEST_SITE = 0x7E57


def test_a_bounded_wait_runs_out_and_is_reported():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    lib = _lib.load()
    ws = torch.empty(256, dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    wsp = ctypes.c_void_p(ws.data_ptr())
    assert lib.fpa_selftest_wait_timeout(wsp, 5_000_000, stream) == _lib.OK   # 5 ms
    torch.cuda.synchronize()
    words = ws[:8].view(torch.int32).cpu()
    assert int(words[1]) == 1, "the waiting kernel did not return through its timeout"
    assert (int(words[0]) >> 16) == _lib.ERR_TIMEOUT and (int(words[0]) & 0xFFFF) == SELFTEST_SITE
    rc = lib.fpa_workspace_status(wsp, stream)
    assert rc == _lib.ERR_TIMEOUT
    assert f"site {SELFTEST_SITE}".encode() in lib.fpa_last_error()
    assert lib.fpa_workspace_status(wsp, stream) == _lib.OK     # the read cleared the word

    # The device is still usable: an ordinary forward + backward matches the oracle.
    g = torch.Generator().manual_seed(3)
    q, k, v, do = (torch.randn(1, 2, 200, 64, generator=g).half() for _ in range(4))
    phi = torch.randn(1, 2, 200, generator=g).cumsum(-1)
    psi = phi + torch.randn(1, 2, 200, generator=g)
    beta = torch.rand(2, generator=g) + 0.5
    leaves = [t.cuda().requires_grad_() for t in (q, k, v, phi, psi, beta)]
    o = first_passage_attention(*leaves, impl="cuda")
    grads = torch.autograd.grad(o, leaves, do.cuda())
    n = [t.double().numpy() for t in (q, k, v, phi, psi, beta, do)]
    ref = [O.forward(*n[:6])[0]] + list(O.backward(*n))
    for name, x, r in zip(("o", "dq", "dk", "dv", "dphi", "dpsi", "dbeta"), [o] + list(grads), ref):
        tol = 1e-2 if name == "dbeta" else 2e-3
        assert O.rel_err(x.detach().double().cpu().numpy(), r) <= tol, name

