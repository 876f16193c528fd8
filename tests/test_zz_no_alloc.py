"""fpa_fwd_noalloc: the forward entry point for callers that cannot allocate device memory.

Such callers (a plugin host that passes only the input and output buffers, a runtime whose device memory is fully
reserved, code that must not allocate once it is running) cannot provide the workspace fpa_fwd asks for. This
entry point keeps that scratch in a device array built into the library instead. The test makes the set-up call
first (which creates the array in this context), then calls the entry point through the C ABI twice in a row, on
different inputs, and checks that each result equals fpa_fwd's with a workspace bit for bit (the same kernels on
the same inputs: any difference would mean the shared scratch leaked state from the previous call), that the
status word in the built-in array reads FPA_OK after each call, and that the device's free memory does not drop
across the calls. It also checks that a call too large for the built-in array is refused without launching anything.

The file name sorts last so that a run stopping at the first failure has run every other test before it.
"""
import ctypes

import pytest
import torch

from first_passage_attention_b200 import _lib

pytestmark = pytest.mark.gpu


def _inputs(B, H, T, D, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, H, T, D, generator=g).half().cuda() for _ in range(3))
    phi = torch.randn(B, H, T, generator=g).cumsum(-1).cuda()
    psi = (phi.cpu() + torch.randn(B, H, T, generator=g)).cuda()
    beta = (torch.rand(H, generator=g) + 0.5).cuda()
    return q, k, v, phi, psi, beta


def _args(q, k, v, phi, psi, beta, o, lse, workspace=None, nbytes=0):
    B, H, T, D = q.shape
    s = lambda t: (ctypes.c_int64 * 4)(*t.stride())  # noqa: E731
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    return _lib.FpaFwdArgs(dtype=_lib.DTYPE_F16, path=_lib.PATH_AUTO, B=B, H=H, T=T, D=D, tau=1.0,
                           q=p(q), q_stride=s(q), k=p(k), k_stride=s(k), v=p(v), v_stride=s(v),
                           phi=p(phi), psi=p(psi), beta=p(beta), o=p(o), o_stride=s(o), lse=p(lse),
                           workspace=None if workspace is None else p(workspace), workspace_bytes=nbytes)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_noalloc_forward_matches_the_workspace_forward():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    lib = _lib.load()
    cases = []
    for call, (B, H, T, D) in enumerate([(2, 3, 640, 64), (1, 4, 300, 128)]):
        q, k, v, phi, psi, beta = _inputs(B, H, T, D, seed=900 + call)
        o_ref = torch.empty_like(q)
        lse_ref = torch.empty(B, H, T, device="cuda")
        nbytes = lib.fpa_fwd_workspace_bytes(_lib.DTYPE_F16, B, H, T, D, _lib.PATH_AUTO)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        a = _args(q, k, v, phi, psi, beta, o_ref, lse_ref, ws, nbytes)
        _lib.check(lib.fpa_fwd(ctypes.byref(a), _stream()))
        o = torch.full_like(q, float("nan"))
        lse = torch.full((B, H, T), float("nan"), device="cuda")
        keep = (q, k, v, phi, psi, beta, ws)   # the argument blocks hold raw pointers: keep the tensors alive
        cases.append((a, o_ref, lse_ref, _args(q, k, v, phi, psi, beta, o, lse), o, lse, keep))
    _lib.check(lib.fpa_fwd_noalloc(None, _stream()))   # set-up: creates the built-in array, launches nothing
    for a, o_ref, lse_ref, b, o, lse, _ in cases:
        # Free device memory right around the call (torch's own allocations for the checks come after).
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        _lib.check(lib.fpa_fwd_noalloc(ctypes.byref(b), _stream()))
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] >= free_before
        assert b.workspace is not None                       # the call reports the built-in array it used
        assert lib.fpa_workspace_status(ctypes.c_void_p(b.workspace), _stream()) == _lib.OK
        assert b.kernels_launched == a.kernels_launched > 0
        assert torch.equal(o, o_ref)
        assert torch.equal(lse, lse_ref)


def test_noalloc_refuses_calls_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    lib = _lib.load()
    B, H, T, D = 64, 16, 4096, 64   # needs far more than the built-in scratch; no tensor is touched
    need = lib.fpa_fwd_workspace_bytes(_lib.DTYPE_F16, B, H, T, D, _lib.PATH_AUTO)
    assert need > _lib.NOALLOC_SCRATCH_BYTES
    dummy = torch.empty(16, device="cuda")
    p = ctypes.c_void_p(dummy.data_ptr())
    z = (ctypes.c_int64 * 4)(T * D * H, T * D, D, 1)
    a = _lib.FpaFwdArgs(dtype=_lib.DTYPE_F16, path=_lib.PATH_AUTO, B=B, H=H, T=T, D=D, tau=1.0,
                        q=p, q_stride=z, k=p, k_stride=z, v=p, v_stride=z, phi=p, psi=p, beta=p,
                        o=p, o_stride=z, lse=p)
    rc = lib.fpa_fwd_noalloc(ctypes.byref(a), _stream())
    assert rc == _lib.ERR_WORKSPACE
    assert a.kernels_launched == 0
    assert b"built into the library" in lib.fpa_last_error()
