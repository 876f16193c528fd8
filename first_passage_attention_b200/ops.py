"""The FPA operator and layer: the drop-in host side of yliu-fort/first-passage-attention's ``kernel.py``.

``first_passage_attention(q, k, v, phi, psi, beta, tau=1.0, impl=None, block=64)`` keeps the reference signature,
argument checks and error messages (kernel.py:458-489). ``impl="cuda"`` (alias ``"triton"``, the reference's name
for its GPU path) runs the native sm_100a kernels of libfpa_b200 through its C ABI; ``impl="reference"`` evaluates
the dense PyTorch definition. ``impl=None`` picks the CUDA kernels for CUDA tensors and the definition otherwise
(kernel.py:463-464). There is no silent fallback: a CUDA request that the library cannot serve raises.
"""
import contextlib
import ctypes
import math
import os

import torch
from torch import nn
from torch.nn import functional as F

from . import _lib
from .reference import first_passage_attention_reference, first_passage_bias  # noqa: F401  (public API)

_KERNEL_IMPLS = ("cuda", "triton")


def _pow2(n):
    return n >= 16 and n & (n - 1) == 0


def _path_from_env():
    p = os.environ.get("FPA_B200_PATH", "auto").lower()
    return {"auto": _lib.PATH_AUTO, "simt": _lib.PATH_SIMT, "tensor": _lib.PATH_TENSOR}[p]


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


_NO_SWITCH = contextlib.nullcontext()


def _on_device(device):
    """Make `device` the current CUDA device for the library call (the context manager costs a few microseconds,
    so it is skipped when the device is current already)."""
    return _NO_SWITCH if device.index == torch.cuda.current_device() else torch.cuda.device(device)


def _tma_ready(t):
    """True if a [B, H, T, D] fp16 tensor can be described by a TMA tensor map as it is (innermost stride 1,
    16-byte aligned base, positive 16-byte multiple outer strides; a broadcast view has stride 0 and is copied)."""
    if t.dtype != torch.float16 or t.stride(-1) != 1:
        return False
    if t.data_ptr() % 16:
        return False
    return all(s > 0 and (s * 2) % 16 == 0 for s in t.stride()[:3])


def _prep_qkv(x, path):
    # The FFMA kernels take any strides; the tensor-core kernels need a TMA-describable layout. A contiguous tensor
    # with a 16-byte aligned base is one (D is a power of two >= 16), which saves the stride checks on the common path.
    if path == _lib.PATH_SIMT or x.dtype != torch.float16 or (
            x.is_contiguous() and x.data_ptr() % 16 == 0 and 0 not in x.stride()):
        return x
    return x if _tma_ready(x) else x.contiguous()


class LaunchStats:
    """Counts of native kernel launches made through this module (read by the benchmark)."""
    fwd_calls = 0
    bwd_calls = 0
    kernels = 0
    last_fwd_path = None

    @classmethod
    def reset(cls):
        cls.fwd_calls = cls.bwd_calls = cls.kernels = 0


def _dtype_code(dt):
    return _lib.DTYPE_F16 if dt == torch.float16 else _lib.DTYPE_F32


def fpa_forward(q, k, v, phi, psi, beta, tau, path=None):
    """Run the native forward: returns (o, lse) with o [B, H, T, D] in q's dtype and lse [B, H, T] float32.

    phi, psi must be float32 contiguous [B, H, T]; beta float32 contiguous [H]."""
    lib = _lib.load()
    path = _path_from_env() if path is None else path
    B, H, T, D = q.shape
    q, k, v = (_prep_qkv(x, path) for x in (q, k, v))
    o = torch.empty((B, H, T, D), dtype=q.dtype, device=q.device)
    lse = torch.empty((B, H, T), dtype=torch.float32, device=q.device)
    dt = _dtype_code(q.dtype)
    nbytes = lib.fpa_fwd_workspace_bytes(dt, B, H, T, D, path)
    if nbytes == 0:
        _lib.check(_lib.ERR_UNSUPPORTED if path == _lib.PATH_TENSOR else _lib.ERR_INVALID)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    a = _lib.FpaFwdArgs()  # filled in one pack_into, in the field order of FpaFwdArgs
    _lib.FWD_PACKER.pack_into(a, 0, dt, path, B, H, T, D, float(tau),
                              q.data_ptr(), *q.stride(), k.data_ptr(), *k.stride(), v.data_ptr(), *v.stride(),
                              phi.data_ptr(), psi.data_ptr(), beta.data_ptr(), o.data_ptr(), *o.stride(),
                              lse.data_ptr(), ws.data_ptr(), nbytes, 0, 0)
    _lib.check(lib.fpa_fwd(ctypes.byref(a), _stream(q.device)))
    LaunchStats.fwd_calls += 1
    LaunchStats.kernels += a.kernels_launched
    LaunchStats.last_fwd_path = a.path_taken
    if os.environ.get("FPA_B200_CHECK") == "1":
        _lib.check(lib.fpa_workspace_status(_ptr(ws), _stream(q.device)))
    return o, lse


def fpa_backward(q, k, v, o, lse, phi, psi, beta, do, tau, path=None):
    """Run the native backward: returns (dq, dk, dv, dphi, dpsi, dbeta)."""
    lib = _lib.load()
    path = _path_from_env() if path is None else path
    B, H, T, D = q.shape
    # q, k, v are the tensors the caller gave the forward (which copied any that TMA cannot describe), and the
    # gradient of o.sum() arrives as a broadcast view (all strides 0). The reference's backward works on contiguous
    # copies too: q, k, v padded in its forward and dO padded on entry (kernel.py:380-384, 402, 429).
    q, k, v, do = (_prep_qkv(x, path) for x in (q, k, v, do))
    dq, dk, dv = (torch.empty((B, H, T, D), dtype=q.dtype, device=q.device) for _ in range(3))
    dphi = torch.empty((B, H, T), dtype=torch.float32, device=q.device)
    dpsi = torch.empty_like(dphi)
    dbeta = torch.empty((H,), dtype=torch.float32, device=q.device)
    dt = _dtype_code(q.dtype)
    nbytes = lib.fpa_bwd_workspace_bytes(dt, B, H, T, D, path)
    if nbytes == 0:
        _lib.check(_lib.ERR_UNSUPPORTED if path == _lib.PATH_TENSOR else _lib.ERR_INVALID)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    a = _lib.FpaBwdArgs()  # filled in one pack_into, in the field order of FpaBwdArgs
    _lib.BWD_PACKER.pack_into(a, 0, dt, path, B, H, T, D, float(tau),
                              q.data_ptr(), *q.stride(), k.data_ptr(), *k.stride(), v.data_ptr(), *v.stride(),
                              o.data_ptr(), *o.stride(), do.data_ptr(), *do.stride(), lse.data_ptr(),
                              phi.data_ptr(), psi.data_ptr(), beta.data_ptr(), dq.data_ptr(), *dq.stride(),
                              dk.data_ptr(), *dk.stride(), dv.data_ptr(), *dv.stride(), dphi.data_ptr(),
                              dpsi.data_ptr(), dbeta.data_ptr(), ws.data_ptr(), nbytes, 0, 0)
    _lib.check(lib.fpa_bwd(ctypes.byref(a), _stream(q.device)))
    LaunchStats.bwd_calls += 1
    LaunchStats.kernels += a.kernels_launched
    if os.environ.get("FPA_B200_CHECK") == "1":
        _lib.check(lib.fpa_workspace_status(_ptr(ws), _stream(q.device)))
    return dq, dk, dv, dphi, dpsi, dbeta


class _FirstPassageAttention(torch.autograd.Function):
    """Autograd node of the native operator (kernel.py:415-451 is the reference's counterpart)."""

    @staticmethod
    def forward(ctx, q, k, v, phi, psi, beta, tau, path):
        phif = phi.float().contiguous()
        psif = psi.float().contiguous()
        betaf = beta.float().contiguous()
        with _on_device(q.device):
            o, lse = fpa_forward(q, k, v, phif, psif, betaf, tau, path)
        ctx.save_for_backward(q, k, v, o, lse, phif, psif, betaf)
        ctx.tau, ctx.path = tau, path
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, phif, psif, betaf = ctx.saved_tensors
        with _on_device(q.device):
            dq, dk, dv, dphi, dpsi, dbeta = fpa_backward(q, k, v, o, lse, phif, psif, betaf, do.to(q.dtype),
                                                         ctx.tau, ctx.path)
        return dq, dk, dv, dphi, dpsi, dbeta, None, None


def first_passage_attention(q, k, v, phi, psi, beta, tau=1.0, impl=None, block=64):
    """o (B, H, T, D) of q, k, v (B, H, T, D), phi, psi (B, H, T) and beta (H,).

    impl: "cuda" (alias "triton"; q, k, v all fp16 or all fp32 CUDA tensors, D a power of two >= 16),
    "reference" (any device), or None for "cuda" on CUDA tensors and "reference" otherwise. block: accepted and
    validated as the reference does (a power of two >= 16, at most 32 in fp32); the native kernels choose their
    own tiling, so it does not change the result."""
    if impl is None:
        impl = "cuda" if q.is_cuda else "reference"
    if impl == "reference":
        return first_passage_attention_reference(q, k, v, phi, psi, beta, tau)
    if impl not in _KERNEL_IMPLS:
        raise ValueError(f"unknown implementation {impl!r}")
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k and v must have the same shape (B, H, T, D)")
    if q.dtype not in (torch.float16, torch.float32) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k and v must all be fp16 or all fp32")
    B, H, T, D = q.shape
    if phi.shape != (B, H, T) or psi.shape != (B, H, T):
        raise ValueError("phi and psi must have shape (B, H, T)")
    if not _pow2(D) or not _pow2(block):
        raise ValueError("the head dimension and the block must be powers of two >= 16")
    if not torch.is_tensor(beta):
        beta = torch.tensor(float(beta), device=q.device)
    beta = beta.reshape(-1)
    if beta.numel() == 1:
        beta = beta.expand(H)
    if beta.shape != (H,):
        raise ValueError("beta must have shape (H,) or a single value")
    if not tau > 0:
        raise ValueError("tau must be positive")
    if not (q.is_cuda and k.is_cuda and v.is_cuda and phi.is_cuda and psi.is_cuda and beta.is_cuda):
        raise ValueError("the CUDA implementation needs q, k, v, phi, psi and beta on a CUDA device")
    if q.dtype == torch.float32:
        block = min(block, 32)
    return _FirstPassageAttention.apply(q, k, v, phi, psi, beta, float(tau), None)


class _FieldFn(torch.autograd.Function):
    """phi, psi [B, H, T] from the Field projection's output proj [B, T, 3H] (fp32, on a CUDA device) in one
    kernel each way (fpa_field_fwd / fpa_field_bwd): the cumsum of delta and the two additions of kernel.py:507-509
    and their backward, with no intermediate tensors."""

    @staticmethod
    def forward(ctx, proj, H):
        lib = _lib.load()
        B, T, _ = proj.shape
        phi = torch.empty((B, H, T), dtype=torch.float32, device=proj.device)
        psi = torch.empty_like(phi)
        a = _lib.FpaFieldArgs(B=B, T=T, H=H, proj=_ptr(proj), proj_stride=(ctypes.c_int64 * 3)(*proj.stride()),
                              phi=_ptr(phi), psi=_ptr(psi))
        _lib.check(lib.fpa_field_fwd(ctypes.byref(a), _stream(proj.device)))
        LaunchStats.kernels += 1
        ctx.shape, ctx.H = proj.shape, H
        return phi, psi

    @staticmethod
    def backward(ctx, dphi, dpsi):
        lib = _lib.load()
        B, T, H3 = ctx.shape
        dev = (dphi if dphi is not None else dpsi).device
        dphi = torch.zeros((B, ctx.H, T), device=dev) if dphi is None else dphi.float().contiguous()
        dpsi = torch.zeros((B, ctx.H, T), device=dev) if dpsi is None else dpsi.float().contiguous()
        dproj = torch.empty((B, T, H3), dtype=torch.float32, device=dev)
        a = _lib.FpaFieldArgs(B=B, T=T, H=ctx.H, dphi=_ptr(dphi), dpsi=_ptr(dpsi), dproj=_ptr(dproj),
                              dproj_stride=(ctypes.c_int64 * 3)(*dproj.stride()))
        _lib.check(lib.fpa_field_bwd(ctypes.byref(a), _stream(dev)))
        LaunchStats.kernels += 1
        return dproj, None


class Field(nn.Module):
    """The per-head field of the layer (kernel.py:492-509). One fp32 projection of x (B, T, d_model) gives three
    values per head and position: an increment delta, and offsets g and h. The walk W is the running sum of delta
    along T; the field is phi = W + g and the levels are psi = W + h, both (B, H, T). The strength is
    beta = softplus(beta_raw) (H,), positive for any parameter value.

    On a CUDA device in fp32 the walk and the two sums run as one kernel each way (fpa_field_fwd / fpa_field_bwd)
    that writes phi and psi in the operator's layout; ``impl = "reference"`` (set by a layer built with it), CPU
    inputs and float64 keep the PyTorch ops."""

    def __init__(self, d_model, n_heads, beta_init=1.0):
        super().__init__()
        self.n_heads = n_heads
        self.proj = nn.Linear(d_model, 3 * n_heads)
        # softplus(beta_raw) = beta_init at initialisation: beta_raw = log(expm1(beta_init)), written stably.
        self.beta_raw = nn.Parameter(torch.full((n_heads,), beta_init + math.log(-math.expm1(-beta_init))))
        self.impl = None

    def forward(self, x):
        B, T, _ = x.shape
        dt = torch.float64 if x.dtype == torch.float64 else torch.float32
        with torch.autocast(device_type=x.device.type, enabled=False):
            out = F.linear(x.to(dt), self.proj.weight.to(dt), self.proj.bias.to(dt))
        if x.is_cuda and dt == torch.float32 and self.impl != "reference":
            phi, psi = _FieldFn.apply(out, self.n_heads)
            return phi, psi, F.softplus(self.beta_raw)
        delta, g, h = out.view(B, T, 3, self.n_heads).permute(2, 0, 3, 1)
        w = torch.cumsum(delta, dim=-1)
        return w + g, w + h, F.softplus(self.beta_raw)


class FirstPassageAttention(nn.Module):
    """Self-attention layer with the first-passage bias in place of a positional encoding (kernel.py:512-530):
    x (B, T, d_model) goes through one bias-free projection to q, k, v of n_heads heads, a Field gives phi, psi and
    beta, the operator combines them, and a bias-free output projection maps the heads back to d_model.

    The q, k, v views of the fused projection are passed to the kernels with their strides (no copy)."""

    def __init__(self, d_model, n_heads, tau=1.0, beta_init=1.0, impl=None, block=64):
        super().__init__()
        if d_model % n_heads:
            raise ValueError("d_model must be a multiple of n_heads")
        self.h, self.d = n_heads, d_model // n_heads
        self.tau, self.impl, self.block = tau, impl, block
        self.qkv = nn.Linear(d_model, 3 * d_model, bias=False)
        self.out = nn.Linear(d_model, d_model, bias=False)
        self.field = Field(d_model, n_heads, beta_init)
        self.field.impl = impl

    def forward(self, x):
        B, T, _ = x.shape
        q, k, v = self.qkv(x).view(B, T, 3, self.h, self.d).permute(2, 0, 3, 1, 4)
        phi, psi, beta = self.field(x)
        o = first_passage_attention(q, k, v, phi, psi, beta, tau=self.tau, impl=self.impl, block=self.block)
        return self.out(o.transpose(1, 2).reshape(B, T, -1))
