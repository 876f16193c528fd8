"""Host-side API: the drop-in surface (names, argument checks and messages of kernel.py:458-530), the PyTorch
definition behind impl="reference" against the reference's golden vectors, and the C ABI library (loads, exports
every symbol include/fpa.h declares, struct layouts agree). CPU only: no kernel is launched."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

import kernel as shim
from first_passage_attention_b200 import FirstPassageAttention, _lib, first_passage_attention, first_passage_bias

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
NAMES = ("o", "dq", "dk", "dv", "dphi", "dpsi", "dbeta")


def _declared_symbols():
    text = open(os.path.join(ROOT, "include", "fpa.h")).read()
    return re.findall(r"FPA_API\s+[\w\s\*]+?\b(fpa_\w+)\s*\(", text)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared_symbols()
    assert set(declared) == set(_lib.EXPORTS)
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.fpa_abi_version() == _lib.ABI_VERSION
    assert lib.fpa_struct_size(0) == ctypes.sizeof(_lib.FpaFwdArgs)
    assert lib.fpa_struct_size(1) == ctypes.sizeof(_lib.FpaBwdArgs)


def test_ffma_backward_workspace_holds_eight_tb_partials_per_tile_pair():
    """The FFMA path's backward workspace (tiles of 64): the status block, the field statistics, delta, W, DPHI2,
    DPHI4, the TB array with eight per-warp partial sums per tile pair (the register-tiled kv-pass writes one per
    warp), dbeta partials and the part-3 scratch, every array 256-byte aligned."""
    lib = _lib.load()
    a256 = lambda n: (n + 255) // 256 * 256  # noqa: E731
    for B, H, T, D in [(2, 8, 1000, 64), (1, 3, 65, 256), (1, 1, 1, 16), (4, 2, 4096, 128)]:
        NB = (T + 63) // 64
        TP, BH = NB * 64, B * H
        stats = 4 * a256(BH * TP * 4) + 2 * a256(BH * NB * 4)
        scratch = 4 * a256(BH * TP * 4) + a256(BH * NB * NB * 8 * 4) + 2 * a256(BH * NB * 4)
        want = 256 + stats + scratch
        assert lib.fpa_bwd_workspace_bytes(_lib.DTYPE_F32, B, H, T, D, _lib.PATH_AUTO) == want, (B, H, T, D)
        assert lib.fpa_bwd_workspace_bytes(_lib.DTYPE_F16, B, H, T, D, _lib.PATH_SIMT) == want, (B, H, T, D)


def test_workspace_queries_and_argument_errors():
    lib = _lib.load()
    assert lib.fpa_fwd_workspace_bytes(_lib.DTYPE_F16, 4, 12, 2048, 64, 0) > 0
    assert lib.fpa_bwd_workspace_bytes(_lib.DTYPE_F32, 2, 8, 1000, 256, 0) > 0
    assert lib.fpa_fwd_workspace_bytes(_lib.DTYPE_F16, 1, 1, 64, 48, 0) == 0      # D not a power of two
    assert lib.fpa_fwd_workspace_bytes(7, 1, 1, 64, 64, 0) == 0                  # bad dtype
    # Invalid arguments are rejected before any CUDA call, so this runs without a GPU.
    a = _lib.FpaFwdArgs(dtype=_lib.DTYPE_F16, path=0, B=1, H=1, T=64, D=64, tau=0.0)
    rc = lib.fpa_fwd(ctypes.byref(a), None)
    assert rc == _lib.ERR_INVALID and b"tau" in lib.fpa_last_error()
    a = _lib.FpaFwdArgs(dtype=_lib.DTYPE_F16, path=0, B=1, H=1, T=64, D=64, tau=1.0)
    assert lib.fpa_fwd(ctypes.byref(a), None) == _lib.ERR_INVALID                 # null pointers
    b = _lib.FpaBwdArgs(dtype=_lib.DTYPE_F32, path=0, B=1, H=1, T=64, D=24, tau=1.0)
    assert lib.fpa_bwd(ctypes.byref(b), None) == _lib.ERR_INVALID
    # Grid limits, as the reference's (tiles, H, B) launches have them: B and H up to 65535 each.
    assert lib.fpa_fwd_workspace_bytes(_lib.DTYPE_F16, 2, 33000, 20, 16, 0) > 0   # B * H above 65535 is fine
    assert lib.fpa_bwd_workspace_bytes(_lib.DTYPE_F16, 1, 70000, 20, 16, 0) == 0
    a = _lib.FpaFwdArgs(dtype=_lib.DTYPE_F32, path=0, B=70000, H=1, T=20, D=16, tau=1.0)
    assert lib.fpa_fwd(ctypes.byref(a), None) == _lib.ERR_UNSUPPORTED and b"65535" in lib.fpa_last_error()
    assert lib.fpa_fwd_workspace_bytes(_lib.DTYPE_F16, 65535, 65535, 1, 16, 0) == 0  # B * H * T above 2^31 - 1
    assert lib.fpa_status_string(_lib.ERR_TIMEOUT) == b"device-side wait timed out"
    # The wait-expiry self-test checks its arguments before any CUDA call.
    assert lib.fpa_selftest_wait_timeout(None, 1000, None) == _lib.ERR_WORKSPACE
    assert lib.fpa_selftest_wait_timeout(ctypes.c_void_p(256), 0, None) == _lib.ERR_INVALID
    assert lib.fpa_selftest_wait_timeout(ctypes.c_void_p(256), 2_000_000_000, None) == _lib.ERR_INVALID
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_INVALID)


def test_shim_exports_the_reference_names():
    for n in ("first_passage_attention", "first_passage_bias", "Field", "FirstPassageAttention"):
        assert hasattr(shim, n)


def _inp(B=1, H=2, T=8, D=16, dtype=torch.float32):
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(B, H, T, D, generator=g).to(dtype) for _ in range(3))
    phi = torch.randn(B, H, T, generator=g).cumsum(-1)
    return q, k, v, phi, phi + 1, torch.ones(H)


def test_validation_messages_match_the_reference():
    """kernel.py:467-486: the same ValueError texts, raised before any device work."""
    q, k, v, phi, psi, beta = _inp()
    with pytest.raises(ValueError, match="unknown implementation 'tpu'"):
        first_passage_attention(q, k, v, phi, psi, beta, impl="tpu")
    with pytest.raises(ValueError, match=r"same shape \(B, H, T, D\)"):
        first_passage_attention(q, k[:, :1], v, phi, psi, beta, impl="triton")
    with pytest.raises(ValueError, match="must all be fp16 or all fp32"):
        first_passage_attention(q.double(), k.double(), v.double(), phi, psi, beta, impl="cuda")
    with pytest.raises(ValueError, match=r"phi and psi must have shape \(B, H, T\)"):
        first_passage_attention(q, k, v, phi[..., :4], psi, beta, impl="triton")
    with pytest.raises(ValueError, match="powers of two >= 16"):
        first_passage_attention(q, k, v, phi, psi, beta, impl="triton", block=48)
    q8, k8, v8, phi8, psi8, beta8 = _inp(D=8)
    with pytest.raises(ValueError, match="powers of two >= 16"):
        first_passage_attention(q8, k8, v8, phi8, psi8, beta8, impl="triton")
    with pytest.raises(ValueError, match=r"beta must have shape \(H,\)"):
        first_passage_attention(q, k, v, phi, psi, torch.ones(3), impl="triton")
    with pytest.raises(ValueError, match="tau must be positive"):
        first_passage_attention(q, k, v, phi, psi, beta, tau=0.0, impl="triton")
    with pytest.raises(ValueError, match="tau must be positive"):
        first_passage_bias(phi, psi, beta, tau=-1.0)
    with pytest.raises(ValueError, match="CUDA device"):     # CPU tensors asked for the CUDA kernels
        first_passage_attention(q, k, v, phi, psi, beta, impl="cuda")


def test_impl_none_on_cpu_is_the_reference():
    q, k, v, phi, psi, beta = _inp()
    a = first_passage_attention(q, k, v, phi, psi, beta)
    b = first_passage_attention(q, k, v, phi, psi, beta, impl="reference")
    assert torch.equal(a, b)
    # scalar beta is broadcast over heads
    c = first_passage_attention(q, k, v, phi, psi, 1.0, impl="reference")
    assert torch.allclose(a, c)


@pytest.mark.parametrize("name", ["t64_d16_fp16_s100", "t96_d16_scale40_s103", "t72_d32_fp32_tau025_s11",
                                  "config1_t256_d32_fp32"])
def test_reference_impl_matches_golden(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    r = [torch.from_numpy(z[n]).double().requires_grad_() for n in ("q", "k", "v", "phi", "psi", "beta")]
    o = first_passage_attention(*r, tau=float(z["tau"]), impl="reference")
    grads = torch.autograd.grad(o, r, torch.from_numpy(z["do"]).double())
    for n, x in zip(NAMES, (o.detach(),) + grads):
        ref = torch.from_numpy(z[n])
        assert ((x - ref).abs().max() / ref.abs().max()).item() < 1e-12, n


def test_reference_layer_matches_golden():
    """The layer built under torch.manual_seed(0) has the reference's parameters and outputs (test.py:177-197)."""
    z = np.load(os.path.join(GOLDEN, "layer_d64_h4_t50.npz"))
    torch.manual_seed(0)
    layer = FirstPassageAttention(64, 4, impl="reference")
    names = [n for n, _ in layer.named_parameters()]
    assert names == list(z["names"])
    for n, p in layer.named_parameters():
        assert torch.equal(p.detach(), torch.from_numpy(z[f"param:{n}"])), n
    x = torch.from_numpy(z["x"])
    y = layer(x)
    assert torch.allclose(y, torch.from_numpy(z["y"]), rtol=1e-5, atol=1e-6)
    grads = torch.autograd.grad(y.float().square().mean(), list(layer.parameters()))
    for n, g in zip(names, grads):
        ref = torch.from_numpy(z[f"grad:{n}"])
        assert ((g - ref).norm() / ref.norm()).item() < 1e-4, n


def test_layout_preparation_for_the_tensor_core_path():
    """Which q, k, v, dO views go to the tensor-core kernels as they are (TMA tensor maps need unit innermost
    stride and positive 16-byte-multiple outer strides) and which are copied first; the FFMA path copies nothing."""
    from first_passage_attention_b200 import ops
    B, T, H, D = 2, 130, 4, 32
    qkv = torch.zeros(B, T, 3, H, D, dtype=torch.float16)
    q = qkv.permute(2, 0, 3, 1, 4)[0]                     # the layer's view of the fused projection
    assert ops._tma_ready(q) and ops._prep_qkv(q, _lib.PATH_AUTO) is q
    k = torch.zeros(B, 1, T, D, dtype=torch.float16).expand(B, H, T, D)    # one head shared by all heads
    assert not ops._tma_ready(k)
    kc = ops._prep_qkv(k, _lib.PATH_TENSOR)
    assert kc.is_contiguous() and kc.shape == k.shape
    do = torch.ones((), dtype=torch.float16).expand(B, H, T, D)            # the gradient of o.sum()
    assert not ops._tma_ready(do) and ops._prep_qkv(do, _lib.PATH_AUTO).is_contiguous()
    assert ops._prep_qkv(do, _lib.PATH_SIMT) is do
    odd = torch.zeros(B, H, T, D + 1, dtype=torch.float16)[..., :D]          # rows not 16-byte multiples
    assert not ops._tma_ready(odd) and ops._prep_qkv(odd, _lib.PATH_AUTO).is_contiguous()
    f32 = torch.zeros(B, 1, T, D).expand(B, H, T, D)
    assert ops._prep_qkv(f32, _lib.PATH_AUTO) is f32     # fp32 runs on the FFMA kernels, which take any strides


def _reference_layer_and_input(T=50, seed=0):
    torch.manual_seed(seed)
    layer = FirstPassageAttention(64, 4, impl="reference")
    x = torch.randn(2, T, 64, generator=torch.Generator().manual_seed(seed + 1))
    return layer, x


def test_reference_layer_is_causal():
    """test.py:184-190: changing the input after position t0 leaves the layer's outputs up to t0 unchanged (the
    field's cumulative sum and the bias's range minimum only look backwards)."""
    layer, x = _reference_layer_and_input()
    t0 = 30
    x2 = x.clone()
    x2[:, t0 + 1:] = torch.randn(x2[:, t0 + 1:].shape, generator=torch.Generator().manual_seed(7)) * 5
    with torch.no_grad():
        assert torch.allclose(layer(x)[:, :t0 + 1], layer(x2)[:, :t0 + 1], rtol=0, atol=1e-6)


def test_reference_layer_gradients_reach_every_parameter():
    """test.py:193-197: every named parameter (qkv, out, field.proj, field.beta_raw) gets a finite, non-zero
    gradient through the bias."""
    layer, x = _reference_layer_and_input()
    layer(x).square().mean().backward()
    for name, p in layer.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all() and p.grad.abs().max() > 0, name


def test_layer_rejects_bad_head_split():
    with pytest.raises(ValueError, match="multiple of n_heads"):
        FirstPassageAttention(65, 4)
