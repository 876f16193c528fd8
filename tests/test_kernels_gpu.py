"""Parity of the native CUDA kernels with the CPU oracle and with the reference's golden vectors.

Tolerances are the reference's (test.py:19-20, README.md:49): max relative error (max|x - ref| / max|ref|)
2e-3 in fp16 (1e-2 for dbeta) and 2e-4 in fp32, against the float64 definition."""
import os

import numpy as np
import pytest
import torch

from first_passage_attention_b200 import FirstPassageAttention, LaunchStats, first_passage_attention
from first_passage_attention_b200 import _lib
from oracle import fpa_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
NAMES = ("o", "dq", "dk", "dv", "dphi", "dpsi", "dbeta")
TOL = {torch.float16: 2e-3, torch.float32: 2e-4}
TOL_DBETA_FP16 = 1e-2
PATHS = {"auto": _lib.PATH_AUTO, "simt": _lib.PATH_SIMT, "tensor": _lib.PATH_TENSOR}


def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")


def make_inputs(B, H, T, D, phi_scale=1.0, ties=False, seed=0, dtype=torch.float16):
    """test.py:108-117 (CPU tensors)."""
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, H, T, D, generator=g).to(dtype) for _ in range(3))
    phi = torch.randn(B, H, T, generator=g).cumsum(-1) * phi_scale
    if ties:
        phi = torch.round(phi)
    psi = phi + 0.5 * torch.randn(B, H, T, generator=g)
    beta = torch.rand(H, generator=g) + 0.5
    do = torch.randn(B, H, T, D, generator=g).to(dtype)
    return q, k, v, phi, psi, beta, do


def run_kernel(q, k, v, phi, psi, beta, do, tau=1.0, path="auto"):
    os.environ["FPA_B200_PATH"] = path
    try:
        a = [t.cuda().clone().requires_grad_() for t in (q, k, v, phi, psi, beta)]
        o = first_passage_attention(*a, tau=tau, impl="triton")
        grads = torch.autograd.grad(o, a, do.cuda())
        torch.cuda.synchronize()
        return [o.detach().cpu()] + [x.cpu() for x in grads]
    finally:
        os.environ.pop("FPA_B200_PATH", None)


def run_oracle(q, k, v, phi, psi, beta, do, tau=1.0):
    n = [t.double().numpy() for t in (q, k, v, phi, psi, beta, do)]
    o, _ = O.forward(*n[:6])
    return [o] + list(O.backward(*n, tau=tau))


def check(kern, ref, dtype, tol=None, floor=0.0):
    """rel_err of test.py:120-121 for every output; `floor` bounds the denominator from below for cases whose exact
    gradients vanish (T = 1: o = v and dS = 0, so only rounding is left to compare)."""
    for name, x, r in zip(NAMES, kern, ref):
        want = dtype if name in ("o", "dq", "dk", "dv") else torch.float32
        assert x.dtype == want, name
        assert torch.isfinite(x).all(), name
        t = tol or (TOL_DBETA_FP16 if (name == "dbeta" and dtype == torch.float16) else TOL[dtype])
        xd = x.double().numpy()
        err = float(np.abs(xd - r).max() / max(np.abs(r).max(), floor, 1e-30))
        assert err <= t, (name, err)


# test.py:134-147, all sizes (the reference marks the last four GPU-only).
CASES = [
    (1, 2, 64, 64, 32, 1.0, False, torch.float16, 100),
    (2, 3, 100, 64, 32, 1.0, False, torch.float16, 101),
    (1, 2, 128, 64, 64, 1.0, False, torch.float16, 102),
    (1, 2, 96, 64, 32, 40.0, False, torch.float16, 103),
    (1, 2, 96, 64, 32, 1.0, True, torch.float16, 104),
    (1, 2, 80, 32, 16, 1.0, False, torch.float16, 110),
    (1, 2, 100, 64, 32, 1.0, False, torch.float32, 111),
    (1, 2, 96, 16, 16, 40.0, False, torch.float32, 112),
    (2, 4, 512, 64, 64, 1.0, False, torch.float16, 105),
    (1, 2, 2048, 64, 64, 1.0, False, torch.float16, 106),
    (1, 2, 2048, 64, 32, 1.0, False, torch.float32, 200),
    (1, 2, 1000, 64, 32, 40.0, False, torch.float32, 201),
]


@pytest.mark.parametrize("path", list(PATHS))
@pytest.mark.parametrize("B,H,T,D,block,scale,ties,dtype,seed", CASES)
def test_kernel_matches_the_oracle(B, H, T, D, block, scale, ties, dtype, seed, path):
    need_gpu()
    if path == "tensor" and dtype != torch.float16:
        pytest.skip("the tensor-core kernels take fp16")
    inp = make_inputs(B, H, T, D, scale, ties, seed=seed, dtype=dtype)
    check(run_kernel(*inp, path=path), run_oracle(*inp), dtype)


@pytest.mark.parametrize("name", sorted(f[:-4] for f in os.listdir(GOLDEN) if f.startswith(("t", "config1"))))
def test_kernel_matches_the_reference_golden(name):
    """Outputs of the reference implementation itself (tests/golden/make_golden.py)."""
    need_gpu()
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    dtype = torch.float16 if str(z["dtype"]) == "f16" else torch.float32
    inp = [torch.from_numpy(z[n]) for n in ("q", "k", "v", "phi", "psi", "beta", "do")]
    inp = [x.to(dtype) if n in ("q", "k", "v", "do") else x for n, x in zip("qkvabcd", inp)]
    kern = run_kernel(*inp, tau=float(z["tau"]))
    check(kern, [z[n] for n in NAMES], dtype)


def test_kernel_temperature():
    """test.py:162-167."""
    need_gpu()
    inp = make_inputs(1, 2, 72, 32, seed=11, dtype=torch.float32)
    check(run_kernel(*inp, tau=0.25), run_oracle(*inp, tau=0.25), torch.float32)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_kernel_deterministic(dtype):
    """test.py:170-174: two runs are bit-identical."""
    need_gpu()
    inp = make_inputs(2, 2, 300, 32, seed=12, dtype=dtype)
    runs = [run_kernel(*inp) for _ in range(2)]
    assert all(torch.equal(x, y) for x, y in zip(*runs))


@pytest.mark.parametrize("D", [32, 64, 128])
def test_persistent_passes_with_several_units_per_cta(D):
    """More work units (a head's 128-row tile) than SMs: B2 H48 T384 gives 288 units per backward pass, a third of
    them one tile long, so each persistent CTA takes two units in a row and the unit-boundary hand-overs (staged or
    shared-memory stationary operands, accumulator read-out, the diagonal soft-min buffer) all run. D = 32 keeps
    K and V in TMEM, D = 64 in shared memory, D = 128 also has the separate diagonal kernel. Against the oracle, and
    bit-identical twice."""
    need_gpu()
    inp = make_inputs(2, 48, 384, D, seed=500 + D)
    kern = run_kernel(*inp, path="tensor")
    check(kern, run_oracle(*inp), torch.float16)
    again = run_kernel(*inp, path="tensor")
    assert all(torch.equal(x, y) for x, y in zip(kern, again))


def test_backward_calls_on_two_streams_at_once():
    """Two forward + backward calls issued on two streams without synchronising in between (each call's q-pass runs
    on an auxiliary stream of its own calling stream) give bit-identical results to the same calls run one after
    the other."""
    need_gpu()
    inputs = [make_inputs(2, 8, 640, 64, seed=700 + n) for n in range(2)]
    seq = [run_kernel(*inp, path="tensor") for inp in inputs]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    os.environ["FPA_B200_PATH"] = "tensor"
    try:
        outs = []
        for inp, st in zip(inputs, streams):
            with torch.cuda.stream(st):
                a = [t.cuda(non_blocking=False).clone().requires_grad_() for t in inp[:6]]
                o = first_passage_attention(*a, impl="triton")
                g = torch.autograd.grad(o, a, inp[6].cuda())
                outs.append([o.detach()] + list(g))
        torch.cuda.synchronize()
    finally:
        os.environ.pop("FPA_B200_PATH", None)
    for got, want in zip(outs, seq):
        assert all(torch.equal(x.cpu(), y) for x, y in zip(got, want))


def test_forward_backward_replayed_from_a_cuda_graph():
    """Forward + backward captured into a CUDA graph (the forked q-pass becomes graph edges) and replayed give the
    eager call's gradients bit for bit."""
    need_gpu()
    inp = [t.cuda() for t in make_inputs(2, 6, 512, 64, seed=800)]
    leaves = [t.clone().requires_grad_() for t in inp[:6]]
    do = inp[6]

    def step():
        for x in leaves:
            x.grad = None
        first_passage_attention(*leaves, impl="triton").backward(do)

    os.environ["FPA_B200_PATH"] = "tensor"
    try:
        step()
        want = [x.grad.clone() for x in leaves]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        assert all(torch.equal(x.grad, w) for x, w in zip(leaves, want))
    finally:
        os.environ.pop("FPA_B200_PATH", None)


@pytest.mark.parametrize("path", ["tensor", "simt"])
def test_long_context_dphi_combination(path):
    """The O(NB^2) evaluation of dphi's strictly-between part (dphi_part3_kernel, which runs on its own beyond 256
    tiles) forced at T = 2048 (16 tiles on the tensor-core path, 32 on the FFMA path): against the oracle and against
    the O(NB^3) evaluation; every other output is bit-identical."""
    need_gpu()
    inp = make_inputs(1, 3, 2048, 64, seed=900)
    cubic = run_kernel(*inp, path=path)
    os.environ["FPA_B200_DPHI_QUADRATIC"] = "1"
    try:
        quad = run_kernel(*inp, path=path)
    finally:
        os.environ.pop("FPA_B200_DPHI_QUADRATIC", None)
    check(quad, run_oracle(*inp), torch.float16)
    for name, x, y in zip(NAMES, quad, cubic):
        if name == "dphi":
            assert (x - y).abs().max() <= 1e-5 * y.abs().max()
        else:
            assert torch.equal(x, y), name


def config3_inputs(D, dtype, seed):
    """Benchmark configuration 3: B2 H8 T1000; phi = cumsum N(-0.05, 1); psi = phi + N(0,1); beta = softplus(N)."""
    g = torch.Generator().manual_seed(seed)
    B, H, T = 2, 8, 1000
    q, k, v = (torch.randn(B, H, T, D, generator=g).to(dtype) for _ in range(3))
    phi = (torch.randn(B, H, T, generator=g) - 0.05).cumsum(-1)
    psi = phi + torch.randn(B, H, T, generator=g)
    beta = torch.nn.functional.softplus(torch.randn(H, generator=g))
    do = torch.randn(B, H, T, D, generator=g).to(dtype)
    return q, k, v, phi, psi, beta, do


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("D", [16, 32, 128, 256])
def test_config3_edge_coverage(D, dtype):
    need_gpu()
    inp = config3_inputs(D, dtype, seed=D)
    kern = run_kernel(*inp)
    check(kern, run_oracle(*inp), dtype)
    again = run_kernel(*inp)
    assert all(torch.equal(x, y) for x, y in zip(kern, again))


@pytest.mark.parametrize("T", [1, 2, 3, 63, 64, 65, 127, 129])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_ragged_and_tiny_lengths(T, dtype):
    """Lengths around the tile sizes (64 for the FFMA kernels, 128 for the tensor-core forward) and the degenerate
    T = 1, 2. For T <= 2 the gradients through dS = P (dP - delta) are pure cancellation: with fp16 inputs, delta
    is formed from the fp16-rounded output o (as kernel.py:174 forms it), so only rounding is left and those
    cases are held to 1e-2 instead of 2e-3."""
    need_gpu()
    inp = make_inputs(1, 3, T, 64, seed=300 + T, dtype=dtype)
    tiny = T <= 2
    tol = 1e-2 if (tiny and dtype == torch.float16) else None
    check(run_kernel(*inp), run_oracle(*inp), dtype, tol=tol, floor=1e-2 if tiny else 0.0)


def test_negative_and_scalar_beta():
    """beta is a free parameter of the operator: a negative strength flips the bias sign (kernel.py:478-484)."""
    need_gpu()
    q, k, v, phi, psi, beta, do = make_inputs(1, 3, 200, 32, seed=41, dtype=torch.float32)
    beta = torch.tensor([-0.7, 0.0, 1.3])
    check(run_kernel(q, k, v, phi, psi, beta, do), run_oracle(q, k, v, phi, psi, beta, do), torch.float32)


def test_strided_qkv_views():
    """The layer's permuted views of the fused projection (kernel.py:527) are read in place."""
    need_gpu()
    B, T, H, D = 2, 130, 4, 32
    g = torch.Generator().manual_seed(5)
    qkv = torch.randn(B, T, 3, H, D, generator=g).half()
    q, k, v = qkv.permute(2, 0, 3, 1, 4)
    _, _, _, phi, psi, beta, do = make_inputs(B, H, T, D, seed=6)
    check(run_kernel(q, k, v, phi, psi, beta, do), run_oracle(q, k, v, phi, psi, beta, do), torch.float16)


@pytest.mark.parametrize("D", [64, 256])
def test_ffma_path_reads_strided_operands(D):
    """fp32 q, k, v and dO stored [B, H, D, T] and passed as transposed views (column stride T, so every tile load
    takes the scalar path; at D = 256 the streamed tiles start at column offsets 64, 128, 192): the same result as
    the oracle and, bit for bit, as contiguous copies."""
    need_gpu()
    B, H, T = 1, 2, 300
    q, k, v, phi, psi, beta, do = make_inputs(B, H, T, D, seed=70 + D, dtype=torch.float32)
    tq, tk, tv, tdo = (x.transpose(-1, -2).contiguous().transpose(-1, -2) for x in (q, k, v, do))
    assert tq.stride()[-1] == T
    kern = run_kernel(tq, tk, tv, phi, psi, beta, tdo)
    check(kern, run_oracle(q, k, v, phi, psi, beta, do), torch.float32)
    dense = run_kernel(q, k, v, phi, psi, beta, do)
    assert all(torch.equal(x, y) for x, y in zip(kern, dense))


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_keys_and_values_shared_across_heads(dtype):
    """k and v given as one head broadcast over all heads (expand, head stride 0): the result equals the oracle's on
    the repeated tensors and, bit for bit, the kernels' own result on contiguous copies."""
    need_gpu()
    B, H, T, D = 1, 3, 200, 64
    q, k, v, phi, psi, beta, do = make_inputs(B, H, T, D, seed=61, dtype=dtype)
    k, v = (x[:, :1].expand(B, H, T, D) for x in (k, v))
    xs = [t.cuda().requires_grad_() for t in (q, k[:, :1], v[:, :1], phi, psi, beta)]
    kb, vb = (x.expand(B, H, T, D) for x in xs[1:3])
    ins = [xs[0], kb, vb] + xs[3:]
    o = first_passage_attention(*ins, impl="triton")
    kern = [o.detach().cpu()] + [g.cpu() for g in torch.autograd.grad(o, ins, do.cuda())]
    torch.cuda.synchronize()
    check(kern, run_oracle(q, k.contiguous(), v.contiguous(), phi, psi, beta, do), dtype)
    again = run_kernel(q, k.contiguous(), v.contiguous(), phi, psi, beta, do)
    for name, a, b in zip(NAMES, kern, again):
        assert torch.equal(a, b), name


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_more_than_65535_heads(dtype):
    """B * H = 66000 heads (the per-head kernels' grid is (tiles, H, B), as the reference's is): every head's
    output and gradients equal, bit for bit, those of a run on a slice of the heads alone, and the oracle's."""
    need_gpu()
    B, H, T, D = 2, 33000, 20, 16
    inp = make_inputs(B, H, T, D, seed=71, dtype=dtype)
    full = run_kernel(*inp)
    for sl in (slice(0, 40), slice(H - 40, H)):
        part_inp = [x[:, sl].contiguous() if x.dim() > 1 else x[sl].contiguous() for x in inp]
        part = run_kernel(*part_inp)
        for name, a, b in zip(NAMES, full, part):
            a = a[sl] if name == "dbeta" else a[:, sl]
            if name == "dbeta":
                assert torch.allclose(a, b, rtol=1e-6, atol=0), name
            else:
                assert torch.equal(a, b), name
    check(part, run_oracle(*part_inp), dtype)


@pytest.mark.parametrize("path", ["auto", "tensor", "simt"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_backward_of_the_sum(dtype, path):
    """o.sum().backward(), the step of the CPU configuration: autograd hands the backward a broadcast gradient of
    ones with all strides 0; the result equals the oracle's with grad_o = ones."""
    need_gpu()
    if path == "tensor" and dtype != torch.float16:
        pytest.skip("the tensor-core kernels take fp16")
    q, k, v, phi, psi, beta, _ = make_inputs(2, 3, 300, 64, seed=51, dtype=dtype)
    os.environ["FPA_B200_PATH"] = path
    try:
        a = [t.cuda().clone().requires_grad_() for t in (q, k, v, phi, psi, beta)]
        o = first_passage_attention(*a, impl="triton")
        o.sum().backward()
        torch.cuda.synchronize()
        kern = [o.detach().cpu()] + [x.grad.cpu() for x in a]
    finally:
        os.environ.pop("FPA_B200_PATH", None)
    check(kern, run_oracle(q, k, v, phi, psi, beta, torch.ones(q.shape, dtype=dtype)), dtype)


def test_long_context_prefix():
    """Configuration 4 (B1 H16 T16383 D128 fp16) at full size. With do = 0 beyond T0 every output and gradient of
    the first T0 positions equals that of the truncated problem (the operator is causal), so the full-size run is
    checked against the oracle on the prefix; the rest of o is checked for finiteness."""
    need_gpu()
    B, H, T, D, T0 = 1, 16, 16383, 128, 640
    g = torch.Generator().manual_seed(0)
    q, k, v = ((0.5 * torch.randn(B, H, T, D, generator=g)).half() for _ in range(3))
    phi = torch.randn(B, H, T, generator=g).cumsum(-1)
    psi = phi + 2 * torch.randn(B, H, T, generator=g)
    beta = 2 * torch.ones(H)
    do = torch.randn(B, H, T, D, generator=g).half()
    do[:, :, T0:] = 0
    kern = run_kernel(q, k, v, phi, psi, beta, do)
    assert torch.isfinite(kern[0]).all()
    heads = [0, 7, 15]
    pre = [x[:, heads, :T0] for x in (q, k, v, phi, psi)] + [beta[heads], do[:, heads, :T0]]
    ref = run_oracle(*pre)
    got = [kern[0][:, heads, :T0], kern[1][:, heads, :T0], kern[2][:, heads, :T0], kern[3][:, heads, :T0],
           kern[4][:, heads, :T0], kern[5][:, heads, :T0], kern[6][heads]]
    check(got, ref, torch.float16)
    for x in kern[1:6]:  # dq, dk, dv, dphi, dpsi vanish exactly where do (and so dS) is zero
        assert torch.count_nonzero(x[:, :, T0:]) == 0
    # Late rows of the full-length forward, where the diagonal-backwards walk carries the running minimum of phi
    # over 31, 63 and 127 key tiles: each against the float64 one-row evaluation (O(T*D) per row).
    for h in heads:
        for t in (4095, 8191, 16382):
            want = O.forward_row(q[0, h].double().numpy(), k[0, h].double().numpy(), v[0, h].double().numpy(),
                                 phi[0, h].double().numpy(), psi[0, h].double().numpy(), float(beta[h]), t)
            err = float(np.abs(kern[0][0, h, t].double().numpy() - want).max() / np.abs(want).max())
            assert err <= TOL[torch.float16], (h, t, err)


@pytest.mark.parametrize("amp", [False, True])
def test_layer_kernel_matches_the_reference(amp):
    """test.py:200-214: the layer on the native kernels against the layer on the PyTorch definition."""
    need_gpu()
    out = []
    for impl in ("triton", "reference"):
        torch.manual_seed(0)
        layer = FirstPassageAttention(64, 4, impl=impl).cuda()
        x = torch.randn(2, 50, 64, generator=torch.Generator().manual_seed(1)).cuda()
        with torch.autocast("cuda", dtype=torch.float16, enabled=amp):
            y = layer(x)
        loss = y.float().square().mean()
        out.append([y.detach().float()] + list(torch.autograd.grad(loss, list(layer.parameters()))))
    tol = 5e-3 if amp else 1e-4
    for a, b in zip(*out):
        assert ((a - b).norm() / b.norm()).item() <= tol


@pytest.mark.parametrize("D", [16, 32, 64, 128])
@pytest.mark.parametrize("T", [100, 128, 255, 256, 384, 700])
def test_tensor_core_forward(T, D):
    """The tcgen05 forward on every head dimension it covers, odd and even numbers of 128-row tiles."""
    need_gpu()
    inp = make_inputs(2, 2, T, D, 1.0, seed=T + D, dtype=torch.float16)
    check(run_kernel(*inp, path="tensor"), run_oracle(*inp), torch.float16)


def test_tensor_core_forward_extreme_field():
    """A field scaled by 40 (test.py:138) through the lazy-rescaling softmax of the tcgen05 forward."""
    need_gpu()
    inp = make_inputs(1, 3, 1000, 64, 40.0, seed=77, dtype=torch.float16)
    check(run_kernel(*inp, path="tensor"), run_oracle(*inp), torch.float16)


def test_native_library_is_what_ran():
    """The CUDA path runs the in-tree libfpa_b200.so and counts its launches; nothing falls back."""
    need_gpu()
    LaunchStats.reset()
    inp = make_inputs(1, 2, 256, 64, seed=9)
    run_kernel(*inp)
    assert LaunchStats.fwd_calls == 1 and LaunchStats.bwd_calls == 1 and LaunchStats.kernels >= 4
    maps = open("/proc/self/maps").read()
    assert _lib.LIB_PATH in maps


@pytest.mark.parametrize("T", [1, 700, 1024, 3000])
def test_field_kernel_matches_the_pytorch_field(T):
    """The Field's walk and sums in one kernel each way (fpa_field_fwd / fpa_field_bwd) against the PyTorch ops of
    kernel.py:504-509 on the same parameters: phi, psi and the gradients of x and of the projection's weight and bias,
    with T below, at and above one 1024-position chunk."""
    need_gpu()
    from first_passage_attention_b200 import Field
    torch.manual_seed(3)
    fk = Field(48, 12).cuda()
    fr = Field(48, 12).cuda()
    fr.load_state_dict(fk.state_dict())
    fr.impl = "reference"
    x = torch.randn(2, T, 48, device="cuda")
    outs = []
    for f in (fk, fr):
        xx = x.clone().requires_grad_()
        phi, psi, beta = f(xx)
        g = torch.Generator(device="cuda").manual_seed(9)
        w_phi = torch.randn(phi.shape, device="cuda", generator=g)
        w_psi = torch.randn(psi.shape, device="cuda", generator=g)
        loss = (phi * w_phi).sum() + (psi * w_psi).sum() + beta.sum()
        grads = torch.autograd.grad(loss, [xx, f.proj.weight, f.proj.bias])
        outs.append([phi.detach(), psi.detach()] + list(grads))
    assert outs[0][0].is_contiguous() and outs[0][0].shape == (2, 12, T)
    for a, b in zip(*outs):
        scale = b.abs().max().clamp_min(1e-6)
        assert ((a - b).abs().max() / scale).item() <= 1e-5
