"""Parity on the benchmark's own inputs: the configuration-2 batch that bench.py times (B4 H12 T2048 D64 fp16,
beta = 1, grad_o = ones, bench.make_inputs), checked against the float64 oracle on sampled heads, and the
strong-scaling split of its 48 heads over 2, 4 and 8 ranks (bench.head_shard / bench.take_heads), whose shards the
CUDA kernels must compute bit for bit as they compute those heads inside the whole batch.

Tolerances are the reference's (test.py:19-20): max relative error 2e-3 in fp16, 1e-2 for dbeta."""
import os

import numpy as np
import pytest
import torch

import bench
from first_passage_attention_b200 import first_passage_attention
from oracle import fpa_oracle as O

pytestmark = pytest.mark.gpu

NAMES = ("o", "dq", "dk", "dv", "dphi", "dpsi", "dbeta")


def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")


def fwd_bwd(q, k, v, phi, psi, beta, do):
    leaves = [t.detach().clone().requires_grad_() for t in (q, k, v, phi, psi, beta)]
    o = first_passage_attention(*leaves, impl="cuda")
    grads = torch.autograd.grad(o, leaves, do)
    torch.cuda.synchronize()
    return [o.detach()] + list(grads)


@pytest.fixture(scope="module")
def config2():
    need_gpu()
    inp = bench.make_inputs(4, 12, 2048, 64, seed=1000, device=torch.device("cuda"))
    return inp, fwd_bwd(*inp)


def _oracle_head(inp, b, h):
    n = [x[b:b + 1, h:h + 1].double().cpu().numpy() for x in (inp[0], inp[1], inp[2], inp[3], inp[4])]
    beta = inp[5][h:h + 1].double().cpu().numpy()
    do = inp[6][b:b + 1, h:h + 1].double().cpu().numpy()
    o, _ = O.forward(*n, beta)
    return [o] + list(O.backward(*n, beta, do))


def test_config2_batch_matches_the_oracle_on_sampled_heads(config2):
    inp, out = config2
    for b, h in ((0, 0), (1, 5), (3, 11)):
        ref = _oracle_head(inp, b, h)
        for name, x, r in zip(NAMES[:6], out[:6], ref[:6]):
            got = x[b:b + 1, h:h + 1].double().cpu().numpy()
            err = O.rel_err(got, r)
            assert err <= 2e-3, (b, h, name, err)
    # dbeta of head 11 sums its four (b, h) heads over the batch (kernel.py:450).
    want = sum(_oracle_head(inp, b, 11)[6][0] for b in range(4))
    err = abs(float(out[6][11]) - want) / abs(want)
    assert err <= 1e-2, err


def _unsplit(fn, *args):
    """fn(*args) with the forward's key-range split turned off (FPA_B200_FWD_SPLIT=0)."""
    os.environ["FPA_B200_FWD_SPLIT"] = "0"
    try:
        return fn(*args)
    finally:
        os.environ.pop("FPA_B200_FWD_SPLIT", None)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_strong_split_shards_match_the_whole_batch_bit_for_bit(config2, world):
    """With the forward's key-range split off, a shard's heads come out bit for bit as inside the whole batch. With
    it on (the default, taken when a shard's grid leaves SMs idle: 12 and 6 heads per GPU here), the forward adds
    the same terms in another order, so every output agrees with the whole batch's to the fp16 tolerance."""
    inp, out = config2
    B, H = 4, 12
    for rank in range(world):
        z0, z1 = bench.head_shard(B, H, rank, world)
        b0, b1, h0, h1 = bench.shard_block(H, z0, z1)
        shard = [bench.take_heads(x, z0, z1, H).contiguous() for x in inp]
        part = _unsplit(fwd_bwd, *shard)
        for name, x, y in zip(NAMES[:6], part[:6], out[:6]):
            assert torch.equal(x, y[b0:b1, h0:h1]), (world, rank, name)
        # dbeta of a shard sums over its own batches only; the shards' sums add up to the whole batch's.
        if b1 - b0 == B:
            assert torch.equal(part[6], out[6][h0:h1])
        split = fwd_bwd(*shard)
        for name, x, y in zip(NAMES[:6], split[:6], out[:6]):
            y = y[b0:b1, h0:h1].double()
            err = float((x.double() - y).abs().max() / y.abs().max())
            assert err <= 2e-3, (world, rank, name, err)
    # Summed over the ranks' partials (another order of the same additions), dbeta agrees to rounding.
    total = torch.zeros(H, device="cuda")
    for rank in range(world):
        z0, z1 = bench.head_shard(B, H, rank, world)
        _, _, h0, h1 = bench.shard_block(H, z0, z1)
        total[h0:h1] += _unsplit(fwd_bwd, *(bench.take_heads(x, z0, z1, H).contiguous() for x in inp))[6]
    assert torch.allclose(total, out[6], rtol=1e-5, atol=0)
