"""Head sharding of the benchmark's multi-GPU runs, checked with 2 CPU ranks over gloo: each rank computes the
forward and backward of its block of heads, and the gathered results equal the single-process computation (the
heads are independent; dbeta, a per-head sum over the batch, is the sum of the ranks' partials). Also checks that
a rank that fails before a collective makes the other rank's collective fail within the process-group timeout
instead of hanging."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench
from first_passage_attention_b200 import first_passage_attention


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(3)
    B, H, T, D = 2, 3, 40, 16
    q, k, v, do = (torch.randn(B, H, T, D, generator=g, dtype=torch.float64) for _ in range(4))
    phi = torch.randn(B, H, T, generator=g, dtype=torch.float64).cumsum(-1)
    psi = phi + torch.randn(B, H, T, generator=g, dtype=torch.float64)
    beta = torch.rand(H, generator=g, dtype=torch.float64) + 0.5
    return q, k, v, phi, psi, beta, do


def _fwd_bwd(q, k, v, phi, psi, beta, do):
    leaves = [t.clone().requires_grad_() for t in (q, k, v, phi, psi, beta)]
    o = first_passage_attention(*leaves, impl="reference")
    grads = torch.autograd.grad(o, leaves, do)
    return [o.detach()] + list(grads)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    q, k, v, phi, psi, beta, do = _inputs()
    B, H = q.shape[:2]
    z0, z1 = bench.head_shard(B, H, rank, world)
    part = _fwd_bwd(*(bench.take_heads(t, z0, z1, H) for t in (q, k, v, phi, psi, beta, do)))
    gathered = []
    for x in part[:6]:                       # o, dq, dk, dv, dphi, dpsi: [1, n, ...] per rank
        bufs = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(bufs, x.contiguous())
        gathered.append(torch.cat(bufs, 1).reshape(B, H, *x.shape[2:]))
    dbeta = torch.zeros(H, dtype=torch.float64)
    dbeta.index_add_(0, torch.arange(z0, z1) % H, part[6])
    dist.all_reduce(dbeta)
    if rank == 0:
        out.put([t.numpy() for t in gathered + [dbeta]])
    dist.destroy_process_group()


def test_head_shards_reassemble_the_full_result():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    world, port = 2, _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    got = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full = _fwd_bwd(*_inputs())
    for a, b in zip(got, full):
        assert torch.allclose(torch.from_numpy(a), b, rtol=1e-12, atol=1e-12)


def test_head_shard_rejects_uneven_split():
    with pytest.raises(ValueError):
        bench.head_shard(4, 12, 0, 5)
    assert bench.head_shard(4, 12, 3, 8) == (18, 24)


def _failing_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(3)                          # dies between steps, before the next collective
    try:
        dist.all_reduce(torch.ones(1))
        out.put("returned")
    except Exception as e:                   # gloo reports the lost peer or the timeout
        out.put(type(e).__name__)


def test_a_dead_rank_fails_the_collective_instead_of_hanging():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    world, port = 2, _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert res != "returned"
