"""Expert-parallel dispatch/combine (the exchange steps of 64-token expert-parallel decode) on CPU: world_size-2 gloo
ranks, each with its own tokens and half of the experts, against the same MoE computed on one process.
The expert compute is a dense fp32 stand-in; the GPU path swaps in the batched MoE kernel."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, I, E, K, N = 32, 16, 8, 3, 5  # per-rank tokens N


def _experts(seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(E, I, H, generator=g) * 0.3, torch.randn(E, I, H, generator=g) * 0.3,
            torch.randn(E, H, I, generator=g) * 0.3)


def _expert(e, x, W):
    wg, wu, wd = W
    return (torch.nn.functional.silu(x @ wg[e].T) * (x @ wu[e].T)) @ wd[e].T


def _routing(rank, seed=1):
    g = torch.Generator().manual_seed(seed + rank)
    x = torch.randn(N, H, generator=g)
    sel = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(N)])
    w = torch.softmax(torch.randn(N, K, generator=g), 1)
    return x, sel, w


def _reference(rank, W):
    x, sel, w = _routing(rank)
    out = torch.zeros(N, H)
    for t in range(N):
        for j in range(K):
            out[t] += w[t, j] * _expert(int(sel[t, j]), x[t], W)
    return out


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from wisp.ep import ExpertParallelMoE

        W = _experts()
        E_local = E // world
        lo = rank * E_local

        def fn(xr, ids, layer):  # dense stand-in for the local experts
            y = torch.zeros_like(xr)
            for r in range(xr.shape[0]):
                if ids[r] >= 0:
                    y[r] = _expert(lo + int(ids[r]), xr[r], W)
            return y

        ep = ExpertParallelMoE(E, K, H, N, fn, device="cpu", dtype=torch.float32)
        x, sel, w = _routing(rank)
        out = ep.forward(x, sel, w)
        q.put((rank, (out - _reference(rank, W)).abs().max().item(), _reference(rank, W).abs().max().item()))
    finally:
        dist.destroy_process_group()


def test_two_rank_dispatch_combine_matches_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, scale in res:
        assert err <= 1e-5 * max(1.0, scale), (rank, err)


def test_single_process_world_one():
    from wisp.ep import ExpertParallelMoE

    W = _experts()

    def fn(xr, ids, layer):
        y = torch.zeros_like(xr)
        for r in range(xr.shape[0]):
            if ids[r] >= 0:
                y[r] = _expert(int(ids[r]), xr[r], W)
        return y

    ep = ExpertParallelMoE(E, K, H, N, fn, device="cpu", dtype=torch.float32)
    x, sel, w = _routing(0)
    assert torch.allclose(ep.forward(x, sel, w), _reference(0, W), atol=1e-5)
