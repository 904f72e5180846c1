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


# ---- the kernel path's bookkeeping across ranks ------------------------------------------------------
def _kernel_layout_worker(rank, world, port, q):
    """The exchange as the CUDA kernel path lays it out (dispatch_plan / combine_plan: receiver routing
    rows [slot_base + local id, 1], capacity slots, src_pos), moved by gloo all-to-alls."""
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from wisp.ep import combine_plan, dispatch_plan

        W = _experts()
        El, C, base = E // world, N * K, 40  # slot of local expert e = base + e on every rank
        x, sel, w = _routing(rank)
        dest, cap, meta, src_pos = dispatch_plan(sel, El, world, C, base)
        send_x = torch.zeros(world, C, H)
        send_x[dest, cap] = x[torch.arange(N * K) // K]
        recv_x, recv_m = torch.empty_like(send_x), torch.empty_like(meta)
        dist.all_to_all_single(recv_x.view(-1), send_x.view(-1))
        dist.all_to_all_single(recv_m.view(-1), meta.view(-1))
        y = torch.zeros(world * C, H)
        rm, rx = recv_m.view(-1, 2), recv_x.view(-1, H)
        for r in range(world * C):
            if rm[r, 0] >= 0:  # slot -> this rank's expert
                y[r] = rm[r, 1] * _expert(rank * El + int(rm[r, 0]) - base, rx[r], W)
        back = torch.empty_like(y)
        dist.all_to_all_single(back.view(-1), y.view(-1))
        out = combine_plan(back, src_pos, w)
        ref = _reference(rank, W)
        unused = int((meta[..., 0] < 0).sum())
        q.put((rank, (out - ref).abs().max().item(), ref.abs().max().item(), unused))
    finally:
        dist.destroy_process_group()


def _spawn(target, world, extra=()):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() * 7 + world * 131 + len(extra) * 17) % 2000
    procs = [ctx.Process(target=target, args=(r, world, port, q, *extra)) for r in range(world)]
    for p in procs:
        p.start()
    return procs, q


def test_two_rank_kernel_layout_matches_single_process():
    procs, q = _spawn(_kernel_layout_worker, 2)
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, scale, unused in res:
        assert err <= 1e-5 * max(1.0, scale), (rank, err)
        assert unused == 2 * N * K - N * K  # every pair takes one capacity slot somewhere


def test_dispatch_plan_layout():
    from wisp.ep import dispatch_plan

    sel = torch.tensor([[0, 5], [6, 1], [7, 4]])
    dest, cap, meta, src_pos = dispatch_plan(sel, 4, 2, 6, 100)
    assert dest.tolist() == [0, 1, 1, 0, 1, 1] and cap.tolist() == [0, 0, 1, 1, 2, 3]
    assert src_pos.tolist() == [0, 6, 7, 1, 8, 9]
    assert meta[0, :2].tolist() == [[100.0, 1.0], [101.0, 1.0]] and meta[1, :4, 0].tolist() == [101.0, 102.0, 103.0, 100.0]
    assert (meta[0, 2:, 0] == -1).all() and (meta[0, 2:, 1] == 0).all()
    with pytest.raises(ValueError):
        dispatch_plan(sel, 4, 2, 5, 0)


# ---- failures seen on the host ----------------------------------------------------------------------
def _failure_worker(rank, world, port, q, mode):
    """Rank 1 leaves after one step ('exit') or stalls past the group's timeout ('stall'); rank 0's next
    exchange must end with an error instead of waiting forever."""
    import time
    from datetime import timedelta

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=4))
    from wisp.ep import ExpertParallelMoE

    W = _experts()

    def fn(xr, ids, layer):
        y = torch.zeros_like(xr)
        for r in range(xr.shape[0]):
            if ids[r] >= 0:
                y[r] = _expert(rank * (E // world) + int(ids[r]), xr[r], W)
        return y

    ep = ExpertParallelMoE(E, K, H, N, fn, device="cpu", dtype=torch.float32)
    x, sel, w = _routing(rank)
    ep.forward(x, sel, w)  # step 1: every rank takes part
    if rank == 1:
        if mode == "stall":
            time.sleep(12)
        q.put((rank, "left", 0.0))
        q.close()
        q.join_thread()  # the message is out before the process goes
        os._exit(0)  # leaves between steps, with nothing in flight
    t0 = time.time()
    try:
        ep.forward(x, sel, w)
        q.put((rank, "no error", time.time() - t0))
    except Exception as e:  # gloo reports the lost or late peer
        q.put((rank, type(e).__name__, time.time() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_lost_rank_ends_the_next_exchange_with_an_error(mode):
    procs, q = _spawn(_failure_worker, 2, (mode,))
    res = dict((r, (what, dt)) for r, what, dt in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
    what, dt = res[0]
    assert what != "no error", res
    assert dt < 60, res  # bounded by the group timeout (4 s) and connection loss, not a hang
