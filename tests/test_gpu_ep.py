"""Expert parallelism on 2 GPUs (NCCL all-to-all over NVLink) with the batched MoE kernel on each
rank's half of the experts, against the batched MoE of all experts on one GPU.  Skipped with fewer
than two GPUs; ranks are child processes with a short process-group timeout."""

import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

H, I, E, K, G, BITS, N = 2048, 768, 16, 8, 128, 4, 16  # N tokens per rank


def _setup(device):
    from wisp import quant

    gen = torch.Generator(device=device).manual_seed(3)
    n = H * I
    pool = quant.quantize_batch((torch.randn(E, 3, n, device=device, generator=gen) * 0.02).to(torch.bfloat16), BITS, G)
    return pool


def _tokens(rank, device):
    gen = torch.Generator(device=device).manual_seed(100 + rank)
    x = torch.randn(N, H, device=device, generator=gen).to(torch.bfloat16)
    sel = torch.stack([torch.randperm(E, device=device, generator=gen)[:K] for _ in range(N)])
    w = torch.softmax(torch.randn(N, K, device=device, generator=gen), 1).to(torch.bfloat16).float()
    return x, sel, w


def _lib_status(dev):
    from wisp import _lib

    return _lib.device_status(dev.index, clear=True)


def _worker(rank, world, port, q):
    from datetime import timedelta

    import torch.distributed as dist

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from wisp import kernels
        from wisp.ep import ExpertParallelMoE, batched_expert_fn

        pool = _setup(dev)
        El = E // world
        local = pool[rank * El : (rank + 1) * El].contiguous()
        fn = batched_expert_fn(local, lambda l, e: l * El + e, H * I, H, I, BITS, G)
        x, sel, w = _tokens(rank, dev)
        meta = torch.cat([sel.float(), w], 1).contiguous()
        ref = kernels.moe_batched(pool, meta, x, K, H * I, H, I, BITS, G)
        errs = []
        # torch bucketing + NCCL, the dispatch/combine kernels + NCCL, then the peer-memory transport
        for slot_base, transport in ((None, "nccl"), (lambda l: l * El, "nccl"), (lambda l: l * El, "p2p")):
            ep = ExpertParallelMoE(E, K, H, N, fn, device=dev, slot_base=slot_base, transport=transport)
            for _ in range(3):  # consecutive calls alternate the p2p buffer sets
                out = ep.forward(x, sel, w)
            torch.cuda.synchronize()
            errs.append((out.float() - ref.float()).abs().max().item() / ref.float().abs().max().item())
            ep.close()
        assert kernels.__name__ and _lib_status(dev) == 0
        q.put((rank, max(errs)))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2 if torch.cuda.is_available() else True, reason="needs 2 GPUs")
def test_two_gpu_expert_parallel_matches_single_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 200
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err in res:
        # each pair's expert output is rounded to bf16 before the weighted sum (the reference's
        # per-expert path rounds the same way); the one-GPU kernel sums in fp32
        assert err < 1e-2, (rank, err)


def test_dispatch_combine_kernels_one_rank():
    """wisp_ep_dispatch / wisp_ep_combine with world = 1 (no process group): the kernel path matches the
    torch bucketing path (the same bf16 expert outputs, summed in a fixed order instead of torch's
    reduction: within one bf16 rounding), and the packed meta rows carry [slot_base + expert, 1] in
    pair order with [-1, 0] nowhere (one rank receives every pair)."""
    from wisp import kernels
    from wisp.ep import ExpertParallelMoE, batched_expert_fn

    dev = torch.device("cuda", 0)
    pool = _setup(dev)
    fn = batched_expert_fn(pool, lambda l, e: l * E + e, H * I, H, I, BITS, G)
    x, sel, w = _tokens(0, dev)
    a = ExpertParallelMoE(E, K, H, N, fn, device=dev).forward(x, sel, w)
    kp = ExpertParallelMoE(E, K, H, N, fn, device=dev, slot_base=lambda l: l * E)
    b = kp.forward(x, sel, w)
    assert (a.float() - b.float()).abs().max().item() <= 2.0**-7 * a.float().abs().max().item()
    meta = kp.send_meta.view(-1, 2).cpu()
    assert torch.equal(meta[:, 0], sel.reshape(-1).float().cpu()) and bool((meta[:, 1] == 1).all())
    assert torch.equal(kp.src_pos.cpu(), torch.arange(N * K, dtype=torch.int32))
    assert torch.equal(kp.send_x.view(N * K, H).cpu(), x.repeat_interleave(K, 0).cpu())


def test_dispatch_buckets_by_destination_rank():
    """world = 4 packing on one GPU (no exchange): every pair lands in its owner's bucket at its rank
    among that owner's pairs, unused capacity is [-1, 0], and combine over a y equal to the packed x
    returns sum_j w_j x (the row each pair carried)."""
    from wisp import kernels

    dev = torch.device("cuda", 0)
    world, El = 4, E // 4
    x, sel, w = _tokens(1, dev)
    C = N * K
    send_x = torch.zeros(world, C, H, dtype=torch.bfloat16, device=dev)
    send_meta = torch.zeros(world, C, 2, dtype=torch.float32, device=dev)
    src_pos = torch.zeros(N * K, dtype=torch.int32, device=dev)
    kernels.ep_dispatch(x, sel.contiguous(), El, world, C, 100, send_x, send_meta, src_pos)
    s, m, sp = sel.cpu().reshape(-1), send_meta.cpu(), src_pos.cpu()
    seen = [0] * world
    for p in range(N * K):
        d = int(s[p]) // El
        assert int(sp[p]) == d * C + seen[d]
        assert m[d, seen[d]].tolist() == [100.0 + int(s[p]) - d * El, 1.0]
        assert torch.equal(send_x[d, seen[d]].cpu(), x[p // K].cpu())
        seen[d] += 1
    for d in range(world):
        assert bool((m[d, seen[d]:, 0] == -1).all()) and bool((m[d, seen[d]:, 1] == 0).all())
    out = torch.empty(N, H, dtype=torch.bfloat16, device=dev)
    kernels.ep_combine(send_x.view(world * C, H), src_pos, w, out)
    want = (w.view(N, K, 1) * x.float().view(N, 1, H)).sum(1)
    assert (out.float() - want).abs().max().item() <= 1e-2 * want.abs().max().item()


def test_p2p_transport_one_rank_matches_kernel_path():
    """The peer-memory transport with world = 1 (the exchange is this GPU's own buffers): the same
    result as the kernel path over consecutive calls (alternating buffer sets, increasing epochs), and
    no wait ran out."""
    from wisp import _lib
    from wisp.ep import ExpertParallelMoE, batched_expert_fn

    dev = torch.device("cuda", 0)
    pool = _setup(dev)
    fn = batched_expert_fn(pool, lambda l, e: l * E + e, H * I, H, I, BITS, G)
    a = ExpertParallelMoE(E, K, H, N, fn, device=dev, slot_base=lambda l: l * E)
    b = ExpertParallelMoE(E, K, H, N, fn, device=dev, slot_base=lambda l: l * E, transport="p2p")
    _lib.device_status(0, clear=True)
    for seed in range(4):
        x, sel, w = _tokens(seed, dev)
        assert torch.equal(a.forward(x, sel, w), b.forward(x, sel, w)), seed
    torch.cuda.synchronize()
    assert _lib.device_status(0) == 0
    b.close()


def test_p2p_wait_runs_out_and_reports():
    """A wait for a flag that nothing raises ends after its bound (2 s) with WISP_STATUS_WAIT_TIMEOUT
    instead of hanging, and the context stays usable."""
    from wisp import _lib, kernels

    dev = torch.device("cuda", 0)
    ex = kernels.P2PExchange(1, 0, 8, 64, dev)
    ex.open([ex.handle])
    x = torch.zeros(1, 64, dtype=torch.bfloat16, device=dev)
    sel = torch.zeros(1, 1, dtype=torch.int64, device=dev)
    src_pos = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.device_status(0, clear=True)
    ex.dispatch(x, sel, 4, 0, 0, src_pos)  # raises the dispatch flag to epoch 1
    ex.wait_dispatch(x)
    torch.cuda.synchronize()
    assert _lib.device_status(0) == 0
    _lib.call("wisp_ep_wait", ex.local, 1, 8, 64, 1, _stream0())  # the return flag is never raised
    torch.cuda.synchronize()
    assert _lib.device_status(0, clear=True) & _lib.STATUS_WAIT_TIMEOUT
    assert (x + 1).sum().item() == 64  # the context still works
    ex.close()


def _stream0():
    return torch.cuda.current_stream(0).cuda_stream


@pytest.mark.parametrize("world", [2, 4, 8])
def test_emulated_ranks_kernel_path_matches_oracle(world):
    """``world`` ranks emulated on one GPU, 32 tokens in total: each rank's pairs go through
    wisp_ep_dispatch (its routing rows, capacity slots and src_pos bit-exact with dispatch_plan, the
    rows equal to the token rows), the all-to-all is a permutation of the send buffers, each rank runs
    the batched MoE on its own contiguous slice of the experts, the results travel back and
    wisp_ep_combine sums them -- the whole against the oracle's batched MoE over all tokens."""
    import numpy as np

    from oracle import wisp_oracle as O
    from wisp import _lib, kernels, quant
    from wisp.ep import dispatch_plan

    dev = torch.device("cuda", 0)
    Hs, Is, Es, Ks, Ntot, bits, G = 256, 128, 16, 4, 32, 4, 128
    n = Hs * Is
    El, Nr = Es // world, Ntot // world
    C = Nr * Ks
    gen = torch.Generator(device="cuda").manual_seed(world)
    pool = quant.quantize_batch((torch.randn(Es, 3, n, device=dev, generator=gen) * 0.05).to(torch.bfloat16), bits, G)
    x = torch.randn(Ntot, Hs, device=dev, generator=gen).to(torch.bfloat16)
    logits = torch.randn(Ntot, Es, device=dev, generator=gen)
    sel_np, rw_np = O.router_topk(logits.to(torch.bfloat16).float().cpu().numpy(), Ks)
    sel = torch.from_numpy(sel_np).to(dev).contiguous()
    w = torch.from_numpy(rw_np).to(dev).float().contiguous()
    _lib.device_status(0)
    sends, metas, srcs = [], [], []
    for r in range(world):
        xr, sr = x[r * Nr : (r + 1) * Nr].contiguous(), sel[r * Nr : (r + 1) * Nr].contiguous()
        sx = torch.zeros(world, C, Hs, dtype=torch.bfloat16, device=dev)
        sm = torch.zeros(world, C, 2, dtype=torch.float32, device=dev)
        sp = torch.zeros(Nr * Ks, dtype=torch.int32, device=dev)
        kernels.ep_dispatch(xr, sr, El, world, C, 0, sx, sm, sp)
        dest, cap, meta, src_pos = dispatch_plan(sr.cpu(), El, world, C, 0)
        assert torch.equal(sm.cpu(), meta) and torch.equal(sp.cpu(), src_pos), r
        assert torch.equal(sx[dest, cap].cpu(), xr.cpu()[torch.arange(Nr * Ks) // Ks]), r
        sends.append(sx)
        metas.append(sm)
        srcs.append(sp)
    ys = []
    for d in range(world):  # rank d receives block d of every source, runs its experts (slots 0..El-1)
        rx = torch.stack([sends[s][d] for s in range(world)]).view(world * C, Hs).contiguous()
        rm = torch.stack([metas[s][d] for s in range(world)]).view(world * C, 2).contiguous()
        ys.append(kernels.moe_batched(pool[d * El : (d + 1) * El].contiguous(), rm, rx, 1, n, Hs, Is, bits, G))
    outs = []
    for s in range(world):  # results of source s come back from every rank d
        back = torch.stack([ys[d][s * C : (s + 1) * C] for d in range(world)]).view(world * C, Hs).contiguous()
        out = torch.empty(Nr, Hs, dtype=torch.bfloat16, device=dev)
        kernels.ep_combine(back, srcs[s], w[s * Nr : (s + 1) * Nr].contiguous(), out)
        outs.append(out)
    got = torch.cat(outs).float().cpu().numpy()
    want = O.moe_batched_ref(pool.cpu().numpy(), sel_np, rw_np, O.bf16_bits_to_f32(x.view(torch.int16).cpu().numpy().view(np.uint16)),
                             n, Hs, Is, bits, G)
    assert float(np.abs(got - want).max() / np.abs(want).max()) < 1e-2
    assert _lib.device_status(0) == 0
