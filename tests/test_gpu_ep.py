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
        ep = ExpertParallelMoE(E, K, H, N, fn, device=dev)
        x, sel, w = _tokens(rank, dev)
        out = ep.forward(x, sel, w)
        meta = torch.cat([sel.float(), w], 1).contiguous()
        ref = kernels.moe_batched(pool, meta, x, K, H * I, H, I, BITS, G)
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs().max().item() / ref.float().abs().max().item()
        q.put((rank, err))
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
