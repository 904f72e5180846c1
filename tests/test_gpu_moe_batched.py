"""GPU parity of the batched MoE (N tokens, each its own top-k; N = 1, 4, 16 and the 64-token
expert-parallel shape) through the C ABI: against the reference PagedMoEBlock outputs
(fixture moe_block.npz, both of its branches), the oracle's fp32 batched reference at the Qwen3 layer
shape, and the bs=1 kernels."""

import numpy as np
import pytest
import torch

from oracle import wisp_oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _np(t):
    return O.bf16_bits_to_f32(t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16))


def _rel(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


@pytest.mark.parametrize("bits", [4, 3, 2])
@pytest.mark.parametrize("N", [1, 4, 16])
def test_matches_reference_paged_block(golden, bits, N):
    from wisp import kernels

    g = golden("moe_block")
    H, I, k, G = int(g["H"]), int(g["I"]), int(g["k"]), int(g["G"])
    pool = torch.from_numpy(g[f"pool_b{bits}"]).cuda()
    x = torch.from_numpy(g[f"x_b{bits}_N{N}"].view(np.int16)).view(torch.bfloat16).cuda()
    sel = g[f"sel_b{bits}_N{N}"]
    rw = O.bf16_bits_to_f32(g[f"rw_b{bits}_N{N}"])
    meta = torch.from_numpy(np.concatenate([sel.astype(np.float32), rw], 1)).cuda().contiguous()
    out = kernels.moe_batched(pool, meta, x, k, H * I, H, I, bits, G)
    ref = O.bf16_bits_to_f32(g[f"out_b{bits}_N{N}"])
    # the reference computes in bf16 (dequantized weights, bf16 matmuls): 2e-2 as in its own tests
    assert _rel(_np(out), ref) < 2e-2
    want = O.moe_batched_ref(g[f"pool_b{bits}"], sel, rw, _np(x), H * I, H, I, bits, G)
    assert _rel(_np(out), want) < TOL


def _routing(N, E, k, seed, zipf=None):
    gen = torch.Generator().manual_seed(seed)
    logits = torch.randn(N, E, generator=gen)
    if zipf is not None:  # popularity ~ Zipf(s) over a seeded permutation of the experts
        rank = torch.randperm(E, generator=gen).float() + 1
        logits = logits + torch.log(rank ** -zipf)[None, :]
    sel, rw = O.router_topk(logits.to(torch.bfloat16).float().numpy(), k)
    return sel, rw


@pytest.mark.parametrize("bits", [4, 3, 2])
@pytest.mark.parametrize("N", [4, 16])
def test_qwen3_layer_vs_oracle(bits, N):
    """Config 2: the Qwen3-30B-A3B layer (H 2048, I 768, 128 experts, top-8), N tokens with their own
    seeded top-8."""
    from wisp import kernels, quant

    H, I, E, k, G = 2048, 768, 128, 8, 128
    n = H * I
    sel, rw = _routing(N, E, k, seed=bits * 10 + N)
    used = np.unique(sel)
    gen = torch.Generator(device="cuda").manual_seed(bits + N)
    pool = torch.zeros((E, quant.expert_nbytes(n, bits, G)), dtype=torch.uint8, device="cuda")
    w3 = (torch.randn(len(used), 3, n, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    pool[torch.from_numpy(used).cuda()] = quant.quantize_batch(w3, bits, G)
    x = torch.randn(N, H, device="cuda", generator=gen).to(torch.bfloat16)
    meta = torch.from_numpy(np.concatenate([sel.astype(np.float32), rw], 1)).cuda().contiguous()
    out = kernels.moe_batched(pool, meta, x, k, n, H, I, bits, G)
    want = O.moe_batched_ref(pool.cpu().numpy(), sel, rw, _np(x), n, H, I, bits, G)
    assert _rel(_np(out), want) < TOL
    # sabotage control: a shifted expert choice misses by far more than the tolerance
    bad = torch.from_numpy(np.concatenate([((sel + 1) % E).astype(np.float32), rw], 1)).cuda().contiguous()
    assert _rel(_np(kernels.moe_batched(pool, bad, x, k, n, H, I, bits, G)), want) > 10 * TOL


def test_batch64_zipf_and_single_token_agreement():
    """Config 4 batch shape (64 tokens, Zipf(1.1) popularity: popular experts get many tokens), and
    N = 1 against the bs=1 decode kernels."""
    from wisp import _lib, kernels, quant

    H, I, E, k, G, bits = 2048, 768, 128, 8, 128, 4
    n = H * I
    sel, rw = _routing(64, E, k, seed=64, zipf=1.1)
    gen = torch.Generator(device="cuda").manual_seed(5)
    w3 = (torch.randn(E, 3, n, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    pool = quant.quantize_batch(w3, bits, G)
    del w3
    x = torch.randn(64, H, device="cuda", generator=gen).to(torch.bfloat16)
    meta = torch.from_numpy(np.concatenate([sel.astype(np.float32), rw], 1)).cuda().contiguous()
    _lib.device_status(0, clear=True)
    out = kernels.moe_batched(pool, meta, x, k, n, H, I, bits, G)
    pn = pool.cpu().numpy()
    want = O.moe_batched_ref(pn, sel, rw, _np(x), n, H, I, bits, G)
    assert _rel(_np(out), want) < TOL
    assert _lib.device_status(0) == 0
    one = kernels.moe_batched(pool, meta[:1].contiguous(), x[:1].contiguous(), k, n, H, I, bits, G)
    dec = kernels.moe_decode_fast(pool, meta[0].contiguous(), x[0], k, n, H, I, bits, G)
    assert _rel(_np(one)[0], _np(dec)) < TOL


def test_invalid_slot_skipped_and_flagged():
    from wisp import _lib, kernels, quant

    H, I, E, k, G, bits = 256, 128, 4, 2, 128, 4
    n = H * I
    gen = torch.Generator(device="cuda").manual_seed(1)
    pool = quant.quantize_batch((torch.randn(E, 3, n, device="cuda", generator=gen) * 0.02).to(torch.bfloat16), bits, G)
    x = torch.randn(3, H, device="cuda", generator=gen).to(torch.bfloat16)
    meta = torch.tensor([[0, 1, 0.5, 0.5], [2, 99, 0.5, 0.5], [3, -1, 0.5, 0.5]], dtype=torch.float32, device="cuda")
    _lib.device_status(0, clear=True)
    kernels.moe_batched(pool, meta[2:].contiguous(), x[2:].contiguous(), k, n, H, I, bits, G)
    assert _lib.device_status(0) == 0  # -1: an empty pair, not an error
    out = kernels.moe_batched(pool, meta, x, k, n, H, I, bits, G)
    assert _lib.device_status(0) & _lib.STATUS_BAD_SLOT  # 99: out of range
    sel = np.array([[0, 1], [2, 2], [3, 3]])
    rw = np.array([[0.5, 0.5], [0.5, 0.0], [0.5, 0.0]], np.float32)
    want = O.moe_batched_ref(pool.cpu().numpy(), sel, rw, _np(x), n, H, I, bits, G)
    assert _rel(_np(out), want) < TOL
    _lib.device_status(0, clear=True)


@pytest.mark.parametrize("N,k", [(16, 2), (11, 3)])
def test_grouping_either_side_of_the_warp_path(N, k):
    """32 pairs are grouped by one warp, 33 by the one-CTA counting sort; both against the oracle, with
    repeated experts (several tokens per group) and one padded pair."""
    from wisp import kernels, quant

    H, I, E, G, bits = 256, 128, 6, 128, 4
    n = H * I
    gen = torch.Generator(device="cuda").manual_seed(N * k)
    pool = quant.quantize_batch((torch.randn(E, 3, n, device="cuda", generator=gen) * 0.02).to(torch.bfloat16), bits, G)
    x = torch.randn(N, H, device="cuda", generator=gen).to(torch.bfloat16)
    rng = np.random.default_rng(N * k)
    sel = np.stack([rng.choice(E, k, replace=False) for _ in range(N)]).astype(np.int64)
    rw = rng.uniform(0.1, 1.0, (N, k)).astype(np.float32)
    meta_np = np.concatenate([sel.astype(np.float32), rw], 1)
    meta_np[N - 1, k - 1] = -1.0  # a padded pair: skipped, contributes nothing
    rw_ref = rw.copy()
    rw_ref[N - 1, k - 1] = 0.0
    sel_ref = sel.copy()
    sel_ref[N - 1, k - 1] = sel[N - 1, 0]
    out = kernels.moe_batched(pool, torch.from_numpy(meta_np).cuda().contiguous(), x, k, n, H, I, bits, G)
    want = O.moe_batched_ref(pool.cpu().numpy(), sel_ref, rw_ref, _np(x), n, H, I, bits, G)
    assert _rel(_np(out), want) < TOL


def test_reference_named_batched_entry():
    """moe_decode_qb (the reference's planned batched name) is the batched kernel, and each of its rows
    agrees with the bs=1 moe_decode_q4_fast of that token."""
    from wisp import kernels, quant

    H, I, E, k, G, N = 256, 128, 8, 2, 128, 3
    n = H * I
    gen = torch.Generator(device="cuda").manual_seed(11)
    pool = quant.quantize_batch((torch.randn(E, 3, n, device="cuda", generator=gen) * 0.02).to(torch.bfloat16), 4, G)
    x = torch.randn(N, H, device="cuda", generator=gen).to(torch.bfloat16)
    sel = torch.stack([torch.randperm(E, generator=torch.Generator().manual_seed(t))[:k] for t in range(N)]).float()
    meta = torch.cat([sel, torch.full((N, k), 0.5)], 1).cuda().contiguous()
    got = kernels.moe_decode_qb(pool, meta, x, k, n, H, I, block_gu=16)
    assert torch.equal(got.view(torch.int16), kernels.moe_batched(pool, meta, x, k, n, H, I, 4, G).view(torch.int16))
    for t in range(N):
        one = kernels.moe_decode_q4_fast(pool, meta[t].contiguous(), x[t], k, n, H, I)
        assert _rel(_np(got)[t], _np(one)) < TOL
