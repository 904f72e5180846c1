"""The batched MoE on the 5th-generation tensor cores (wisp_moe_batched_variant path 2: TMA-fed
dequantization to fp16 in shared memory, tcgen05.mma with TMEM accumulators) against the oracle's fp32
batched reference and the warp-level tensor-core path (path 1), through the C ABI.  Cases: the Qwen3
layer at 1 to 256 tokens (uniform and Zipf routing), an expert receiving more tokens than one N tile
holds, empty pairs, several weight-row tiles at a small shape, 4-bit and 2-bit codes, repeatability,
and a sabotage control."""

import numpy as np
import pytest
import torch

from oracle import wisp_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2  # relative to max |oracle|


def _np(t):
    return O.bf16_bits_to_f32(t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16))


def _rel(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def _routing(N, E, k, seed, zipf=None):
    gen = torch.Generator().manual_seed(seed)
    logits = torch.randn(N, E, generator=gen)
    if zipf is not None:
        rank = torch.randperm(E, generator=gen).float() + 1
        logits = logits + torch.log(rank ** -zipf)[None, :]
    return O.router_topk(logits.to(torch.bfloat16).float().numpy(), k)


def _pool(E, n, bits, G, used, seed, std=0.02):
    from wisp import quant

    gen = torch.Generator(device="cuda").manual_seed(seed)
    pool = torch.zeros((E, quant.expert_nbytes(n, bits, G)), dtype=torch.uint8, device="cuda")
    w3 = (torch.randn(len(used), 3, n, device="cuda", generator=gen) * std).to(torch.bfloat16)
    pool[torch.as_tensor(used, device="cuda")] = quant.quantize_batch(w3, bits, G)
    return pool, gen


def _meta(sel, rw):
    return torch.from_numpy(np.concatenate([sel.astype(np.float32), rw.astype(np.float32)], 1)).cuda().contiguous()


@pytest.mark.parametrize("bits", [4, 2])
@pytest.mark.parametrize("N,zipf", [(1, None), (8, None), (64, 1.1), (256, None)])
def test_qwen3_layer_paths_match_oracle(bits, N, zipf):
    from wisp import _lib, kernels

    if N == 256 and bits == 2:
        pytest.skip("one prefill-sized case is enough")
    H, I, E, k, G = 2048, 768, 128, 8, 128
    n = H * I
    sel, rw = _routing(N, E, k, seed=100 + N + bits, zipf=zipf)
    used = np.unique(sel)
    pool, gen = _pool(E, n, bits, G, used, seed=bits * 7 + N)
    x = torch.randn(N, H, device="cuda", generator=gen).to(torch.bfloat16)
    meta = _meta(sel, rw)
    _lib.device_status(0)
    want = O.moe_batched_ref(pool.cpu().numpy(), sel, rw, _np(x), n, H, I, bits, G)
    got2 = kernels.moe_batched(pool, meta, x, k, n, H, I, bits, G, variant=2)
    got1 = kernels.moe_batched(pool, meta, x, k, n, H, I, bits, G, variant=1)
    assert _rel(_np(got2), want) < TOL, _rel(_np(got2), want)
    assert _rel(_np(got1), want) < TOL
    assert torch.equal(kernels.moe_batched(pool, meta, x, k, n, H, I, bits, G, variant=2), got2)  # repeatable
    assert _lib.device_status(0) == 0
    # sabotage: a shifted expert choice misses by far more than the tolerance
    bad = _meta((sel + 1) % E, rw)
    assert _rel(_np(kernels.moe_batched(pool, bad, x, k, n, H, I, bits, G, variant=2)), want) > 10 * TOL


@pytest.mark.parametrize("bits", [4, 2])
def test_expert_with_several_token_tiles(bits):
    """One expert receives 300 tokens (four N tiles of 64 and one of 44), another 17, with k = 1."""
    from wisp import _lib, kernels

    H, I, E, k, G = 256, 128, 4, 1, 128
    n = H * I
    N = 317
    sel = np.full((N, 1), 2, np.int64)
    sel[::19] = 1
    rw = np.random.default_rng(3).uniform(0.2, 1.0, (N, 1)).astype(np.float32)
    rw = O.bf16_bits_to_f32(O.f32_to_bf16_bits(rw))
    pool, gen = _pool(E, n, bits, G, [1, 2], seed=5, std=0.05)
    x = torch.randn(N, H, device="cuda", generator=gen).to(torch.bfloat16)
    _lib.device_status(0)
    got = kernels.moe_batched(pool, _meta(sel, rw), x, k, n, H, I, bits, G, variant=2)
    want = O.moe_batched_ref(pool.cpu().numpy(), sel, rw, _np(x), n, H, I, bits, G)
    assert (sel == 2).sum() > 256
    assert _rel(_np(got), want) < TOL
    assert _lib.device_status(0) == 0


def test_empty_pairs_and_several_row_tiles():
    """H = 384 and I = 256: three down tiles and two gate/up tiles of 128 rows; pairs with slot -1 (the
    padding of an expert-parallel buffer) contribute nothing and raise no flag."""
    from wisp import _lib, kernels

    H, I, E, k, G, bits = 384, 256, 6, 3, 128, 4
    n = H * I
    N = 40
    rng = np.random.default_rng(9)
    sel = np.stack([rng.choice(E, k, replace=False) for _ in range(N)])
    rw = O.bf16_bits_to_f32(O.f32_to_bf16_bits(rng.uniform(0.1, 0.6, (N, k)).astype(np.float32)))
    empty = rng.random((N, k)) < 0.3
    pool, gen = _pool(E, n, bits, G, list(range(E)), seed=11, std=0.05)
    x = torch.randn(N, H, device="cuda", generator=gen).to(torch.bfloat16)
    msel = np.where(empty, -1, sel)
    mrw = np.where(empty, 0.0, rw).astype(np.float32)
    _lib.device_status(0)
    got = kernels.moe_batched(pool, _meta(msel, mrw), x, k, n, H, I, bits, G, variant=2)
    want = O.moe_batched_ref(pool.cpu().numpy(), np.where(empty, 0, sel), mrw, _np(x), n, H, I, bits, G)
    assert _rel(_np(got), want) < TOL
    assert _lib.device_status(0) == 0


def test_path_two_needs_its_formats():
    from wisp import kernels, quant
    from wisp._lib import WispError

    H, I, E, k, G = 256, 128, 2, 1, 128
    n = H * I
    pool = quant.quantize_batch(torch.randn(E, 3, n, device="cuda").to(torch.bfloat16) * 0.02, 3, G)
    x = torch.randn(4, H, device="cuda").to(torch.bfloat16)
    meta = _meta(np.zeros((4, 1), np.int64), np.ones((4, 1), np.float32))
    with pytest.raises(WispError, match="tensor-core path"):
        kernels.moe_batched(pool, meta, x, k, n, H, I, 3, G, variant=2)
    kernels.moe_batched(pool, meta, x, k, n, H, I, 3, G, variant=0)  # automatic falls back
