"""Chunked prefill of the decoder (the reference's GraphDecoder.prefill, wisp/graphdec.py:99-152):
the prompt in chunks through GEMMs, the q/k norm + rotary + cache-write rows kernel, causal attention
and the batched MoE kernel, against the same prompt fed one decode step per token.  The two paths
round differently (GEMM vs GEMV accumulation order, the MoE kernels' fixed point), so logits and
caches agree to a tolerance, and the routing they lead to must agree."""

import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 3e-2  # relative to max |logit| / max |cache entry|


def _cfg(**kw):
    from wisp.model import DecoderConfig

    base = dict(vocab=2000, hidden=2048, layers=2, heads=32, kv_heads=4, head_dim=128, experts=32, top_k=8, moe_inter=768)
    base.update(kw)
    return DecoderConfig(**base)


def _close(a, b, tol=TOL):
    a, b = a.float(), b.float()
    return (a - b).abs().max().item() <= tol * b.abs().max().item()


@pytest.mark.parametrize("chunk", [16, 256])
def test_chunked_prefill_matches_stepwise(chunk):
    from wisp.graphdec import GraphDecoder
    from wisp.model import DecoderWeights

    cfg = _cfg()
    w = DecoderWeights.random(cfg, seed=21)
    ids = torch.randint(0, cfg.vocab, (41,), device="cuda", generator=torch.Generator("cuda").manual_seed(2))
    a = GraphDecoder(w, tmax=128)
    b = GraphDecoder(w, tmax=128)
    la = a.prefill(ids, chunk=chunk).clone()  # 41 = 16 + 16 + 9 at chunk 16: a ragged last chunk
    lb = None
    for t in ids:
        lb = b.next(t.reshape(1))
    assert a.pos == b.pos == 41
    assert _close(la, lb)
    T = 41
    assert _close(a.kc[:, :, :T], b.kc[:, :, :T]) and _close(a.vc[:, :, :T], b.vc[:, :, :T])
    # continuing from either context gives the same greedy tokens
    t0 = lb.argmax().reshape(1)
    assert torch.equal(a.greedy(t0, 6), b.greedy(t0, 6))


def test_prefill_continues_a_context():
    """Two prefills in a row (the second reusing the first's KV, as prefix reuse does) equal one."""
    from wisp.graphdec import GraphDecoder
    from wisp.model import DecoderWeights

    cfg = _cfg(layers=1)
    w = DecoderWeights.random(cfg, seed=4)
    ids = torch.randint(0, cfg.vocab, (30,), device="cuda", generator=torch.Generator("cuda").manual_seed(8))
    a = GraphDecoder(w, tmax=64)
    b = GraphDecoder(w, tmax=64)
    a.prefill(ids[:17])
    la = a.prefill(ids[17:])
    lb = b.prefill(ids)
    assert a.pos == b.pos == 30
    assert torch.equal(la, lb) or _close(la, lb, 1e-2)
    assert _close(a.kc[:, :, :30], b.kc[:, :, :30], 1e-2)


def test_prefill_with_a_capped_cache():
    """Device-paged decoder with 10% of the experts resident: the prefill pages each layer's experts in
    groups the pool can hold; the logits equal the all-resident decoder's prefill."""
    from wisp.cache import ExpertCache
    from wisp.graphdec import DevicePagedDecoder, GraphDecoder
    from wisp.model import DecoderWeights
    from wisp.store import ExpertStore

    cfg = _cfg(layers=3)
    w = DecoderWeights.random(cfg, seed=11)
    store = ExpertStore.from_pool(w.pool, cfg.hidden * cfg.moe_inter, cfg.bits, cfg.group, cfg.layers, cfg.experts)
    cache = ExpertCache(store, nslots=int(0.1 * cfg.layers * cfg.experts))
    ids = torch.randint(0, cfg.vocab, (24,), device="cuda", generator=torch.Generator("cuda").manual_seed(9))
    a = GraphDecoder(w, tmax=64)
    b = DevicePagedDecoder(w, cache, tmax=64)
    la = a.prefill(ids).clone()
    lb = b.prefill(ids)
    assert _close(la, lb, 1e-2)
    assert cache.stats["misses"] > 0
    # the paged prefill sums groups of experts in bf16, so its cache differs from the resident one by
    # rounding; with the same cache contents the paged decode steps are bit-identical to the resident ones
    b.kc.copy_(a.kc)
    b.vc.copy_(a.vc)
    t = la.argmax().reshape(1)
    for _ in range(4):
        x, y = a.next(t).clone(), b.next(t)
        assert torch.equal(x, y)
        t = x.argmax().reshape(1)


def test_resize_keeps_the_context():
    from wisp.graphdec import GraphDecoder
    from wisp.model import DecoderWeights

    cfg = _cfg(layers=1)
    w = DecoderWeights.random(cfg, seed=6)
    ids = torch.randint(0, cfg.vocab, (20,), device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    a = GraphDecoder(w, tmax=64)
    b = GraphDecoder(w, tmax=64)
    a.prefill(ids)
    b.prefill(ids)
    t = torch.tensor([7], device="cuda")
    b.next(t)  # captures a graph at the old capacity
    b = GraphDecoder(w, tmax=64)
    b.prefill(ids)
    b.resize(200)
    assert b.tmax == 256 and b.pos == 20 and b.kc.shape[2] == 256
    assert torch.equal(a.next(t), b.next(t))
