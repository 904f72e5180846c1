"""The package drop-in on the GPU, driven the way the reference's own callers drive it:

  - ``wisp.moe.PagedMoEBlock`` against the reference block's frozen outputs (moe_block.npz) for every
    WISP_FUSED mode, with the cache all-resident, thrashing in chunks, and the hybrid miss policy;
  - an HF Qwen3-MoE model with ``attach()``ed blocks (prefill through the batched kernel, decode steps
    through the fused ones) against the same HF model running the dequantized experts, over the
    policies of the reference's tests/test_paged_moe.py (lru / wsa / hybrid / prefetch / decode_on_load),
    with a sabotage control;
  - ``GraphDecoder(model, rt, tmax)`` (the reference's constructor): chunked prefill and decode steps
    against HF;
  - ``ExpertCache``: weights_batched / weights / cpu_weights / resize / decode_on_load;
  - ``wisp.gptoss.PagedGptOssBlock`` against the reference block's outputs (gptoss.npz)."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import wisp_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2  # relative to max |reference|: the bar of the MoE tests


def _bf(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16).cuda()


def _np(t):
    return O.bf16_bits_to_f32(t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16))


def _rel(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def _store_cache(rows, n, bits, group, E, nslots, policy="lru", **kw):
    from wisp.cache import ExpertCache
    from wisp.store import ExpertStore

    st = ExpertStore.from_pool(rows.cpu(), n, bits, group, rows.shape[0] // E, E)
    return st, ExpertCache(st, nslots, "cuda", policy, admit_after=1.0, **kw)


# ---- PagedMoEBlock against the reference block's outputs -------------------------------------------
@pytest.mark.parametrize("bits", [4, 3, 2])
@pytest.mark.parametrize("fused", [0, 1, 2])
@pytest.mark.parametrize("nslots,miss", [(16, "transfer"), (6, "transfer"), (6, "hybrid")])
def test_block_matches_reference_outputs(golden, bits, fused, nslots, miss):
    from wisp.moe import PagedMoEBlock, Runtime

    g = golden("moe_block")
    H, I, E, k, G = (int(g[c]) for c in ("H", "I", "E", "k", "G"))
    st, cache = _store_cache(torch.from_numpy(g[f"pool_b{bits}"]), H * I, bits, G, E, nslots)
    rt = Runtime(st, cache, miss_policy=miss, chunk=4, fused=fused)
    rt.fused = fused
    gate = torch.nn.Linear(H, E, bias=False).to("cuda", torch.bfloat16)
    gate.weight.data.copy_(_bf(g[f"gate_b{bits}"]))
    cfg = SimpleNamespace(num_experts=E, num_experts_per_tok=k, norm_topk_prob=True, hidden_size=H, moe_intermediate_size=I)
    blk = PagedMoEBlock(gate, 0, rt, cfg)
    for N in (1, 4, 16):
        x = _bf(g[f"x_b{bits}_N{N}"])[None]
        with torch.no_grad():
            out, logits = blk(x)
        assert torch.equal(logits.view(torch.int16).cpu(), torch.from_numpy(g[f"logits_b{bits}_N{N}"].view(np.int16)))
        # the block's own routing (CUDA topk); bf16 logits can tie at the k-th place, and a tie may break
        # differently than on the reference's CPU, so the frozen output is compared only where they agree
        with torch.no_grad():
            _, sel, rw = blk._route(x[0])
        sel_np, rw_np = sel.cpu().numpy(), rw.float().cpu().numpy()
        want = O.moe_batched_ref(g[f"pool_b{bits}"], sel_np, rw_np, _np(x[0]), H * I, H, I, bits, G)
        assert _rel(_np(out[0]), want) < TOL, (N, _rel(_np(out[0]), want))
        same = (np.sort(sel_np, 1) == np.sort(g[f"sel_b{bits}_N{N}"], 1)).all(1)
        assert same.sum() >= N - 1, N  # at most one tie in a fixture
        ref = O.bf16_bits_to_f32(g[f"out_b{bits}_N{N}"])
        assert _rel(_np(out[0])[same], ref[same]) < 2 * TOL, N
    if nslots < E:
        assert cache.stats["misses"] > 0
    if miss == "hybrid":
        assert rt.stats["cpu_experts"] > 0  # misses of single-token calls served from host memory
    from wisp import _lib

    assert _lib.device_status(0) == 0


# ---- an HF Qwen3-MoE model with attached blocks ---------------------------------------------------------
def _tiny_hf(seed=0, layers=3, boost=True):
    from transformers import AutoModelForCausalLM, Qwen3MoeConfig

    cfg = Qwen3MoeConfig(vocab_size=256, hidden_size=256, intermediate_size=512, moe_intermediate_size=128,
                         num_hidden_layers=layers, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                         num_experts=8, num_experts_per_tok=2, decoder_sparse_step=1, mlp_only_layers=[],
                         norm_topk_prob=True, max_position_embeddings=256, rms_norm_eps=1e-6)
    torch.manual_seed(seed)
    m = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16).cuda().eval()
    if boost:
        with torch.no_grad():  # make the experts matter: default init leaves the MoE almost irrelevant
            for layer in m.model.layers:
                layer.mlp.experts.gate_up_proj.mul_(6)
                layer.mlp.experts.down_proj.mul_(30)
    return m, cfg


def _experts_of(model, cfg):
    """Per layer the (gate [I, H], up [I, H], down [H, I]) weights of every expert of the HF model."""
    I = cfg.moe_intermediate_size
    out = []
    for layer in model.model.layers:
        ex = layer.mlp.experts
        out.append([(ex.gate_up_proj[e, :I], ex.gate_up_proj[e, I:], ex.down_proj[e]) for e in range(cfg.num_experts)])
    return out


def _quantized_hf(bits, group=128, seed=0, shuffle=False, boost=True):
    """The tiny HF model with its experts replaced by their dequantized packed form (both sides then
    compute the same function), and the packed store."""
    from wisp import quant
    from wisp.store import ExpertStore

    model, cfg = _tiny_hf(seed, boost=boost)
    store = ExpertStore.from_experts(_experts_of(model, cfg), bits, group=group, device="cuda")
    E, I, H = cfg.num_experts, cfg.moe_intermediate_size, cfg.hidden_size
    with torch.no_grad():
        for l, layer in enumerate(model.model.layers):
            W = quant.dequant(store.host[l * E : (l + 1) * E].cuda(), H * I, bits, group)  # [E, 3, n]
            ex = layer.mlp.experts
            ex.gate_up_proj.copy_(torch.cat([W[:, 0].view(E, I, H), W[:, 1].view(E, I, H)], 1))
            ex.down_proj.copy_(W[:, 2].view(E, H, I))
        if shuffle:  # sabotage: the store's experts of every layer in the wrong order
            for l in range(cfg.num_hidden_layers):
                rows = store.host[l * E : (l + 1) * E].clone()
                store.host[l * E : (l + 1) * E].copy_(rows.roll(1, 0))
    return model, cfg, store


def _logits(model, ids, split):
    """HF prefill of ids[:split], then one token at a time with the HF cache."""
    with torch.no_grad():
        out = model(ids[:, :split], use_cache=True)
        pk, res = out.past_key_values, [out.logits]
        for t in range(split, ids.shape[1]):
            o = model(ids[:, t : t + 1], past_key_values=pk, use_cache=True)
            pk = o.past_key_values
            res.append(o.logits)
    return torch.cat(res, 1).float()


def _attach(model, store, nslots, policy="lru", miss="transfer", prefetch=False, fused=0, dol=False):
    from wisp.cache import ExpertCache
    from wisp.moe import Runtime, attach

    rt = Runtime(store, miss_policy=miss, cpu_threshold=4, prefetch=prefetch, chunk=4, fused=fused)
    rt.fused = fused
    rt.cache = ExpertCache(store, nslots, "cuda", policy, admit_after=1.0, decode_on_load=dol, staging_rows=3)
    attach(model, rt)
    return rt


@pytest.mark.parametrize(
    "nslots,policy,miss,prefetch,fused,dol",
    [
        (24, "lru", "transfer", False, 0, False),  # everything resident
        (6, "lru", "transfer", False, 0, False),  # thrashing
        (6, "wsa", "transfer", False, 2, False),
        (6, "lru", "hybrid", False, 0, False),  # misses served from host memory
        (6, "wsa", "hybrid", False, 1, False),
        (8, "lru", "transfer", True, 2, False),  # next-layer prefetch
        (8, "lru", "transfer", False, 1, False),
        (8, "lru", "transfer", False, 0, True),  # bf16 slots decoded on arrival
    ],
)
def test_attached_model_matches_hf(nslots, policy, miss, prefetch, fused, dol):
    model, cfg, store = _quantized_hf(4)
    ids = torch.randint(0, 256, (1, 14), device="cuda", generator=torch.Generator("cuda").manual_seed(3))
    with torch.no_grad():
        ref = model(ids).logits.float()
    rt = _attach(model, store, nslots, policy, miss, prefetch, fused, dol)
    got = _logits(model, ids, split=9)  # 9-token prefill (batched kernel) + 5 decode steps (fused kernels)
    err = (got - ref).abs().max().item()
    assert err < 3 * TOL * ref.abs().max().item(), err
    if nslots < 24:
        assert rt.cache.stats["misses"] > 0
    if miss == "hybrid":
        assert rt.stats["cpu_experts"] > 0
    if prefetch:
        assert rt.stats["prefetched"] > 0
    from wisp import _lib

    assert _lib.device_status(0) == 0


def test_attached_model_sabotage_is_caught():
    """Experts shuffled inside the store: the same comparison must fail by a wide margin."""
    model, cfg, store = _quantized_hf(4, shuffle=True)
    ids = torch.randint(0, 256, (1, 14), device="cuda", generator=torch.Generator("cuda").manual_seed(3))
    with torch.no_grad():
        ref = model(ids).logits.float()
    _attach(model, store, 24)
    got = _logits(model, ids, split=9)
    assert (got - ref).abs().max().item() > 10 * TOL * ref.abs().max().item()


@pytest.mark.parametrize("nslots", [24, 10])
def test_graph_decoder_from_model(nslots):
    """GraphDecoder(model, rt, tmax): chunked prefill, then teacher-forced decode steps through the
    whole-token graph (device slot table; with 10 of 24 experts resident the rest are read from the
    pinned host store and paged in one token behind).  Bit-identical to the decoder built from the
    same weights with every expert resident, and close to HF itself.  (The HF comparison uses the
    default expert scale: with boosted experts a last-bit difference in attention can flip a top-2
    choice, which the test of the attached blocks avoids by running HF's own attention.)"""
    from wisp.graphdec import GraphDecoder
    from wisp.model import DecoderWeights

    model, cfg, store = _quantized_hf(4, boost=False)
    ids = torch.randint(0, 256, (1, 16), device="cuda", generator=torch.Generator("cuda").manual_seed(5))
    with torch.no_grad():
        ref = model(ids).logits.float()[0]
    w = DecoderWeights.from_hf(model, None, bits=4, group=128)
    w.pool = store.host.cuda()  # every expert resident, slot = key: the store's own bytes
    resident = GraphDecoder(w, tmax=64)
    rt = _attach(model, store, nslots)
    dec = GraphDecoder(model, rt, tmax=64)
    scale = ref.abs().max().item()
    lg = dec.prefill(ids[0, :9], chunk=4)  # chunks of 4, 4, 1
    want = resident.prefill(ids[0, :9], chunk=4)
    assert lg.shape == (1, cfg.vocab_size)
    assert torch.equal(lg[0], want)
    # against HF only a gross-error bound: in a random-init model every top-2 choice is a near tie that a
    # last-bit difference can flip (tests/test_gpu_decoder.py replays HF's routing for a tight bound)
    assert (lg.float()[0] - ref[8]).abs().max().item() < 15 * TOL * scale
    for t in range(9, 16):
        lg = dec.next(ids[0, t : t + 1])
        assert torch.equal(lg[0], resident.next(ids[0, t : t + 1])), t
        assert (lg.float()[0] - ref[t]).abs().max().item() < 15 * TOL * scale, t
    dec.flush()
    assert rt.stats["layer_calls"] > 0
    if nslots < 24:
        assert dec.host_reads_total() > 0 or rt.cache.stats["misses"] > 0
    from wisp import _lib

    assert _lib.device_status(0) == 0


# ---- ExpertCache API --------------------------------------------------------------------------------
def test_cache_weights_resize_and_decode_on_load():
    from wisp import quant

    torch.manual_seed(1)
    H, I, E, bits, G = 256, 128, 12, 4, 128
    n = H * I
    rows = quant.quantize_batch((torch.randn(E, 3, n, device="cuda") * 0.05).to(torch.bfloat16), bits, G)
    st, cache = _store_cache(rows, n, bits, G, E, 8)
    slots = cache.ensure([3, 7, 1])
    want = quant.dequant(rows, n, bits, G)
    got = cache.weights_batched(torch.tensor(slots, device="cuda"))
    assert torch.equal(got, want[[3, 7, 1]])
    for s, key, W in zip(slots, (3, 7, 1), cache.weights(slots)):
        assert torch.equal(W, want[key])
    assert torch.equal(cache.cpu_weights(5), want[5].cpu())
    # resize: the kept experts are the most recently used, their bytes re-copied from the host store
    for key in (0, 2, 4, 5, 6):
        cache.ensure([key])
    cache.resize(4)
    assert cache.gpu.shape[0] == 4 and len(cache.core.key2slot) == 4
    for key, s in cache.core.key2slot.items():
        assert torch.equal(cache.gpu[s].cpu(), st.host[key])
    assert set(cache.core.key2slot) == {2, 4, 5, 6}
    cache.resize(10)
    assert cache.gpu.shape[0] == 10 and set(cache.core.key2slot) == {2, 4, 5, 6}
    # decode_on_load: bf16 slots hold exactly the dequantized experts
    _, dol = _store_cache(rows, n, bits, G, E, 5, decode_on_load=True, staging_rows=2)
    ds = dol.ensure([9, 0, 11])
    assert dol.gpu.shape[1] == 3 * n * 2
    for s, key in zip(ds, (9, 0, 11)):
        assert torch.equal(dol.gpu[s].view(torch.bfloat16).view(3, n), want[key])
    assert torch.equal(dol.weights_batched(torch.tensor(ds, device="cuda")), want[[9, 0, 11]])


# ---- gpt-oss block ------------------------------------------------------------------------------------
@pytest.mark.parametrize("nslots", [8, 3])
def test_gptoss_block_matches_reference_outputs(golden, nslots):
    from wisp.gptoss import PagedGptOssBlock
    from wisp.moe import Runtime

    g = golden("gptoss")
    H, I, E, k, G = (int(g[c]) for c in ("H", "I", "E", "k", "G"))
    st, cache = _store_cache(torch.from_numpy(g["pool"]), H * I, 4, G, E, nslots)
    rt = Runtime(st, cache, chunk=2)
    router = torch.nn.Linear(H, E).to("cuda", torch.bfloat16)
    router.weight.data.copy_(_bf(g["router_w"]))
    router.bias.data.copy_(_bf(g["router_b"]))
    cfg = SimpleNamespace(num_local_experts=E, num_experts_per_tok=k, hidden_size=H, intermediate_size=I, swiglu_limit=7.0)
    blk = PagedGptOssBlock(router, 0, rt, cfg)
    blk.gub.copy_(_bf(g["gub"]))
    blk.db.copy_(_bf(g["db"]))
    for N in (1, 5):
        x = _bf(g[f"x_N{N}"])[None]
        with torch.no_grad():
            y, sc = blk(x)
        tv, _ = torch.topk(F.linear(x[0], router.weight, router.bias), k, dim=-1)
        assert torch.equal(sc, F.softmax(tv, dim=1, dtype=tv.dtype))
        assert _rel(_np(y[0]), O.bf16_bits_to_f32(g[f"out_N{N}"])) < 2 * TOL, N
    if nslots < E:
        assert cache.stats["misses"] > 0
