"""End-to-end decode steps of the CUDA-graph decoder against the HF Qwen3-MoE model (the modules the
reference's GraphDecoder wraps, wisp/graphdec.py), following the reference's own decoder test
(tests/test_graphdec.py:49-82 in the reference): HF prefill, KV handed over, then each decode step's
logits compared with HF's.  The HF model's MoE blocks use the experts dequantized from the same
packed pool the decoder streams, so both sides compute the same function."""

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
transformers = pytest.importorskip("transformers")


class PoolMoE(nn.Module):
    """HF-side MoE block: the layer's router + experts dequantized from the packed pool (the math of
    the reference PagedMoEBlock's non-fused path, wisp/moe.py:62-137, in fp32)."""

    def __init__(self, gate_w, pool, layer, cfg, gate_b=None):
        super().__init__()
        from wisp import quant

        E, H, I = cfg.experts, cfg.hidden, cfg.moe_inter
        self.gate = nn.Linear(H, E, bias=gate_b is not None).to(device=gate_w.device, dtype=gate_w.dtype)
        self.gate.weight.data.copy_(gate_w)
        if gate_b is not None:
            self.gate.bias.data.copy_(gate_b)
        deq = quant.dequant(pool[layer * E : (layer + 1) * E], H * I, cfg.bits, cfg.group).float()
        self.wg, self.wu, self.wd = deq[:, 0].view(E, I, H), deq[:, 1].view(E, I, H), deq[:, 2].view(E, H, I)
        self.k, self.norm_topk = cfg.top_k, cfg.norm_topk
        self.forced = None  # (experts, weights) of one token ([k]) or of every token ([N, k]): replay another router's choice
        self.margin = 0.0  # how far the replayed choice is from HF's own top-k (probability units)

    def forward(self, h):
        x = h.reshape(-1, h.shape[-1])
        p = F.softmax(self.gate(x), dim=1, dtype=torch.float32)
        rw, sel = torch.topk(p, self.k, -1)
        if self.norm_topk:
            rw = rw / rw.sum(-1, keepdim=True)
        rw = rw.to(x.dtype).float()
        if self.forced is not None:
            fsel, frw = self.forced
            fsel, frw = (fsel[None], frw[None]) if fsel.dim() == 1 else (fsel, frw)
            assert fsel.shape[0] == x.shape[0]
            self.margin = 0.0
            for i in range(x.shape[0]):
                chosen = torch.zeros_like(p[i], dtype=torch.bool)
                chosen[fsel[i]] = True
                # > 0 when an expert outside HF's own choice beats one inside it
                self.margin = max(self.margin, (p[i][~chosen].max() - p[i][chosen].min()).item())
            sel, rw = fsel, frw.float()
        out = torch.zeros(x.shape, dtype=torch.float32, device=x.device)
        xf = x.float()
        for i in range(x.shape[0]):
            for j in range(self.k):
                e = int(sel[i, j])
                a = F.silu(self.wg[e] @ xf[i]) * (self.wu[e] @ xf[i])
                out[i] += rw[i, j] * (self.wd[e] @ a)
        return out.to(h.dtype).view_as(h)


def _kv(pk, i):
    if hasattr(pk, "layers"):
        return pk.layers[i].keys, pk.layers[i].values
    if hasattr(pk, "key_cache"):
        return pk.key_cache[i], pk.value_cache[i]
    return pk[i][0], pk[i][1]


def _model(H, I, layers, heads, kv_heads, D, E, k, vocab, seed=0):
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    torch.manual_seed(seed)
    hc = Qwen3MoeConfig(
        vocab_size=vocab, hidden_size=H, intermediate_size=2 * H, moe_intermediate_size=I, num_hidden_layers=layers,
        num_attention_heads=heads, num_key_value_heads=kv_heads, head_dim=D, num_experts=E, num_experts_per_tok=k,
        norm_topk_prob=True, max_position_embeddings=4096, decoder_sparse_step=1, mlp_only_layers=[],
    )
    model = Qwen3MoeForCausalLM(hc).to(device="cuda", dtype=torch.bfloat16).eval()
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    experts = [
        (
            torch.randn(E, I, H, device="cuda", generator=g) * 0.1,
            torch.randn(E, I, H, device="cuda", generator=g) * 0.1,
            torch.randn(E, H, I, device="cuda", generator=g) * 0.1,
        )
        for _ in range(layers)
    ]
    return model, experts


def _decoder_vs_hf(H, I, layers, heads, kv_heads, D, E, k, vocab, group, prompt=7, steps=6, tol=3e-2):
    from wisp.graphdec import GraphDecoder
    from wisp.model import DecoderWeights

    model, experts = _model(H, I, layers, heads, kv_heads, D, E, k, vocab)
    w = DecoderWeights.from_hf(model, lambda l: experts[l], bits=4, group=group)
    for l, layer in enumerate(model.model.layers):
        layer.mlp = PoolMoE(w.layers[l]["router"], w.pool, l, w.cfg)
    ids = torch.randint(0, vocab, (1, prompt), device="cuda")
    with torch.no_grad():
        out = model(input_ids=ids, use_cache=True)
        pk = out.past_key_values
        dec = GraphDecoder(w, tmax=256)
        ks = torch.stack([_kv(pk, i)[0][0] for i in range(layers)])
        vs = torch.stack([_kv(pk, i)[1][0] for i in range(layers)])
        dec.load_kv(ks, vs, prompt)
        t = out.logits[:, -1].argmax(-1)
        agree = 0
        for _ in range(steps):
            got = dec.next(t).float()
            # the HF side replays the decoder's routing (near-ties among many experts may order
            # differently under different rounding); the choice itself must be HF's top-k up to a
            # small probability margin
            for l, layer in enumerate(model.model.layers):
                layer.mlp.forced = (dec.rows[l, :k].long(), dec.rows[l, k:])
            ref = model(input_ids=t[:, None], past_key_values=pk, use_cache=True)
            pk = ref.past_key_values
            for layer in model.model.layers:
                assert layer.mlp.margin < 1e-3, layer.mlp.margin
            want = ref.logits[0, -1].float()
            err = (got - want).abs().max().item() / want.abs().max().item()
            assert err < tol, err
            agree += int(got.argmax() == want.argmax())
            t = want.argmax(-1).reshape(1)
        assert agree >= steps - 1
    return dec


def test_tiny_decoder_matches_hf():
    """The reference test's shapes (head_dim raised to 32, the attention kernel's granularity); MoE on
    the CUDA-core kernels (H, I not multiples of 128)."""
    _decoder_vs_hf(H=64, I=32, layers=3, heads=4, kv_heads=2, D=32, E=8, k=2, vocab=100, group=32)


def test_qwen3_layer_shapes_match_hf():
    """Two layers at the Qwen3-30B-A3B widths (H 2048, 32/4 heads x 128, 128 experts top-8, I 768,
    4-bit g128): every production kernel path (bulk-copy GEMVs, tensor-core MoE, 8-way GQA)."""
    _decoder_vs_hf(H=2048, I=768, layers=2, heads=32, kv_heads=4, D=128, E=128, k=8, vocab=4096, group=128)


def test_greedy_graph_matches_stepwise():
    from wisp.graphdec import GraphDecoder
    from wisp.model import DecoderConfig, DecoderWeights

    cfg = DecoderConfig(vocab=1000, hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, experts=16, top_k=4, moe_inter=128)
    w = DecoderWeights.random(cfg, seed=5)
    a = GraphDecoder(w, tmax=128)
    b = GraphDecoder(w, tmax=128)
    t0 = torch.tensor([17], device="cuda")
    ids = a.greedy(t0, 10).tolist()
    t, want = t0, []
    for _ in range(10):
        t = b.next(t).argmax().reshape(1)
        want.append(int(t))
    assert ids == want
    assert torch.equal(a.kc, b.kc) and torch.equal(a.vc, b.vc)


@pytest.mark.parametrize("prefetch", [False, True])
def test_paged_decoder_matches_resident(prefetch):
    """40% of the experts resident, the rest paged in per layer from pinned host memory: the same
    tokens and (up to the routing weights' last bit) the same logits as with every expert resident."""
    from wisp.cache import ExpertCache
    from wisp.graphdec import GraphDecoder, PagedGraphDecoder
    from wisp.model import DecoderConfig, DecoderWeights
    from wisp.store import ExpertStore

    cfg = DecoderConfig(vocab=2000, hidden=2048, layers=3, heads=32, kv_heads=4, head_dim=128, experts=32, top_k=8,
                        moe_inter=768)
    w = DecoderWeights.random(cfg, seed=11)
    store = ExpertStore.from_pool(w.pool, cfg.hidden * cfg.moe_inter, cfg.bits, cfg.group, cfg.layers, cfg.experts)
    cache = ExpertCache(store, nslots=int(0.4 * cfg.layers * cfg.experts))
    a = GraphDecoder(w, tmax=128)
    b = PagedGraphDecoder(w, cache, tmax=128, prefetch=prefetch)
    t = torch.tensor([5], device="cuda")
    for step in range(8):
        la = a.next(t).float().clone()
        lb = b.next(t).float()
        assert (la - lb).abs().max().item() <= 2e-2 * la.abs().max().item(), step
        assert torch.equal(a.rows, b.rows) or (a.rows[:, : cfg.top_k] == b.rows[:, : cfg.top_k]).all()
        t = la.argmax().reshape(1)
    st = cache.stats
    assert st["misses"] > 0 and st["hits"] + st["misses"] == 8 * cfg.layers * cfg.top_k
    assert cache.bytes_h2d >= st["misses"] * store.nbytes


@pytest.mark.parametrize("frac,admit", [(0.4, "all"), (0.1, "all"), (0.4, "hot")])
def test_device_paged_decoder_matches_resident(frac, admit):
    """Part of the experts resident, residency in a device slot table, misses read by the MoE kernels
    from the pinned host store, page-ins published one token behind: the logits are bit-identical to
    the all-resident decoder's, and after a flush the table, the policy and the slot bytes agree."""
    from wisp.cache import ExpertCache
    from wisp.graphdec import DevicePagedDecoder, GraphDecoder
    from wisp.model import DecoderConfig, DecoderWeights
    from wisp.store import ExpertStore

    cfg = DecoderConfig(vocab=2000, hidden=2048, layers=3, heads=32, kv_heads=4, head_dim=128, experts=32, top_k=8,
                        moe_inter=768)
    w = DecoderWeights.random(cfg, seed=11)
    store = ExpertStore.from_pool(w.pool, cfg.hidden * cfg.moe_inter, cfg.bits, cfg.group, cfg.layers, cfg.experts)
    cache = ExpertCache(store, nslots=max(cfg.top_k, int(frac * cfg.layers * cfg.experts)))
    a = GraphDecoder(w, tmax=128)
    b = DevicePagedDecoder(w, cache, tmax=128, admit=admit)
    t = torch.tensor([5], device="cuda")
    steps = 12
    for step in range(steps):
        la = a.next(t).clone()
        lb = b.next(t)
        assert torch.equal(la, lb), step
        t = la.argmax().reshape(1)
    b.flush()
    torch.cuda.synchronize()
    tbl = b.pager.table.cpu()
    core = cache.core
    assert int((tbl >= 0).sum()) == len(core.key2slot)
    for key, slot in core.key2slot.items():
        assert int(tbl[key]) == slot
        assert torch.equal(cache.gpu[slot].cpu(), store.host[key]), key
    st = cache.stats
    assert st["hits"] + st["misses"] == steps * cfg.layers * cfg.top_k
    assert st["misses"] > 0 and b.host_reads_total() > 0
    if admit == "all":
        assert cache.n_loads > 0
