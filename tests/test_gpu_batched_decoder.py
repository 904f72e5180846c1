"""The batched Qwen3-MoE decoder (B sequences per step, one CUDA graph) against the HF Qwen3-MoE model
run on the same batch: HF prefill of B prompts, the KV handed over, then every decode step's logits of
every sequence compared with HF's.  HF's MoE blocks use the experts dequantized from the decoder's
packed pool and replay the decoder's routing (experts and weights) for each token, with a check that
the replayed choice is HF's own top-k up to a small probability margin; the router's logit bias (the
benchmark's Zipf popularity) sits in HF's gate as its bias."""

import pytest
import torch

from test_gpu_decoder import PoolMoE, _kv, _model

pytestmark = pytest.mark.gpu


def _setup(B, prompt, bias, layers=2, seed=0):
    from wisp.batched_decoder import zipf_bias
    from wisp.model import DecoderWeights

    H, I, heads, kv_heads, D, E, k, vocab = 256, 128, 4, 2, 128, 16, 4, 300
    model, experts = _model(H, I, layers, heads, kv_heads, D, E, k, vocab, seed=seed)
    w = DecoderWeights.from_hf(model, lambda l: experts[l], bits=4, group=128)
    zb = zipf_bias(layers, E, device="cuda").to(torch.bfloat16) if bias else None
    for l, layer in enumerate(model.model.layers):
        layer.mlp = PoolMoE(w.layers[l]["router"], w.pool, l, w.cfg, gate_b=None if zb is None else zb[l])
    ids = torch.randint(0, vocab, (B, prompt), device="cuda", generator=torch.Generator(device="cuda").manual_seed(seed + 5))
    return model, w, zb, ids


@pytest.mark.parametrize("B,bias", [(3, False), (4, True)])
def test_batched_decoder_matches_hf(B, bias):
    from wisp import _lib
    from wisp.batched_decoder import BatchedDecoder

    prompt, steps, k = 6, 5, 4
    model, w, zb, ids = _setup(B, prompt, bias)
    with torch.no_grad():
        out = model(input_ids=ids, use_cache=True)
        pk = out.past_key_values
        dec = BatchedDecoder(w, batch=B, tmax=64, expert_bias=zb)
        L = w.cfg.layers
        ks = torch.stack([_kv(pk, i)[0] for i in range(L)])
        vs = torch.stack([_kv(pk, i)[1] for i in range(L)])
        dec.load_kv(ks, vs, prompt)
        t = out.logits[:, -1].argmax(-1)
        _lib.device_status(0)
        agree = 0
        for _ in range(steps):
            got = dec.step(t).float()
            for l, layer in enumerate(model.model.layers):
                layer.mlp.forced = (dec.routes[l], dec.rweights[l])
            ref = model(input_ids=t[:, None], past_key_values=pk, use_cache=True)
            pk = ref.past_key_values
            for layer in model.model.layers:
                assert layer.mlp.margin < 1e-3, layer.mlp.margin
            want = ref.logits[:, -1].float()
            for b in range(B):
                err = (got[b] - want[b]).abs().max().item() / want[b].abs().max().item()
                assert err < 3e-2, (b, err)
            agree += int((got.argmax(-1) == want.argmax(-1)).sum())
            assert torch.equal(dec.next_token, got.argmax(-1))
            t = want.argmax(-1)
        assert agree >= B * steps - 2
        assert _lib.device_status(0) == 0
        assert dec.pos.tolist() == [prompt + steps] * B


def test_sequences_are_independent():
    """Sequence b's logits do not depend on what the other sequences hold: the batch of 3 against each
    sequence decoded alone (batch 1) with the same cache, token and position (cuBLAS may tile a 1-row and
    a 3-row GEMM differently, so the logits are compared to bf16 rounding)."""
    from wisp.batched_decoder import BatchedDecoder

    model, w, _, ids = _setup(3, 6, False)
    with torch.no_grad():
        out = model(input_ids=ids, use_cache=True)
        pk = out.past_key_values
        L = w.cfg.layers
        ks = torch.stack([_kv(pk, i)[0] for i in range(L)])
        vs = torch.stack([_kv(pk, i)[1] for i in range(L)])
        t = out.logits[:, -1].argmax(-1)
        dec = BatchedDecoder(w, batch=3, tmax=64)
        dec.load_kv(ks, vs, 6)
        both = dec.step(t).float().clone()
        for b in range(3):
            one = BatchedDecoder(w, batch=1, tmax=64)
            one.load_kv(ks[:, b : b + 1], vs[:, b : b + 1], 6)
            got = one.step(t[b : b + 1]).float()
            assert (got[0] - both[b]).abs().max().item() <= 2e-2 * both[b].abs().max().item(), b


def test_expert_parallel_path_on_one_rank():
    """The decoder's expert-parallel branch (router rows -> dispatch -> batched experts -> combine, one
    rank owning every expert) against its resident branch on the same weights, routing and cache."""
    from wisp.batched_decoder import BatchedDecoder, zipf_bias
    from wisp.ep import ExpertParallelMoE, batched_expert_fn

    model, w, _, ids = _setup(4, 6, True)
    c = w.cfg
    with torch.no_grad():
        out = model(input_ids=ids, use_cache=True)
        pk = out.past_key_values
        ks = torch.stack([_kv(pk, i)[0] for i in range(c.layers)])
        vs = torch.stack([_kv(pk, i)[1] for i in range(c.layers)])
        t = out.logits[:, -1].argmax(-1)
        zb = zipf_bias(c.layers, c.experts, device="cuda")
        fn = batched_expert_fn(w.pool, lambda l, e: l * c.experts + e, c.hidden * c.moe_inter, c.hidden, c.moe_inter, c.bits,
                               c.group)
        ep = ExpertParallelMoE(c.experts, c.top_k, c.hidden, 4, fn, device="cuda", slot_base=lambda l: l * c.experts)
        a = BatchedDecoder(w, batch=4, tmax=64, expert_bias=zb)
        b = BatchedDecoder(w, batch=4, tmax=64, expert_bias=zb, ep=ep)
        for dec in (a, b):
            dec.load_kv(ks, vs, 6)
        for _ in range(3):
            la = a.step(t).float()
            lb = b.step(t).float()
            assert torch.equal(a.routes, b.routes)
            assert (la - lb).abs().max().item() <= 2e-2 * la.abs().max().item()
            t = la.argmax(-1)
        ep.close()
