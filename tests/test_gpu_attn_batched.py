"""Batched decode attention and the batched q/k norm + rotary + cache write (one token of each of B
sequences, each with its own position and cache), through the C ABI: against an fp32 restatement of
masked softmax attention with gpt-oss's sliding window and attention sinks (the HF GptOssAttention
math), and against the single-sequence kernels."""

import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 1e-2  # relative to max |reference| (bf16 output)


def _ref_attn(q, kc, vc, pos, scale, window, sinks):
    """fp32: out[b, head] = sum_t p_t v_t over t in [lo, pos[b]], p = softmax over those scores plus an
    optional per-head sink logit that takes part in the normalisation only."""
    B, Hq, D = q.shape
    Hk = kc.shape[1]
    G = Hq // Hk
    out = torch.zeros(B, Hq, D)
    for b in range(B):
        p = int(pos[b])
        lo = max(0, p - window + 1) if window > 0 else 0
        for hd in range(Hq):
            k = kc[b, hd // G, lo : p + 1].float()
            v = vc[b, hd // G, lo : p + 1].float()
            s = (k @ q[b, hd].float()) * scale
            if sinks is not None:
                s = torch.cat([s, sinks[hd : hd + 1].float()])
            w = torch.softmax(s, 0)[: k.shape[0]]
            out[b, hd] = w @ v
    return out


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("window,use_sinks", [(0, False), (128, True), (100, False), (0, True)])
def test_batched_attention_matches_reference(D, window, use_sinks):
    from wisp import _lib, kernels

    g = torch.Generator(device="cuda").manual_seed(D + window)
    B, Hq, Hk, tmax = 4, 8, 2, 320
    q = torch.randn(B, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(B, Hk, tmax, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hk, tmax, D, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.tensor([0, 63, 191, 319], dtype=torch.int64, device="cuda")  # chunk edges and the last slot
    sinks = torch.randn(Hq, device="cuda", generator=g).float() * 2 if use_sinks else None
    scale = D ** -0.5
    _lib.device_status(0)
    out = kernels.gqa_decode_attn_batched(q, Hq, Hk, D, kc, vc, pos, scale, window=window, sinks=sinks)
    ref = _ref_attn(q.cpu(), kc.cpu(), vc.cpu(), pos.cpu(), scale, window, None if sinks is None else sinks.cpu())
    err = (out.float().cpu() - ref).abs().max().item() / ref.abs().max().item()
    assert err < TOL, err
    assert _lib.device_status(0) == 0
    if window == 0 and not use_sinks:  # one sequence at a time through the single-sequence entry point: the same bits
        for b in range(B):
            one = kernels.gqa_decode_attn(q[b].reshape(-1).contiguous(), Hq, Hk, D, kc[b].contiguous(), vc[b].contiguous(),
                                          pos[b : b + 1], scale)
            assert torch.equal(one.view(Hq, D), out[b]), b


@pytest.mark.parametrize("norm", [True, False])
def test_batched_rope_kv_write(norm):
    from wisp import kernels
    from wisp.model import rotary_tables

    g = torch.Generator(device="cuda").manual_seed(3)
    B, Hq, Hk, D, tmax = 3, 8, 2, 64, 96
    qkv = torch.randn(B, (Hq + 2 * Hk) * D, device="cuda", generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).to(torch.bfloat16) if norm else None
    kn = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).to(torch.bfloat16) if norm else None
    cos, sin = rotary_tables(D, tmax, 150000.0, "cuda")
    pos = torch.tensor([5, 0, 95], dtype=torch.int64, device="cuda")
    kc = torch.zeros(B, Hk, tmax, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    q = kernels.qk_norm_rope_kv_batched(qkv, Hq, Hk, D, qn, kn, 1e-6, cos, sin, pos, kc, vc)
    for b in range(B):
        p = int(pos[b])
        v = qkv[b, (Hq + Hk) * D :].view(Hk, D)
        assert torch.equal(vc[b, :, p], v)
        if norm:  # the single-token kernel on that sequence's cache gives the same bits
            kc1 = torch.zeros(Hk, tmax, D, dtype=torch.bfloat16, device="cuda")
            vc1 = torch.zeros_like(kc1)
            q1 = kernels.qk_norm_rope_kv(qkv[b].contiguous(), Hq, Hk, D, qn, kn, 1e-6, cos, sin, pos[b : b + 1], kc1, vc1)
            assert torch.equal(q1.view(Hq, D), q[b]) and torch.equal(kc1[:, p], kc[b, :, p])
        else:  # plain rotate-half rotary in fp32
            x = qkv[b, : Hq * D].view(Hq, D).float()
            rot = torch.cat([-x[:, D // 2 :], x[:, : D // 2]], 1)
            want = x * cos[p].float() + rot * sin[p].float()
            assert (q[b].float() - want).abs().max().item() <= 1e-2 * want.abs().max().item()
        others = [t for t in range(tmax) if t != p]
        assert (kc[b, :, others] == 0).all()  # nothing else of that cache was written


@pytest.mark.parametrize("D,norm,window,use_sinks", [(128, True, 0, False), (64, False, 8, True), (64, False, 0, True)])
def test_fused_rotary_attention_equals_two_calls(D, norm, window, use_sinks):
    """wisp_attn_decode_batched (norm + rotary + cache write inside the attention kernel) against
    qk_norm_rope_kv_batched + gqa_decode_attn_batched: the same bits in the output and in both caches,
    sequences at their own positions (one at a chunk's first row, one at the cache's last)."""
    from wisp import kernels
    from wisp.model import rotary_tables

    g = torch.Generator(device="cuda").manual_seed(D + window)
    B, Hq, Hk, tmax = 4, 8, 2, 192
    qkv = torch.randn(B, (Hq + 2 * Hk) * D, device="cuda", generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).to(torch.bfloat16) if norm else None
    kn = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).to(torch.bfloat16) if norm else None
    cos, sin = rotary_tables(D, tmax, 150000.0, "cuda")
    pos = torch.tensor([0, 64, 100, 191], dtype=torch.int64, device="cuda")
    kc = torch.randn(B, Hk, tmax, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hk, tmax, D, device="cuda", generator=g).to(torch.bfloat16)
    sinks = torch.randn(Hq, device="cuda", generator=g).float() if use_sinks else None
    kc2, vc2 = kc.clone(), vc.clone()
    q = kernels.qk_norm_rope_kv_batched(qkv, Hq, Hk, D, qn, kn, 1e-6, cos, sin, pos, kc, vc)
    want = kernels.gqa_decode_attn_batched(q, Hq, Hk, D, kc, vc, pos, D ** -0.5, window=window, sinks=sinks)
    got = kernels.attn_decode_batched(qkv, Hq, Hk, D, qn, kn, 1e-6, cos, sin, pos, kc2, vc2, D ** -0.5, window=window, sinks=sinks)
    assert torch.equal(got, want)
    assert torch.equal(kc2, kc) and torch.equal(vc2, vc)


def _ref_attn_gpu(q, kc, vc, pos, scale, window, sinks):
    """_ref_attn on the GPU in fp32, all heads of a sequence at once (for long caches)."""
    B, Hq, D = q.shape
    Hk, tmax = kc.shape[1], kc.shape[2]
    G = Hq // Hk
    out = torch.zeros(B, Hq, D, device=q.device)
    t = torch.arange(tmax, device=q.device)
    for b in range(B):
        p = int(pos[b])
        lo = max(0, p - window + 1) if window > 0 else 0
        s = torch.einsum("hgd,htd->hgt", q[b].float().view(Hk, G, D), kc[b].float()) * scale
        s = s.masked_fill(((t < lo) | (t > p))[None, None], float("-inf"))
        if sinks is not None:
            s = torch.cat([s, sinks.float().view(Hk, G, 1)], -1)
        w = torch.softmax(s, -1)[..., :tmax]
        out[b] = torch.einsum("hgt,htd->hgd", w, vc[b].float()).reshape(Hq, D)
    return out


@pytest.mark.parametrize("D,Hq,Hk,B,tmax,window,use_sinks", [(128, 32, 4, 64, 4096, 0, False), (128, 32, 4, 64, 4096, 1000, True),
                                                            (64, 64, 8, 32, 2048, 128, True)])
def test_long_context_several_chunks_per_cta(D, Hq, Hk, B, tmax, window, use_sinks):
    """At many sequences and long caches each attention CTA takes several consecutive chunks (an online
    softmax across them) and writes one record for all of them: the output still matches the fp32
    restatement, for positions at chunk edges, mid-chunk and at the cache's last slot, with a sliding
    window that starts mid-chunk; the fused rotary form stays bit-identical to the two calls there."""
    from wisp import _lib, kernels
    from wisp.model import rotary_tables

    g = torch.Generator(device="cuda").manual_seed(D + B + window)
    q = torch.randn(B, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(B, Hk, tmax, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hk, tmax, D, device="cuda", generator=g).to(torch.bfloat16)
    edges = [0, 63, 64, 255, 256, 257, tmax - 1, tmax - 64, 1000, 1023, 1024, 2047]
    rnd = torch.randint(0, tmax, (B,), device="cuda", generator=g)
    pos = torch.tensor([edges[i] if i < len(edges) else int(rnd[i]) for i in range(B)], dtype=torch.int64, device="cuda")
    sinks = torch.randn(Hq, device="cuda", generator=g).float() * 2 if use_sinks else None
    scale = D ** -0.5
    _lib.device_status(0, clear=True)
    out = kernels.gqa_decode_attn_batched(q, Hq, Hk, D, kc, vc, pos, scale, window=window, sinks=sinks)
    ref = _ref_attn_gpu(q, kc, vc, pos, scale, window, sinks)
    err = ((out.float() - ref).abs().amax(-1) / ref.abs().amax(-1).clamp_min(1e-6)).max().item()
    assert err < 2 * TOL, err
    assert _lib.device_status(0) == 0
    # the fused rotary form at the same shape: the same bits as the two calls
    qkv = torch.randn(B, (Hq + 2 * Hk) * D, device="cuda", generator=g).to(torch.bfloat16)
    cos, sin = rotary_tables(D, tmax, 150000.0, "cuda")
    kc2, vc2 = kc.clone(), vc.clone()
    qr = kernels.qk_norm_rope_kv_batched(qkv, Hq, Hk, D, None, None, 1e-6, cos, sin, pos, kc, vc)
    want = kernels.gqa_decode_attn_batched(qr, Hq, Hk, D, kc, vc, pos, scale, window=window, sinks=sinks)
    got = kernels.attn_decode_batched(qkv, Hq, Hk, D, None, None, 1e-6, cos, sin, pos, kc2, vc2, scale, window=window, sinks=sinks)
    assert torch.equal(got, want)
    assert torch.equal(kc2, kc) and torch.equal(vc2, vc)
