"""GPU parity of the decode-step kernels (GEMV with fused residual/RMSNorm, q/k norm + rotary + cache
write, GQA decode attention, router top-k, embedding, argmax) through the C ABI, against plain torch
fp32 references of the same rounding steps, the oracle, and the reference's SDPA fixture."""

import numpy as np
import pytest
import torch

from oracle import wisp_oracle as O

pytestmark = pytest.mark.gpu


def _bf(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16).cuda()


def _np(t):
    return O.bf16_bits_to_f32(t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16))


def _gen(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


def _ref_gemv(W, x, x_add=None, norm_w=None, eps=1e-6, res=None):
    """torch fp32 reference with the kernel's rounding steps (bf16 after every named op)."""
    xs = x.float()
    if x_add is not None:
        xs = (xs + x_add.float()).to(torch.bfloat16).float()
    xn = xs
    if norm_w is not None:
        inv = torch.rsqrt((xs * xs).mean() + eps)
        xn = (norm_w.float() * (xs * inv).to(torch.bfloat16).float()).to(torch.bfloat16).float()
    y = (W.float() @ xn).to(torch.bfloat16).float()
    if res is not None:
        y = (res.float() + y).to(torch.bfloat16).float()
    return xs, xn, y


@pytest.mark.parametrize("N,K", [(5120, 2048), (2048, 4096), (128, 2048), (1000, 64), (37, 1024), (151936 // 16, 2048)])
def test_gemv_plain(N, K):
    from wisp import kernels

    g = _gen(N + K)
    W = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(K, device="cuda", generator=g).to(torch.bfloat16)
    y = kernels.gemv(W, x)
    _, _, ref = _ref_gemv(W, x)
    # fp32 sums in another order: at most one bf16 rounding step apart
    tol = 2.0**-7 * ref.abs().max().item()
    assert (y.float() - ref).abs().max().item() <= tol


@pytest.mark.parametrize("K", [2048, 64])
def test_gemv_fused_residual_norm(K):
    from wisp import kernels

    N = 3 * K
    g = _gen(K)
    W = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(K, device="cuda", generator=g).to(torch.bfloat16)
    xa = torch.randn(K, device="cuda", generator=g).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(K, device="cuda", generator=g)).to(torch.bfloat16)
    res = torch.randn(N, device="cuda", generator=g).to(torch.bfloat16)
    xs_out = torch.empty(K, dtype=torch.bfloat16, device="cuda")
    xn_out = torch.empty(K, dtype=torch.bfloat16, device="cuda")
    y = kernels.gemv(W, x, x_add=xa, x_sum_out=xs_out, norm_w=nw, eps=1e-6, xn_out=xn_out, res=res)
    xs, xn, ref = _ref_gemv(W, x, xa, nw, 1e-6, res)
    assert torch.equal(xs_out.float(), xs)  # bf16 add: exact
    assert (xn_out.float() - xn).abs().max().item() <= 2.0**-7 * xn.abs().max().item()  # rsqrt rounding
    assert (y.float() - ref).abs().max().item() <= 2.0**-6 * ref.abs().max().item()


@pytest.mark.parametrize("N,K", [(5120, 2880), (2880, 4096)])
def test_gemv_bias_and_residual(N, K):
    """y = bf16(res + bf16(W x + bias)): the biased gpt-oss projections (fp32 sum and bias, one rounding)."""
    from wisp import kernels

    g = _gen(N + 7)
    W = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(K, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(N, device="cuda", generator=g).to(torch.bfloat16)
    res = torch.randn(N, device="cuda", generator=g).to(torch.bfloat16)
    lin = (W.float() @ x.float() + b.float()).to(torch.bfloat16).float()
    y = kernels.gemv(W, x, bias=b)
    assert (y.float() - lin).abs().max().item() <= 2.0**-7 * lin.abs().max().item()
    y2 = kernels.gemv(W, x, bias=b, res=res)
    want = (res.float() + y.float()).to(torch.bfloat16)
    assert torch.equal(y2, want)  # the residual add is one bf16 add on the same biased product


@pytest.mark.parametrize("B,H,E,k,mode", [(1, 2880, 32, 4, "selected"), (32, 2880, 32, 4, "selected"), (5, 2048, 128, 8, True),
                                          (3, 64, 8, 2, False)])
def test_router_rows(B, H, E, k, mode):
    """RMSNorm + biased gate + top-k + weights for B tokens in one launch, against torch fp32 with the
    kernel's rounding steps; the selection and weights also against the single-token router kernel on
    the same logits."""
    from wisp import kernels

    g = _gen(B * 1000 + E)
    x = torch.randn(B, H, device="cuda", generator=g).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).to(torch.bfloat16)
    W = (torch.randn(E, H, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    bias = (torch.randn(E, device="cuda", generator=g) * 0.1).to(torch.bfloat16) if mode == "selected" else None
    xn = torch.empty_like(x)
    experts = torch.empty(B, k, dtype=torch.int32, device="cuda")
    row = torch.empty(B, 2 * k, dtype=torch.float32, device="cuda")
    meta = kernels.router_rows(x, W, k, mode, norm_w=nw, eps=1e-5, bias=bias, xn_out=xn, base=7 * E, experts=experts, row=row)
    xs = x.float()
    inv = torch.rsqrt((xs * xs).mean(-1, keepdim=True) + 1e-5)
    xn_ref = (nw.float() * (xs * inv).to(torch.bfloat16).float()).to(torch.bfloat16)
    assert (xn.float() - xn_ref.float()).abs().max().item() <= 2.0**-7 * xn_ref.float().abs().max().item()
    logits = xn.float() @ W.float().t() + (0 if bias is None else bias.float())
    lg = logits.to(torch.bfloat16)
    for b in range(B):
        want = torch.empty(2 * k, dtype=torch.float32, device="cuda")
        kernels.router_topk(lg[b].contiguous(), k, mode, row=want)
        # the kernel's own logits may differ from torch's by one bf16 step; compare where the top-k has
        # no near-tie at that resolution
        srt = lg[b].float().sort(descending=True).values
        if (srt[k - 1] - srt[k]).abs().item() > 2 * 2.0**-7 * srt[0].abs().item():
            assert set(row[b, :k].long().tolist()) == set(want[:k].long().tolist()), b
            assert (row[b, k:].sort().values - want[k:].sort().values).abs().max().item() <= 0.02
    assert torch.equal(experts.long(), row[:, :k].long())
    assert torch.equal(meta[:, :k].long(), row[:, :k].long() + 7 * E) and torch.equal(meta[:, k:], row[:, k:])
    assert torch.allclose(row[:, k:].sum(-1), torch.ones(B, device="cuda"), atol=2e-2) or mode is False


@pytest.mark.parametrize("B,H,E,k,mode", [(1, 2880, 32, 4, "selected"), (64, 2048, 128, 8, True), (3, 256, 10, 3, False)])
def test_router_split_matches_one_cta(B, H, E, k, mode):
    """The gate split over CTAs (four experts each, the last CTA of a token runs the top-k) against the
    one-CTA router: the same experts and weights (the RMSNorm's sum of squares is added in another order,
    so the normed rows may differ by a bf16 step), and the workspace is left ready: a second launch on
    it gives the same result."""
    from wisp import kernels

    g = _gen(B * 7 + E)
    x = torch.randn(B, H, device="cuda", generator=g).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).to(torch.bfloat16)
    W = (torch.randn(E, H, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    bias = (torch.randn(E, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    ws = kernels.router_workspace(B, E, "cuda")
    outs = []
    for workspace in (None, ws, ws):
        xn = torch.empty_like(x)
        row = torch.empty(B, 2 * k, dtype=torch.float32, device="cuda")
        experts = torch.empty(B, k, dtype=torch.int32, device="cuda")
        meta = kernels.router_rows(x, W, k, mode, norm_w=nw, eps=1e-5, bias=bias, xn_out=xn, base=3 * E, experts=experts, row=row,
                                   workspace=workspace)
        outs.append((xn, row, experts, meta))
    assert torch.equal(outs[1][1], outs[2][1]) and torch.equal(outs[1][0], outs[2][0])  # repeatable on the same workspace
    assert torch.count_nonzero(ws[-4 * B:]) == 0  # arrival counters back at zero
    (xa, ra, ea, ma), (xb, rb, eb, mb) = outs[0], outs[1]
    assert (xa.float() - xb.float()).abs().max().item() <= 2.0**-7 * xa.float().abs().max().item()
    same = (ra[:, :k] == rb[:, :k]).all(-1)
    assert same.float().mean().item() >= 0.9, same  # a near-tie may flip with a one-step difference in xn
    assert (ra[same, k:] - rb[same, k:]).abs().max().item() <= 0.02
    assert torch.equal(eb.long(), rb[:, :k].long()) and torch.equal(mb[:, :k].long(), rb[:, :k].long() + 3 * E)


def test_gemv_rejects_aliasing():
    from wisp import kernels
    from wisp._lib import WispError

    W = torch.zeros(64, 64, dtype=torch.bfloat16, device="cuda")
    x = torch.zeros(64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(WispError, match="alias"):
        kernels.gemv(W, x, out=x)


@pytest.mark.parametrize("pos", [0, 5, 700])
def test_qk_norm_rope_kv(pos):
    from wisp import kernels
    from wisp.model import rotary_tables

    Hq, Hk, D, tmax, eps = 32, 4, 128, 1024, 1e-6
    g = _gen(pos)
    qkv = torch.randn((Hq + 2 * Hk) * D, device="cuda", generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).to(torch.bfloat16)
    cos, sin = rotary_tables(D, tmax, 1e6, "cuda")
    kc = torch.zeros(Hk, tmax, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    p = torch.tensor([pos], dtype=torch.int64, device="cuda")
    q = kernels.qk_norm_rope_kv(qkv, Hq, Hk, D, qn, kn, eps, cos, sin, p, kc, vc)
    heads = _np(qkv).reshape(Hq + 2 * Hk, D)
    c, s = _np(cos[pos]), _np(sin[pos])

    def normed(x, w):
        inv = 1.0 / np.sqrt(np.mean(x * x, -1, keepdims=True) + np.float32(eps))
        return O.round_bf16(_np(w) * O.round_bf16(x * inv))

    want_q = O.round_bf16(O.rope(normed(heads[:Hq], qn), c, s))
    want_k = O.round_bf16(O.rope(normed(heads[Hq : Hq + Hk], kn), c, s))
    got_q = _np(q).reshape(Hq, D)
    got_k = _np(kc[:, pos])
    # rsqrt and the fp32 products may round one bf16 ulp apart
    assert np.abs(got_q - want_q).max() <= 2.0**-6 * np.abs(want_q).max()
    assert np.abs(got_k - want_k).max() <= 2.0**-6 * np.abs(want_k).max()
    assert np.array_equal(_np(vc[:, pos]), heads[Hq + Hk :])
    others = torch.ones(tmax, dtype=torch.bool)
    others[pos] = False
    assert not kc[:, others].any() and not vc[:, others].any()


def test_attention_matches_reference_fixture(golden):
    """The reference graph decoder's masked GQA SDPA on the fixture's cache (tmax 64)."""
    from wisp import kernels

    a = golden("attn")
    Hq, D = a["q"].shape
    Hk = a["kc"].shape[0]
    q, kc, vc = _bf(a["q"]), _bf(a["kc"]), _bf(a["vc"])
    pos = torch.tensor([int(a["pos"])], dtype=torch.int64, device="cuda")
    out = kernels.gqa_decode_attn(q.reshape(-1), Hq, Hk, D, kc, vc, pos, D**-0.5)
    ref = a["out"]
    assert np.abs(_np(out).reshape(Hq, D) - ref).max() <= 1e-2 * np.abs(ref).max()


@pytest.mark.parametrize("pos", [0, 1, 63, 64, 65, 777, 4095])
@pytest.mark.parametrize("G,D", [(8, 128), (8, 64), (2, 32)])
def test_attention_vs_oracle(pos, G, D):
    from wisp import kernels

    Hk, tmax = 4, 4096
    Hq = Hk * G
    g = _gen(pos + D)
    q = torch.randn(Hq * D, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(Hk, tmax, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(Hk, tmax, D, device="cuda", generator=g).to(torch.bfloat16)
    p = torch.tensor([pos], dtype=torch.int64, device="cuda")
    out = kernels.gqa_decode_attn(q, Hq, Hk, D, kc, vc, p, D**-0.5)
    want = O.gqa_decode_attention(_np(q).reshape(Hq, D), _np(kc), _np(vc), pos, D**-0.5)
    assert np.abs(_np(out).reshape(Hq, D) - want).max() <= 1e-2 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("E,k", [(128, 8), (32, 4), (8, 2)])
def test_router_topk_vs_oracle(E, k):
    from wisp import kernels

    for seed in range(5):
        g = _gen(seed * 100 + E)
        logits = (torch.randn(E, device="cuda", generator=g) * 2).to(torch.bfloat16)
        row = torch.empty(2 * k, dtype=torch.float32, device="cuda")
        meta = kernels.router_topk(logits, k, True, base=5 * E, row=row)
        sel, rw = O.router_topk(_np(logits)[None], k)
        got_sel = row[:k].long().cpu().numpy()
        assert np.array_equal(np.sort(got_sel), np.sort(sel[0]))
        order = np.argsort(sel[0])
        gorder = np.argsort(got_sel)
        assert np.abs(row[k:].cpu().numpy()[gorder] - rw[0][order]).max() <= 2.0**-8
        assert np.array_equal(meta[:k].long().cpu().numpy(), got_sel + 5 * E)
        assert torch.equal(meta[k:], row[k:])


def test_router_slot_table():
    from wisp import kernels

    E, k = 16, 2
    logits = torch.zeros(E, dtype=torch.bfloat16, device="cuda")
    logits[3], logits[9] = 4.0, 3.0
    table = torch.arange(100, 100 + 2 * E, dtype=torch.int32, device="cuda")
    table[E + 9] = -1
    meta = kernels.router_topk(logits, k, True, slot_table=table, base=E)
    assert meta[:k].tolist() == [100.0 + E + 3, -1.0]


def test_embed_and_argmax():
    from wisp import kernels

    V, H = 5000, 2048
    g = _gen(3)
    table = torch.randn(V, H, device="cuda", generator=g).to(torch.bfloat16)
    tok = torch.tensor([4321], dtype=torch.int64, device="cuda")
    assert torch.equal(kernels.embed(table, tok), table[4321])
    x = torch.randn(151936, device="cuda", generator=g).to(torch.bfloat16)
    assert int(kernels.argmax(x)) == int(torch.argmax(x.float()))
    x[7] = x[100000] = 50.0  # tie: the lower index wins
    assert int(kernels.argmax(x)) == 7
    x[3] = float("nan")
    assert int(kernels.argmax(x)) == 7


@pytest.mark.parametrize("pos", [0, 1, 7, 127, 128, 700, 1031, 4095])
@pytest.mark.parametrize("Hq,Hk", [(32, 4), (16, 4), (4, 4)])
def test_fused_attention_matches_two_kernel_path(pos, Hq, Hk):
    """One-launch norm/rotary/cache-write/attention (cluster + distributed shared memory merge) against
    the two separate kernels and the oracle: the cache rows are bit-identical, the output within
    tolerance."""
    from wisp import kernels
    from wisp.model import rotary_tables

    D, tmax, eps = 128, 4096, 1e-6
    g = _gen(pos + Hq)
    qkv = torch.randn((Hq + 2 * Hk) * D, device="cuda", generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).to(torch.bfloat16)
    cos, sin = rotary_tables(D, tmax, 1e6, "cuda")
    kc = torch.randn(Hk, tmax, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(Hk, tmax, D, device="cuda", generator=g).to(torch.bfloat16)
    kc2, vc2 = kc.clone(), vc.clone()
    p = torch.tensor([pos], dtype=torch.int64, device="cuda")
    out = kernels.attn_decode(qkv, Hq, Hk, D, qn, kn, eps, cos, sin, p, kc, vc, D**-0.5)
    q = kernels.qk_norm_rope_kv(qkv, Hq, Hk, D, qn, kn, eps, cos, sin, p, kc2, vc2)
    ref = kernels.gqa_decode_attn(q, Hq, Hk, D, kc2, vc2, p, D**-0.5)
    torch.cuda.synchronize()
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    want = O.gqa_decode_attention(_np(q).reshape(Hq, D), _np(kc2), _np(vc2), pos, D**-0.5)
    got = _np(out).reshape(Hq, D)
    assert np.abs(got - want).max() <= 1e-2 * max(1.0, np.abs(want).max())
    assert np.abs(got - _np(ref).reshape(Hq, D)).max() <= 1e-2 * max(1.0, np.abs(want).max())
