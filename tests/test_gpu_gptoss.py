"""GPU parity of the gpt-oss expert kernels (gpt-oss-20b shape) through the C ABI: against the reference
PagedGptOssBlock outputs (fixture gptoss.npz: its decode branch N=1 and grouped branch N=5) and the
oracle at the gpt-oss-20b layer shape (H = I = 2880, 32 experts, top-4) for N = 1 and 32."""

import numpy as np
import pytest
import torch

from oracle import wisp_oracle as O

pytestmark = pytest.mark.gpu


def _np(t):
    return O.bf16_bits_to_f32(t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16))


def _bf(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16).cuda()


def _rel(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def _route(logits, k):
    """Router of gpt-oss through the library: top-k of the logits, softmax over the selected."""
    from wisp import kernels

    rows = []
    for t in range(logits.shape[0]):
        row = torch.empty(2 * k, dtype=torch.float32, device="cuda")
        kernels.router_topk(logits[t].contiguous(), k, "selected", row=row)
        rows.append(row)
    row = torch.stack(rows)
    return row[:, :k].to(torch.int32).contiguous(), row[:, k:].contiguous()


@pytest.mark.parametrize("N", [1, 5])
def test_matches_reference_block(golden, N):
    from wisp import kernels

    g = golden("gptoss")
    H, I, k, G = int(g["H"]), int(g["I"]), int(g["k"]), int(g["G"])
    x = _bf(g[f"x_N{N}"])
    logits = torch.nn.functional.linear(x, _bf(g["router_w"]), _bf(g["router_b"]))
    experts, w = _route(logits, k)
    # the reference: torch.topk of the logits, softmax over them in bf16
    tv, ti = torch.topk(logits, k, dim=-1)
    sc = torch.softmax(tv, dim=1, dtype=tv.dtype).float()
    assert torch.equal(experts.long().sort(1).values, ti.sort(1).values)
    order = torch.argsort(experts.long(), 1)
    assert (w.gather(1, order) - sc.gather(1, torch.argsort(ti, 1))).abs().max().item() <= 2.0**-7
    pool = torch.from_numpy(g["pool"]).cuda()
    meta = torch.cat([experts.float(), w], 1).contiguous()
    out = kernels.moe_gptoss(pool, meta, experts, x, k, H, I, 4, _bf(g["gub"]), _bf(g["db"]), G)
    ref = O.bf16_bits_to_f32(g[f"out_N{N}"])
    assert _rel(_np(out), ref) < 2e-2
    want = O.gptoss_ref(g["pool"], experts.cpu().numpy(), w.cpu().numpy(), _np(x), H, I, 4, G, g["gub"], g["db"])
    assert _rel(_np(out), want) < 1e-2


@pytest.mark.parametrize("N", [1, 32])
def test_gptoss_20b_layer_vs_oracle(N):
    from wisp import kernels, quant

    H = I = 2880
    E, k, G, bits = 32, 4, 128, 4
    n = H * I
    gen = torch.Generator(device="cuda").manual_seed(N)
    logits = torch.randn(N, E, device="cuda", generator=gen).to(torch.bfloat16)
    experts, w = _route(logits, k)
    used = torch.unique(experts.long()).tolist()
    nb = quant.expert_nbytes(n, bits, G)
    pool = torch.zeros((E, nb), dtype=torch.uint8, device="cuda")
    for e in used:
        w3 = (torch.randn(1, 3, n, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
        pool[e : e + 1] = quant.quantize_batch(w3, bits, G)
    gub = (torch.randn(E, 2 * I, device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
    db = (torch.randn(E, H, device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
    x = torch.randn(N, H, device="cuda", generator=gen).to(torch.bfloat16)
    meta = torch.cat([experts.float(), w], 1).contiguous()
    out = kernels.moe_gptoss(pool, meta, experts, x, k, H, I, bits, gub, db, G)
    tok = list(range(N)) if N <= 4 else [0, 7, 31]  # the oracle dequantizes per token: sample a few
    want = O.gptoss_ref(pool.cpu().numpy(), experts.cpu().numpy()[tok], w.cpu().numpy()[tok], _np(x)[tok], H, I, bits, G,
                        gub.view(torch.int16).cpu().numpy().view(np.uint16), db.view(torch.int16).cpu().numpy().view(np.uint16))
    assert _rel(_np(out)[tok], want) < 1e-2


def _layer_case(H, bits, G, N, E, k, seed, hot=None, top=False):
    """One gpt-oss layer of shape H = I through the library and the oracle on a sample of tokens, and the
    same call twice (bitwise equal). `hot` routes every token to experts drawn from the first `hot`
    ids, so each expert's tokens span several 8-token passes."""
    from wisp import kernels, quant

    I = H
    n = H * I
    gen = torch.Generator(device="cuda").manual_seed(seed)
    logits = torch.randn(N, E, device="cuda", generator=gen)
    if hot is not None:
        logits[:, hot:] -= 100.0
    if top:  # only the last k + 2 experts of the pool can win
        logits[:, : E - k - 2] -= 100.0
    experts, w = _route(logits.to(torch.bfloat16), k)
    used = torch.unique(experts.long()).tolist()
    nb = quant.expert_nbytes(n, bits, G)
    pool = torch.zeros((E, nb), dtype=torch.uint8, device="cuda")
    for e in used:
        w3 = (torch.randn(1, 3, n, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
        pool[e : e + 1] = quant.quantize_batch(w3, bits, G)
    gub = (torch.randn(E, 2 * I, device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
    db = (torch.randn(E, H, device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
    x = torch.randn(N, H, device="cuda", generator=gen).to(torch.bfloat16)
    meta = torch.cat([experts.float(), w], 1).contiguous()
    out = kernels.moe_gptoss(pool, meta, experts, x, k, H, I, bits, gub, db, G)
    again = kernels.moe_gptoss(pool, meta, experts, x, k, H, I, bits, gub, db, G)
    assert torch.equal(out.view(torch.int16), again.view(torch.int16)), "two calls differ"
    tok = list(range(N)) if N <= 4 else [0, N // 2, N - 1]
    want = O.gptoss_ref(pool.cpu().numpy(), experts.cpu().numpy()[tok], w.cpu().numpy()[tok], _np(x)[tok], H, I, bits, G,
                        gub.view(torch.int16).cpu().numpy().view(np.uint16), db.view(torch.int16).cpu().numpy().view(np.uint16))
    return _rel(_np(out)[tok], want)


@pytest.mark.parametrize("bits,G", [(8, 128), (3, 128), (2, 128), (4, 32)])
def test_column_path_other_formats(bits, G):
    """Formats outside the row-streaming kernel (other widths, groups below 64) take the column kernel."""
    assert _layer_case(512, bits, G, N=3, E=8, k=2, seed=bits * 100 + G) < 1e-2


@pytest.mark.parametrize("G", [64, 256])
def test_row_path_ragged_slab_and_groups(G):
    """H = 640: gate_up has 1280 columns (slabs of 960 and 320) and down 640 (one narrower slab)."""
    assert _layer_case(640, 4, G, N=2, E=8, k=2, seed=G) < 1e-2


def test_row_path_many_passes():
    """24 tokens on 3 hot experts: each expert's tokens span several 8-token passes."""
    assert _layer_case(512, 4, 128, N=24, E=16, k=2, seed=7, hot=3) < 1e-2


def test_row_path_last_slots_of_a_larger_pool():
    """Experts in the last slots of a 64-slot pool: the tensor maps' slot coordinate at its far end."""
    assert _layer_case(512, 4, 128, N=3, E=64, k=2, seed=5, top=True) < 1e-2
