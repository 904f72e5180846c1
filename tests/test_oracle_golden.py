"""Pin the numpy oracle to the reference: golden vectors made by running the reference itself
(tests/golden/make_golden.py) and the reference's own known-answer tests.  CPU only."""

import numpy as np
import pytest

from oracle import wisp_oracle as O


@pytest.mark.parametrize("group", [128, 32])
@pytest.mark.parametrize("bits", [16, 8, 4, 3, 2])
@pytest.mark.parametrize("src", ["f32", "bf16"])
def test_quantize_bit_exact(golden, group, bits, src):
    g = golden(f"quant_g{group}")
    n = int(g["n"])
    w = g["w_f32"] if src == "f32" else O.bf16_bits_to_f32(g["w_bf16"])
    buf = O.quantize(w.reshape(3, n), bits, group)
    assert buf.size == int(g[f"nbytes_b{bits}"]) == O.expert_nbytes(n, bits, group)
    np.testing.assert_array_equal(buf, g[f"buf_b{bits}_{src}"])


@pytest.mark.parametrize("group", [128, 32])
@pytest.mark.parametrize("bits", [16, 8, 4, 3, 2])
def test_dequant_and_codes_bit_exact(golden, group, bits):
    g = golden(f"quant_g{group}")
    n = int(g["n"])
    for src in ("f32", "bf16"):
        buf = g[f"buf_b{bits}_{src}"]
        np.testing.assert_array_equal(O.dequant(buf[None], n, bits, group)[0].reshape(-1), g[f"deq_b{bits}_{src}"].reshape(-1))
        if bits < 16:
            ncode = (3 * n * bits) // 8
            np.testing.assert_array_equal(O.unpack_codes(buf[None, :ncode], bits)[0], g[f"codes_b{bits}_{src}"])


@pytest.mark.parametrize("bits", [8, 4, 3, 2])
def test_pack_roundtrip(bits):
    """Reference tests/test_quant.py:9-12."""
    rng = np.random.default_rng(bits)
    q = rng.integers(0, 2**bits, 4096, dtype=np.uint8)
    np.testing.assert_array_equal(O.unpack_codes(O.pack_codes(q, bits)[None], bits)[0], q)


def test_known_answer_sizes(golden):
    """Reference tests/test_quant.py:37-40 and the per-expert byte table of the Qwen3-30B-A3B shape."""
    g = golden("nbytes_qwen3")
    for b in (16, 8, 4, 3, 2):
        assert O.expert_nbytes(1572864, b, 128) == int(g[f"b{b}"])
    assert O.expert_nbytes(1572864, 16, 128) == 9437184
    assert abs(O.expert_nbytes(1572864, 4, 128) / O.expert_nbytes(1572864, 16, 128) - 0.265) < 0.01
    assert O.expert_nbytes(1572864, 4, 128) == 2506752
    assert O.expert_nbytes(1572864, 3, 128) == 1916928
    assert O.expert_nbytes(1572864, 2, 128) == 1327104


@pytest.mark.parametrize("bits", [16, 8, 4, 3, 2])
def test_error_bounds(bits):
    """Reference tests/test_quant.py:15-24 (size + relative error bound per bit-width)."""
    rng = np.random.default_rng(0)
    n, group = 2048, 32
    w = (rng.standard_normal((3, n)) * 0.02).astype(np.float32)
    buf = O.quantize(w, bits, group)
    assert buf.size == O.expert_nbytes(n, bits, group)
    r = O.bf16_bits_to_f32(O.dequant(buf[None], n, bits, group)[0])
    rel = np.linalg.norm(r - w) / np.linalg.norm(w)
    assert rel < {16: 0.01, 8: 0.01, 4: 0.12, 3: 0.25, 2: 0.6}[bits]


def test_fused_kernel_goldens(golden):
    """The reference Triton kernels (run under the Triton interpreter) and its dequant+einsum oracle
    agree with this oracle's dequant-then-matmul (reference tests/test_kernels.py: < 2e-2)."""
    g = golden("kernels")
    H, I = int(g["H"]), int(g["I"])
    n = H * I
    for bits in (4, 3):
        pool, slots = g[f"pool_b{bits}"], g[f"slots_b{bits}"]
        x = O.bf16_bits_to_f32(g[f"x_b{bits}"])
        w = g[f"w_b{bits}"]
        ours = O.moe_decode_ref(pool, slots, x, w, n, H, I, bits)
        ref = g[f"ref_b{bits}"]
        assert np.abs(ours - ref).max() <= 1e-5 * np.abs(ref).max()
        tri = [O.bf16_bits_to_f32(g[k]) for k in (("q4_v1", "q4_fast") if bits == 4 else ("q3_fast",))]
        for t in tri:
            assert np.abs(t - ref).max() / np.abs(ref).max() < 2e-2


def test_moe_block_goldens(golden):
    """The reference PagedMoEBlock (bf16 torch path: decode branch N<=4, per-expert branch N>4) agrees
    with the fp32 oracle's routed MoE within the bf16 tolerance.  The oracle's router reproduces the
    reference's top-k weights exactly; expert ids may differ only where bf16 logits tie."""
    g = golden("moe_block")
    H, I, k, G = int(g["H"]), int(g["I"]), int(g["k"]), int(g["G"])
    n = H * I
    for bits in (4, 3, 2):
        pool = g[f"pool_b{bits}"]
        for N in (1, 4, 16):
            x = O.bf16_bits_to_f32(g[f"x_b{bits}_N{N}"])
            sel, rw = O.router_topk(O.bf16_bits_to_f32(g[f"logits_b{bits}_N{N}"]), k)
            rsel, rrw = g[f"sel_b{bits}_N{N}"], O.bf16_bits_to_f32(g[f"rw_b{bits}_N{N}"])
            # routing: same top-k weights; the chosen experts differ only inside bf16 logit ties
            np.testing.assert_array_equal(np.sort(rw, -1), np.sort(rrw, -1))
            lg = O.bf16_bits_to_f32(g[f"logits_b{bits}_N{N}"])
            np.testing.assert_array_equal(
                np.sort(np.take_along_axis(lg, sel, -1), -1), np.sort(np.take_along_axis(lg, rsel, -1), -1)
            )
            ours = O.moe_batched_ref(pool, rsel, rrw, x, n, H, I, bits, G)
            ref = O.bf16_bits_to_f32(g[f"out_b{bits}_N{N}"])
            err = np.abs(ours - ref).max() / np.abs(ref).max()
            assert err < 2e-2, (bits, N, err)


def test_rope_and_norm_goldens(golden):
    r = golden("rope")
    D = 128
    cos = O.bf16_bits_to_f32(r["cos"]).reshape(D)
    sin = O.bf16_bits_to_f32(r["sin"]).reshape(D)
    for name in ("q", "k"):
        x = O.bf16_bits_to_f32(r[name]).reshape(-1, D)
        ours = O.round_bf16(O.rope(x, cos, sin))
        for ref_key in (f"{name}_hf", f"{name}_wisp"):
            ref = O.bf16_bits_to_f32(r[ref_key]).reshape(-1, D)
            assert np.abs(ours - ref).max() < 3e-2 * np.abs(ref).max()
        # the reference one-kernel rotary computes in fp32 and stores once; the fixture was made under
        # the Triton interpreter, whose fp32->bf16 store truncates, so truncating the oracle's fp32
        # result must reproduce it bit for bit (this pins the fp32 rotary math exactly)
        f = O.rope(x, cos, sin)
        trunc = ((f.view(np.uint32) >> 16) << 16).view(np.float32)
        np.testing.assert_array_equal(trunc, O.bf16_bits_to_f32(r[f"{name}_wisp"]).reshape(-1, D))
    nm = golden("norm")
    for H in (2048, 128):
        x, w = O.bf16_bits_to_f32(nm[f"x_{H}"]), O.bf16_bits_to_f32(nm[f"w_{H}"])
        # patched form: bf16(w * bf16(rms_norm(x)))
        ours = O.round_bf16(w * O.round_bf16(O.rmsnorm(x, np.ones(H, np.float32))))
        ref = O.bf16_bits_to_f32(nm[f"wisp_{H}"])
        assert np.abs(ours - ref).max() <= 2e-2 * max(1.0, np.abs(ref).max())
        hf = O.bf16_bits_to_f32(nm[f"hf_{H}"])
        assert np.abs(ours - hf).max() < 2e-2 * max(1.0, np.abs(hf).max())


def test_attention_golden(golden):
    a = golden("attn")
    q = O.bf16_bits_to_f32(a["q"])
    kc, vc = O.bf16_bits_to_f32(a["kc"]), O.bf16_bits_to_f32(a["vc"])
    ours = O.gqa_decode_attention(q, kc, vc, int(a["pos"]), 128**-0.5)
    np.testing.assert_allclose(ours, a["out"], atol=2e-5, rtol=1e-4)


def test_sabotage_detected(golden):
    """Control (pattern of the reference tests/test_paged_moe.py:114-126): a planted mistake in the
    oracle -- shuffled experts -- must miss the reference by far more than the tolerance."""
    g = golden("kernels")
    H, I = int(g["H"]), int(g["I"])
    pool, slots = g["pool_b4"], g["slots_b4"]
    x, w, ref = O.bf16_bits_to_f32(g["x_b4"]), g["w_b4"], g["ref_b4"]
    shuffled = (slots + 1) % pool.shape[0]  # every token routed to the wrong expert
    bad = O.moe_decode_ref(pool, shuffled, x, w, H * I, H, I, 4)
    assert np.abs(bad - ref).max() > 10 * 2e-2 * np.abs(ref).max()


def test_gptoss_oracle_matches_reference_block(golden):
    """The oracle's gpt-oss expert math against PagedGptOssBlock (wisp/gptoss.py:111-143) on the
    fixture, routing as the reference does it (top-k of the bf16 logits, softmax over them in bf16)."""
    import torch

    g = golden("gptoss")
    H, I, k, G = int(g["H"]), int(g["I"]), int(g["k"]), int(g["G"])
    for N in (1, 5):
        x = O.bf16_bits_to_f32(g[f"x_N{N}"])
        xb = torch.from_numpy(g[f"x_N{N}"].view(np.int16)).view(torch.bfloat16)
        wr = torch.from_numpy(g["router_w"].view(np.int16)).view(torch.bfloat16)
        br = torch.from_numpy(g["router_b"].view(np.int16)).view(torch.bfloat16)
        logits = torch.nn.functional.linear(xb, wr, br)
        tv, ti = torch.topk(logits, k, dim=-1)
        sc = torch.softmax(tv, dim=1, dtype=tv.dtype).float().numpy()
        out = O.gptoss_ref(g["pool"], ti.numpy(), sc, x, H, I, 4, G, g["gub"], g["db"])
        ref = O.bf16_bits_to_f32(g[f"out_N{N}"])
        assert np.abs(out - ref).max() <= 2e-2 * np.abs(ref).max()
