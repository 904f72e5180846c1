"""GPU parity of the packed-format kernels (quantize, dequant, code unpack) through the C ABI:
bit-exact against the reference fixtures and against the oracle at the full Qwen3-30B-A3B expert size."""

import numpy as np
import pytest
import torch

from oracle import wisp_oracle as O

pytestmark = pytest.mark.gpu

FULL_N = 2048 * 768


def _t(a, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _bf16_tensor(bits_u16):
    return torch.from_numpy(np.ascontiguousarray(bits_u16).view(np.int16)).view(torch.bfloat16).cuda()


@pytest.mark.parametrize("group", [128, 32])
@pytest.mark.parametrize("bits", [16, 8, 4, 3, 2])
def test_quantize_matches_reference_fixture(golden, group, bits):
    from wisp import quant

    g = golden(f"quant_g{group}")
    n = int(g["n"])
    for src in ("f32", "bf16"):
        w = _t(g["w_f32"]) if src == "f32" else _bf16_tensor(g["w_bf16"])
        buf = quant.quantize(w.reshape(3, n), bits, group).cpu().numpy()
        np.testing.assert_array_equal(buf, g[f"buf_b{bits}_{src}"])


@pytest.mark.parametrize("group", [128, 32])
@pytest.mark.parametrize("bits", [16, 8, 4, 3, 2])
def test_dequant_and_codes_match_reference_fixture(golden, group, bits):
    from wisp import quant

    g = golden(f"quant_g{group}")
    n = int(g["n"])
    for src in ("f32", "bf16"):
        buf = _t(g[f"buf_b{bits}_{src}"])[None]
        deq = quant.dequant(buf, n, bits, group)
        got = deq.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
        np.testing.assert_array_equal(got, g[f"deq_b{bits}_{src}"].reshape(-1))
        if bits < 16:
            codes = quant.unpack_codes(buf, n, bits).cpu().numpy()[0]
            np.testing.assert_array_equal(codes, g[f"codes_b{bits}_{src}"])


@pytest.mark.parametrize("bits", [8, 4, 3, 2])
def test_full_size_expert_bit_exact_vs_oracle(bits):
    """One Qwen3-30B-A3B expert (3 x 2048 x 768): quantize, codes and dequant all bit-exact."""
    from wisp import quant

    gen = torch.Generator(device="cuda").manual_seed(100 + bits)
    w = (torch.randn(3, FULL_N, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    buf = quant.quantize(w, bits, 128)
    wn = O.bf16_bits_to_f32(w.view(torch.int16).cpu().numpy().view(np.uint16))
    ref = O.quantize(wn, bits, 128)
    np.testing.assert_array_equal(buf.cpu().numpy(), ref)
    codes = quant.unpack_codes(buf[None], FULL_N, bits).cpu().numpy()[0]
    ncode = 3 * FULL_N * bits // 8
    np.testing.assert_array_equal(codes, O.unpack_codes(ref[None, :ncode], bits)[0])
    deq = quant.dequant(buf[None], FULL_N, bits, 128).view(torch.int16).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(deq.reshape(-1), O.dequant(ref[None], FULL_N, bits, 128).reshape(-1))


def test_batched_quantize_and_gathered_dequant():
    """Several experts per launch, and dequant of a row selection (the weights_batched gather)."""
    from wisp import quant

    n, bits, G = 256 * 128, 4, 128
    gen = torch.Generator(device="cuda").manual_seed(5)
    w = torch.randn(6, 3, n, device="cuda", generator=gen) * 0.05
    pool = quant.quantize_batch(w, bits, G)
    for e in range(6):
        assert torch.equal(pool[e], quant.quantize(w[e], bits, G))
    idx = torch.tensor([4, 1, 1, 5], device="cuda")
    got = quant.dequant(pool, n, bits, G, rows=idx)
    assert torch.equal(got, quant.dequant(pool[idx], n, bits, G))


def test_bad_row_is_flagged_not_faulted():
    from wisp import _lib, quant

    n, bits, G = 256 * 128, 4, 128
    pool = quant.quantize_batch(torch.randn(2, 3, n, device="cuda"), bits, G)
    _lib.device_status(0, clear=True)
    quant.dequant(pool, n, bits, G, rows=torch.tensor([0, 7], device="cuda"))
    assert _lib.device_status(0) & _lib.STATUS_BAD_SLOT
    assert _lib.device_status(0) == 0  # cleared by the read
