"""GPU parity of the decode-side ops (one-kernel rotary, RMSNorm with fused residual add) against the
reference fixtures and the oracle."""

import numpy as np
import pytest
import torch

from oracle import wisp_oracle as O

pytestmark = pytest.mark.gpu


def _bf(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16).cuda()


def _np(t):
    return O.bf16_bits_to_f32(t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16))


def test_rope_decode_matches_fixture_and_oracle(golden):
    from wisp.kernels import rope_decode

    r = golden("rope")
    D, Hq, Hk = 128, 32, 4
    q = _bf(r["q"]).reshape(1, Hq, 1, D)
    k = _bf(r["k"]).reshape(1, Hk, 1, D)
    # the HF layout: [1,H,1,D] views of a [1,1,H,D] tensor (non-contiguous head stride)
    qv = q.reshape(1, 1, Hq, D).transpose(1, 2)
    kv = k.reshape(1, 1, Hk, D).transpose(1, 2)
    qo, ko = rope_decode(qv, kv, _bf(r["cos"]).reshape(1, 1, D), _bf(r["sin"]).reshape(1, 1, D))
    cos, sin = O.bf16_bits_to_f32(r["cos"]).reshape(D), O.bf16_bits_to_f32(r["sin"]).reshape(D)
    for got, name in ((qo, "q"), (ko, "k")):
        x = O.bf16_bits_to_f32(r[name]).reshape(-1, D)
        want = O.round_bf16(O.rope(x, cos, sin))
        np.testing.assert_array_equal(_np(got).reshape(-1, D), want)  # fp32 math, one RNE rounding
        hf = O.bf16_bits_to_f32(r[f"{name}_hf"]).reshape(-1, D)
        assert np.abs(_np(got).reshape(-1, D) - hf).max() < 3e-2 * np.abs(hf).max()


def test_rmsnorm_matches_fixture(golden):
    from wisp.kernels import rmsnorm

    nm = golden("norm")
    for H in (2048, 128):
        x, w = _bf(nm[f"x_{H}"]), _bf(nm[f"w_{H}"])
        got = _np(rmsnorm(x, w, 1e-6))
        ref = O.bf16_bits_to_f32(nm[f"wisp_{H}"])
        assert np.abs(got - ref).max() <= 2e-2 * max(1.0, np.abs(ref).max())
        # at most a one-ulp bf16 difference from rsqrt rounding, on a small fraction of elements
        assert (got != ref).mean() < 0.05


@pytest.mark.parametrize("H", [2048, 1000, 100, 12288])
def test_rmsnorm_fused_residual(H):
    """Vector path (H % 8 == 0, H/8 <= 1024) and the generic loop path (H = 100, H = 12288)."""
    from wisp.kernels import rmsnorm

    gen = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(3, H, device="cuda", generator=gen).to(torch.bfloat16)
    d = torch.randn(3, H, device="cuda", generator=gen).to(torch.bfloat16)
    w = (torch.randn(H, device="cuda", generator=gen) * 0.3 + 1).to(torch.bfloat16)
    s = torch.empty_like(x)
    out = rmsnorm(x, w, 1e-6, delta=d, sum_out=s)
    assert torch.equal(s, x + d)  # bf16 add, same rounding as torch
    hs = _np(x + d)
    want = O.round_bf16(_np(w) * O.round_bf16(O.rmsnorm(hs, np.ones(H, np.float32))))
    assert np.abs(_np(out) - want).max() <= 2e-2 * np.abs(want).max()
