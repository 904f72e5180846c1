"""wisp_moe_decode_noalloc: the fused MoE decode with its fp32 intermediate in the library's built-in
per-device array instead of caller scratch.  Compared through the C ABI with wisp_moe_decode on the same
inputs, two calls in a row (the second reuses the array the first wrote).  The file name sorts last so
the array is also exercised after every other GPU test has run in the same process."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import wisp_oracle as O

TOL = 1e-2  # relative to max |reference|, the bar of the other MoE decode tests


def _bf16_np(t):
    return O.bf16_bits_to_f32(t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16))


def _rel(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def test_noalloc_rejects_oversize_on_host():
    """k*I above the built-in array is refused before any device work (no GPU needed)."""
    from wisp import _lib

    L = _lib.lib()
    fake = ctypes.c_void_p(256)  # never dereferenced: the size check comes first
    k, H, I = 17, 128, 4096
    assert k * I > _lib.MOE_NOALLOC_MAX_SCRATCH
    rc = L.wisp_moe_decode_noalloc(fake, 1, 16, fake, k, fake, H, I, 4, 128, fake, None)
    assert rc == _lib.WISP_ERR_INVALID
    assert b"exceeds the built-in scratch" in L.wisp_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [4, 3, 8])
def test_noalloc_matches_moe_decode_twice(bits):
    """Qwen3-30B-A3B layer shape (H=2048, I=768, top-8 of 16 experts).  Bits 4/3 run the tensor-core
    kernels, 8 the CUDA-core ones; both read and write the built-in array.  Every call is checked
    against wisp_moe_decode (caller scratch) and against the CPU oracle.  The third call uses k=2
    after two calls with k=8, so values a larger call left in the array beyond k*I must not leak."""
    from wisp import _lib, kernels, quant

    H, I, E, G = 2048, 768, 16, 128
    n = H * I
    gen = torch.Generator(device="cuda").manual_seed(7 + bits)
    w3 = (torch.randn(E, 3, n, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    pool = quant.quantize_batch(w3, bits, G)
    pool_np = pool.cpu().numpy()
    _lib.device_status(0)
    for call, k in enumerate((8, 8, 2)):
        x = torch.randn(H, device="cuda", generator=gen).to(torch.bfloat16)
        slots = torch.randperm(E, device="cuda", generator=gen)[:k]
        wts = torch.softmax(torch.randn(k, device="cuda", generator=gen), 0)
        meta = torch.cat([slots.float(), wts.float()])
        want = _bf16_np(kernels.moe_decode_fast(pool, meta, x, k, n, H, I, bits, G))
        out = torch.full((H,), float("nan"), dtype=torch.bfloat16, device="cuda")
        got = _bf16_np(kernels.moe_decode_noalloc(pool, meta, x, k, n, H, I, bits, G, out=out))
        ref = O.moe_decode_ref(pool_np, slots.cpu().numpy(), _bf16_np(x), wts.cpu().numpy(), n, H, I, bits, G)
        assert np.isfinite(got).all(), f"call {call}"
        assert _rel(got, want) < TOL, f"call {call}: against wisp_moe_decode"
        assert _rel(got, ref) < TOL, f"call {call}: against the oracle"
    assert _lib.device_status(0) == 0


@pytest.mark.gpu
def test_noalloc_rejects_oversize_on_device_tensors():
    from wisp import kernels
    from wisp._lib import WispError

    k, H, I = 17, 128, 4096
    pool = torch.zeros((1, 16), dtype=torch.uint8, device="cuda")
    meta = torch.zeros(2 * k, dtype=torch.float32, device="cuda")
    x = torch.zeros(H, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(WispError, match="exceeds the built-in scratch"):
        kernels.moe_decode_noalloc(pool, meta, x, k, H * I, H, I, 4, 128)


def test_context_table_keys_on_context_id(tmp_path):
    """The per-context address table behind wisp_moe_decode_noalloc (csrc/ctx_cache.h), compiled with
    g++ on the CPU: each context id keeps its own address, a re-put replaces it, an id never seen (a
    context rebuilt by cudaDeviceReset gets a new id) finds nothing, and a full table overwrites its
    oldest entry first."""
    import os
    import shutil
    import subprocess

    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    src = tmp_path / "t.cpp"
    src.write_text(
        """
#include "ctx_cache.h"
#include <cstdio>
int main() {
  wisp::ContextAddressTable<4> t;
  int a, b, c, d, e, f;
  if (t.find(1)) return 1;
  t.put(1, &a); t.put(2, &b);
  if (t.find(1) != &a || t.find(2) != &b) return 2;
  t.put(1, &c);                       // same context, new address
  if (t.find(1) != &c || t.find(2) != &b) return 3;
  if (t.find(3)) return 4;            // a context id never recorded
  t.put(3, &d); t.put(4, &e);         // table now full: ids 1, 2, 3, 4
  t.put(5, &f);                       // overwrites the oldest slot (id 1)
  if (t.find(1) || t.find(5) != &f || t.find(2) != &b || t.find(4) != &e) return 5;
  std::puts("ok");
  return 0;
}
"""
    )
    exe = tmp_path / "t"
    inc = os.path.join(root, "wisp-runtime_b200", "csrc")
    subprocess.run([gxx, "-std=c++17", "-I", inc, str(src), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0 and r.stdout.strip() == "ok", (r.returncode, r.stdout)
