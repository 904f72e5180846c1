"""Packed expert format (drop-in for the reference ``wisp.quant``, wisp/quant.py).

Layout per expert (byte-identical to the reference store and its on-disk ``.u8`` files):
  bits == 16 : raw bf16                                  -> 3*n*2 bytes
  bits <  16 : [ codes (packed) | fp16 scales [3n/G] | fp16 mins [3n/G] ]
An expert holds 3 matrices of n = I*H elements (gate [I,H], up [I,H], down [H,I]) -> flat [3, n];
element e sits at bit bits*e of the little-endian code stream.

quantize / dequant / unpack run on the GPU through libwisp_b200 and are bit-exact with the reference;
CPU tensors are moved to the current CUDA device and the result moved back (a GPU is required).
"""

from __future__ import annotations

import torch

from . import _lib

SUPPORTED_BITS = (16, 8, 4, 3, 2)


def expert_nbytes(n: int, bits: int, group: int) -> int:
    """Bytes of one packed expert.  Reference: wisp/quant.py:17-22."""
    assert bits in SUPPORTED_BITS, bits
    nb = _lib.lib().wisp_expert_nbytes(int(n), int(bits), int(group))
    if nb < 0:
        raise AssertionError("3*n must be divisible by group and by 8/bits")
    return int(nb)


def _on_gpu(t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        return t
    if not torch.cuda.is_available():
        raise _lib.WispError("wisp.quant needs a CUDA device (there is no CPU path)")
    return t.cuda()


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


@torch.no_grad()
def quantize_batch(w3: torch.Tensor, bits: int, group: int = 128) -> torch.Tensor:
    """[B, 3, n] float (fp32 or bf16, any device) -> [B, nbytes] uint8 on the same device."""
    dev = w3.device
    w = _on_gpu(w3)
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.float()
    w = w.contiguous()
    B, n = w.shape[0], w.shape[-1]
    assert w.numel() == B * 3 * n
    nb = expert_nbytes(n, bits, group)
    out = torch.empty((B, nb), dtype=torch.uint8, device=w.device)
    dt = _lib.DTYPE_F32 if w.dtype == torch.float32 else _lib.DTYPE_BF16
    _lib.call("wisp_quantize", w.data_ptr(), dt, B, n, bits, group, out.data_ptr(), _stream(w))
    return out if out.device == dev else out.to(dev)


@torch.no_grad()
def quantize(w3: torch.Tensor, bits: int, group: int = 128) -> torch.Tensor:
    """w3: [3, n] (any float dtype, any device) -> flat uint8 buffer on the same device.
    Reference: wisp/quant.py:60-73."""
    n = w3.shape[-1]
    return quantize_batch(w3.reshape(1, 3, n), bits, group).reshape(-1)


def _rows_call(name, buf, n, bits, group, out_shape, out_dtype, idx=None):
    dev = buf.device
    b = _on_gpu(buf)
    if b.dim() == 1:
        b = b.reshape(1, -1)
    b = b.contiguous()
    if idx is None:
        nrows, rows_ptr = b.shape[0], None
    else:
        idx = _on_gpu(idx).to(torch.int64).contiguous()
        nrows, rows_ptr = idx.numel(), idx.data_ptr()
    out = torch.empty((nrows, *out_shape), dtype=out_dtype, device=b.device)
    if name == "wisp_dequant":
        _lib.call(name, b.data_ptr(), b.shape[0], b.shape[1], rows_ptr, nrows, n, bits, group, out.data_ptr(), _stream(b))
    else:
        _lib.call(name, b.data_ptr(), b.shape[0], b.shape[1], rows_ptr, nrows, n, bits, out.data_ptr(), _stream(b))
    return out if out.device == dev else out.to(dev)


@torch.no_grad()
def dequant(buf: torch.Tensor, n: int, bits: int, group: int = 128, rows: torch.Tensor | None = None) -> torch.Tensor:
    """buf: [B, nbytes] uint8 -> [B, 3, n] bfloat16 (same device as buf), bit-exact with the reference.
    ``rows`` (int64) optionally selects rows of ``buf`` (a fused gather).  Reference: wisp/quant.py:76-87."""
    if bits == 16 and rows is None:
        B = buf.shape[0]
        return buf.contiguous().view(torch.bfloat16).view(B, 3, n)
    return _rows_call("wisp_dequant", buf, n, bits, group, (3, n), torch.bfloat16, rows)


def dequant_fast(buf, n, bits, group=128):
    """Same as dequant (one CUDA kernel already).  Reference: wisp/quant.py:94-111."""
    return dequant(buf, n, bits, group)


@torch.no_grad()
def unpack_codes(buf: torch.Tensor, n: int, bits: int, rows: torch.Tensor | None = None) -> torch.Tensor:
    """Integer codes [B, 3n] uint8 of packed experts [B, nbytes].  Reference: wisp/quant.py:44-57."""
    return _rows_call("wisp_unpack_codes", buf, n, bits, 0, (3 * n,), torch.uint8, rows)
