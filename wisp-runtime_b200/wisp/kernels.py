"""Drop-in for the reference ``wisp.kernels`` (wisp/kernels.py): the same entry points and argument
meaning, computed by hand-written sm_100a CUDA kernels in libwisp_b200.so.

    moe_decode_q4(pool, slots, x, w, n, H, I, group=128, ...)       wisp/kernels.py:115-137
    moe_decode_q4_fast(pool, meta, x, k, n, H, I, group=128, ...)   wisp/kernels.py:188-203
    moe_decode_q3_fast(pool, meta, x, k, n, H, I, group=128, ...)   wisp/kernels.py:310-322
    moe_decode_q2_fast(pool, meta, x, k, n, H, I, group=128, ...)   (new: the reference has no 2-bit kernel)
    rope_decode(q, k, cos, sin)                                      wisp/kernels.py:352-371

The Triton tuning keywords (block_r, block_gu, block_down, num_warps) are accepted and ignored.
Outputs and the fp32 intermediate are allocated with torch.empty on the caller's stream, so every call
can be captured in a CUDA graph.  Preconditions raise AssertionError like the reference; a kernel-side
failure raises WispError.  There is no CPU path.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import WispError

__all__ = [
    "moe_decode_q4",
    "moe_decode_q4_fast",
    "moe_decode_q3_fast",
    "moe_decode_q2_fast",
    "moe_decode_fast",
    "moe_decode_routed",
    "moe_decode_paged",
    "moe_batched",
    "moe_gptoss",
    "ep_dispatch",
    "ep_combine",
    "P2PExchange",
    "rope_decode",
    "rmsnorm",
    "gemv",
    "qk_norm_rope_kv",
    "qk_norm_rope_kv_rows",
    "qk_norm_rope_kv_batched",
    "gqa_decode_attn_batched",
    "gqa_decode_attn",
    "attn_decode",
    "router_topk",
    "embed",
    "argmax",
    "WispError",
]


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if not (isinstance(t, torch.Tensor) and t.is_cuda):
            raise WispError("wisp kernels need CUDA tensors (there is no CPU path)")


def moe_scratch(k, I, device, H=None, bits=4, group=128):
    """Scratch for the fused MoE calls (k*I floats: the intermediate a = silu(g) * u, what
    wisp_moe_scratch_floats reports); reusable by calls that do not overlap."""
    n = k * I
    if H is not None:
        with torch.cuda.device(torch.device(device)) if torch.device(device).type == "cuda" else _null():
            n = max(n, int(_lib.lib().wisp_moe_scratch_floats(k, H, I, bits, group)))
    return torch.empty(n, dtype=torch.float32, device=device)


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def moe_decode_fast(pool, meta, x, k, n, H, I, bits, group=128, out=None, scratch=None, variant=0):
    """Fused dequant + GEMV MoE of one token over the k experts named by ``meta`` (fp32 [2k] =
    [slots..., weights...]).  pool: uint8 [nslots, nbytes]; x: bf16 [H].  Returns bf16 [H].
    ``variant``: 0 automatic, 1 warp-per-row CUDA-core kernels, 2 TMA bulk copies + integer MMA in
    two chained kernels.  ``scratch`` (reusable across calls that do not overlap) comes from
    ``moe_scratch``; one is allocated per call when omitted."""
    assert H % group == 0 and I % group == 0 and n == H * I
    _need_cuda(pool, meta, x)
    assert pool.dtype == torch.uint8 and pool.dim() == 2 and pool.is_contiguous()
    assert meta.dtype == torch.float32 and meta.numel() >= 2 * k and meta.is_contiguous()
    if x.dtype != torch.bfloat16:
        raise WispError(f"x must be bfloat16 (got {x.dtype})")
    x = x.contiguous()
    if scratch is None:
        scratch = moe_scratch(k, I, x.device, H, bits, group)
    elif scratch.numel() < k * I or scratch.dtype != torch.float32 or not scratch.is_contiguous():
        raise WispError(f"scratch must be a contiguous float32 tensor of >= {k * I} elements")
    if out is None:
        out = torch.empty((H,), dtype=x.dtype, device=x.device)
    _lib.call(
        "wisp_moe_decode_variant",
        pool.data_ptr(),
        pool.shape[0],
        pool.shape[1],
        meta.data_ptr(),
        k,
        x.data_ptr(),
        H,
        I,
        bits,
        group,
        scratch.data_ptr(),
        scratch.numel(),
        out.data_ptr(),
        variant,
        _stream(x),
    )
    return out


def moe_decode_routed(pool, logits, x, k, n, H, I, bits, group=128, norm_topk=True, slot_table=None, base=0, row=None,
                      out=None, scratch=None):
    """moe_decode_fast with the router's softmax / top-k computed inside the MoE kernels from the
    router logits (bf16 [E]); ``row`` (fp32 [2k]) optionally receives [experts | weights]."""
    assert H % group == 0 and I % group == 0 and n == H * I
    _need_cuda(pool, logits, x)
    _bf16(logits)
    if x.dtype != torch.bfloat16:
        raise WispError(f"x must be bfloat16 (got {x.dtype})")
    if slot_table is not None and (slot_table.dtype != torch.int32 or not slot_table.is_contiguous()):
        raise WispError("slot_table must be contiguous int32")
    x = x.contiguous()
    if scratch is None:
        scratch = moe_scratch(k, I, x.device, H, bits, group)
    if out is None:
        out = torch.empty((H,), dtype=x.dtype, device=x.device)
    _lib.call(
        "wisp_moe_decode_routed", pool.data_ptr(), pool.shape[0], pool.shape[1], logits.data_ptr(), logits.numel(), k,
        1 if norm_topk else 0, _ptr(slot_table), int(base), _ptr(row), x.data_ptr(), H, I, bits, group, scratch.data_ptr(),
        scratch.numel(), out.data_ptr(), _stream(x),
    )
    return out


def moe_decode_paged(pool, logits, x, k, n, H, I, bits, group=128, norm_topk=True, slot_table=None, base=0,
                     store_host=None, miss_count=None, row=None, out=None, scratch=None):
    """moe_decode_routed over a partially resident pool: ``slot_table`` (int32 [L*E] on the device)
    maps key = base + e to a slot, or to -1 when the expert is not resident; those experts are read
    by the kernels straight from ``store_host`` (the pinned uint8 [L*E, nbytes] host store), so no
    host decision sits between the router and the MoE.  ``miss_count`` (int32 [1], nullable) counts
    the experts read from the host store."""
    assert H % group == 0 and I % group == 0 and n == H * I
    _need_cuda(pool, logits, x, slot_table)
    _bf16(logits)
    if x.dtype != torch.bfloat16:
        raise WispError(f"x must be bfloat16 (got {x.dtype})")
    if slot_table.dtype != torch.int32 or not slot_table.is_contiguous():
        raise WispError("slot_table must be contiguous int32")
    if not (isinstance(store_host, torch.Tensor) and store_host.device.type == "cpu" and store_host.is_pinned()):
        raise WispError("store_host must be a pinned host tensor")
    if store_host.dtype != torch.uint8 or store_host.dim() != 2 or not store_host.is_contiguous():
        raise WispError("store_host must be contiguous uint8 [rows, nbytes]")
    if store_host.shape[1] != pool.shape[1]:
        raise WispError(f"store_host rows of {store_host.shape[1]} bytes, pool slots of {pool.shape[1]}")
    if slot_table.numel() < store_host.shape[0]:
        raise WispError("slot_table must cover every row of store_host")
    if miss_count is not None:
        _need_cuda(miss_count)
        if miss_count.dtype != torch.int32:
            raise WispError("miss_count must be int32")
    x = x.contiguous()
    if scratch is None:
        scratch = moe_scratch(k, I, x.device, H, bits, group)
    if out is None:
        out = torch.empty((H,), dtype=x.dtype, device=x.device)
    _lib.call(
        "wisp_moe_decode_paged", pool.data_ptr(), pool.shape[0], pool.shape[1], logits.data_ptr(), logits.numel(), k,
        1 if norm_topk else 0, slot_table.data_ptr(), int(base), store_host.data_ptr(), store_host.shape[0],
        _ptr(miss_count), _ptr(row), x.data_ptr(), H, I, bits, group, scratch.data_ptr(), scratch.numel(), out.data_ptr(),
        _stream(x),
    )
    return out


def moe_batched_workspace(N, k, H, I, device):
    nb = _lib.lib().wisp_moe_batched_workspace_bytes(N, k, H, I)
    if nb < 0:
        raise WispError("moe_batched: N*k must be in [1, 2048]")
    return torch.empty(nb, dtype=torch.uint8, device=device)


def moe_batched(pool, meta, x, k, n, H, I, bits, group=128, out=None, workspace=None, variant=0):
    """MoE of N tokens (x bf16 [N, H], meta fp32 [N, 2k] = per token [slots | weights]) -> bf16 [N, H].
    ``variant``: 0 automatic, 1 warp-level tensor-core kernels, 2 tcgen05 (4/2-bit, groups of 128k)."""
    assert H % group == 0 and I % group == 0 and n == H * I
    _need_cuda(pool, meta, x)
    _bf16(x)
    N = x.shape[0]
    assert meta.dtype == torch.float32 and meta.is_contiguous() and meta.numel() == N * 2 * k
    if workspace is None:
        workspace = moe_batched_workspace(N, k, H, I, x.device)
    if out is None:
        out = torch.empty((N, H), dtype=torch.bfloat16, device=x.device)
    _lib.call(
        "wisp_moe_batched_variant", pool.data_ptr(), pool.shape[0], pool.shape[1], meta.data_ptr(), N, k, x.data_ptr(), H, I,
        bits, group, workspace.data_ptr(), workspace.numel(), out.data_ptr(), int(variant), _stream(x),
    )
    return out


def moe_gptoss(pool, meta, experts, x, k, H, I, bits, gate_up_bias, down_bias, group=128, out=None, workspace=None):
    """gpt-oss experts of N tokens (x bf16 [N, H]; meta fp32 [N, 2k] = per token [slots | weights];
    experts int32 [N, k] = expert ids for the biases) -> bf16 [N, H]."""
    _need_cuda(pool, meta, x, experts)
    _bf16(x, gate_up_bias, down_bias)
    N = x.shape[0]
    assert meta.dtype == torch.float32 and meta.is_contiguous() and meta.numel() == N * 2 * k
    assert experts.dtype == torch.int32 and experts.is_contiguous() and experts.numel() == N * k
    if workspace is None:
        nb = _lib.lib().wisp_moe_gptoss_workspace_bytes(N, k, H, I)
        if nb < 0:
            raise WispError("moe_gptoss: N*k must be in [1, 2048]")
        workspace = torch.empty(nb, dtype=torch.uint8, device=x.device)
    if out is None:
        out = torch.empty((N, H), dtype=torch.bfloat16, device=x.device)
    _lib.call(
        "wisp_moe_gptoss", pool.data_ptr(), pool.shape[0], pool.shape[1], meta.data_ptr(), experts.data_ptr(), N, k,
        x.data_ptr(), H, I, bits, group, gate_up_bias.data_ptr(), down_bias.data_ptr(), workspace.data_ptr(),
        workspace.numel(), out.data_ptr(), _stream(x),
    )
    return out


def ep_dispatch(x, sel, E_local, world, capacity, slot_base, send_x, send_meta, src_pos):
    """Pack this rank's (token, choice) pairs for the dispatch all-to-all (wisp_ep_dispatch): x bf16
    [N, H], sel int64 [N, k] global expert ids -> send_x [world, capacity, H], send_meta [world,
    capacity, 2] ([slot_base + local id, 1], [-1, 0] when unused), src_pos int32 [N*k]."""
    _need_cuda(x, sel, send_x, send_meta, src_pos)
    _bf16(x, send_x)
    if sel.dtype != torch.int64 or not sel.is_contiguous():
        raise WispError("sel must be contiguous int64")
    if send_meta.dtype != torch.float32 or src_pos.dtype != torch.int32:
        raise WispError("send_meta must be float32 and src_pos int32")
    N, k = sel.shape
    H = x.shape[-1]
    assert send_x.numel() == world * capacity * H and send_meta.numel() == world * capacity * 2 and src_pos.numel() == N * k
    _lib.call(
        "wisp_ep_dispatch", x.data_ptr(), N, H, sel.data_ptr(), k, E_local, world, capacity, int(slot_base), send_x.data_ptr(),
        send_meta.data_ptr(), src_pos.data_ptr(), _stream(x),
    )


def ep_combine(y_back, src_pos, w, out):
    """out[t] = bf16(sum_j w[t, j] * y_back[src_pos[t*k + j]]), choices in order (wisp_ep_combine)."""
    _need_cuda(y_back, src_pos, w, out)
    _bf16(y_back, out)
    if w.dtype != torch.float32 or not w.is_contiguous():
        raise WispError("w must be contiguous float32")
    N, k = w.shape
    _lib.call("wisp_ep_combine", y_back.data_ptr(), N, k, out.shape[-1], src_pos.data_ptr(), w.data_ptr(), out.data_ptr(), _stream(out))
    return out


class _DevArray:
    """A device range described by __cuda_array_interface__ (to view library-owned memory as a tensor)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False), "version": 3}


class P2PExchange:
    """One rank's side of the peer-memory expert-parallel exchange (wisp_ep_*_p2p): a library-owned
    device allocation mapped by every peer through CUDA IPC.  ``open(handles)`` maps the peers' handles
    (gathered from all ranks, in rank order); ``recv_x(set)`` / ``recv_meta(set)`` view the receive
    buffers the batched MoE reads.  Layout as p2p_layout in csrc/ep.cuh."""

    def __init__(self, world, rank, capacity, hidden, device):
        import ctypes

        self.world, self.rank, self.C, self.H, self.device = world, rank, capacity, hidden, torch.device(device)
        nb = _lib.lib().wisp_ep_p2p_bytes(world, capacity, hidden)
        if nb < 0:
            raise WispError(f"ep p2p: world {world} outside [1, 8]")
        self.nbytes = nb
        ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
        with torch.cuda.device(self.device):
            _lib.call("wisp_ipc_alloc", nb, ctypes.byref(ptr), handle)
        self.local = ptr.value
        self.handle = handle.raw
        self.peers = None
        self._opened = []
        self._views()

    def open(self, handles):
        import ctypes

        assert len(handles) == self.world
        bases = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self.local)
                    continue
                p = ctypes.c_void_p()
                _lib.call("wisp_ipc_open", h, ctypes.byref(p))
                self._opened.append(p.value)
                bases.append(p.value)
        self.peers = (ctypes.c_void_p * self.world)(*bases)

    def _off(self):
        W, C, H = self.world, self.C, self.H
        r256 = lambda v: (v + 255) // 256 * 256  # noqa: E731
        recv_meta = r256(2 * W * C * H * 2)
        y_back = r256(recv_meta + 2 * W * C * 2 * 4)
        return 0, recv_meta, y_back

    def _views(self):
        W, C, H = self.world, self.C, self.H
        o = self._off()
        self._rx = [torch.as_tensor(_DevArray(self.local + o[0] + st * W * C * H * 2, (W * C, H), "<i2"), device=self.device)
                    .view(torch.bfloat16) for st in (0, 1)]
        self._rm = [torch.as_tensor(_DevArray(self.local + o[1] + st * W * C * 2 * 4, (W * C, 2), "<f4"), device=self.device)
                    for st in (0, 1)]

    def recv_x(self, st):
        return self._rx[st]

    def recv_meta(self, st):
        return self._rm[st]

    def dispatch(self, x, sel, E_local, slot_base, st, src_pos):
        _need_cuda(x, sel, src_pos)
        _bf16(x)
        N, k = sel.shape
        _lib.call(
            "wisp_ep_dispatch_p2p", x.data_ptr(), N, self.H, sel.data_ptr(), k, E_local, self.world, self.rank, self.C,
            int(slot_base), st, self.peers, src_pos.data_ptr(), _stream(x),
        )

    def wait_dispatch(self, stream_of):
        _lib.call("wisp_ep_wait", self.local, self.world, self.C, self.H, 0, _stream(stream_of))

    def give_back(self, y, st):
        _bf16(y)
        _lib.call("wisp_ep_return_p2p", y.data_ptr(), self.world, self.rank, self.C, self.H, st, self.peers, _stream(y))

    def combine(self, st, src_pos, w, out):
        N, k = w.shape
        _lib.call(
            "wisp_ep_combine_p2p", self.local, self.world, self.C, self.H, st, N, k, src_pos.data_ptr(), w.data_ptr(),
            out.data_ptr(), _stream(out),
        )
        return out

    def close_peers(self):
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.call("wisp_ipc_close", p)
        self._opened = []
        self.peers = None

    def close(self):
        """Unmap the peers and free the local allocation (every peer must have unmapped it first)."""
        self.close_peers()
        self._rx = self._rm = None  # views of the allocation go first
        if self.local:
            with torch.cuda.device(self.device):
                _lib.call("wisp_ipc_free", self.local)
            self.local = None


def moe_decode_noalloc(pool, meta, x, k, n, H, I, bits, group=128, out=None):
    """moe_decode_fast through wisp_moe_decode_noalloc: the fp32 intermediate lives in the library's
    built-in per-device array (k*I <= MOE_NOALLOC_MAX_SCRATCH), so the call allocates nothing on the
    device when ``out`` is given.  Calls on one device that can overlap race on that array."""
    assert H % group == 0 and I % group == 0 and n == H * I
    _need_cuda(pool, meta, x)
    assert pool.dtype == torch.uint8 and pool.dim() == 2 and pool.is_contiguous()
    assert meta.dtype == torch.float32 and meta.numel() >= 2 * k and meta.is_contiguous()
    if x.dtype != torch.bfloat16:
        raise WispError(f"x must be bfloat16 (got {x.dtype})")
    x = x.contiguous()
    if out is None:
        out = torch.empty((H,), dtype=x.dtype, device=x.device)
    _lib.call(
        "wisp_moe_decode_noalloc",
        pool.data_ptr(),
        pool.shape[0],
        pool.shape[1],
        meta.data_ptr(),
        k,
        x.data_ptr(),
        H,
        I,
        bits,
        group,
        out.data_ptr(),
        _stream(x),
    )
    return out


def moe_decode_q4_fast(pool, meta, x, k, n, H, I, group=128, block_gu=32, block_down=8, num_warps=4):
    """4-bit fused MoE decode (2 launches), meta = fp32 [slot_0..slot_{k-1}, w_0..w_{k-1}].
    Reference: wisp/kernels.py:188-203."""
    return moe_decode_fast(pool, meta, x, k, n, H, I, 4, group)


def moe_decode_q3_fast(pool, meta, x, k, n, H, I, group=128, block_gu=8, block_down=8, num_warps=4):
    """3-bit twin of moe_decode_q4_fast.  Reference: wisp/kernels.py:310-322."""
    return moe_decode_fast(pool, meta, x, k, n, H, I, 3, group)


def moe_decode_q2_fast(pool, meta, x, k, n, H, I, group=128, block_gu=8, block_down=8, num_warps=4):
    """2-bit fused MoE decode; the reference runs 2-bit experts through dequant + bmm
    (wisp/moe.py:122-130), this is the same math fused."""
    return moe_decode_fast(pool, meta, x, k, n, H, I, 2, group)


def moe_decode_qb(pool, meta, x, k, n, H, I, bits=4, group=128, out=None, workspace=None, **tuning):
    """Batched MoE decode of N tokens in the reference's naming (the batched entry it plans beside the
    bs=1 ``moe_decode_q*_fast``): meta fp32 [N, 2k] = per token [slots | weights], x bf16 [N, H] ->
    bf16 [N, H].  The reference's own batched path is dequant + bmm / per-expert MLPs
    (wisp/moe.py:122-137); tuning keyword arguments are accepted and ignored, like the bs=1 names'."""
    return moe_batched(pool, meta, x, k, n, H, I, bits, group, out=out, workspace=workspace)


def moe_decode_q4(pool, slots, x, w, n, H, I, group=128, block_r=32, num_warps=4):
    """pool uint8 [nslots, nbytes] (4-bit experts); slots int64 [k]; x [H] bf16; w [k] routing weights.
    Returns [H] in x.dtype.  Reference: wisp/kernels.py:115-137."""
    assert H % group == 0 and I % group == 0 and n == H * I
    _need_cuda(pool, slots, x, w)
    k = slots.numel()
    meta = torch.cat([slots.reshape(-1).to(torch.float32), w.reshape(-1).to(torch.float32)])
    return moe_decode_fast(pool, meta, x, k, n, H, I, 4, group)


def rope_decode(q, k, cos, sin):
    """q: [1,Hq,1,D], k: [1,Hk,1,D] bf16 (any head stride, e.g. HF's transposed views), cos/sin [1,1,D]
    -> rotated (qo, ko), contiguous, same shapes.  Reference: wisp/kernels.py:352-371."""
    _need_cuda(q, k, cos, sin)
    Hq, D = q.shape[1], q.shape[3]
    Hk = k.shape[1]
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        raise WispError("rope_decode: q and k must be bfloat16")
    assert q.stride(3) == 1 and k.stride(3) == 1, "rope_decode: the head dimension must be contiguous"
    cos = cos.reshape(-1).to(torch.bfloat16).contiguous()
    sin = sin.reshape(-1).to(torch.bfloat16).contiguous()
    qo = torch.empty((1, Hq, 1, D), dtype=q.dtype, device=q.device)
    ko = torch.empty((1, Hk, 1, D), dtype=k.dtype, device=k.device)
    _lib.call(
        "wisp_rope_decode",
        q.data_ptr(),
        q.stride(1),
        Hq,
        k.data_ptr(),
        k.stride(1),
        Hk,
        D,
        cos.data_ptr(),
        sin.data_ptr(),
        qo.data_ptr(),
        ko.data_ptr(),
        _stream(q),
    )
    return qo, ko


def rmsnorm(x, weight, eps=1e-6, delta=None, sum_out=None, out=None):
    """weight * rms_norm(x) over the last dim (the patched Qwen3MoeRMSNorm, wisp/model.py:101-102),
    optionally with the residual add fused: x := x + delta (written to ``sum_out`` when given)."""
    _need_cuda(x, weight)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise WispError("rmsnorm: bfloat16 tensors expected")
    H = x.shape[-1]
    x = x.contiguous()
    rows = x.numel() // H
    if out is None:
        out = torch.empty_like(x)
    if delta is not None:
        delta = delta.contiguous()
    _lib.call(
        "wisp_rmsnorm",
        x.data_ptr(),
        delta.data_ptr() if delta is not None else None,
        sum_out.data_ptr() if sum_out is not None else None,
        weight.contiguous().data_ptr(),
        rows,
        H,
        float(eps),
        out.data_ptr(),
        _stream(x),
    )
    return out


# ------------------------------------------------------------------------------------------------
# decoder step (bs = 1)
# ------------------------------------------------------------------------------------------------
def _ptr(t):
    return t.data_ptr() if t is not None else None


def _bf16(*ts):
    for t in ts:
        if t is not None and (t.dtype != torch.bfloat16 or not t.is_contiguous()):
            raise WispError("contiguous bfloat16 tensors expected")


def gemv(W, x, x_add=None, x_sum_out=None, norm_w=None, eps=1e-6, xn_out=None, res=None, out=None, bias=None):
    """y = [res +] (W x' [+ bias]) (W [N, K] bf16, one token), x' = rmsnorm(x + x_add) as requested; see
    wisp_gemv / wisp_gemv_bias."""
    _need_cuda(W, x)
    _bf16(W, x, x_add, x_sum_out, norm_w, xn_out, res, out, bias)
    N, K = W.shape
    if out is None:
        out = torch.empty(N, dtype=torch.bfloat16, device=x.device)
    if bias is None:
        _lib.call(
            "wisp_gemv", W.data_ptr(), N, K, x.data_ptr(), _ptr(x_add), _ptr(x_sum_out), _ptr(norm_w), float(eps),
            _ptr(xn_out), _ptr(res), out.data_ptr(), _stream(x),
        )
    else:
        _lib.call(
            "wisp_gemv_bias", W.data_ptr(), N, K, x.data_ptr(), _ptr(x_add), _ptr(x_sum_out), _ptr(norm_w), float(eps),
            _ptr(xn_out), bias.data_ptr(), _ptr(res), out.data_ptr(), _stream(x),
        )
    return out


def qk_norm_rope_kv(qkv, Hq, Hk, D, qn_w, kn_w, eps, cos_t, sin_t, pos, k_cache, v_cache, q_out=None):
    """Per-head q/k RMSNorm, rotary at position ``pos`` (int64 device scalar), K/V cache write."""
    _need_cuda(qkv, pos)
    _bf16(qkv, qn_w, kn_w, cos_t, sin_t, k_cache, v_cache)
    if q_out is None:
        q_out = torch.empty(Hq * D, dtype=torch.bfloat16, device=qkv.device)
    tmax = k_cache.shape[-2]
    _lib.call(
        "wisp_qk_norm_rope_kv", qkv.data_ptr(), Hq, Hk, D, qn_w.data_ptr(), kn_w.data_ptr(), float(eps), cos_t.data_ptr(),
        sin_t.data_ptr(), pos.data_ptr(), tmax, q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), _stream(qkv),
    )
    return q_out


def qk_norm_rope_kv_rows(qkv, Hq, Hk, D, qn_w, kn_w, eps, cos_t, sin_t, pos0, k_cache, v_cache, q_out=None):
    """qk_norm_rope_kv for the T tokens of ``qkv`` [T, (Hq + 2 Hk) D] at positions *pos0 .. *pos0 + T - 1
    (``pos0`` an int64 device scalar) -> q [T, Hq, D]; K/V rows go into the caches [Hk, tmax, D]."""
    _need_cuda(qkv, pos0)
    _bf16(qkv, qn_w, kn_w, cos_t, sin_t, k_cache, v_cache)
    T = qkv.shape[0]
    if q_out is None:
        q_out = torch.empty((T, Hq, D), dtype=torch.bfloat16, device=qkv.device)
    tmax = k_cache.shape[-2]
    _lib.call(
        "wisp_qk_norm_rope_kv_rows", qkv.data_ptr(), T, qkv.stride(0), Hq, Hk, D, qn_w.data_ptr(), kn_w.data_ptr(), float(eps),
        cos_t.data_ptr(), sin_t.data_ptr(), pos0.data_ptr(), tmax, q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        _stream(qkv),
    )
    return q_out


def qk_norm_rope_kv_batched(qkv, Hq, Hk, D, qn_w, kn_w, eps, cos_t, sin_t, pos, k_cache, v_cache, q_out=None):
    """One token of each of B sequences: qkv [B, (Hq + 2 Hk) D] at positions pos (int64 [B] on the device)
    -> q [B, Hq, D]; K/V rows go into the caches [B, Hk, tmax, D].  qn_w = kn_w = None: no q/k norm."""
    _need_cuda(qkv, pos)
    _bf16(qkv, cos_t, sin_t, k_cache, v_cache)
    B = qkv.shape[0]
    if q_out is None:
        q_out = torch.empty((B, Hq, D), dtype=torch.bfloat16, device=qkv.device)
    tmax = k_cache.shape[-2]
    _lib.call(
        "wisp_qk_norm_rope_kv_batched", qkv.data_ptr(), B, qkv.stride(0), Hq, Hk, D, _ptr(qn_w), _ptr(kn_w), float(eps),
        cos_t.data_ptr(), sin_t.data_ptr(), pos.data_ptr(), tmax, q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        _stream(qkv),
    )
    return q_out


def attn_batched_workspace(B, Hq, Hk, D, tmax, device):
    nf = _lib.lib().wisp_attn_batched_workspace_floats(B, Hq, Hk, D, tmax)
    if nf < 0:
        raise WispError("attn_batched_workspace: bad shape")
    return torch.empty(nf, dtype=torch.float32, device=device)


def gqa_decode_attn_batched(q, Hq, Hk, D, k_cache, v_cache, pos, scale, window=0, sinks=None, workspace=None, out=None):
    """q [B, Hq, D] (one token per sequence) over sequence b's cached positions up to pos[b] (int64 [B]),
    the last ``window`` of them when window > 0; ``sinks`` fp32 [Hq] per-head softmax sinks -> [B, Hq, D]."""
    _need_cuda(q, k_cache, v_cache, pos)
    _bf16(q, k_cache, v_cache)
    B = q.shape[0]
    tmax = k_cache.shape[-2]
    if workspace is None:
        workspace = attn_batched_workspace(B, Hq, Hk, D, tmax, q.device)
    if out is None:
        out = torch.empty((B, Hq, D), dtype=torch.bfloat16, device=q.device)
    if sinks is not None and (sinks.dtype != torch.float32 or not sinks.is_contiguous()):
        raise WispError("sinks must be contiguous float32")
    _lib.call(
        "wisp_gqa_decode_attn_batched", q.data_ptr(), B, Hq, Hk, D, k_cache.data_ptr(), v_cache.data_ptr(), tmax, pos.data_ptr(),
        int(window), _ptr(sinks), float(scale), workspace.data_ptr(), workspace.numel(), out.data_ptr(), _stream(q),
    )
    return out


def attn_decode_batched(qkv, Hq, Hk, D, qn_w, kn_w, eps, cos_t, sin_t, pos, k_cache, v_cache, scale, window=0, sinks=None,
                        workspace=None, out=None):
    """qk_norm_rope_kv_batched + gqa_decode_attn_batched in one pass (wisp_attn_decode_batched): qkv
    [B, (Hq + 2 Hk) D] raw projections -> attention output [B, Hq, D]; the new K/V rows go into the
    caches.  Same bits as the two calls.  D = 64 or 128."""
    _need_cuda(qkv, pos, k_cache, v_cache)
    _bf16(qkv, cos_t, sin_t, k_cache, v_cache, qn_w, kn_w)
    B = qkv.shape[0]
    tmax = k_cache.shape[-2]
    if workspace is None:
        workspace = attn_batched_workspace(B, Hq, Hk, D, tmax, qkv.device)
    if out is None:
        out = torch.empty((B, Hq, D), dtype=torch.bfloat16, device=qkv.device)
    if sinks is not None and (sinks.dtype != torch.float32 or not sinks.is_contiguous()):
        raise WispError("sinks must be contiguous float32")
    _lib.call(
        "wisp_attn_decode_batched", qkv.data_ptr(), qkv.stride(0), B, Hq, Hk, D, _ptr(qn_w), _ptr(kn_w), float(eps), cos_t.data_ptr(),
        sin_t.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), tmax, pos.data_ptr(), int(window), _ptr(sinks), float(scale),
        workspace.data_ptr(), workspace.numel(), out.data_ptr(), _stream(qkv),
    )
    return out


def attn_workspace(Hq, Hk, D, tmax, device):
    n = _lib.lib().wisp_attn_workspace_floats(Hq, Hk, D, tmax)
    if n < 0:
        raise WispError("attn_workspace: bad shape")
    return torch.empty(n, dtype=torch.float32, device=device)


def gqa_decode_attn(q, Hq, Hk, D, k_cache, v_cache, pos, scale, workspace=None, out=None):
    """Decode attention of one token over cache positions 0..pos; q [Hq*D], caches [Hk, tmax, D]."""
    _need_cuda(q, pos)
    _bf16(q, k_cache, v_cache)
    tmax = k_cache.shape[-2]
    if workspace is None:
        workspace = attn_workspace(Hq, Hk, D, tmax, q.device)
    if out is None:
        out = torch.empty(Hq * D, dtype=torch.bfloat16, device=q.device)
    _lib.call(
        "wisp_gqa_decode_attn", q.data_ptr(), Hq, Hk, D, k_cache.data_ptr(), v_cache.data_ptr(), tmax, pos.data_ptr(),
        float(scale), workspace.data_ptr(), out.data_ptr(), _stream(q),
    )
    return out


def attn_decode(qkv, Hq, Hk, D, qn_w, kn_w, eps, cos_t, sin_t, pos, k_cache, v_cache, scale, out=None):
    """qk_norm_rope_kv + gqa_decode_attn in one cluster launch (D = 128): returns attention out [Hq*D]."""
    _need_cuda(qkv, pos)
    _bf16(qkv, qn_w, kn_w, cos_t, sin_t, k_cache, v_cache)
    if out is None:
        out = torch.empty(Hq * D, dtype=torch.bfloat16, device=qkv.device)
    tmax = k_cache.shape[-2]
    _lib.call(
        "wisp_attn_decode", qkv.data_ptr(), Hq, Hk, D, qn_w.data_ptr(), kn_w.data_ptr(), float(eps), cos_t.data_ptr(),
        sin_t.data_ptr(), pos.data_ptr(), tmax, k_cache.data_ptr(), v_cache.data_ptr(), float(scale), out.data_ptr(),
        _stream(qkv),
    )
    return out


def router_topk(logits, k, norm_topk=True, slot_table=None, base=0, row=None, meta=None):
    """softmax -> top-k -> renormalise -> bf16 of one token's router logits (bf16 [E]); fills the
    routing row [experts | weights] and the MoE meta [slots | weights] (fp32).  ``norm_topk``:
    True (Qwen3 norm_topk_prob), False, or "selected" (gpt-oss: softmax over the k selected logits)."""
    _need_cuda(logits)
    _bf16(logits)
    E = logits.numel()
    if meta is None:
        meta = torch.empty(2 * k, dtype=torch.float32, device=logits.device)
    if slot_table is not None and (slot_table.dtype != torch.int32 or not slot_table.is_contiguous()):
        raise WispError("slot_table must be contiguous int32")
    mode = 2 if norm_topk == "selected" else (1 if norm_topk else 0)
    _lib.call(
        "wisp_router_topk", logits.data_ptr(), E, k, mode, _ptr(slot_table), int(base), _ptr(row),
        meta.data_ptr(), _stream(logits),
    )
    return meta


def router_workspace(B, E, device):
    """Zero-filled workspace of the split router (router_rows(..., workspace=)); reusable by calls that
    do not overlap (each launch leaves it zeroed again)."""
    nb = _lib.lib().wisp_router_workspace_bytes(B, E)
    if nb < 0:
        raise WispError("router_workspace: bad shape")
    return torch.zeros(nb, dtype=torch.uint8, device=device)


def router_rows(x, W, k, norm_topk, norm_w=None, eps=1e-6, bias=None, xn_out=None, slot_table=None, base=0, meta=None,
                experts=None, row=None, workspace=None):
    """Router of B tokens (x bf16 [B, H]) in one launch: RMSNorm (norm_w), gate logits W [E, H] (+ bias),
    top-k and weights (norm_topk 0 / 1 / 2 as in router_topk) -> meta fp32 [B, 2k] = [slots | weights];
    optionally experts int32 [B, k], row fp32 [B, 2k] = [ids | weights], xn_out = the normed rows.  With
    ``workspace`` (router_workspace) the gate is split over CTAs, four experts each."""
    _need_cuda(x, W)
    _bf16(x, W, norm_w, bias, xn_out)
    B, H = x.shape
    E = W.shape[0]
    if meta is None:
        meta = torch.empty((B, 2 * k), dtype=torch.float32, device=x.device)
    mode = 2 if norm_topk == "selected" else (1 if norm_topk else 0)
    for t, dt in ((slot_table, torch.int32), (experts, torch.int32), (row, torch.float32), (meta, torch.float32)):
        if t is not None and (t.dtype != dt or not t.is_contiguous()):
            raise WispError("router_rows: slot_table / experts int32, meta / row float32, contiguous")
    if workspace is None:
        _lib.call(
            "wisp_router_rows", x.data_ptr(), B, H, _ptr(norm_w), float(eps), _ptr(xn_out), W.data_ptr(), _ptr(bias), E, k,
            int(mode), _ptr(slot_table), int(base), meta.data_ptr(), _ptr(experts), _ptr(row), _stream(x),
        )
    else:
        _lib.call(
            "wisp_router_rows_ws", x.data_ptr(), B, H, _ptr(norm_w), float(eps), _ptr(xn_out), W.data_ptr(), _ptr(bias), E, k,
            int(mode), _ptr(slot_table), int(base), meta.data_ptr(), _ptr(experts), _ptr(row), workspace.data_ptr(),
            workspace.numel(), _stream(x),
        )
    return meta


def embed(table, token, out=None):
    """out = table[token] for an int64 device scalar ``token``."""
    _need_cuda(table, token)
    _bf16(table)
    V, H = table.shape
    if out is None:
        out = torch.empty(H, dtype=torch.bfloat16, device=table.device)
    _lib.call("wisp_embed", table.data_ptr(), V, H, token.data_ptr(), out.data_ptr(), _stream(table))
    return out


def argmax(x, workspace=None, out=None):
    """Index of the largest bf16 value (ties: lowest index) as an int64 device scalar."""
    _need_cuda(x)
    _bf16(x)
    if workspace is None:
        workspace = torch.empty(_lib.ARGMAX_WORKSPACE, dtype=torch.int64, device=x.device)
    if out is None:
        out = torch.empty(1, dtype=torch.int64, device=x.device)
    _lib.call("wisp_argmax", x.data_ptr(), x.numel(), workspace.data_ptr(), out.data_ptr(), _stream(x))
    return out
