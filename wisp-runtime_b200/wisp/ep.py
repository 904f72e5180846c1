"""Expert parallelism for batched decode: the experts of every layer are split
contiguously over the ranks of a process group (E / P each); every rank keeps its own tokens
(data-parallel attention), and per MoE layer

    1. buckets its (token, choice) pairs by the rank that owns the chosen expert,
    2. dispatch all-to-all: token vectors + local expert ids, fixed capacity per destination,
    3. runs its local experts on what it received (the batched MoE kernel, each pair weight 1),
    4. combine all-to-all: the expert outputs go back to the pair's source rank,
    5. sums w[t, j] * y[t, j] over the choices in a fixed order.

Buffers have a fixed capacity C = (tokens per rank) * k per destination (the worst case: every pair to
one rank), so all shapes are static: no host synchronisation, and the whole exchange can be captured
in a CUDA graph with NCCL.  Empty capacity slots carry expert id -1 (the kernels skip them).  The
collective is torch.distributed's all_to_all_single (NCCL over NVLink on the GPU, gloo on CPU).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class ExpertParallelMoE:
    def __init__(self, experts_per_layer, k, hidden, tokens_per_rank, expert_fn, group=None, device="cuda",
                 dtype=torch.bfloat16):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        assert experts_per_layer % self.world == 0, "experts must split evenly over the ranks"
        self.E, self.k, self.H = experts_per_layer, k, hidden
        self.E_local = experts_per_layer // self.world
        self.lo = self.rank * self.E_local
        self.N = tokens_per_rank
        self.C = tokens_per_rank * k
        self.expert_fn = expert_fn  # (x [R, H], local ids float [R] (-1 = empty), layer) -> y [R, H]
        W, C = self.world, self.C
        self.send_x = torch.zeros(W, C, hidden, dtype=dtype, device=device)
        self.recv_x = torch.zeros_like(self.send_x)
        self.send_id = torch.full((W, C), -1.0, dtype=torch.float32, device=device)
        self.recv_id = torch.full_like(self.send_id, -1.0)
        self.y_back = torch.zeros_like(self.send_x)
        self.ranks = torch.arange(W, device=device)

    def _a2a(self, out, inp):
        if self.world == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, group=self.group)

    def forward(self, x, sel, w, layer=0):
        """x [N, H]; sel int64 [N, k] global expert ids; w float32 [N, k] -> [N, H] (x.dtype)."""
        N, k, W, C = x.shape[0], self.k, self.world, self.C
        assert N == self.N and sel.shape == (N, k)
        P = N * k
        dest = (sel // self.E_local).reshape(P)
        local = (sel - dest.view(N, k) * self.E_local).reshape(P).to(torch.float32)
        onehot = (dest[:, None] == self.ranks[None, :]).to(torch.int64)  # [P, W], no host-side checks
        pos = (torch.cumsum(onehot, 0) - 1).gather(1, dest[:, None])[:, 0]  # rank of the pair in its bucket
        tok = torch.arange(P, device=x.device) // k
        # 1-2. dispatch
        self.send_id.fill_(-1.0)
        self.send_id[dest, pos] = local
        self.send_x[dest, pos] = x[tok]
        self._a2a(self.recv_x.view(-1), self.send_x.view(-1))
        self._a2a(self.recv_id.view(-1), self.send_id.view(-1))
        # 3. local experts
        y = self.expert_fn(self.recv_x.view(W * C, self.H), self.recv_id.view(W * C), layer)
        # 4. combine exchange: row (src, pos) of y returns to rank src at (my rank, pos)
        self._a2a(self.y_back.view(-1), y.reshape(-1).to(self.y_back.dtype))
        # 5. weighted sum over the choices, fixed order
        yb = self.y_back[dest, pos].view(N, k, self.H).float()
        out = (yb * w.view(N, k, 1)).sum(1)
        return out.to(x.dtype)


def batched_expert_fn(pool, layer_slots, n, H, I, bits, group):
    """expert_fn running this rank's experts with the batched MoE kernel: local id e of layer l is slot
    layer_slots(l, e) of ``pool``; every received pair gets weight 1 (the source applies w)."""
    from . import kernels

    def fn(xr, ids, layer):
        R = xr.shape[0]
        base = float(layer_slots(layer, 0))
        slots = torch.where(ids >= 0, ids + base, torch.full_like(ids, -1.0))
        meta = torch.stack([slots, torch.ones_like(ids)], 1).contiguous()
        return kernels.moe_batched(pool, meta, xr.contiguous(), 1, n, H, I, bits, group)

    return fn
