"""Expert parallelism for batched decode (64 tokens per step over all ranks): the experts of every layer are split
contiguously over the ranks of a process group (E / P each); every rank keeps its own tokens
(data-parallel attention), and per MoE layer

    1. buckets its (token, choice) pairs by the rank that owns the chosen expert,
    2. dispatch all-to-all: token vectors + routing of the receiving rank, fixed capacity per destination,
    3. runs its local experts on what it received (the batched MoE kernel, each pair weight 1),
    4. combine all-to-all: the expert outputs go back to the pair's source rank,
    5. sums w[t, j] * y[t, j] over the choices in a fixed order.

Buffers have a fixed capacity C = (tokens per rank) * k per destination (the worst case: every pair to
one rank), so all shapes are static: no host synchronisation, and the whole exchange can be captured
in a CUDA graph with NCCL.  The collective is torch.distributed's all_to_all_single (NCCL over NVLink
on the GPU, gloo on CPU).

On CUDA tensors with a ``slot_base`` (layer -> slot of the layer's first local expert, the same on every
rank), steps 1 and 5 are single kernels (wisp_ep_dispatch / wisp_ep_combine) and the receiver's routing
travels as the batched MoE's meta rows [slot, 1] ([-1, 0] for unused capacity), so ``expert_fn`` gets
(x, meta, layer).  Otherwise (the gloo tests on CPU) the bucketing is plain torch indexing and
``expert_fn`` gets (x, local expert ids as float with -1 for unused capacity, layer).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class ExpertParallelMoE:
    def __init__(self, experts_per_layer, k, hidden, tokens_per_rank, expert_fn, group=None, device="cuda",
                 dtype=torch.bfloat16, slot_base=None, transport="nccl"):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        assert experts_per_layer % self.world == 0, "experts must split evenly over the ranks"
        self.E, self.k, self.H = experts_per_layer, k, hidden
        self.E_local = experts_per_layer // self.world
        self.lo = self.rank * self.E_local
        self.N = tokens_per_rank
        self.C = tokens_per_rank * k
        self.expert_fn = expert_fn
        self.slot_base = slot_base
        self.kernel_mode = torch.device(device).type == "cuda" and slot_base is not None
        W, C = self.world, self.C
        self.send_x = torch.zeros(W, C, hidden, dtype=dtype, device=device)
        self.recv_x = torch.zeros_like(self.send_x) if W > 1 else self.send_x
        if self.kernel_mode:
            self.send_meta = torch.zeros(W, C, 2, dtype=torch.float32, device=device)
            self.recv_meta = torch.zeros_like(self.send_meta) if W > 1 else self.send_meta
            self.src_pos = torch.zeros(tokens_per_rank * k, dtype=torch.int32, device=device)
            self.out = torch.zeros(tokens_per_rank, hidden, dtype=dtype, device=device)
        else:
            self.send_id = torch.full((W, C), -1.0, dtype=torch.float32, device=device)
            self.recv_id = torch.full_like(self.send_id, -1.0)
            self.ranks = torch.arange(W, device=device)
        self.y_back = torch.zeros(W, C, hidden, dtype=dtype, device=device)
        # transport "p2p": the exchanges are kernel stores into peer memory (CUDA IPC over NVLink) with
        # flags instead of NCCL all-to-alls; buffer set = call index % 2 (so a captured step must make an
        # even number of calls, e.g. one per layer of an even layer count)
        self.p2p = None
        self.calls = 0
        if transport == "p2p":
            assert self.kernel_mode, "the p2p transport needs CUDA tensors and slot_base"
            from .kernels import P2PExchange

            self.p2p = P2PExchange(W, self.rank, C, hidden, device)
            handles = [None] * W
            if W > 1:
                dist.all_gather_object(handles, self.p2p.handle, group=self.group)
            else:
                handles = [self.p2p.handle]
            self.p2p.open(handles)
            if W > 1:
                dist.barrier(group=self.group)  # every rank has mapped every allocation

    def _a2a(self, out, inp):
        if self.world == 1:
            if out.data_ptr() != inp.data_ptr():
                out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, group=self.group)

    def forward(self, x, sel, w, layer=0):
        """x [N, H]; sel int64 [N, k] global expert ids; w float32 [N, k] -> [N, H] (x.dtype)."""
        if self.kernel_mode:
            return self._forward_kernels(x, sel, w, layer)
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

    def _forward_p2p(self, x, sel, w, layer):
        N, k, W, C = x.shape[0], self.k, self.world, self.C
        assert N == self.N and sel.shape == (N, k)
        st = self.calls % 2
        self.calls += 1
        ex = self.p2p
        ex.dispatch(x.contiguous(), sel.contiguous(), self.E_local, self.slot_base(layer), st, self.src_pos)
        ex.wait_dispatch(x)
        y = self.expert_fn(ex.recv_x(st), ex.recv_meta(st), layer)
        ex.give_back(y.contiguous(), st)
        return ex.combine(st, self.src_pos, w.contiguous(), self.out)

    def close(self):
        """Unmap the peers' buffers, wait for every rank to do the same, then free this rank's buffer."""
        if self.p2p is not None:
            torch.cuda.synchronize(self.out.device)
            self.p2p.close_peers()
            if self.world > 1:
                dist.barrier(group=self.group)
            self.p2p.close()
            self.p2p = None

    def _forward_kernels(self, x, sel, w, layer):
        from . import kernels

        if self.p2p is not None:
            return self._forward_p2p(x, sel, w, layer)
        N, k, W, C = x.shape[0], self.k, self.world, self.C
        assert N == self.N and sel.shape == (N, k)
        kernels.ep_dispatch(x.contiguous(), sel.contiguous(), self.E_local, W, C, self.slot_base(layer), self.send_x,
                            self.send_meta, self.src_pos)
        self._a2a(self.recv_x.view(-1), self.send_x.view(-1))
        self._a2a(self.recv_meta.view(-1), self.send_meta.view(-1))
        y = self.expert_fn(self.recv_x.view(W * C, self.H), self.recv_meta.view(W * C, 2), layer)
        if W > 1:
            self._a2a(self.y_back.view(-1), y.reshape(-1))
            y = self.y_back.view(W * C, self.H)
        return kernels.ep_combine(y, self.src_pos, w.contiguous(), self.out)


def dispatch_plan(sel, E_local, world, capacity, slot_base):
    """The bookkeeping of the kernel-path dispatch as plain tensor operations (any device): exactly what
    wisp_ep_dispatch writes besides the token rows.  For pair p = t*k + j of this rank's tokens
    (sel int64 [N, k] global expert ids): destination d = sel // E_local, capacity slot c = the pair's
    rank among the pairs bound for d (pair order).  Returns

      dest, cap  int64 [N*k]
      meta       fp32 [world, capacity, 2]: [slot_base + sel - d*E_local, 1] at (d, c), [-1, 0] elsewhere
                 (the receiver's batched-MoE routing rows, k = 1)
      src_pos    int32 [N*k] = d*capacity + c (where the pair's result comes back)"""
    sel = sel.reshape(-1)
    P = sel.numel()
    if P > capacity:
        raise ValueError(f"capacity {capacity} is below the {P} pairs of this rank")
    dest = sel // E_local
    onehot = (dest[:, None] == torch.arange(world, device=sel.device)[None, :]).to(torch.int64)
    cap = (torch.cumsum(onehot, 0) - 1).gather(1, dest[:, None])[:, 0]
    meta = torch.zeros(world, capacity, 2, dtype=torch.float32, device=sel.device)
    meta[..., 0] = -1.0
    meta[dest, cap, 0] = (slot_base + sel - dest * E_local).to(torch.float32)
    meta[dest, cap, 1] = 1.0
    src_pos = (dest * capacity + cap).to(torch.int32)
    return dest, cap, meta, src_pos


def combine_plan(y_back, src_pos, w):
    """What wisp_ep_combine computes, in fp32: out[t] = sum_j w[t, j] * y_back[src_pos[t*k + j]], the
    choices summed in order (y_back [world * capacity, H], w fp32 [N, k])."""
    N, k = w.shape
    rows = y_back.reshape(-1, y_back.shape[-1])[src_pos.long()].float().view(N, k, -1)
    out = torch.zeros(N, rows.shape[-1], dtype=torch.float32, device=rows.device)
    for j in range(k):
        out += w[:, j : j + 1].float() * rows[:, j]
    return out


def batched_expert_fn(pool, layer_slots, n, H, I, bits, group, variant=0):
    """expert_fn running this rank's experts with the batched MoE kernel: local id e of layer l is slot
    layer_slots(l, e) of ``pool``; every received pair gets weight 1 (the source applies w).  Takes the
    receiver meta rows [slot, 1] (kernel mode) or local ids (-1 = unused capacity)."""
    from . import kernels

    def fn(xr, ids_or_meta, layer):
        if ids_or_meta.dim() == 2:  # meta rows from wisp_ep_dispatch
            return kernels.moe_batched(pool, ids_or_meta, xr, 1, n, H, I, bits, group, variant=variant)
        ids = ids_or_meta
        base = float(layer_slots(layer, 0))
        slots = torch.where(ids >= 0, ids + base, torch.full_like(ids, -1.0))
        meta = torch.stack([slots, torch.ones_like(ids)], 1).contiguous()
        return kernels.moe_batched(pool, meta, xr.contiguous(), 1, n, H, I, bits, group, variant=variant)

    return fn
