"""Paged MoE block, a drop-in for HF ``Qwen3MoeSparseMoeBlock``, and the shared ``Runtime`` (drop-in for
the reference ``wisp.moe``, wisp/moe.py).

The block keeps the reference's control flow -- route in fp32 (softmax, top-k, renormalise, cast),
one device-to-host read of the routing per call, ``cache.ensure`` per chunk of experts, optional
next-layer prefetch and the hybrid miss policy -- while every expert product runs in this package's
CUDA kernels straight from the packed slots:

  1 token                 wisp_moe_decode (gate/up + SwiGLU, down + weighted combine, two launches)
  several tokens          wisp_moe_batched (pairs grouped by slot on the device, tensor-core MLPs)
  hybrid misses, 1 token  wisp_moe_decode_paged: hit experts from their slots, missed ones read by the
                          same kernels straight from the pinned host store (the reference computes
                          those on the CPU instead, wisp/moe.py:152-164)

bf16 experts (``bits == 16``) or bf16 slots (``cache.decode_on_load``) have nothing to dequantize; they
go through batched cuBLAS products of the slot views, as in the reference.  ``rt.fused`` (env
``WISP_FUSED``) keeps its meaning: 2 = the one-sync two-launch path for single tokens
(``_forward_fast``), 1 = fused kernels per chunk, 0 = the chunked decode / per-expert paths (here also
fused kernels: there is no Triton or torch dequant path to fall back to).
"""

from __future__ import annotations

import os
import time

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import kernels


class Runtime:
    """State shared by all paged blocks of a model (flags, cache, statistics).  Mutable, so a runner can
    reconfigure without rebuilding the store.  Reference: wisp/moe.py:11-39."""

    def __init__(self, store, cache=None, miss_policy="transfer", cpu_threshold=4, prefetch=False, chunk=8,
                 cpu_threads=None, fused=False):
        self.fused = int(fused) or int(os.environ.get("WISP_FUSED", "0") or 0)
        self.store, self.cache = store, cache
        self.miss_policy = miss_policy  # 'transfer' | 'hybrid' (misses served from host memory during decode)
        self.cpu_threshold = cpu_threshold  # tokens per call that count as decode
        self.prefetch = prefetch
        self.chunk = chunk
        self.recorder = None  # a list collects (layer, sel [N, k]) routing traces
        self.reset_stats()
        if cpu_threads:
            torch.set_num_threads(cpu_threads)

    def reset_stats(self):
        # cpu_experts: experts served from host memory (the reference's CPU-computed misses)
        self.stats = dict(layer_calls=0, cpu_experts=0, gpu_experts=0, cpu_time=0.0, admitted=0, prefetched=0)


def _mlp(x, W3, I, H):
    """SwiGLU expert on bf16 weights [3, n] (gate [I, H], up [I, H], down [H, I]).  wisp/moe.py:42-45."""
    g = F.linear(x, W3[0].view(I, H))
    u = F.linear(x, W3[1].view(I, H))
    return F.linear(F.silu(g) * u, W3[2].view(H, I))


class PagedMoEBlock(nn.Module):
    def __init__(self, gate, layer_idx, rt, cfg):
        super().__init__()
        self.gate = gate
        self.layer_idx, self.rt = layer_idx, rt
        self.E, self.top_k = cfg.num_experts, cfg.num_experts_per_tok
        self.norm_topk = cfg.norm_topk_prob
        self.H, self.I = cfg.hidden_size, cfg.moe_intermediate_size
        self.next_gate = None
        self.return_logits = True  # forward returns (out, router logits) as the reference does
        self._ws = {}  # per-device reusable buffers

    def set_next_gate(self, gate):
        # another block's parameter: kept out of this module's registration (state_dict stays the same)
        object.__setattr__(self, "next_gate", gate)

    # ---- routing -------------------------------------------------------------------------------------
    def _logits(self, x):
        g = self.gate
        if isinstance(g, nn.Linear):
            return g(x)
        # a router module that returns more than logits (transformers >= 5 Qwen3MoeTopKRouter): its weight
        return F.linear(x, g.weight.to(x.dtype), None if getattr(g, "bias", None) is None else g.bias.to(x.dtype))

    def _route(self, x):
        logits = self._logits(x)
        rw = F.softmax(logits, dim=1, dtype=torch.float32)
        rw, sel = torch.topk(rw, self.top_k, dim=-1)
        if self.norm_topk:
            rw = rw / rw.sum(dim=-1, keepdim=True)
        return logits, sel, rw.to(x.dtype)

    def _packed(self):
        c = self.rt.cache
        return c.store.bits < 16 and not c.decode_on_load

    def _scratch(self, dev):
        s = self._ws.get(("scratch", dev))
        if s is None:
            c = self.rt.cache
            s = self._ws[("scratch", dev)] = kernels.moe_scratch(self.top_k, self.I, dev, self.H, c.store.bits, c.store.group)
        return s

    # ---- forward ---------------------------------------------------------------------------------------
    def forward(self, hidden_states):
        rt, cache = self.rt, self.rt.cache
        B, T, H = hidden_states.shape
        x = hidden_states.reshape(-1, H)
        N, k = x.shape[0], self.top_k
        logits, sel, rw = self._route(x)
        decode = N <= rt.cpu_threshold
        hybrid = decode and rt.miss_policy == "hybrid"
        do_pf = rt.prefetch and decode and self.next_gate is not None
        pred = torch.topk(self._next_logits(x), k, dim=-1).indices if do_pf else None
        if rt.fused == 2 and N == 1 and not hybrid and self._packed():
            out = self._forward_fast(x, rw, sel, pred, B, T, H)
            return (out, logits) if self.return_logits else out

        # ---- the one device-to-host read of this call: routing (and the prefetch prediction) -----------
        parts = [sel.float(), rw.float()] + ([pred.float()] if do_pf else [])
        row = torch.cat(parts, 1).cpu()
        sel_c, rw_c = row[:, :k].to(torch.int64), row[:, k : 2 * k]
        if rt.recorder is not None:
            rt.recorder.append((self.layer_idx, sel_c.numpy().copy()))
        base = self.layer_idx * self.E
        keys = [base + e for e in torch.unique(sel_c).tolist()]
        st = rt.stats
        st["layer_calls"] += 1
        out = torch.zeros_like(x)
        used = []

        served = False
        if hybrid:
            hit_keys, hit_slots, miss_keys = cache.split(keys)
            if miss_keys:
                served = self._hybrid(x, logits, hit_keys, miss_keys, out)
            else:  # every expert is resident
                cache.sync_compute()
                self._run(x, sel_c, rw_c, list(zip(hit_keys, hit_slots)), out)
                st["gpu_experts"] += len(hit_keys)
                served = True
            if served:
                used = list(hit_slots)
                if miss_keys:
                    t0 = time.perf_counter()
                    st["admitted"] += cache.admit_async(miss_keys, used)
                    st["cpu_time"] += time.perf_counter() - t0
        if not served:  # transfer policy (or a hybrid call whose shape the host-reading kernels do not take)
            for i in range(0, len(keys), rt.chunk):
                ck = keys[i : i + rt.chunk]
                cs = cache.ensure(ck)
                self._run(x, sel_c, rw_c, list(zip(ck, cs)), out)
                st["gpu_experts"] += len(ck)
                used = list(cs)  # only the newest chunk is still to be protected: older ones are queued

        if do_pf:
            nb = (self.layer_idx + 1) * self.E
            pk = [nb + e for e in torch.unique(row[:, 2 * k : 3 * k].to(torch.int64)).tolist()]
            st["prefetched"] += cache.prefetch(pk, used)
        out = out.view(B, T, H)
        return (out, logits) if self.return_logits else out

    def _next_logits(self, x):
        g = self.next_gate
        if isinstance(g, nn.Linear):
            return g(x)
        return F.linear(x, g.weight.to(x.dtype))

    def _run(self, x, sel_c, rw_c, chunk, out):
        """Adds the contribution of the experts in ``chunk`` ([(key, slot)]) to ``out``."""
        cache, k, N, H, I = self.rt.cache, self.top_k, x.shape[0], self.H, self.I
        st = cache.store
        base = self.layer_idx * self.E
        slot_of = {kk - base: s for kk, s in chunk}
        if not self._packed():
            return self._run_bf16(x, sel_c, rw_c, slot_of, out)
        dev = x.device
        if N == 1:
            j = [c for c in range(k) if int(sel_c[0, c]) in slot_of]
            meta = torch.tensor([float(slot_of[int(sel_c[0, c])]) for c in j] + [float(rw_c[0, c]) for c in j],
                                dtype=torch.float32)
            meta = meta.pin_memory().to(dev, non_blocking=True) if dev.type == "cuda" else meta
            if self.rt.fused == 1 and st.bits == 4:
                y = kernels.moe_decode_q4(cache.gpu, meta[: len(j)], x[0], meta[len(j):], st.n, H, I, st.group)
            else:
                y = kernels.moe_decode_fast(cache.gpu, meta, x[0], len(j), st.n, H, I, st.bits, st.group,
                                            scratch=self._scratch(dev))
            out[0].add_(y)
            return
        # several tokens: pairs whose expert is not in this chunk carry slot -1 and are skipped
        meta = torch.empty((N, 2 * k), dtype=torch.float32)
        for t in range(N):
            for c in range(k):
                s = slot_of.get(int(sel_c[t, c]))
                meta[t, c], meta[t, k + c] = (-1.0, 0.0) if s is None else (float(s), float(rw_c[t, c]))
        meta = meta.pin_memory().to(dev, non_blocking=True)
        step = max(1, 2048 // k)  # the batched kernel takes up to 2048 (token, choice) pairs per call
        for t0 in range(0, N, step):
            t1 = min(N, t0 + step)
            y = kernels.moe_batched(cache.gpu, meta[t0:t1].contiguous(), x[t0:t1].contiguous(), k, st.n, H, I,
                                    st.bits, st.group)
            out[t0:t1].add_(y)

    def _run_bf16(self, x, sel_c, rw_c, slot_of, out):
        """bf16 slots: batched products of the slot views (cuBLAS), per expert."""
        cache, H, I = self.rt.cache, self.H, self.I
        experts = sorted(slot_of)
        Ws = cache.weights([slot_of[e] for e in experts])
        dev = x.device
        sel_d = sel_c.to(dev)
        rw_d = rw_c.to(dev)
        for e, W3 in zip(experts, Ws):
            tok, pos = torch.where(sel_d == e)
            y = _mlp(x[tok], W3, I, H) * rw_d[tok, pos].unsqueeze(-1).to(x.dtype)
            out.index_add_(0, tok, y.to(out.dtype))

    def _hybrid(self, x, logits, hit_keys, miss_keys, out):
        """Decode with misses served from host memory: per token, the paged MoE kernels read hit experts
        from their slots and missed ones from the pinned host store.  False when the shape is not one
        the host-reading kernels take (the caller pages the misses in instead)."""
        cache = self.rt.cache
        st = cache.store
        if not (self._packed() and st.bits in (4, 3, 2) and st.host.is_pinned()):
            return False
        dev = x.device
        table = cache.table()
        base = self.layer_idx * self.E
        try:
            for t in range(x.shape[0]):
                y = kernels.moe_decode_paged(cache.gpu, logits[t].contiguous(), x[t], self.top_k, st.n, self.H, self.I,
                                             st.bits, st.group, norm_topk=self.norm_topk, slot_table=table, base=base,
                                             store_host=st.host, scratch=self._scratch(dev))
                out[t].add_(y)
        except kernels.WispError:
            return False
        self.rt.stats["cpu_experts"] += len(miss_keys)
        self.rt.stats["gpu_experts"] += len(hit_keys)
        return True

    def _forward_fast(self, x, rw, sel, pred, B, T, H):
        """One token: one device-to-host read of the routing, one host-to-device copy of the slots and
        weights, two kernel launches.  Reference: wisp/moe.py:174-204."""
        rt, cache, k = self.rt, self.rt.cache, self.top_k
        parts = [sel.float(), rw.float()] + ([pred.float()] if pred is not None else [])
        row = torch.cat(parts, 1).cpu()[0].tolist()
        ex = [int(v) for v in row[:k]]
        base = self.layer_idx * self.E
        if rt.recorder is not None:
            import numpy as np

            rt.recorder.append((self.layer_idx, np.array([ex])))
        st = rt.stats
        st["layer_calls"] += 1
        slots = cache.ensure([base + e for e in ex])
        mm = self._ws.get("meta")
        if mm is None or mm[0].numel() != 2 * k or mm[2].device != x.device:
            host = torch.empty(2 * k, dtype=torch.float32, pin_memory=True)
            mm = self._ws["meta"] = (host, host.numpy(), torch.empty(2 * k, dtype=torch.float32, device=x.device))
        host, hnp, dev = mm
        hnp[:k] = slots  # same-stream order: the previous call's copy of this buffer has finished
        hnp[k:] = row[k : 2 * k]
        dev.copy_(host, non_blocking=True)
        s = cache.store
        y = kernels.moe_decode_fast(cache.gpu, dev, x[0], k, s.n, H, self.I, s.bits, s.group, scratch=self._scratch(x.device))
        st["gpu_experts"] += k
        if pred is not None:
            nb = (self.layer_idx + 1) * self.E
            st["prefetched"] += cache.prefetch([nb + int(e) for e in set(row[2 * k :])], list(slots))
        return y.view(B, T, H)


def _layer_unpacks_tuple(layer):
    """True when the HF decoder layer unpacks (hidden, router_logits) from its MLP (transformers 4.x);
    transformers 5 layers add the MLP output straight to the residual."""
    import inspect

    try:
        src = inspect.getsource(type(layer).forward)
    except (OSError, TypeError):
        return True
    return "isinstance(hidden_states, tuple)" in src


def attach(model, rt):
    """Replace every sparse-MoE block of an HF Qwen3-MoE model with a PagedMoEBlock (keeping its gate;
    the expert weights are dropped, they live in the store) and link each block to the next layer's
    gate for prefetch.  Reference: wisp/moe.py:207-222."""
    cfg = model.config
    blocks = []
    for i, layer in enumerate(model.model.layers):
        old = layer.mlp
        if not hasattr(old, "gate"):
            blocks.append(None)
            continue
        blk = PagedMoEBlock(old.gate, i, rt, cfg)
        blk.return_logits = _layer_unpacks_tuple(layer)
        layer.mlp = blk
        blocks.append(blk)
    for i, b in enumerate(blocks[:-1]):
        if b is not None:
            b.set_next_gate(blocks[i + 1].gate if blocks[i + 1] is not None else None)
    return model
