"""CUDA-graph decode of one token at a time (bs = 1), every op a libwisp_b200 kernel.

Drop-in for the reference ``wisp.graphdec.GraphDecoder`` (wisp/graphdec.py): static buffers (KV
cache [L, Hk, tmax, D], position and token in ``ctl``, routing in ``meta``) so that nothing captured
depends on the current length.  The reference cuts a token at its 48 host decisions (expert paging)
and records the pieces between them; with the experts resident (or a device-side slot table) there
is no host decision, so a whole token is one graph:

    embed -> per layer: [RMSNorm+qkv GEMV] [q/k norm, rotary, cache write, attention]
                        [o GEMV + residual] [RMSNorm+router GEMV] [MoE gate/up (top-k inside), down]
          -> [residual + final RMSNorm + lm_head GEMV] [argmax]

Each kernel is launched with programmatic dependent launch, so its prologue (and the weight stream of
the GEMVs) overlaps the tail of the kernel before it.  ``greedy`` appends the position/token update
to the graph, so a whole generation runs with no host round trip per token.

Two constructors:

  GraphDecoder(weights: DecoderWeights, tmax=...)   the weights in the layout the kernels stream
  GraphDecoder(model, rt, tmax)                     the reference's form: an HF Qwen3-MoE model (its
                                                    MoE blocks attached or not) whose experts live in
                                                    ``rt.cache`` / ``rt.store``; residency is a device
                                                    slot table, misses are read from the pinned host
                                                    store and paged in one token behind

``prefill`` runs the prompt in chunks (the reference's chunked prefill, wisp/graphdec.py:99-152): per
layer the q/k/v, o and router products as GEMMs over the chunk, q/k RMSNorm + rotary + cache write
for all its tokens in one kernel, causal attention over the cache, and the batched MoE kernel.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import kernels
from .model import DecoderWeights, rotary_tables


def _get_kv(pk, i):
    """(keys, values) [1, Hk, T, D] of layer i from an HF cache object or a legacy tuple list."""
    if hasattr(pk, "layers"):
        return pk.layers[i].keys, pk.layers[i].values
    if hasattr(pk, "key_cache"):
        return pk.key_cache[i], pk.value_cache[i]
    return pk[i][0], pk[i][1]


class GraphDecoder:
    def __init__(self, w, rt=None, tmax=2048, use_graph=True, slot_table=None, pool=None, store_host=None, pager=None):
        self.model, self.rt = None, rt
        if not isinstance(w, DecoderWeights):  # the reference's GraphDecoder(model, rt, tmax)
            self.model = w
            if rt is None or getattr(rt, "cache", None) is None:
                raise kernels.WispError("GraphDecoder(model, rt, tmax): the experts come from rt.cache")
            cache = rt.cache
            st = cache.store
            if cache.decode_on_load or st.bits not in (4, 3, 2):
                raise kernels.WispError("GraphDecoder(model, rt): needs packed 4/3/2-bit slots (no decode_on_load)")
            from .cache import SlotTablePager

            w = DecoderWeights.from_hf(self.model, None, bits=st.bits, group=st.group)
            self.cache = cache
            pager = SlotTablePager(cache)
            slot_table, pool, store_host = pager.table, cache.gpu, st.host
        cfg = w.cfg
        self.w, self.cfg = w, cfg
        self.pool = w.pool if pool is None else pool
        self.store_host = store_host  # pinned host store: non-resident experts are read from it
        self.pager = pager
        dev = w.embed.device
        self.dev = dev
        self.L, self.H = cfg.layers, cfg.hidden
        self.Hq, self.Hk, self.D = cfg.heads, cfg.kv_heads, cfg.head_dim
        self.k, self.E, self.I = cfg.top_k, cfg.experts, cfg.moe_inter
        self.tmax = (tmax + 63) // 64 * 64
        self.use_graph = use_graph
        self.slot_table = slot_table
        bf, H = torch.bfloat16, self.H
        d = dict(device=dev, dtype=bf)
        self.kc = torch.zeros(self.L, self.Hk, self.tmax, self.D, **d)
        self.vc = torch.zeros(self.L, self.Hk, self.tmax, self.D, **d)
        self.cos, self.sin = self._rotary(self.tmax)
        self.ctl = torch.zeros(2, dtype=torch.int64, device=dev)  # [token, position]
        self.h_emb = torch.zeros(H, **d)
        self.h_res = torch.zeros(H, **d)  # residual stream entering a layer
        self.h_mid = torch.zeros(H, **d)  # residual stream after attention
        self.xn = torch.zeros(H, **d)  # MoE input (post-attention RMSNorm)
        self.moe = torch.zeros(H, **d)
        self.qkv = torch.zeros((self.Hq + 2 * self.Hk) * self.D, **d)
        self.q = torch.zeros(self.Hq * self.D, **d)
        self.att = torch.zeros(self.Hq * self.D, **d)
        self.rlog = torch.zeros(self.E, **d)
        self.rows = torch.zeros(self.L, 2 * self.k, dtype=torch.float32, device=dev)  # per layer [experts | weights]
        self.meta = torch.zeros(2 * self.k, dtype=torch.float32, device=dev)
        self.scratch = kernels.moe_scratch(self.k, self.I, dev, self.H, cfg.bits, cfg.group)
        self.miss_count = torch.zeros(1, dtype=torch.int32, device=dev) if store_host is not None else None
        self.attn_ws = kernels.attn_workspace(self.Hq, self.Hk, self.D, self.tmax, dev)
        self.argmax_ws = torch.zeros(256, dtype=torch.int64, device=dev)
        self.logits = torch.zeros(cfg.vocab, **d)
        self.next_token = torch.zeros(1, dtype=torch.int64, device=dev)
        self.scale = self.D ** -0.5
        self.pos = 0
        self.graph = self.greedy_graph = None
        if self.pager is not None:  # routing rows of the last tokens, for the policy one token behind
            self.rows_host = [torch.zeros(self.L, 2 * self.k, dtype=torch.float32, pin_memory=True) for _ in range(2)]
            self.turn = 0
            self.waiting = None  # (rows_host index, event) of the last replayed token, not yet planned
        # router top-k folded into the MoE kernels where the tensor-core MoE path takes the shape
        self.routed_moe = self._try_routed_moe()

    def _rotary(self, tmax):
        """cos / sin [tmax, D] bf16: the HF model's own rotary embedding when there is a model, else the
        rotate-half tables of the configured base."""
        if self.model is not None and hasattr(self.model.model, "rotary_emb"):
            pos = torch.arange(tmax, device=self.dev)[None]
            cos, sin = self.model.model.rotary_emb(torch.zeros(1, 1, self.H, device=self.dev, dtype=torch.bfloat16), pos)
            return cos[0].to(torch.bfloat16).contiguous(), sin[0].to(torch.bfloat16).contiguous()
        return rotary_tables(self.D, tmax, self.cfg.rope_theta, self.dev)

    def _out_logits(self):
        return self.logits.view(1, -1) if self.model is not None else self.logits

    # ---------------------------------------------------------------------------------------------
    def _layer(self, l):
        w, c, lw = self.w, self.cfg, self.w.layers[l]
        pos = self.ctl[1:2]
        first = l == 0
        # residual add of the previous MoE + input RMSNorm + q/k/v projections
        kernels.gemv(
            lw["wqkv"], self.h_emb if first else self.h_mid, x_add=None if first else self.moe,
            x_sum_out=None if first else self.h_res, norm_w=lw["in_norm"], eps=c.eps, out=self.qkv,
        )
        if self.D == 128 and self.Hq // self.Hk <= 8:  # one cluster launch: norms, rotary, cache write, attention
            kernels.attn_decode(
                self.qkv, self.Hq, self.Hk, self.D, lw["q_norm"], lw["k_norm"], c.eps, self.cos, self.sin, pos,
                self.kc[l], self.vc[l], self.scale, out=self.att,
            )
        else:
            kernels.qk_norm_rope_kv(
                self.qkv, self.Hq, self.Hk, self.D, lw["q_norm"], lw["k_norm"], c.eps, self.cos, self.sin, pos,
                self.kc[l], self.vc[l], q_out=self.q,
            )
            kernels.gqa_decode_attn(
                self.q, self.Hq, self.Hk, self.D, self.kc[l], self.vc[l], pos, self.scale, workspace=self.attn_ws, out=self.att
            )
        # o projection + residual, then post-attention RMSNorm + router
        kernels.gemv(lw["wo"], self.att, res=self.h_emb if first else self.h_res, out=self.h_mid)
        kernels.gemv(lw["router"], self.h_mid, norm_w=lw["post_norm"], eps=c.eps, xn_out=self.xn, out=self.rlog)
        if self.store_host is not None:
            kernels.moe_decode_paged(
                self.pool, self.rlog, self.xn, self.k, self.H * self.I, self.H, self.I, c.bits, c.group, norm_topk=c.norm_topk,
                slot_table=self.slot_table, base=l * self.E, store_host=self.store_host, miss_count=self.miss_count,
                row=self.rows[l], out=self.moe, scratch=self.scratch,
            )
        elif self.routed_moe:
            kernels.moe_decode_routed(
                self.pool, self.rlog, self.xn, self.k, self.H * self.I, self.H, self.I, c.bits, c.group, norm_topk=c.norm_topk,
                slot_table=self.slot_table, base=l * self.E, row=self.rows[l], out=self.moe, scratch=self.scratch,
            )
        else:
            kernels.router_topk(
                self.rlog, self.k, c.norm_topk, slot_table=self.slot_table, base=l * self.E, row=self.rows[l], meta=self.meta
            )
            kernels.moe_decode_fast(
                self.pool, self.meta, self.xn, self.k, self.H * self.I, self.H, self.I, c.bits, c.group, out=self.moe,
                scratch=self.scratch,
            )

    def _try_routed_moe(self):
        c = self.cfg
        if self.store_host is not None:  # the paged kernels need the tensor-core path: no fallback
            kernels.moe_decode_paged(
                self.pool, self.rlog, self.xn, self.k, self.H * self.I, self.H, self.I, c.bits, c.group,
                norm_topk=c.norm_topk, slot_table=self.slot_table, store_host=self.store_host, out=self.moe,
                scratch=self.scratch,
            )
            torch.cuda.synchronize()
            return True
        try:
            kernels.moe_decode_routed(
                self.pool, self.rlog, self.xn, self.k, self.H * self.I, self.H, self.I, c.bits, c.group,
                norm_topk=c.norm_topk, slot_table=self.slot_table, out=self.moe, scratch=self.scratch,
            )
            torch.cuda.synchronize()
            return True
        except kernels.WispError:
            return False

    def kernels_per_step(self):
        """Kernels launched by one decode step (what the graph replays, torch copies excluded)."""
        attn = 1 if (self.D == 128 and self.Hq // self.Hk <= 8) else 3
        moe = 2 if self.routed_moe else 3
        return 1 + self.L * (attn + 3 + moe) + 3

    def _step(self):
        kernels.embed(self.w.embed, self.ctl[0:1], out=self.h_emb)
        for l in range(self.L):
            self._layer(l)
        kernels.gemv(
            self.w.lm_head, self.h_mid, x_add=self.moe, x_sum_out=self.h_res, norm_w=self.w.final_norm,
            eps=self.cfg.eps, out=self.logits,
        )
        kernels.argmax(self.logits, workspace=self.argmax_ws, out=self.next_token)

    def _advance(self):
        self.ctl[0:1].copy_(self.next_token)
        self.ctl[1:2].add_(1)

    def _capture(self, body):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        saved = self.ctl.clone()
        with torch.cuda.stream(s):  # warm-up outside capture (aims the cache write at the last slot)
            self.ctl[1] = self.tmax - 1
            self._step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.ctl.copy_(saved)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            body()
        return g

    def capture(self):
        """Record one decode step (and the greedy variant that also advances token and position)."""
        self.graph = self._capture(self._step)

        def greedy():
            self._step()
            self._advance()

        self.greedy_graph = self._capture(greedy)

    # ---------------------------------------------------------------------------------------------
    @torch.no_grad()
    def load_kv(self, pk, v=None, T=None):
        """Hand over a context of T positions: ``load_kv(hf_cache, T)`` (the reference's form, an HF
        cache object or per-layer (k, v) pairs of [1, Hk, T, D]) or ``load_kv(k, v, T)`` with
        k, v [L, Hk, T, D]."""
        if T is None:  # load_kv(pk, T)
            T = int(v)
            assert T < self.tmax, f"context {T} >= tmax {self.tmax}"
            for i in range(self.L):
                k_i, v_i = _get_kv(pk, i)
                self.kc[i, :, :T].copy_(k_i.reshape(self.Hk, -1, self.D)[:, :T])
                self.vc[i, :, :T].copy_(v_i.reshape(self.Hk, -1, self.D)[:, :T])
        else:
            assert T < self.tmax, f"context {T} >= tmax {self.tmax}"
            self.kc[:, :, :T].copy_(pk)
            self.vc[:, :, :T].copy_(v)
        self.pos = int(T)

    @torch.no_grad()
    def next(self, token):
        """token: LongTensor [1] on the device -> logits (bf16 [V]; [1, V] for a model-built decoder)
        for the following position."""
        assert self.pos < self.tmax, "context full"
        if self.use_graph and self.graph is None:
            self.capture()
        self.ctl[0:1].copy_(token.reshape(1))
        self.ctl[1].fill_(self.pos)
        if self.use_graph:
            self.graph.replay()
        else:
            self._step()
        self.pos += 1
        if self.pager is not None:
            self._after_replay()
        return self._out_logits()

    @torch.no_grad()
    def greedy(self, token, steps):
        """Greedy generation of ``steps`` tokens after ``token`` without host round trips; returns the
        generated ids (device tensor)."""
        assert self.pos + steps <= self.tmax, "context full"
        if self.greedy_graph is None:
            self.capture()
        out = torch.empty(steps, dtype=torch.int64, device=self.dev)
        self.ctl[0:1].copy_(token.reshape(1))
        self.ctl[1].fill_(self.pos)
        for i in range(steps):
            self.greedy_graph.replay()
            out[i : i + 1].copy_(self.next_token)
            if self.pager is not None:
                self._after_replay()
        self.pos += steps
        return out

    @torch.no_grad()
    def step_greedy(self):
        """One greedy token from the device-side token and position (no host input)."""
        if self.greedy_graph is None:
            self.capture()
        self.greedy_graph.replay()
        self.pos += 1
        if self.pager is not None:
            self._after_replay()

    # ---- chunked prefill -------------------------------------------------------------------------
    @torch.no_grad()
    def prefill(self, ids, start=None, chunk=None):
        """Run prompt tokens ``ids`` at positions start .. start + T - 1 (default: the current position,
        so earlier context is reused), writing K/V straight into the static cache, in chunks of at most
        ``chunk`` tokens (<= 2048 / top_k, the batched MoE kernel's pair limit).  Returns the logits of
        the last token.  Reference: wisp/graphdec.py:99-152."""
        start = self.pos if start is None else int(start)
        ids = ids.reshape(-1).to(self.dev)
        n = ids.numel()
        assert start + n <= self.tmax, f"context {start + n} > capacity {self.tmax}"
        if self.pager is not None:
            self.flush()  # every page-in landed and published: residency is settled
        most = max(1, 2048 // self.k)
        chunk = most if chunk is None else max(1, min(int(chunk), most))
        for c0 in range(0, n, chunk):
            self._prefill_chunk(ids[c0 : c0 + chunk], start + c0)
        self.pos = start + n
        return self._out_logits()

    def _chunk_moe(self, l, sel, rw, xn):
        """MoE of the chunk's tokens in layer l (routing sel [T, k], rw fp32 [T, k]) with the batched
        kernel.  Its experts must be resident in the pool it reads: with an expert cache they are paged
        in as one request per layer, or in groups the pool can hold (pairs outside a group carry slot
        -1, and the groups' outputs are summed) when the layer's working set is larger than the cache."""
        c, H, I, k = self.cfg, self.H, self.I, self.k
        cache = getattr(self, "cache", None)
        if cache is None:
            slots = (sel + l * self.E).float() if self.slot_table is None else self.slot_table[sel + l * self.E].float()
            meta = torch.cat([slots, rw], 1).contiguous()
            return kernels.moe_batched(self.pool, meta, xn, k, H * I, H, I, c.bits, c.group)
        base = l * self.E
        sel_c = sel.cpu()
        uniq = torch.unique(sel_c).tolist()
        room = max(1, cache.core.nslots - cache.core.n_static)
        out = None
        for i in range(0, len(uniq), room):
            group = uniq[i : i + room]
            slot_of = torch.full((self.E,), -1.0)
            slot_of[group] = torch.tensor(cache.ensure([base + e for e in group]), dtype=torch.float32)
            slots = slot_of[sel_c].to(self.dev, non_blocking=True)
            meta = torch.cat([slots, torch.where(slots >= 0, rw, torch.zeros_like(rw))], 1).contiguous()
            y = kernels.moe_batched(cache.gpu, meta, xn, k, H * I, H, I, c.bits, c.group)
            out = y if out is None else out + y
        return out

    def _prefill_chunk(self, part, s0):
        c, w = self.cfg, self.w
        T, H, Hq, Hk, D, k = part.numel(), self.H, self.Hq, self.Hk, self.D, self.k
        pos0 = torch.full((1,), s0, dtype=torch.int64, device=self.dev)
        S = s0 + T
        mask = torch.arange(S, device=self.dev)[None, :] <= (s0 + torch.arange(T, device=self.dev))[:, None]
        h = w.embed.index_select(0, part)  # [T, H]
        for l in range(self.L):
            lw = w.layers[l]
            xn = kernels.rmsnorm(h, lw["in_norm"], c.eps)
            qkv = xn @ lw["wqkv"].t()
            q = kernels.qk_norm_rope_kv_rows(qkv, Hq, Hk, D, lw["q_norm"], lw["k_norm"], c.eps, self.cos, self.sin, pos0,
                                            self.kc[l], self.vc[l])
            o = F.scaled_dot_product_attention(q.transpose(0, 1)[None], self.kc[l, :, :S][None], self.vc[l, :, :S][None],
                                               attn_mask=mask, scale=self.scale, enable_gqa=True)
            h = h + o[0].transpose(0, 1).reshape(T, Hq * D) @ lw["wo"].t()
            xn2 = kernels.rmsnorm(h, lw["post_norm"], c.eps)
            p = F.softmax(xn2 @ lw["router"].t(), dim=-1, dtype=torch.float32)
            rw, sel = torch.topk(p, k, dim=-1)
            if c.norm_topk:
                rw = rw / rw.sum(-1, keepdim=True)
            h = h + self._chunk_moe(l, sel, rw.to(torch.bfloat16).float(), xn2)
        kernels.gemv(w.lm_head, h[-1].contiguous(), norm_w=w.final_norm, eps=c.eps, out=self.logits)

    # ---- capacity ----------------------------------------------------------------------------------
    @torch.no_grad()
    def resize(self, tmax):
        """Change the context capacity, keeping the first ``pos`` positions; graphs are re-captured on
        the next step.  Reference: wisp/graphdec.py:87-97."""
        tmax = (tmax + 63) // 64 * 64
        if tmax == self.tmax:
            return
        if self.pager is not None:
            self.flush()
        torch.cuda.synchronize()
        keep = min(self.pos, tmax)
        d = dict(device=self.dev, dtype=torch.bfloat16)
        kc = torch.zeros(self.L, self.Hk, tmax, self.D, **d)
        vc = torch.zeros(self.L, self.Hk, tmax, self.D, **d)
        kc[:, :, :keep].copy_(self.kc[:, :, :keep])
        vc[:, :, :keep].copy_(self.vc[:, :, :keep])
        self.kc, self.vc = kc, vc
        self.tmax, self.pos = tmax, keep
        self.cos, self.sin = self._rotary(tmax)
        self.attn_ws = kernels.attn_workspace(self.Hq, self.Hk, self.D, tmax, self.dev)
        self.graph = self.greedy_graph = None
        torch.cuda.empty_cache()

    # ---- paging one token behind (decoders with a SlotTablePager) ----------------------------------
    def _after_replay(self):
        i = self.turn
        self.turn ^= 1
        self.rows_host[i].copy_(self.rows, non_blocking=True)
        evt = torch.cuda.Event()
        evt.record()
        prev, self.waiting = self.waiting, (i, evt)
        if prev is not None:
            self._plan(*prev)

    def _plan(self, j, e):
        e.synchronize()  # that token has finished; the one replayed after it keeps the GPU busy
        rows = self.rows_host[j][:, : self.k].to(torch.int64).tolist()
        self.pager.apply(rows)
        if self.rt is not None:
            st = self.rt.stats
            st["layer_calls"] += self.L
            st["gpu_experts"] += self.L * self.k
            if self.rt.recorder is not None:
                import numpy as np

                for l, r in enumerate(rows):
                    self.rt.recorder.append((l, np.array([r])))

    @torch.no_grad()
    def flush(self):
        """Run the policy on the last replayed token and wait for every page-in."""
        if self.pager is None:
            return
        if self.waiting is not None:
            j, e = self.waiting
            self.waiting = None
            self._plan(j, e)
        self.pager.drain()

    def host_reads_total(self):
        """Experts read from the host store so far (synchronises)."""
        return int(self.miss_count.item()) if self.miss_count is not None else 0


class PagedGraphDecoder(GraphDecoder):
    """Decode with only part of the experts resident: the reference's segmented scheme
    (wisp/graphdec.py:1-16, :215-308).  A token is cut at its L routing decisions; the pieces between
    them are CUDA graphs:

        graph[0]   embed -> layer 0 attention block -> router(0)                 -> row(0) to the host
        graph[i]   MoE(i-1) -> layer i attention block -> router(i)              -> row(i) to the host
        graph[L]   MoE(L-1) -> final norm -> lm_head -> argmax

    Between graph[i] and graph[i+1] the host reads row(i), ``cache.ensure`` picks slots and copies the
    missing experts in on the cache's copy stream (pinned cudaMemcpyAsync), and the slots + weights go
    to the device meta buffer ahead of graph[i+1] on the compute stream.  With ``prefetch`` the next
    layer's router is also applied to this layer's MoE input and its top-k are paged in without waiting
    (the reference's next_gate predictor), overlapping PCIe with the compute of this layer."""

    def __init__(self, w: DecoderWeights, cache, tmax=2048, prefetch=False):
        super().__init__(w, tmax=tmax, use_graph=True)
        self.cache = cache
        self.prefetch = prefetch
        self.row_host = torch.zeros(self.L, 2 * self.k, dtype=torch.float32, pin_memory=True)
        self.pred_host = torch.zeros(self.L, self.k, dtype=torch.float32, pin_memory=True)
        self.pred_log = torch.zeros(self.E, dtype=torch.bfloat16, device=self.dev)
        self.meta_pred = torch.zeros(2 * self.k, dtype=torch.float32, device=self.dev)
        self.meta_host = torch.zeros(2 * self.k, dtype=torch.float32, pin_memory=True)
        self.segs = None
        self.evt = [torch.cuda.Event() for _ in range(self.L)]

    def _try_routed_moe(self):
        return False  # routing comes from the host (slots of the paged pool)

    def kernels_per_step(self):
        attn = 1 if (self.D == 128 and self.Hq // self.Hk <= 8) else 3
        return 1 + self.L * (attn + 3 + 1 + 2) + 3 + (2 * (self.L - 1) if self.prefetch else 0)

    def _attn_router(self, l):
        """Layer l up to its routing row (copied to pinned host memory)."""
        c, lw = self.cfg, self.w.layers[l]
        pos = self.ctl[1:2]
        first = l == 0
        kernels.gemv(
            lw["wqkv"], self.h_emb if first else self.h_mid, x_add=None if first else self.moe,
            x_sum_out=None if first else self.h_res, norm_w=lw["in_norm"], eps=c.eps, out=self.qkv,
        )
        if self.D == 128 and self.Hq // self.Hk <= 8:
            kernels.attn_decode(
                self.qkv, self.Hq, self.Hk, self.D, lw["q_norm"], lw["k_norm"], c.eps, self.cos, self.sin, pos,
                self.kc[l], self.vc[l], self.scale, out=self.att,
            )
        else:
            kernels.qk_norm_rope_kv(
                self.qkv, self.Hq, self.Hk, self.D, lw["q_norm"], lw["k_norm"], c.eps, self.cos, self.sin, pos,
                self.kc[l], self.vc[l], q_out=self.q,
            )
            kernels.gqa_decode_attn(
                self.q, self.Hq, self.Hk, self.D, self.kc[l], self.vc[l], pos, self.scale, workspace=self.attn_ws, out=self.att
            )
        kernels.gemv(lw["wo"], self.att, res=self.h_emb if first else self.h_res, out=self.h_mid)
        kernels.gemv(lw["router"], self.h_mid, norm_w=lw["post_norm"], eps=c.eps, xn_out=self.xn, out=self.rlog)
        kernels.router_topk(self.rlog, self.k, c.norm_topk, row=self.rows[l], meta=self.meta)
        if self.prefetch and l + 1 < self.L:  # next layer's router on this layer's MoE input
            kernels.gemv(self.w.layers[l + 1]["router"], self.xn, out=self.pred_log)
            kernels.router_topk(self.pred_log, self.k, c.norm_topk, meta=self.meta_pred)  # base 0: expert ids
            self.pred_host[l].copy_(self.meta_pred[: self.k], non_blocking=True)
        self.row_host[l].copy_(self.rows[l], non_blocking=True)

    def _moe(self, l):
        c = self.cfg
        kernels.moe_decode_fast(
            self.cache.gpu, self.meta, self.xn, self.k, self.H * self.I, self.H, self.I, c.bits, c.group, out=self.moe,
            scratch=self.scratch,
        )

    def _seg(self, j):
        if j == 0:
            kernels.embed(self.w.embed, self.ctl[0:1], out=self.h_emb)
        else:
            self._moe(j - 1)
        if j < self.L:
            self._attn_router(j)
        else:
            kernels.gemv(
                self.w.lm_head, self.h_mid, x_add=self.moe, x_sum_out=self.h_res, norm_w=self.w.final_norm,
                eps=self.cfg.eps, out=self.logits,
            )
            kernels.argmax(self.logits, workspace=self.argmax_ws, out=self.next_token)

    def capture(self):
        # warm-up (aims the cache write at the last slot; experts 0..k-1 of the pool as routing)
        saved = self.ctl.clone()
        self.ctl[1] = self.tmax - 1
        self.meta.copy_(torch.cat([torch.arange(self.k, device=self.dev).float(), torch.full((self.k,), 1.0 / self.k, device=self.dev)]))
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for j in range(self.L + 1):
                self._seg(j)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.ctl.copy_(saved)
        pool = torch.cuda.graph_pool_handle()
        self.segs = []
        for j in range(self.L + 1):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                self._seg(j)
            self.segs.append(g)
        torch.cuda.synchronize()

    def _prepare(self, l):
        """Host side of layer l: routing row -> resident slots (+ prefetch of the predicted next layer)."""
        self.evt[l].synchronize()
        row = self.row_host[l]
        k = self.k
        base = l * self.E
        experts = [int(v) for v in row[:k].tolist()]
        slots = self.cache.ensure([base + e for e in experts])
        self.meta_host[:k] = torch.tensor(slots, dtype=torch.float32)
        self.meta_host[k:] = row[k:]
        self.meta.copy_(self.meta_host, non_blocking=True)  # ordered before the next replay on this stream
        if self.prefetch and l + 1 < self.L:
            nb = (l + 1) * self.E
            self.cache.prefetch([nb + int(e) for e in self.pred_host[l].tolist()], slots)

    @torch.no_grad()
    def next(self, token):
        assert self.pos < self.tmax, "context full"
        if self.segs is None:
            self.capture()
        self.ctl[0:1].copy_(token.reshape(1))
        self.ctl[1].fill_(self.pos)
        self.segs[0].replay()
        self.evt[0].record()
        for l in range(self.L):
            self._prepare(l)
            self.segs[l + 1].replay()
            if l + 1 < self.L:
                self.evt[l + 1].record()
        self.pos += 1
        return self.logits


class DevicePagedDecoder(GraphDecoder):
    """Decode with only part of the experts resident and no host decision inside a token.

    Residency is a device slot table (``SlotTablePager.table``) read by the MoE kernels; an expert that
    is not resident is read straight from the pinned host store by the same kernels
    (wisp_moe_decode_paged), so a whole token -- embed, 48 layers, lm_head, argmax -- is one CUDA graph
    as in the all-resident decoder.  The cache policy runs one token behind on the host: after token t
    is replayed, the routing rows of token t-1 (copied to pinned memory when that token ran) go
    through the policy while the GPU computes token t, and the page-ins it decides are copied on the
    cache's side stream and published into the table once they have landed.  The reference's paged
    decoder (wisp/graphdec.py:216-235, :296-308) instead stops at every layer for the host to read the
    routing, page experts in and write the slots back."""

    def __init__(self, w: DecoderWeights, cache, tmax=2048, admit="all"):
        from .cache import SlotTablePager

        self.cache = cache
        pager = SlotTablePager(cache, admit)
        super().__init__(w, tmax=tmax, use_graph=True, slot_table=pager.table, pool=cache.gpu,
                         store_host=cache.store.host, pager=pager)
