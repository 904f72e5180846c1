"""Batched decode of the Qwen3-30B-A3B-shaped model: B sequences, one token each per step, each at its own
position with its own KV cache, all through one CUDA graph (the batched counterpart of the reference's
bs=1 GraphDecoder, wisp/graphdec.py:140-220, which decodes one sequence).

Per layer, for the B tokens at once:

    xn  = RMSNorm(h)                      (the previous layer's residual add fused in: wisp_rmsnorm)
    qkv = xn Wqkv^T                       (cuBLAS over the batch)
    q   = rotary(q_norm(q)); k/v -> cache (wisp_qk_norm_rope_kv_batched, per-sequence positions)
    att = GQA attention over [0, pos[b]]  (wisp_gqa_decode_attn_batched)
    h'  = h + att Wo^T
    xn  = RMSNorm(h'); router logits (+ an optional per-expert bias) -> softmax, top-8, renormalise
                                          (wisp_router_rows: one launch for the batch)
    moe = the routed experts of the B tokens: wisp_moe_batched on this GPU's resident pool, or an
          ExpertParallelMoE (experts sharded over the ranks, dispatch / combine exchanges)
    h   = h' + moe

With expert parallelism every rank decodes its own B sequences (data-parallel attention) and the
experts of each layer are split contiguously over the ranks.  ``expert_bias`` [L, E] adds a fixed bias
to the router logits (the benchmark biases them so expert popularity follows Zipf(1.1)).
"""

from __future__ import annotations

import torch

from . import kernels
from .model import DecoderWeights, rotary_tables


class BatchedDecoder:
    def __init__(self, w: DecoderWeights, batch, tmax=512, ep=None, expert_bias=None, use_graph=True, variant=0):
        """``w.pool`` holds every expert of every layer (slot l * E + e) when ``ep`` is None; with an
        ExpertParallelMoE it holds this rank's experts and ``ep``'s expert function reads them."""
        cfg = w.cfg
        self.w, self.cfg, self.B, self.ep, self.variant = w, cfg, batch, ep, variant
        dev = w.embed.device
        self.dev = dev
        self.L, self.H, self.Hq, self.Hk, self.D = cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim
        self.E, self.k, self.I = cfg.experts, cfg.top_k, cfg.moe_inter
        self.tmax = (tmax + 63) // 64 * 64
        self.use_graph = use_graph
        B = batch
        d = dict(device=dev, dtype=torch.bfloat16)
        self.kc = torch.zeros(self.L, B, self.Hk, self.tmax, self.D, **d)
        self.vc = torch.zeros_like(self.kc)
        self.cos, self.sin = rotary_tables(self.D, self.tmax, cfg.rope_theta, dev)
        self.bias = None if expert_bias is None else expert_bias.to(device=dev, dtype=torch.bfloat16).contiguous()
        self.tokens = torch.zeros(B, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int64, device=dev)
        self.h = torch.zeros(B, self.H, **d)
        self.h_mid = torch.zeros(B, self.H, **d)
        self.xn = torch.zeros(B, self.H, **d)
        self.qkv = torch.zeros(B, (self.Hq + 2 * self.Hk) * self.D, **d)
        self.q = torch.zeros(B, self.Hq, self.D, **d)
        self.att = torch.zeros(B, self.Hq, self.D, **d)
        self.tmp = torch.zeros(B, self.H, **d)
        self.moe = torch.zeros(B, self.H, **d)
        self.logits = torch.zeros(B, cfg.vocab, **d)
        self.next_token = torch.zeros(B, dtype=torch.int64, device=dev)
        self.meta = torch.zeros(B, 2 * self.k, dtype=torch.float32, device=dev)
        self.rrow = torch.zeros(self.L, B, 2 * self.k, dtype=torch.float32, device=dev)  # per layer [experts | weights]
        self.sel = torch.zeros(B, self.k, dtype=torch.int64, device=dev)
        self.rw = torch.zeros(B, self.k, dtype=torch.float32, device=dev)
        self.attn_ws = kernels.attn_batched_workspace(B, self.Hq, self.Hk, self.D, self.tmax, dev)
        self.router_ws = kernels.router_workspace(B, self.E, dev)
        self.moe_ws = None if ep is not None else kernels.moe_batched_workspace(B, self.k, self.H, self.I, dev)
        self.scale = self.D ** -0.5
        self.graph = None
        self.steps = 0

    @property
    def routes(self):
        """The experts each layer chose for each sequence in the last step, int64 [L, B, k]."""
        return self.rrow[..., : self.k].long()

    @property
    def rweights(self):
        """Their weights (renormalised top-k probabilities rounded to bf16, held in fp32), [L, B, k]."""
        return self.rrow[..., self.k :]

    @torch.no_grad()
    def load_kv(self, ks, vs, length):
        """Cached keys / values of positions [0, length) for every layer and sequence: [L, B, Hk, length, D];
        every sequence continues at position ``length``."""
        self.kc[:, :, :, :length].copy_(ks)
        self.vc[:, :, :, :length].copy_(vs)
        self.pos.fill_(length)

    # ---- one token of every sequence -----------------------------------------------------------------
    def _layer(self, l):
        c, lw, eps = self.cfg, self.w.layers[l], self.cfg.eps
        if l == 0:
            kernels.rmsnorm(self.h, lw["in_norm"], eps, out=self.xn)
        else:
            kernels.rmsnorm(self.h_mid, lw["in_norm"], eps, delta=self.moe, sum_out=self.h, out=self.xn)
        torch.matmul(self.xn, lw["wqkv"].t(), out=self.qkv)
        q = kernels.qk_norm_rope_kv_batched(self.qkv, self.Hq, self.Hk, self.D, lw["q_norm"], lw["k_norm"], eps, self.cos,
                                            self.sin, self.pos, self.kc[l], self.vc[l], q_out=self.q)
        kernels.gqa_decode_attn_batched(q, self.Hq, self.Hk, self.D, self.kc[l], self.vc[l], self.pos, self.scale,
                                        workspace=self.attn_ws, out=self.att)
        torch.matmul(self.att.view(self.B, -1), lw["wo"].t(), out=self.tmp)
        torch.add(self.h, self.tmp, out=self.h_mid)
        bias = None if self.bias is None else self.bias[l]
        if self.ep is None:
            kernels.router_rows(self.h_mid, lw["router"], self.k, c.norm_topk, norm_w=lw["post_norm"], eps=eps, bias=bias,
                                xn_out=self.xn, base=l * self.E, meta=self.meta, row=self.rrow[l], workspace=self.router_ws)
            kernels.moe_batched(self.w.pool, self.meta, self.xn, self.k, self.H * self.I, self.H, self.I, c.bits, c.group,
                                out=self.moe, workspace=self.moe_ws, variant=self.variant)
        else:
            kernels.router_rows(self.h_mid, lw["router"], self.k, c.norm_topk, norm_w=lw["post_norm"], eps=eps, bias=bias,
                                xn_out=self.xn, meta=self.meta, row=self.rrow[l], workspace=self.router_ws)
            self.sel.copy_(self.rrow[l, :, : self.k])
            self.rw.copy_(self.rrow[l, :, self.k :])
            self.moe.copy_(self.ep.forward(self.xn, self.sel, self.rw, layer=l))

    def _step(self):
        torch.index_select(self.w.embed, 0, self.tokens, out=self.h)
        for l in range(self.L):
            self._layer(l)
        xf = kernels.rmsnorm(self.h_mid, self.w.final_norm, self.cfg.eps, delta=self.moe, sum_out=self.h, out=self.xn)
        torch.matmul(xf, self.w.lm_head.t(), out=self.logits)
        torch.argmax(self.logits, dim=-1, out=self.next_token)
        self.pos.add_(1)

    def capture(self):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        saved = self.pos.clone()
        with torch.cuda.stream(s):  # warm-up aimed at the last cache slot, which a later step overwrites before reading
            self.pos.fill_(self.tmax - 1)
            self._step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.pos.copy_(saved)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()

    @torch.no_grad()
    def step(self, tokens=None):
        """One token of every sequence (``tokens`` int64 [B] on the device, or the last greedy choice);
        returns the logits [B, V]."""
        self.tokens.copy_(self.next_token if tokens is None else tokens)
        if self.use_graph:
            if self.graph is None:
                self.capture()
            self.graph.replay()
        else:
            self._step()
        self.steps += 1
        return self.logits

    def release(self):
        self.graph = None


def zipf_bias(layers, experts, s=1.1, seed=7, device="cuda"):
    """[L, E] router-logit biases log(r^-s) for a seeded random popularity rank r of each expert per layer:
    with unit-variance router logits, expert popularity then follows Zipf(s)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    ranks = torch.stack([torch.randperm(experts, generator=g) for _ in range(layers)]).float() + 1
    return (-s * torch.log(ranks)).to(device)
