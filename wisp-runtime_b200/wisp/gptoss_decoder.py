"""A gpt-oss-shaped decoder (openai/gpt-oss-20b: 24 layers, hidden 2880, 64 query / 8 KV heads of 64,
32 experts top-4 of intermediate 2880, vocab 201088) on this package's kernels, for B sequences decoded
together (B = 1 and 32 in the benchmark configurations), one CUDA graph per token step.

The reference runs gpt-oss through HF modules with its paged expert block swapped in
(wisp/gptoss.py:93-183); the math per layer is HF GptOss's:

    x   = RMSNorm(h)                                   (eps 1e-5)
    qkv = x W_qkv^T + b_qkv                            (q 64x64, k 8x64, v 8x64, all with biases)
    q,k = rotary (YaRN tables), k/v -> the cache at the sequence's position
    att = softmax over [q.k * D^-1/2 over the window | sink_head]  (drop the sink) . v
          (even layers: sliding window of 128 positions; odd layers: full attention)
    h   = h + att W_o^T + b_o
    x   = RMSNorm(h);  logits = x W_r^T + b_r;  top-4 of the logits, softmax over those four
    h   = h + sum_j w_j * (act(x W_gu_j + b_gu_j) W_d_j + b_d_j)   (clamped SwiGLU, wisp_moe_gptoss)
    out = RMSNorm(h) W_lm^T -> greedy argmax

Kernels: this package's RMSNorm (with the residual add fused), q/k rotary + cache write, batched GQA
decode attention with sinks and windows, the fused router (RMSNorm, biased gate, top-k, softmax over
the k: one launch for all sequences) and the gpt-oss expert kernels (wisp_moe_gptoss).  At one sequence
the q/k/v and o projections are the GEMV kernel with the previous residual add, the RMSNorm, the bias
and the next residual add fused; for several sequences they are cuBLAS GEMMs over the batch.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _lib, kernels, quant
from .gptoss import expert_w3


@dataclass
class GptOssDecoderConfig:
    vocab: int = 201088
    hidden: int = 2880
    layers: int = 24
    heads: int = 64
    kv_heads: int = 8
    head_dim: int = 64
    experts: int = 32
    top_k: int = 4
    inter: int = 2880
    window: int = 128
    layer_types: list = field(default_factory=list)  # "sliding_attention" / "full_attention" per layer
    rope_theta: float = 150000.0
    rope_scaling: dict = field(default_factory=lambda: dict(rope_type="yarn", factor=32.0, beta_fast=32.0, beta_slow=1.0,
                                                            truncate=False, original_max_position_embeddings=4096))
    eps: float = 1e-5
    bits: int = 4
    group: int = 128

    def __post_init__(self):
        if not self.layer_types:
            self.layer_types = ["sliding_attention" if l % 2 == 0 else "full_attention" for l in range(self.layers)]

    def hf(self, max_positions=131072):
        """The matching transformers GptOssConfig (used for the rotary tables)."""
        from transformers import GptOssConfig

        rp = dict(self.rope_scaling, rope_theta=self.rope_theta)
        return GptOssConfig(vocab_size=self.vocab, hidden_size=self.hidden, num_hidden_layers=self.layers,
                            num_attention_heads=self.heads, num_key_value_heads=self.kv_heads, head_dim=self.head_dim,
                            num_local_experts=self.experts, num_experts_per_tok=self.top_k, intermediate_size=self.inter,
                            sliding_window=self.window, layer_types=list(self.layer_types), rms_norm_eps=self.eps,
                            rope_parameters=rp, max_position_embeddings=max_positions)


def gptoss_rotary_half(cfg: GptOssDecoderConfig, tmax, device):
    """cos / sin fp32 [tmax, D/2]: HF GptOssRotaryEmbedding's tables (YaRN frequencies, the attention
    factor folded in)."""
    from transformers.models.gpt_oss.modeling_gpt_oss import GptOssRotaryEmbedding

    rot = GptOssRotaryEmbedding(cfg.hf(), device=device)
    pos = torch.arange(tmax, device=device)[None]
    cos, sin = rot(torch.zeros(1, 1, cfg.hidden, device=device, dtype=torch.float32), pos)
    return cos[0].float(), sin[0].float()


def gptoss_rotary_tables(cfg: GptOssDecoderConfig, tmax, device):
    """bf16 [tmax, D] tables for the rotary kernel: gpt-oss rotates the halves x1, x2 of a head as
    x1 c - x2 s, x2 c + x1 s, which is rotate-half rotary with the half-width table repeated."""
    cos, sin = gptoss_rotary_half(cfg, tmax, device)
    return (torch.cat([cos, cos], -1).to(torch.bfloat16).contiguous(), torch.cat([sin, sin], -1).to(torch.bfloat16).contiguous())


class GptOssWeights:
    """Seeded random-init weights of the gpt-oss shape; experts packed in the wisp.quant layout of
    ``expert_w3`` (gate_up [H, 2I] interleaved, down [I, H], input-major) in a resident pool, slot
    l * E + e."""

    def __init__(self, cfg):
        self.cfg = cfg
        self.layers = []

    @staticmethod
    @torch.no_grad()
    def random(cfg: GptOssDecoderConfig, device="cuda", seed=0, std=0.02, expert_std=0.02):
        w = GptOssWeights(cfg)
        g = torch.Generator(device=device).manual_seed(seed)
        H, D, Hq, Hk, E, I, V = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.experts, cfg.inter, cfg.vocab
        bf = torch.bfloat16
        resid = std / (2 * cfg.layers) ** 0.5  # projections into the residual stream (scaled init)

        def rnd(*shape, s=std):
            return (torch.randn(*shape, device=device, generator=g) * s).to(bf)

        def norm(n):
            return (1.0 + 0.1 * torch.randn(n, device=device, generator=g)).to(bf)

        w.embed = rnd(V, H, s=1.0)
        w.lm_head = rnd(V, H)
        w.final_norm = norm(H)
        nq = (Hq + 2 * Hk) * D
        for _ in range(cfg.layers):
            w.layers.append(dict(
                in_norm=norm(H), wqkv=rnd(nq, H), bqkv=rnd(nq, s=0.1), wo=rnd(H, Hq * D, s=resid), bo=rnd(H, s=0.01),
                sinks=(torch.randn(Hq, device=device, generator=g) * 0.5).float(), post_norm=norm(H),
                router=rnd(E, H, s=0.05), router_b=rnd(E, s=0.1),
                gub=rnd(E, 2 * I, s=0.1), db=rnd(E, H, s=0.01),
            ))
        n = H * I
        w.nbytes = quant.expert_nbytes(n, cfg.bits, cfg.group)
        w.pool = torch.empty((cfg.layers * E, w.nbytes), dtype=torch.uint8, device=device)
        for l in range(cfg.layers):
            for e0 in range(0, E, 8):
                e1 = min(E, e0 + 8)
                gu = torch.randn(e1 - e0, H, 2 * I, device=device, generator=g) * expert_std
                dn = torch.randn(e1 - e0, I, H, device=device, generator=g) * (expert_std / (2 * cfg.layers) ** 0.5)
                w3 = torch.stack([expert_w3(gu[i], dn[i]) for i in range(e1 - e0)]).to(bf)
                w.pool[l * E + e0 : l * E + e1].copy_(quant.quantize_batch(w3, cfg.bits, cfg.group))
                del gu, dn, w3
        return w


class GptOssDecoder:
    """B sequences decoded one token per step through one CUDA graph (static buffers: tokens and
    positions on the device, KV caches [L, B, Hk, tmax, D])."""

    def __init__(self, w: GptOssWeights, batch=1, tmax=512, use_graph=True):
        cfg = w.cfg
        self.w, self.cfg, self.B = w, cfg, batch
        dev = w.embed.device
        self.dev = dev
        self.L, self.H, self.Hq, self.Hk, self.D = cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim
        self.E, self.k, self.I = cfg.experts, cfg.top_k, cfg.inter
        self.tmax = (tmax + 63) // 64 * 64
        self.use_graph = use_graph
        B, bf = batch, torch.bfloat16
        d = dict(device=dev, dtype=bf)
        self.kc = torch.zeros(self.L, B, self.Hk, self.tmax, self.D, **d)
        self.vc = torch.zeros_like(self.kc)
        self.cos, self.sin = gptoss_rotary_tables(cfg, self.tmax, dev)
        self.tokens = torch.zeros(B, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int64, device=dev)
        self.h = torch.zeros(B, self.H, **d)
        self.h_mid = torch.zeros(B, self.H, **d)
        self.xn = torch.zeros(B, self.H, **d)
        self.qkv = torch.zeros(B, (self.Hq + 2 * self.Hk) * self.D, **d)
        self.q = torch.zeros(B, self.Hq, self.D, **d)
        self.att = torch.zeros(B, self.Hq, self.D, **d)
        self.moe = torch.zeros(B, self.H, **d)
        self.logits = torch.zeros(B, cfg.vocab, **d)
        self.next_token = torch.zeros(B, dtype=torch.int64, device=dev)
        self.meta = torch.zeros(B, 2 * self.k, dtype=torch.float32, device=dev)  # [slots | weights] of the layer
        self.experts = torch.zeros(B, self.k, dtype=torch.int32, device=dev)
        self.rrow = torch.zeros(self.L, B, 2 * self.k, dtype=torch.float32, device=dev)  # per layer [experts | weights]
        self.attn_ws = kernels.attn_batched_workspace(B, self.Hq, self.Hk, self.D, self.tmax, dev)
        self.router_ws = kernels.router_workspace(B, self.E, dev)
        self.moe_ws = torch.empty(_lib.lib().wisp_moe_gptoss_workspace_bytes(B, self.k, self.H, self.I), dtype=torch.uint8,
                                  device=dev)
        self.tmp = torch.zeros(B, self.H, **d)
        self.argmax_ws = torch.zeros(_lib.ARGMAX_WORKSPACE, dtype=torch.int64, device=dev)
        self.scale = self.D ** -0.5
        self.graph = None
        self.steps = 0

    @property
    def routes(self):
        """The experts each layer chose for each sequence in the last step, int64 [L, B, k]."""
        return self.rrow[..., : self.k].long()

    @property
    def rweights(self):
        """Their weights (bf16 softmax over the chosen logits, held in fp32), [L, B, k]."""
        return self.rrow[..., self.k :]

    # ---- one token of every sequence -----------------------------------------------------------------
    def _layer(self, l):
        """Attention then MoE of layer l.  The residual stream arrives as h (layer 0) or as h_mid + moe
        of the previous layer, whose sum is formed inside this layer's first kernel (stored to h)."""
        c, lw, B, eps = self.cfg, self.w.layers[l], self.B, self.cfg.eps
        if B == 1:
            if l == 0:
                kernels.gemv(lw["wqkv"], self.h[0], norm_w=lw["in_norm"], eps=eps, bias=lw["bqkv"], out=self.qkv[0])
            else:
                kernels.gemv(lw["wqkv"], self.h_mid[0], x_add=self.moe[0], x_sum_out=self.h[0], norm_w=lw["in_norm"], eps=eps,
                             bias=lw["bqkv"], out=self.qkv[0])
        else:
            if l == 0:
                kernels.rmsnorm(self.h, lw["in_norm"], eps, out=self.xn)
            else:
                kernels.rmsnorm(self.h_mid, lw["in_norm"], eps, delta=self.moe, sum_out=self.h, out=self.xn)
            torch.addmm(lw["bqkv"], self.xn, lw["wqkv"].t(), out=self.qkv)
        q = kernels.qk_norm_rope_kv_batched(self.qkv, self.Hq, self.Hk, self.D, None, None, eps, self.cos, self.sin, self.pos,
                                            self.kc[l], self.vc[l], q_out=self.q)
        window = c.window if c.layer_types[l] == "sliding_attention" else 0
        kernels.gqa_decode_attn_batched(q, self.Hq, self.Hk, self.D, self.kc[l], self.vc[l], self.pos, self.scale, window=window,
                                        sinks=lw["sinks"], workspace=self.attn_ws, out=self.att)
        if B == 1:
            kernels.gemv(lw["wo"], self.att.view(-1), bias=lw["bo"], res=self.h[0], out=self.h_mid[0])
        else:
            torch.addmm(lw["bo"], self.att.view(B, -1), lw["wo"].t(), out=self.tmp)
            torch.add(self.h, self.tmp, out=self.h_mid)
        kernels.router_rows(self.h_mid, lw["router"], self.k, "selected", norm_w=lw["post_norm"], eps=eps, bias=lw["router_b"],
                            xn_out=self.xn, base=l * self.E, meta=self.meta, experts=self.experts, row=self.rrow[l],
                            workspace=self.router_ws)
        kernels.moe_gptoss(self.w.pool, self.meta, self.experts, self.xn, self.k, self.H, self.I, c.bits, lw["gub"], lw["db"],
                           c.group, out=self.moe, workspace=self.moe_ws)

    def _step(self):
        if self.B == 1:
            kernels.embed(self.w.embed, self.tokens, out=self.h[0])
        else:
            torch.index_select(self.w.embed, 0, self.tokens, out=self.h)
        for l in range(self.L):
            self._layer(l)
        xf = kernels.rmsnorm(self.h_mid, self.w.final_norm, self.cfg.eps, delta=self.moe, sum_out=self.h, out=self.xn)
        if self.B == 1:
            kernels.gemv(self.w.lm_head, xf[0], out=self.logits[0])
            kernels.argmax(self.logits[0], workspace=self.argmax_ws, out=self.next_token[0:1])
        else:
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
        if tokens is not None:
            self.tokens.copy_(tokens)
        else:
            self.tokens.copy_(self.next_token)
        if self.use_graph:
            if self.graph is None:
                self.capture()
            self.graph.replay()
        else:
            self._step()
        self.steps += 1
        return self.logits

    @torch.no_grad()
    def prompt(self, ids):
        """Feed prompts ids [B, T] one position per step (the cache fills as in decoding)."""
        for t in range(ids.shape[1]):
            self.step(ids[:, t].contiguous())
        return self.logits
