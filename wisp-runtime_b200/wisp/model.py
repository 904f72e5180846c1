"""Weights of a Qwen3-MoE-shaped decoder laid out for the bs=1 decode step.

The reference runs the HF ``Qwen3MoeForCausalLM`` modules and swaps in its paged MoE block
(wisp/model.py, wisp/moe.py); the decode step reads the same tensors (wisp/graphdec.py:155-213).  Here
they are gathered once into the layout the kernels stream:

  embed [V, H], lm_head [V, H], final_norm [H]                            bf16
  per layer: in_norm [H], wqkv [(Hq + 2 Hk) D, H] (q, k, v rows stacked), q_norm [D], k_norm [D],
             wo [H, Hq D], post_norm [H], router [E, H]                     bf16
  experts: one packed slot per (layer, expert) in ``pool`` (wisp.quant layout), slot = l * E + e
  rotary tables cos / sin [tmax, D] (bf16, the HF rotary embedding evaluated at every position)

``DecoderWeights.random`` builds seeded random-init weights (no checkpoints are needed for the
benchmark shapes); ``DecoderWeights.from_hf`` takes them from an HF model whose MoE blocks expose
per-expert gate/up/down weights.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import quant


@dataclass
class DecoderConfig:
    vocab: int = 151936
    hidden: int = 2048
    layers: int = 48
    heads: int = 32
    kv_heads: int = 4
    head_dim: int = 128
    experts: int = 128
    top_k: int = 8
    moe_inter: int = 768
    rope_theta: float = 1e6
    eps: float = 1e-6
    norm_topk: bool = True
    bits: int = 4
    group: int = 128

    @staticmethod
    def qwen3_30b_a3b(**kw):
        return DecoderConfig(**kw)


def rotary_tables(D, tmax, theta, device):
    """cos / sin [tmax, D] bf16 of the rotate-half rotary embedding (HF Qwen3: fp32, then bf16)."""
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64, device=device).float() / D))
    pos = torch.arange(tmax, device=device, dtype=torch.float32)
    f = torch.outer(pos, inv)
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(torch.bfloat16).contiguous(), emb.sin().to(torch.bfloat16).contiguous()


class DecoderWeights:
    def __init__(self, cfg: DecoderConfig):
        self.cfg = cfg
        self.layers = []

    # ------------------------------------------------------------------------------------------------
    @staticmethod
    @torch.no_grad()
    def random(cfg: DecoderConfig, device="cuda", seed=0, std=0.02, expert_std=0.02, resid_scale=False, local_experts=None,
               router_std=0.5):
        """Seeded random-init weights of the given shape; experts quantized into a resident pool.
        ``resid_scale``: the projections that write into the residual stream (attention o_proj, the
        experts' down) start at std / sqrt(2 * layers), the scaled initialisation of GPT-2-style models,
        so the stream stays dominated by the token's own embedding and routing follows the token.
        ``local_experts`` = (first, count): the pool holds only experts [first, first + count) of every
        layer, slot l * count + (e - first) (one rank's share under expert parallelism; their weights
        come from a generator seeded with ``seed`` + first)."""
        w = DecoderWeights(cfg)
        g = torch.Generator(device=device).manual_seed(seed)
        H, D, Hq, Hk, E, I, V = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.experts, cfg.moe_inter, cfg.vocab
        bf = torch.bfloat16

        def rnd(*shape, s=std):
            return (torch.randn(*shape, device=device, generator=g) * s).to(bf)

        def norm(n):
            return (1.0 + 0.1 * torch.randn(n, device=device, generator=g)).to(bf)

        w.embed = rnd(V, H, s=1.0)
        w.lm_head = rnd(V, H)
        w.final_norm = norm(H)
        for _ in range(cfg.layers):
            w.layers.append(
                dict(
                    in_norm=norm(H),
                    wqkv=rnd((Hq + 2 * Hk) * D, H),
                    q_norm=norm(D),
                    k_norm=norm(D),
                    wo=rnd(H, Hq * D, s=std / (2 * cfg.layers) ** 0.5 if resid_scale else std),
                    post_norm=norm(H),
                    router=rnd(E, H, s=router_std),
                )
            )
        n = H * I
        w.nbytes = quant.expert_nbytes(n, cfg.bits, cfg.group)
        first, count = (0, E) if local_experts is None else local_experts
        if local_experts is not None:
            g = torch.Generator(device=device).manual_seed(seed + first)
        w.pool = torch.empty((cfg.layers * count, w.nbytes), dtype=torch.uint8, device=device)
        chunk = 32
        for l in range(cfg.layers):
            for e0 in range(0, count, chunk):
                e1 = min(count, e0 + chunk)
                w3 = torch.randn(e1 - e0, 3, n, device=device, generator=g) * expert_std
                if resid_scale:
                    w3[:, 2] /= (2 * cfg.layers) ** 0.5
                w3 = w3.to(bf)
                w.pool[l * count + e0 : l * count + e1].copy_(quant.quantize_batch(w3, cfg.bits, cfg.group))
                del w3
        return w

    # ------------------------------------------------------------------------------------------------
    @staticmethod
    @torch.no_grad()
    def from_hf(model, experts, bits=4, group=128, device="cuda"):
        """Weights of an HF Qwen3-MoE causal LM.  ``experts(l)`` returns the layer's expert weights as
        three tensors gate [E, I, H], up [E, I, H], down [E, H, I]; they are quantized into the pool.
        With ``experts=None`` only the dense weights are taken (the experts live in an expert store)
        and ``pool`` is None.  The router is ``layer.mlp.gate.weight`` (an HF gate or router module,
        or the gate a PagedMoEBlock kept)."""
        hc = model.config
        cfg = DecoderConfig(
            vocab=hc.vocab_size,
            hidden=hc.hidden_size,
            layers=hc.num_hidden_layers,
            heads=hc.num_attention_heads,
            kv_heads=hc.num_key_value_heads,
            head_dim=getattr(hc, "head_dim", None) or hc.hidden_size // hc.num_attention_heads,
            experts=hc.num_experts,
            top_k=hc.num_experts_per_tok,
            moe_inter=hc.moe_intermediate_size,
            rope_theta=float(getattr(hc, "rope_theta", None) or hc.rope_parameters["rope_theta"]),
            eps=hc.rms_norm_eps,
            norm_topk=bool(hc.norm_topk_prob),
            bits=bits,
            group=group,
        )
        w = DecoderWeights(cfg)
        bf = torch.bfloat16

        def t(x):
            return x.detach().to(device=device, dtype=bf).contiguous()

        m = model.model
        w.embed = t(m.embed_tokens.weight)
        w.lm_head = t(model.lm_head.weight)
        w.final_norm = t(m.norm.weight)
        E, n = cfg.experts, cfg.hidden * cfg.moe_inter
        w.nbytes = quant.expert_nbytes(n, bits, group)
        w.pool = None if experts is None else torch.empty((cfg.layers * E, w.nbytes), dtype=torch.uint8, device=device)
        for l, layer in enumerate(m.layers):
            at = layer.self_attn
            w.layers.append(
                dict(
                    in_norm=t(layer.input_layernorm.weight),
                    wqkv=t(torch.cat([at.q_proj.weight, at.k_proj.weight, at.v_proj.weight], 0)),
                    q_norm=t(at.q_norm.weight),
                    k_norm=t(at.k_norm.weight),
                    wo=t(at.o_proj.weight),
                    post_norm=t(layer.post_attention_layernorm.weight),
                    router=t(layer.mlp.gate.weight),
                )
            )
            if experts is None:
                continue
            gate, up, down = experts(l)
            w3 = torch.stack([gate.reshape(E, n), up.reshape(E, n), down.reshape(E, n)], 1).to(device=device, dtype=torch.float32)
            w.pool[l * E : (l + 1) * E].copy_(quant.quantize_batch(w3, bits, group))
        return w
