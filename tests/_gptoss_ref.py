"""fp32 restatement of HF GptOssForCausalLM decoding one token per step with a KV cache (eager
attention: scores over the window plus a per-head sink logit in the softmax, the sink dropped; top-k
router with softmax over the chosen logits; clamped SwiGLU experts with biases).  The weights are a dict
of fp32 tensors in HF's shapes.  ``step(..., force=(experts, weights))`` takes the experts and their weights from a decoder instead of
its own top-k and softmax: a decoder's router logits are bf16, and at the logit magnitudes of a router
the bf16 step already moves the softmax weights by percents, which would mask every other difference.
Pinned against transformers' own GptOssForCausalLM in tests/test_gptoss_decoder_cpu.py."""

import torch


def rmsnorm(x, w, eps):
    return w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))


def rotate(x, cos, sin):
    """gpt-oss rotary on the two halves of a head: x1 c - x2 s, x2 c + x1 s (cos/sin half-width)."""
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1)


class RefGptOss:
    def __init__(self, p, cfg, cos, sin, batch, tmax):
        """p: embed [V, H], lm_head [V, H], final_norm [H], layers[l]: in_norm, wq [Hq D, H], bq, wk, bk, wv,
        bv, wo [H, Hq D], bo, sinks [Hq], post_norm, router [E, H], router_b [E], gate_up [E, H, 2I], gub [E, 2I],
        down [E, I, H], db [E, H].  cos / sin: half-width tables [tmax, D/2] (with the YaRN attention factor)."""
        self.p, self.c, self.cos, self.sin = p, cfg, cos, sin
        L, Hk, D = cfg.layers, cfg.kv_heads, cfg.head_dim
        self.kc = torch.zeros(L, batch, Hk, tmax, D)
        self.vc = torch.zeros(L, batch, Hk, tmax, D)

    def _attn(self, l, x, pos):
        c, lw = self.c, self.p["layers"][l]
        B = x.shape[0]
        Hq, Hk, D = c.heads, c.kv_heads, c.head_dim
        q = (x @ lw["wq"].T + lw["bq"]).view(B, Hq, D)
        k = (x @ lw["wk"].T + lw["bk"]).view(B, Hk, D)
        v = (x @ lw["wv"].T + lw["bv"]).view(B, Hk, D)
        out = torch.zeros(B, Hq, D)
        window = c.window if c.layer_types[l] == "sliding_attention" else 0
        for b in range(B):
            p = int(pos[b])
            qb = rotate(q[b], self.cos[p], self.sin[p])
            self.kc[l, b, :, p] = rotate(k[b], self.cos[p], self.sin[p])
            self.vc[l, b, :, p] = v[b]
            lo = max(0, p - window + 1) if window else 0
            for h in range(Hq):
                kv = h // (Hq // Hk)
                s = self.kc[l, b, kv, lo : p + 1] @ qb[h] * D ** -0.5
                s = torch.cat([s, lw["sinks"][h : h + 1]])
                pr = torch.softmax(s - s.max(), 0)[:-1]
                out[b, h] = pr @ self.vc[l, b, kv, lo : p + 1]
        return out.view(B, -1) @ lw["wo"].T + lw["bo"]

    def _moe(self, l, x, force=None):
        c, lw = self.c, self.p["layers"][l]
        logits = x @ lw["router"].T + lw["router_b"]
        tv, own = torch.topk(logits, c.top_k, dim=-1)
        own_w = torch.softmax(tv, -1)
        ti, w = (own, own_w) if force is None else (force[0].to(torch.int64), force[1].float())
        y = torch.zeros_like(x)
        for t in range(x.shape[0]):
            for j in range(c.top_k):
                e = int(ti[t, j])
                gu = x[t] @ lw["gate_up"][e] + lw["gub"][e]
                gate = gu[0::2].clamp(max=7.0)
                up = gu[1::2].clamp(-7.0, 7.0)
                act = (up + 1) * gate * torch.sigmoid(gate * 1.702)
                y[t] += w[t, j] * (act @ lw["down"][e] + lw["db"][e])
        return y, own, own_w

    @torch.no_grad()
    def step(self, tokens, pos, force=None):
        """tokens [B], pos [B] -> (logits [B, V], routes [L, B, k], weights [L, B, k]); the routes and weights
        are the reference's own top-k and softmax at each layer, also when ``force`` replaced them."""
        c, p = self.c, self.p
        h = p["embed"][tokens]
        routes, weights = [], []
        for l in range(c.layers):
            lw = p["layers"][l]
            h = h + self._attn(l, rmsnorm(h, lw["in_norm"], c.eps), pos)
            y, ti, w = self._moe(l, rmsnorm(h, lw["post_norm"], c.eps), None if force is None else (force[0][l], force[1][l]))
            routes.append(ti)
            weights.append(w)
            h = h + y
        return rmsnorm(h, p["final_norm"], c.eps) @ p["lm_head"].T, torch.stack(routes), torch.stack(weights)
