"""gpt-oss adapter (drop-in for the reference ``wisp.gptoss``, wisp/gptoss.py): MXFP4 checkpoint ->
expert store in the wisp.quant layout, and a paged MoE block whose expert math runs in
``wisp_moe_gptoss`` (this package's CUDA kernels) straight from the packed slots.

An expert is gate_up [H, 2I] (gate/up interleaved on the last axis) and down [I, H] plus two biases;
with I == H it is stored as the flat [3, n] stream ``[gate_up.flat[:n] | gate_up.flat[n:] | down.flat]``
(``expert_w3``), so the quantization groups run along the output axis.  The biases stay on the GPU for
every expert.  Routing is the gpt-oss one: top-k of the router logits, then softmax over those k.
"""

from __future__ import annotations

import json
import os
import time

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import kernels
from .store import ExpertStore

# the 16 values of an fp4 (e2m1) code, low code first: the MXFP4 element format
FP4_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


def mxfp4_to_bf16(blocks, scales):
    """blocks uint8 [..., G, 16] (two fp4 codes per byte, low nibble first) and scales uint8 [..., G]
    (power-of-two exponents, bias 127) -> bf16 [..., G * 32].  Reference: wisp/gptoss.py:22-29."""
    table = torch.tensor(FP4_VALUES, dtype=torch.float32, device=blocks.device)
    b = blocks.to(torch.int64)
    v = torch.stack([table[b & 0xF], table[b >> 4]], -1).reshape(*blocks.shape[:-1], 32)
    v = torch.ldexp(v, (scales.to(torch.int32) - 127).unsqueeze(-1).to(torch.float32))
    return v.reshape(*blocks.shape[:-2], -1).to(torch.bfloat16)


def expert_w3(gate_up, down):
    """gate_up [H, 2I], down [I, H] -> [3, n] (n = H * I).  Reference: wisp/gptoss.py:32-37."""
    H, I2 = gate_up.shape
    n = H * (I2 // 2)
    f = gate_up.reshape(-1)
    return torch.stack([f[:n], f[n:], down.reshape(-1)])


def _reader(model_dir):
    from safetensors import safe_open

    index = json.load(open(os.path.join(model_dir, "model.safetensors.index.json")))["weight_map"]
    files = {}

    def get(name):
        f = index[name]
        if f not in files:
            files[f] = safe_open(os.path.join(model_dir, f), framework="pt", device="cpu")
        return files[f].get_tensor(name)

    return get, (lambda name: name in index), index


def _layer_experts(get, has, l, device):
    """Dequantized gate_up [E, H, 2I] and down [E, I, H] of one layer (MXFP4 or plain bf16 checkpoints)."""
    p = f"model.layers.{l}.mlp.experts."
    if has(p + "gate_up_proj_blocks"):
        gu = mxfp4_to_bf16(get(p + "gate_up_proj_blocks").to(device), get(p + "gate_up_proj_scales").to(device))
        dn = mxfp4_to_bf16(get(p + "down_proj_blocks").to(device), get(p + "down_proj_scales").to(device))
        return gu.transpose(1, 2).contiguous(), dn.transpose(1, 2).contiguous()  # [E, out, K] -> [E, K, out]
    return get(p + "gate_up_proj").to(device), get(p + "down_proj").to(device)


def build_store(model_dir, cfg, bits, group=128, device="cuda", cache_dir=None, pin=True):
    """Every expert of a gpt-oss checkpoint quantized into an ExpertStore (a layer per quantizer launch);
    with ``cache_dir`` the packed store is loaded from / saved to ``store_gptoss_b{bits}_g{group}_...u8``."""
    L, E, H, I = cfg.num_hidden_layers, cfg.num_local_experts, cfg.hidden_size, cfg.intermediate_size
    assert H == I, "the [3, n] expert layout needs intermediate_size == hidden_size (true for gpt-oss)"
    st = ExpertStore(L, E, H * I, bits, group, pin)
    path = None
    if cache_dir and bits < 16:
        os.makedirs(cache_dir, exist_ok=True)
        path = st.cache_path(cache_dir, prefix="store_gptoss")
        if os.path.exists(path) and os.path.getsize(path) == st.host.numel():
            st._load(path)
            return st
    get, has, _ = _reader(model_dir)
    t0 = time.time()
    for l in range(L):
        gu, dn = _layer_experts(get, has, l, device)
        st.put_layer(l, torch.stack([expert_w3(gu[e], dn[e]) for e in range(E)]), device)
        del gu, dn
        if l % 4 == 3 or l == L - 1:
            print(f"[store] gpt-oss bits={bits} layer {l + 1}/{L}  {time.time() - t0:.0f}s", flush=True)
    if path:
        st._save(path)
    return st


class PagedGptOssBlock(nn.Module):
    """Drop-in for HF ``GptOssMLP``: the router stays resident, experts are paged through the cache and
    computed by ``wisp_moe_gptoss`` (clamped SwiGLU with alpha 1.702, ``(up + 1)``, both biases, the
    weighted sum).  Returns (output, router scores) like HF.  Reference: wisp/gptoss.py:93-143."""

    def __init__(self, router, layer_idx, rt, cfg, device="cuda"):
        super().__init__()
        self.router, self.layer_idx, self.rt = router, layer_idx, rt
        self.E, self.top_k = cfg.num_local_experts, cfg.num_experts_per_tok
        self.H, self.I = cfg.hidden_size, cfg.intermediate_size
        self.alpha, self.limit = 1.702, float(getattr(cfg, "swiglu_limit", 7.0))
        self.register_buffer("gub", torch.zeros(self.E, 2 * self.I, dtype=torch.bfloat16, device=device), persistent=False)
        self.register_buffer("db", torch.zeros(self.E, self.H, dtype=torch.bfloat16, device=device), persistent=False)
        self._ws = {}

    def _workspace(self, N, dev):
        ws = self._ws.get((N, dev))
        if ws is None:
            from . import _lib

            nb = _lib.lib().wisp_moe_gptoss_workspace_bytes(N, self.top_k, self.H, self.I)
            if nb < 0:
                raise kernels.WispError("moe_gptoss: N * k must be in [1, 2048]")
            ws = self._ws[(N, dev)] = torch.empty(nb, dtype=torch.uint8, device=dev)
        return ws

    def forward(self, hidden_states):
        rt, cache = self.rt, self.rt.cache
        B, T, H = hidden_states.shape
        x = hidden_states.reshape(-1, H)
        N, k = x.shape[0], self.top_k
        logits = F.linear(x, self.router.weight, self.router.bias)
        tv, ti = torch.topk(logits, k, dim=-1)
        sc = F.softmax(tv, dim=1, dtype=tv.dtype)
        base = self.layer_idx * self.E
        rt.stats["layer_calls"] += 1
        row = torch.cat([ti.float(), sc.float()], 1).cpu()  # the one device-to-host read of this call
        ti_c, sc_c = row[:, :k].to(torch.int64), row[:, k:]
        if rt.recorder is not None:
            rt.recorder.append((self.layer_idx, ti_c.numpy().copy()))
        uniq = torch.unique(ti_c).tolist()
        experts = ti.to(torch.int32).contiguous()
        y = torch.zeros_like(x)
        st = cache.store
        step = max(1, 2048 // k)
        for i in range(0, len(uniq), rt.chunk):
            ce = uniq[i : i + rt.chunk]
            slot_of = dict(zip(ce, cache.ensure([base + e for e in ce])))
            meta = torch.empty((N, 2 * k), dtype=torch.float32)
            for t in range(N):
                for j in range(k):
                    s = slot_of.get(int(ti_c[t, j]))
                    meta[t, j], meta[t, k + j] = (-1.0, 0.0) if s is None else (float(s), float(sc_c[t, j]))
            meta = meta.pin_memory().to(x.device, non_blocking=True)
            for t0 in range(0, N, step):
                t1 = min(N, t0 + step)
                y[t0:t1].add_(kernels.moe_gptoss(cache.gpu, meta[t0:t1].contiguous(), experts[t0:t1].contiguous(),
                                                 x[t0:t1].contiguous(), k, H, self.I, st.bits, self.gub, self.db, st.group,
                                                 workspace=self._workspace(t1 - t0, x.device)))
            rt.stats["gpu_experts"] += len(ce)
        return y.view(B, T, H), sc


def load_skeleton_gptoss(model_dir, rt, device="cuda"):
    """Meta-initialised HF gpt-oss with every MLP swapped for a PagedGptOssBlock, all non-expert tensors
    and the expert biases loaded.  Reference: wisp/gptoss.py:146-183."""
    from safetensors import safe_open
    from transformers import AutoConfig, AutoModelForCausalLM

    cfg = AutoConfig.from_pretrained(model_dir)
    with torch.device("meta"):
        model = AutoModelForCausalLM.from_config(cfg, torch_dtype=torch.bfloat16)
    blocks = []
    for i, layer in enumerate(model.model.layers):
        blk = PagedGptOssBlock(layer.mlp.router, i, rt, cfg, device)
        layer.mlp = blk
        blocks.append(blk)
    get, _, index = _reader(model_dir)
    wanted = {k: f for k, f in index.items() if ".mlp.experts." not in k}
    sd = {}
    for f in sorted(set(wanted.values())):
        with safe_open(os.path.join(model_dir, f), framework="pt", device=device) as h:
            for k in h.keys():
                if k in wanted:
                    sd[k] = h.get_tensor(k)
    res = model.load_state_dict(sd, strict=False, assign=True)
    bad = [k for k in res.missing_keys if "rotary" not in k]
    assert not bad, f"missing keys: {bad[:5]}"
    for l, blk in enumerate(blocks):
        p = f"model.layers.{l}.mlp.experts."
        blk.gub.copy_(get(p + "gate_up_proj_bias").to(device))
        blk.db.copy_(get(p + "down_proj_bias").to(device))
    model.model.rotary_emb = type(model.model.rotary_emb)(config=cfg, device=device)
    model.eval()
    return model, cfg
