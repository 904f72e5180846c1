"""Host-side store of every expert in the packed wisp.quant layout (drop-in for the reference
``wisp.store.ExpertStore``, wisp/store.py).

One pinned uint8 tensor ``host [L * E, nbytes]``, row ``key = layer * E + expert``: a page-in is one
cudaMemcpyAsync of a row, and the MoE kernels can read a row in place (the pinned tensor is mapped
into the device address space).  Experts are quantized on the GPU by the CUDA quantizer
(``wisp.quant.quantize_batch``, byte-identical to the reference's ``quantize``), a whole layer per
launch.  The on-disk cache ``store_b{bits}_g{group}_{L}x{E}x{n}.u8`` is the raw ``host`` array, the
reference's file format (wisp/store.py:54-110), written to ``.tmp`` and renamed into place.
"""

from __future__ import annotations

import json
import os
import time

import torch

from . import quant


def _host_buffer(rows, nbytes, pin):
    """uint8 [rows, nbytes] in pinned memory when possible (pageable if pinning is refused)."""
    if pin:
        try:
            return torch.empty((rows, nbytes), dtype=torch.uint8, pin_memory=True), True
        except RuntimeError as e:  # a container can refuse page-locked memory
            print(f"[store] pin_memory failed ({e}); using pageable memory", flush=True)
    return torch.empty((rows, nbytes), dtype=torch.uint8), False


class ExpertStore:
    def __init__(self, n_layers, n_experts, n, bits, group=128, pin=True):
        self.L, self.E, self.n, self.bits, self.group = int(n_layers), int(n_experts), int(n), int(bits), int(group)
        self.nbytes = quant.expert_nbytes(self.n, self.bits, self.group)
        t0 = time.time()
        self.host, self.pinned = _host_buffer(self.L * self.E, self.nbytes, pin)
        print(f"[store] {self.host.numel() / 2**30:.2f} GiB host (pinned={self.pinned}) in {time.time() - t0:.1f}s",
              flush=True)

    # the names the rest of this package uses
    @property
    def layers(self):
        return self.L

    @property
    def experts(self):
        return self.E

    @property
    def total_gib(self):
        return self.host.numel() / 2**30

    def key(self, l, e):
        return l * self.E + e

    # ---- filling ---------------------------------------------------------------------------------
    @torch.no_grad()
    def put(self, l, e, w3, device="cuda"):
        """Quantize one expert (w3: [3, n] = gate | up | down flattened) into row (l, e)."""
        self.put_layer(l, w3.reshape(1, 3, self.n), device, first=e)

    @torch.no_grad()
    def put_layer(self, l, w3s, device="cuda", first=0):
        """Quantize experts [B, 3, n] of layer l (experts first .. first+B-1) in one launch."""
        B = w3s.shape[0]
        assert w3s.numel() == B * 3 * self.n and first + B <= self.E
        buf = quant.quantize_batch(w3s.to(device), self.bits, self.group)
        r0 = l * self.E + first
        self.host[r0 : r0 + B].copy_(buf, non_blocking=False)

    # ---- builders ----------------------------------------------------------------------------------
    @classmethod
    def from_experts(cls, layers, bits, group=128, device="cuda", pin=True):
        """layers: per layer a list of (gate [I, H], up [I, H], down [H, I]) tensors."""
        L, E = len(layers), len(layers[0])
        n = layers[0][0][0].numel()
        st = cls(L, E, n, bits, group, pin)
        for l, exps in enumerate(layers):
            w3s = torch.stack([torch.stack([g.reshape(-1), u.reshape(-1), d.reshape(-1)]) for g, u, d in exps])
            st.put_layer(l, w3s, device)
        return st

    @classmethod
    def from_pool(cls, pool, n, bits, group, layers, experts, pin=True):
        """Host copy of an already packed pool (device or host) whose row l*E + e is expert e of layer l."""
        st = cls.__new__(cls)
        st.L, st.E, st.n, st.bits, st.group = int(layers), int(experts), int(n), int(bits), int(group)
        st.nbytes = quant.expert_nbytes(st.n, st.bits, st.group)
        assert tuple(pool.shape) == (st.L * st.E, st.nbytes), (tuple(pool.shape), st.L * st.E, st.nbytes)
        st.host, st.pinned = _host_buffer(st.L * st.E, st.nbytes, pin)
        st.host.copy_(pool)
        return st

    def cache_path(self, cache_dir, prefix="store"):
        return os.path.join(cache_dir, f"{prefix}_b{self.bits}_g{self.group}_{self.L}x{self.E}x{self.n}.u8")

    @classmethod
    def from_safetensors(cls, model_dir, cfg, bits, group=128, device="cuda", cache_dir=None, pin=True):
        """Every expert of an HF Qwen3-MoE checkpoint (``model.layers.{l}.mlp.experts.{e}.{gate,up,down}_proj``),
        quantized a layer at a time; with ``cache_dir`` the packed store is loaded from / saved to its .u8 file."""
        from safetensors import safe_open

        L, E = cfg.num_hidden_layers, cfg.num_experts
        n = cfg.moe_intermediate_size * cfg.hidden_size
        st = cls(L, E, n, bits, group, pin)
        path = None
        if cache_dir and bits < 16:
            os.makedirs(cache_dir, exist_ok=True)
            path = st.cache_path(cache_dir)
            if os.path.exists(path) and os.path.getsize(path) == st.host.numel():
                st._load(path)
                return st
        index = json.load(open(os.path.join(model_dir, "model.safetensors.index.json")))["weight_map"]
        files = {}

        def tensor(name):
            f = index[name]
            if f not in files:
                files[f] = safe_open(os.path.join(model_dir, f), framework="pt", device="cpu")
            return files[f].get_tensor(name)

        t0 = time.time()
        for l in range(L):
            w3s = torch.empty((E, 3, n), dtype=torch.bfloat16)
            for e in range(E):
                p = f"model.layers.{l}.mlp.experts.{e}."
                for j, m in enumerate(("gate_proj", "up_proj", "down_proj")):
                    w3s[e, j].copy_(tensor(p + m + ".weight").reshape(-1))
            st.put_layer(l, w3s, device)
            if l % 4 == 3 or l == L - 1:
                print(f"[store] bits={bits} layer {l + 1}/{L}  {time.time() - t0:.0f}s", flush=True)
        if path:
            st._save(path)
        return st

    # ---- persistence: the raw host array -------------------------------------------------------------
    def _save(self, path, rows=256):
        a = self.host.numpy()
        tmp = path + ".tmp"
        with open(tmp, "wb") as f:
            for i in range(0, a.shape[0], rows):
                f.write(memoryview(a[i : i + rows]))
        os.replace(tmp, path)  # a reader never sees a half-written file under the final name

    def _load(self, path, rows=256):
        a = self.host.numpy()
        if os.path.getsize(path) != a.nbytes:
            raise ValueError(f"{path}: {os.path.getsize(path)} bytes, the store holds {a.nbytes}")
        with open(path, "rb") as f:
            for i in range(0, a.shape[0], rows):
                f.readinto(memoryview(a[i : i + rows]))

    @classmethod
    def load(cls, path, n_layers, n_experts, n, bits, group=128, pin=True):
        """A store read back from its .u8 file."""
        st = cls(n_layers, n_experts, n, bits, group, pin)
        st._load(path)
        return st
