"""Host-side store of packed experts (the reference ``wisp.store`` keeps every layer's experts in host
RAM in the wisp.quant layout and the cache pages them into GPU slots).  Here: one pinned uint8 tensor
[L * E, nbytes], key = layer * E + expert, so a page-in is a single cudaMemcpyAsync per expert."""

from __future__ import annotations

import torch

from . import quant


class ExpertStore:
    def __init__(self, host, n, bits, group, layers, experts):
        self.host = host  # pinned uint8 [layers * experts, nbytes]
        self.n, self.bits, self.group = n, bits, group
        self.layers, self.experts = layers, experts
        self.nbytes = host.shape[1]
        assert self.nbytes == quant.expert_nbytes(n, bits, group)

    @staticmethod
    def from_pool(pool, n, bits, group, layers, experts):
        """Pinned host copy of a device (or host) pool whose row l*E + e is expert e of layer l."""
        host = torch.empty(pool.shape, dtype=torch.uint8, pin_memory=True)
        host.copy_(pool)
        return ExpertStore(host, n, bits, group, layers, experts)
