"""GPU expert cache: one uint8 slot pool on the device, pages copied in from the pinned host store
with cudaMemcpyAsync on a side stream (drop-in for the reference ``wisp.cache.ExpertCache``).

``ensure(keys)`` makes the keys resident (CacheCore policy), issues one async copy per miss on the copy
stream after the work already queued on the compute stream (a victim slot may still be read), and makes
the compute stream wait for the copies.  ``prefetch(keys, protected)`` issues copies without waiting,
so they overlap the compute queued meanwhile.  Slot ids go to the MoE kernels through the routing meta.
"""

from __future__ import annotations

import torch

from .cache_core import CacheCore


class ExpertCache:
    def __init__(self, store, nslots, device="cuda", policy="lru", decay=0.9995, n_static=0, admit_after=2.0,
                 preload_keys=None):
        self.store, self.device = store, torch.device(device)
        self.core = CacheCore(nslots, policy, decay, n_static, admit_after)
        self.nslots = nslots
        self.gpu = torch.empty((nslots, store.nbytes), dtype=torch.uint8, device=self.device)
        self.gpu_rows = self.gpu.unbind(0)  # pre-built views: no indexing work per copy
        self.host_rows = store.host.unbind(0)
        self.copy_stream = torch.cuda.Stream(self.device)
        self.evt = None
        self.bytes_h2d = 0
        self.n_loads = 0
        if n_static:
            assert preload_keys is not None and len(preload_keys) <= n_static
            self._issue(self.core.preload(list(preload_keys)))
            torch.cuda.synchronize(self.device)

    def _issue(self, pairs):
        """Async host -> device copies of [(key, slot)] on the copy stream, after the queued compute."""
        if not pairs:
            return
        e = torch.cuda.Event()
        e.record(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.copy_stream):
            self.copy_stream.wait_event(e)
            gr, hr = self.gpu_rows, self.host_rows
            for k, s in pairs:
                gr[s].copy_(hr[k], non_blocking=True)
        done = torch.cuda.Event()
        done.record(self.copy_stream)
        self.evt = done
        self.bytes_h2d += len(pairs) * self.store.nbytes
        self.n_loads += len(pairs)

    def sync_compute(self):
        """The compute stream waits for every copy issued so far."""
        if self.evt is not None:
            torch.cuda.current_stream(self.device).wait_event(self.evt)

    def ensure(self, keys):
        slots, loads = self.core.ensure(keys)
        self._issue(loads)
        self.sync_compute()
        return slots

    def prefetch(self, keys, protected_slots):
        """Copy not-yet-resident keys in without waiting (never evicting ``protected_slots``)."""
        prot, pairs = set(protected_slots), []
        for k in keys:
            if self.core.lookup(k) is not None:
                continue
            try:
                s = self.core.acquire(k, prot)
            except RuntimeError:
                break
            prot.add(s)
            pairs.append((k, s))
        self._issue(pairs)
        return len(pairs)

    @property
    def stats(self):
        return self.core.stats
