"""GPU expert cache: one uint8 slot pool on the device, pages copied in from the pinned host store
with cudaMemcpyAsync on a side stream (drop-in for the reference ``wisp.cache.ExpertCache``).

``ensure(keys)`` makes the keys resident (CacheCore policy), issues one async copy per miss on the copy
stream after the work already queued on the compute stream (a victim slot may still be read), and makes
the compute stream wait for the copies.  ``prefetch(keys, protected)`` issues copies without waiting,
so they overlap the compute queued meanwhile.  Slot ids go to the MoE kernels through the routing meta.

``SlotTablePager`` is the other way to drive the same cache: residency lives in a device slot table
that the MoE kernels read themselves (a non-resident expert is read from the pinned host store), so a
decode step needs no host decision; the policy runs one token behind on the host and its page-ins are
published into the table by the copy stream once they have landed.
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


def plan_token(core, rows, experts, busy, admit="all"):
    """Cache policy for one decoded token whose routing is already known (``rows[l]`` = the experts
    layer l chose): per layer, in order, one clock tick and the hit / miss counts of the reference's
    per-layer ``cache.ensure`` (wisp/cache.py:87-91, wisp/cache_core.py:64-106).  A miss is admitted
    -- a slot acquired, evicting the policy's victim -- when a slot outside this layer's resident
    experts and ``busy`` (slots whose page-in is still in flight, grown by this call) can be had; with
    admit="hot" only keys whose decayed frequency reached ``core.admit_after`` (the hybrid policy's
    admit_async, wisp/cache.py:96-104).  Returns (evicted keys, [(key, slot)] page-ins)."""
    if admit not in ("all", "hot"):
        raise AssertionError(admit)
    evicted, loads = [], []
    for l, row in enumerate(rows):
        keys = [l * experts + int(e) for e in row]
        core.step()
        core.note(keys)
        core.stats["calls"] += 1
        prot, miss = set(busy), []
        for k in keys:
            s = core.lookup(k)
            if s is None:
                miss.append(k)
            else:
                prot.add(s)
        core.stats["hits"] += len(keys) - len(miss)
        core.stats["misses"] += len(miss)
        for k in miss:
            if admit == "hot" and not core.should_admit(k):
                continue
            try:
                s = core.acquire(k, prot)
            except RuntimeError:  # every candidate is in use or in flight: stays host-served for now
                continue
            prot.add(s)
            busy.add(s)
            if core.last_evicted is not None:
                evicted.append(core.last_evicted)
            loads.append((k, s))
    return evicted, loads


class SlotTablePager:
    """Device-side residency for a whole-token decode graph (no host decision between router and MoE).

    ``table`` (int32 [L*E] on the device) maps key = layer * E + expert to its slot, -1 when it is not
    resident; the MoE kernels (wisp_moe_decode_paged) read non-resident experts from the pinned host
    store.  After a token, ``apply(rows)`` runs the policy on that token's routing (``plan_token``) and:

      1. on the compute stream, after the work already queued: table[victim] = -1 for every eviction,
         so steps enqueued later read a victim from the host store;
      2. on the copy stream, after (1): one cudaMemcpyAsync per page-in (host row -> slot), then
         table[key] = slot for those keys, so a kernel sees a slot only once its bytes have landed.

    A slot being filled is never a victim (``busy`` until its copy stream event has completed), and a
    kernel that reads a table entry while it changes finds either source of the same bytes."""

    def __init__(self, cache, admit="all"):
        import torch

        self.cache, self.admit = cache, admit
        st = cache.store
        self.E, self.L = st.experts, st.layers
        self.table = torch.full((self.L * self.E,), -1, dtype=torch.int32, device=cache.device)
        if cache.core.key2slot:
            keys = torch.tensor(list(cache.core.key2slot.keys()), dtype=torch.int64)
            slots = torch.tensor(list(cache.core.key2slot.values()), dtype=torch.int32)
            self.table[keys.to(cache.device)] = slots.to(cache.device)
        self.pending = []  # (event, slots, tensors kept alive until the copy stream is past them)
        self.busy = set()

    def reap(self):
        keep = []
        for evt, slots, hold in self.pending:
            if evt.query():
                self.busy.difference_update(slots)
            else:
                keep.append((evt, slots, hold))
        self.pending = keep

    def apply(self, rows):
        """Policy + page-ins for one decoded token; rows[l] = the experts layer l routed to."""
        import torch

        self.reap()
        evicted, loads = plan_token(self.cache.core, rows, self.E, self.busy, self.admit)
        if not loads:
            return 0
        c, dev = self.cache, self.cache.device
        hold = []
        if evicted:
            ev = torch.tensor(evicted, dtype=torch.int64).pin_memory()
            evd = ev.to(dev, non_blocking=True)
            self.table.index_fill_(0, evd, -1)
            hold += [ev, evd]
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(dev))
        keys = torch.tensor([k for k, _ in loads], dtype=torch.int64).pin_memory()
        slots = torch.tensor([s for _, s in loads], dtype=torch.int32).pin_memory()
        with torch.cuda.stream(c.copy_stream):
            c.copy_stream.wait_event(ready)
            gr, hr = c.gpu_rows, c.host_rows
            for k, s in loads:
                gr[s].copy_(hr[k], non_blocking=True)
            kd, sd = keys.to(dev, non_blocking=True), slots.to(dev, non_blocking=True)
            self.table.index_copy_(0, kd, sd)
            done = torch.cuda.Event()
            done.record(c.copy_stream)
        hold += [keys, slots, kd, sd]
        self.pending.append((done, [s for _, s in loads], hold))
        c.bytes_h2d += len(loads) * c.store.nbytes
        c.n_loads += len(loads)
        return len(loads)

    def drain(self):
        """Wait for every page-in issued so far (host side)."""
        for evt, _, _ in self.pending:
            evt.synchronize()
        self.reap()
