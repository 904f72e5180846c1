"""GPU expert cache: one uint8 slot pool on the device, pages copied in from the pinned host store
with cudaMemcpyAsync on a side stream (drop-in for the reference ``wisp.cache.ExpertCache``).

``ensure(keys)`` makes the keys resident (CacheCore policy), issues the copies for the misses on the
copy stream after the work already queued on the compute stream (a victim slot may still be read),
and makes the compute stream wait for them.  ``prefetch`` and ``admit_async`` issue copies without
waiting, so they overlap the compute queued meanwhile.  Slot ids go to the MoE kernels through the
routing meta.

``SlotTablePager`` is the other way to drive the same cache: residency lives in a device slot table
that the MoE kernels read themselves (a non-resident expert is read from the pinned host store), so a
decode step needs no host decision; the policy runs one token behind on the host and its page-ins are
published into the table by the copy stream once they have landed.
"""

from __future__ import annotations

import torch

from .cache_core import CacheCore


class ExpertCache:
    """Slot pool ``gpu [nslots, slot_bytes]`` over an ``ExpertStore``.

    Copies.  A batch of (key, slot) page-ins is issued as one unit on ``copy_stream``: it first waits
    for an event recorded on the compute stream (a victim slot may still be read by queued kernels),
    then copies runs of consecutive keys that land in consecutive slots with one cudaMemcpyAsync each
    (preload and resize produce long runs; decode misses are single rows), and records ``evt``;
    ``sync_compute`` makes the compute stream wait for it.

    ``decode_on_load``: experts still cross PCIe packed, into a small device staging area, and are
    dequantized once on arrival (the bit-exact ``wisp_dequant`` kernel) into bf16 slots of 3n*2 bytes,
    so hits cost no dequant at all (the reference's arrival-time decode, wisp/cache.py:25-37, :62-71).
    """

    def __init__(self, store, nslots, device="cuda", policy="lru", decay=0.9995, n_static=0, admit_after=2.0,
                 preload_keys=None, cpu_store=None, decode_on_load=False, staging_rows=8):
        from .cache_core import CacheCore

        self.store, self.device = store, torch.device(device)
        self.decode_on_load = bool(decode_on_load) and store.bits < 16
        self.cpu_store = cpu_store
        self.core = CacheCore(nslots, policy, decay, n_static, admit_after)
        self.nslots = int(nslots)
        self.slot_bytes = 3 * store.n * 2 if self.decode_on_load else store.nbytes
        self.gpu = torch.empty((self.nslots, self.slot_bytes), dtype=torch.uint8, device=self.device)
        self.staging = (torch.empty((staging_rows, store.nbytes), dtype=torch.uint8, device=self.device)
                        if self.decode_on_load else None)
        self.copy_stream = torch.cuda.Stream(self.device)
        self.evt = None
        self.bytes_h2d = 0
        self.n_loads = 0
        self.n_copies = 0  # cudaMemcpyAsync calls issued (runs of rows)
        self._table = None
        self.timeline = None  # a list: (start event, end event, bytes) of every page-in batch on the copy stream
        if n_static:
            assert preload_keys is not None and len(preload_keys) <= n_static
            self._issue(self.core.preload(list(preload_keys)))
            self.sync_all()

    # ---- copies ------------------------------------------------------------------------------------
    @staticmethod
    def _runs(pairs):
        """Split [(key, slot)] into runs where both key and slot go up by one."""
        runs, i = [], 0
        while i < len(pairs):
            j = i + 1
            while j < len(pairs) and pairs[j][0] == pairs[j - 1][0] + 1 and pairs[j][1] == pairs[j - 1][1] + 1:
                j += 1
            runs.append((pairs[i][0], pairs[i][1], j - i))
            i = j
        return runs

    def _issue(self, pairs):
        """Queue the page-ins [(key, slot)] on the copy stream, after the compute queued so far; with a
        device table, the keys are published into it on the copy stream once their bytes have landed,
        before ``evt`` is recorded (so a slot whose event has completed is also published)."""
        if not pairs:
            return
        after = torch.cuda.Event()
        after.record(torch.cuda.current_stream(self.device))
        host = self.store.host
        with torch.cuda.stream(self.copy_stream):
            self.copy_stream.wait_event(after)
            if self.timeline is not None:
                t0 = torch.cuda.Event(enable_timing=True)
                t0.record(self.copy_stream)
            if not self.decode_on_load:
                for k0, s0, n in self._runs(pairs):
                    self.gpu[s0 : s0 + n].copy_(host[k0 : k0 + n], non_blocking=True)
                    self.n_copies += 1
            else:
                self._decode_in(pairs)
            if self._table is not None:
                keys = torch.tensor([k for k, _ in pairs], dtype=torch.int64).pin_memory()
                slots = torch.tensor([s for _, s in pairs], dtype=torch.int32).pin_memory()
                self._table.index_copy_(0, keys.to(self.device, non_blocking=True), slots.to(self.device, non_blocking=True))
            done = torch.cuda.Event(enable_timing=self.timeline is not None)
            done.record(self.copy_stream)
        if self.timeline is not None:
            self.timeline.append((t0, done, len(pairs) * self.store.nbytes))
        self.evt = done
        self.bytes_h2d += len(pairs) * self.store.nbytes
        self.n_loads += len(pairs)

    def _decode_in(self, pairs):
        """decode_on_load: packed rows through the staging area, dequantized into their bf16 slots
        (runs on the copy stream)."""
        from . import _lib

        st, R = self.store, self.staging.shape[0]
        sp = self.copy_stream.cuda_stream
        for i in range(0, len(pairs), R):
            part = pairs[i : i + R]
            for j, (k, _) in enumerate(part):
                self.staging[j].copy_(st.host[k], non_blocking=True)
                self.n_copies += 1
            for j, (_, s) in enumerate(part):
                _lib.call("wisp_dequant", self.staging[j].data_ptr(), 1, st.nbytes, None, 1, st.n, st.bits, st.group,
                          self.gpu[s].data_ptr(), sp)

    def sync_compute(self):
        """The compute stream waits for every copy issued so far."""
        if self.evt is not None:
            torch.cuda.current_stream(self.device).wait_event(self.evt)

    def sync_all(self):
        torch.cuda.synchronize(self.device)

    # ---- device residency table ---------------------------------------------------------------------
    def table(self):
        """int32 [L * E] on the device: slot of each resident key, -1 otherwise (what
        ``wisp_moe_decode_paged`` reads).  Created on first use and then kept current: page-ins are
        published by the copy stream after they land, evictions before (on the compute stream)."""
        if self._table is None:
            torch.cuda.synchronize(self.device)  # every page-in issued so far has landed: all may be published
            t = self.core.table(self.store.L * self.store.E)
            self._table = torch.from_numpy(t).to(self.device)
        return self._table

    def _unpublish(self, keys):
        """Mark ``keys`` not resident in the device table, on the compute stream (after the work queued
        so far, which may still read them from their slots)."""
        if self._table is not None and keys:
            kd = torch.tensor(keys, dtype=torch.int64).pin_memory().to(self.device, non_blocking=True)
            self._table.index_fill_(0, kd, -1)

    # ---- policies ------------------------------------------------------------------------------------
    def _acquire_all(self, keys, protected, stop_on_full):
        prot, pairs, gone = set(protected), [], []
        for k in keys:
            try:
                s = self.core.acquire(k, prot)
            except RuntimeError:
                if stop_on_full:
                    break
                continue
            if self.core.last_evicted is not None:
                gone.append(self.core.last_evicted)
            prot.add(s)
            pairs.append((k, s))
        return pairs, gone

    def ensure(self, keys):
        """Make ``keys`` resident; returns their slots (the compute stream waits for the copies)."""
        owners = self.core.owner.copy() if self._table is not None else None
        slots, loads = self.core.ensure(keys)
        if owners is not None:  # victims leave the table now; the page-ins enter it once they land
            self._unpublish([int(owners[s]) for _, s in loads if owners[s] >= 0])
        self._issue(loads)
        self.sync_compute()
        return slots

    def split(self, keys):
        """(hit keys, hit slots, miss keys); nothing is loaded (the hybrid policy)."""
        return self.core.split(keys)

    def admit_async(self, miss_keys, protected_slots):
        """Page in the misses that have become hot enough (never into ``protected_slots``); not
        waited for here -- the next ``ensure`` / ``sync_compute`` does.  Returns how many."""
        prot, pairs, gone = set(protected_slots), [], []
        for k in miss_keys:
            s = self.core.admit(k, prot)
            if s is not None:
                if self.core.last_evicted is not None:
                    gone.append(self.core.last_evicted)
                prot.add(s)
                pairs.append((k, s))
        self._unpublish(gone)
        self._issue(pairs)
        return len(pairs)

    def prefetch(self, keys, protected_slots):
        """Copy not-yet-resident keys in without waiting (never evicting ``protected_slots``); stops at
        the first key no slot can be found for.  Returns how many were issued."""
        todo = [k for k in keys if self.core.lookup(k) is None]
        pairs, gone = self._acquire_all(todo, protected_slots, stop_on_full=True)
        self._unpublish(gone)
        self._issue(pairs)
        return len(pairs)

    # ---- weights -------------------------------------------------------------------------------------
    def weights_batched(self, idx):
        """idx: int64 slots on the device -> bf16 [k, 3, n] (one gather + dequant kernel, or a view
        of bf16 slots)."""
        from . import quant

        st = self.store
        idx = torch.as_tensor(idx, device=self.device).to(torch.int64)
        if st.bits == 16 or self.decode_on_load:
            return self.gpu.index_select(0, idx).view(torch.bfloat16).view(idx.numel(), 3, st.n)
        return quant.dequant(self.gpu, st.n, st.bits, st.group, rows=idx)

    def weights(self, slots):
        """[3, n] bf16 weights per slot (views of bf16 slots, else dequantized copies)."""
        st = self.store
        if st.bits == 16 or self.decode_on_load:
            return [self.gpu[s].view(torch.bfloat16).view(3, st.n) for s in slots]
        return list(self.weights_batched(torch.as_tensor(list(slots), dtype=torch.int64)).unbind(0))

    def cpu_weights(self, key):
        """[3, n] bf16 weights of ``key`` from the host store, as a CPU tensor (dequantized by the GPU
        kernel; there is no CPU compute path)."""
        from . import quant

        st = self.cpu_store if self.cpu_store is not None else self.store
        row = st.host[key]
        if st.bits == 16:
            return row.view(torch.bfloat16).view(3, st.n)
        return quant.dequant(row.to(self.device).reshape(1, -1), st.n, st.bits, st.group)[0].cpu()

    # ---- capacity ------------------------------------------------------------------------------------
    def resize(self, nslots):
        """Grow or shrink the pool, keeping the hottest experts.  The old pool is released before the
        new one is allocated (so it fits under a tight allocator cap); kept experts are copied back
        from the host store in as few copies as their key runs allow."""
        nslots = int(nslots)
        if nslots == self.nslots:
            return
        torch.cuda.synchronize(self.device)
        self.core, loads = self.core.resized(nslots)
        self.gpu, self.evt = None, None
        torch.cuda.empty_cache()
        self.nslots = nslots
        self.gpu = torch.empty((nslots, self.slot_bytes), dtype=torch.uint8, device=self.device)
        if self._table is not None:
            self._table.fill_(-1)
        self._issue(sorted(loads, key=lambda p: p[1]))
        self.sync_all()

    def free(self):
        self.gpu = None
        self._table = None

    @property
    def stats(self):
        return self.core.stats


LFU_MARGIN = 1.25  # admit="lfu": a miss replaces a resident expert only when used this much more often


def plan_token(core, rows, experts, busy, admit="all"):
    """Cache policy for one decoded token whose routing is already known (``rows[l]`` = the experts
    layer l chose): per layer, in order, one clock tick and the hit / miss counts of the reference's
    per-layer ``cache.ensure`` (wisp/cache.py:87-91, wisp/cache_core.py:64-106).  A miss is admitted
    -- a slot acquired, evicting the policy's victim -- when a slot outside this layer's resident
    experts and ``busy`` (slots whose page-in is still in flight, grown by this call) can be had; with
    admit="hot" only keys whose decayed frequency reached ``core.admit_after`` (the hybrid policy's
    admit_async, wisp/cache.py:96-104); with admit="lfu" only keys whose decayed use frequency is
    LFU_MARGIN times that of the expert they would evict (TinyLFU-style admission: under routing with
    little reuse a page-in that is evicted before its next use only costs PCIe bandwidth, since the
    MoE kernels read a non-resident expert from host memory anyway); admit="none" never pages in (the
    residency stays what it was, a pinned working set).  Returns (evicted keys, [(key, slot)] page-ins)."""
    if admit not in ("all", "hot", "lfu", "none"):
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
            if admit == "none" or (admit == "hot" and not core.should_admit(k)):
                continue
            if admit == "lfu":
                v = core.victim(prot)
                if v is None or (v[1] >= 0 and core.norm_freq(k) <= LFU_MARGIN * core.norm_freq(v[1])):
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

    ``table`` (int32 [L*E] on the device, the cache's own table) maps key = layer * E + expert to its
    slot, -1 when it is not resident; the MoE kernels (wisp_moe_decode_paged) read non-resident experts
    from the pinned host store.  After a token, ``apply(rows)`` runs the policy on that token's routing
    (``plan_token``) and:

      1. on the compute stream, after the work already queued: table[victim] = -1 for every eviction,
         so steps enqueued later read a victim from the host store;
      2. on the copy stream, after (1): the page-ins (host rows -> slots, consecutive runs as one copy),
         then table[key] = slot for those keys, so a kernel sees a slot only once its bytes have landed.

    A slot being filled is never a victim (``busy`` until its copy stream event has completed), and a
    kernel that reads a table entry while it changes finds either source of the same bytes."""

    def __init__(self, cache, admit="all"):
        self.cache, self.admit = cache, admit
        st = cache.store
        self.E, self.L = st.E, st.L
        self.table = cache.table()
        self.pending = []  # (event, slots) of page-ins not yet known to have landed
        self.busy = set()

    def reap(self):
        keep = []
        for evt, slots in self.pending:
            if evt.query():
                self.busy.difference_update(slots)
            else:
                keep.append((evt, slots))
        self.pending = keep

    def apply(self, rows):
        """Policy + page-ins for one decoded token; rows[l] = the experts layer l routed to."""
        self.reap()
        evicted, loads = plan_token(self.cache.core, rows, self.E, self.busy, self.admit)
        if not loads:
            return 0
        self.cache._unpublish(evicted)
        self.cache._issue(loads)
        self.pending.append((self.cache.evt, [s for _, s in loads]))
        return len(loads)

    def drain(self):
        """Wait for every page-in issued so far (host side)."""
        for evt, _ in self.pending:
            evt.synchronize()
        self.reap()
