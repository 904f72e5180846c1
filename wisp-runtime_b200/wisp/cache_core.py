"""Slot bookkeeping of the expert cache (drop-in for the reference ``wisp.cache_core``).

Keys are ints, ``layer * n_experts + expert``.  Slots [0, n_static) hold a pinned resident set (the
'static' profile-then-pin policy); slots [n_static, nslots) are managed by the dynamic policy:

  lru     evict the least recently used slot
  wsa     evict the lowest exponentially-decayed access frequency (working-set style)
  static  nothing dynamic beyond the pinned set (misses still need a dynamic slot)

Semantics follow wisp/cache_core.py (CacheCore: ensure / split / admit / preload / acquire / resized,
hit / miss / eviction statistics); no torch here, so the host logic is tested on CPU.
"""

from __future__ import annotations

from collections import defaultdict

import numpy as np


class CacheCore:
    def __init__(self, nslots, policy="lru", decay=0.9995, n_static=0, admit_after=2.0):
        if policy not in ("lru", "wsa", "static"):
            raise AssertionError(policy)
        if not 0 <= n_static <= nslots:
            raise AssertionError("n_static must be within [0, nslots]")
        self.nslots, self.policy, self.decay = int(nslots), policy, float(decay)
        self.n_static, self.admit_after = int(n_static), float(admit_after)
        self.slot_key = np.full(self.nslots, -1, dtype=np.int64)
        self.last = np.zeros(self.nslots)  # tick of the last use (lru)
        self.score = np.zeros(self.nslots)  # decayed frequency at the last use (wsa)
        self.key2slot = {}
        self.free = list(range(self.nslots - 1, self.n_static - 1, -1))  # pop() hands out low slots first
        self.tick, self.inc = 0, 1.0
        self.freq = defaultdict(float)
        self.stats = dict(hits=0, misses=0, evictions=0, calls=0)
        self.last_evicted = None  # key that the last acquire() evicted (None: it took a free slot)

    # ---- clock and frequency --------------------------------------------------------------------
    def step(self):
        """One routing decision: advance the clock; frequencies decay by ``decay`` per step (kept as a
        growing increment, renormalised before it overflows)."""
        self.tick += 1
        self.inc /= self.decay
        if self.inc > 1e100:
            for k in self.freq:
                self.freq[k] /= 1e100
            self.score /= 1e100
            self.inc /= 1e100

    def note(self, keys):
        for k in keys:
            self.freq[k] += self.inc
            s = self.key2slot.get(k)
            if s is not None:
                self.last[s] = self.tick
                self.score[s] = self.freq[k]

    def norm_freq(self, k):
        return self.freq.get(k, 0.0) / self.inc

    def should_admit(self, k):
        return self.norm_freq(k) >= self.admit_after

    # ---- residency ----------------------------------------------------------------------------------
    def lookup(self, k):
        return self.key2slot.get(k)

    def preload(self, keys):
        """Pin ``keys`` into the static region, in order; returns the (key, slot) copies to issue."""
        if len(keys) > self.n_static:
            raise AssertionError("more preload keys than static slots")
        out = []
        for s, k in enumerate(keys):
            self.slot_key[s] = k
            self.key2slot[k] = s
            out.append((k, s))
        return out

    def acquire(self, key, protected):
        """A slot for ``key``: a free one, else the dynamic slot the policy ranks lowest outside
        ``protected`` (slots the current request already uses)."""
        self.last_evicted = None
        if self.free:
            s = self.free.pop()
        else:
            base = self.n_static
            rank = (self.last if self.policy == "lru" else self.score)[base:].copy()
            for p in protected:
                if p >= base:
                    rank[p - base] = np.inf
            j = int(np.argmin(rank))
            if not np.isfinite(rank[j]):
                raise RuntimeError("no evictable slot: dynamic region smaller than the working request")
            s = base + j
            self.last_evicted = int(self.slot_key[s])
            del self.key2slot[self.last_evicted]
            self.stats["evictions"] += 1
        self.slot_key[s] = key
        self.key2slot[key] = s
        self.last[s] = self.tick
        self.score[s] = self.freq[key]
        return s

    # ---- policies ----------------------------------------------------------------------------------
    def ensure(self, keys):
        """Transfer policy: every key becomes resident.  Returns (slots aligned with keys, [(key, slot)]
        copies to issue for the misses)."""
        self.step()
        self.note(keys)
        self.stats["calls"] += 1
        slots, loads, prot = [None] * len(keys), [], set()
        for i, k in enumerate(keys):
            s = self.key2slot.get(k)
            if s is not None:
                slots[i] = s
                prot.add(s)
                self.stats["hits"] += 1
        for i, k in enumerate(keys):
            if slots[i] is None:
                s = self.acquire(k, prot)
                slots[i] = s
                prot.add(s)
                loads.append((k, s))
                self.stats["misses"] += 1
        return slots, loads

    def split(self, keys):
        """Hybrid policy: (hit keys, hit slots, miss keys); nothing is loaded."""
        self.step()
        self.note(keys)
        self.stats["calls"] += 1
        hk, hs, mk = [], [], []
        for k in keys:
            s = self.key2slot.get(k)
            if s is None:
                mk.append(k)
            else:
                hk.append(k)
                hs.append(s)
        self.stats["hits"] += len(hk)
        self.stats["misses"] += len(mk)
        return hk, hs, mk

    def admit(self, key, protected):
        """Bring a key computed elsewhere into the cache when it is hot enough; slot or None."""
        if key in self.key2slot or not self.should_admit(key):
            return None
        try:
            return self.acquire(key, protected)
        except RuntimeError:
            return None

    def resized(self, nslots):
        """A new core of ``nslots`` keeping the hottest resident keys (lru: most recent, wsa: highest
        score).  Returns (core, [(key, new_slot)]) -- the copies into the new pool."""
        if self.n_static:
            raise AssertionError("resize is not supported with a static region")
        nc = CacheCore(nslots, self.policy, self.decay, 0, self.admit_after)
        nc.tick, nc.inc, nc.freq, nc.stats = self.tick, self.inc, self.freq, self.stats
        resident = [s for s in range(self.nslots) if self.slot_key[s] >= 0]
        rank = self.last if self.policy == "lru" else self.score
        resident.sort(key=lambda s: -rank[s])
        loads = []
        for s in resident[:nslots]:
            k = int(self.slot_key[s])
            ns = nc.free.pop()
            nc.slot_key[ns] = k
            nc.key2slot[k] = ns
            nc.last[ns], nc.score[ns] = self.last[s], self.score[s]
            loads.append((k, ns))
        return nc, loads
