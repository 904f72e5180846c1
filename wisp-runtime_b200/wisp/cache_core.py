"""Slot bookkeeping of the expert cache (drop-in for the reference ``wisp.cache_core.CacheCore``).

Keys are ints, ``layer * n_experts + expert``.  Slots [0, n_static) hold a pinned resident set (the
'static' profile-then-pin policy); slots [n_static, nslots) are managed by the dynamic policy:

  lru     evict the slot used longest ago
  wsa     evict the slot whose key has the lowest exponentially decayed use frequency
  static  nothing dynamic beyond the pinned set (misses still take a dynamic slot)

The structure is the host half of the device slot table that the MoE kernels read
(``wisp_moe_decode_paged``): residency is a dense int array over the key space, ``slot_of[key]`` =
slot or -1, exactly the layout of the int32 table on the GPU (``table()`` hands it over), plus its
inverse ``owner[slot]``.  Around it:

  - ``rank[slot]``: the eviction order of the policy -- the clock tick of the slot's last use (lru) or
    its key's decayed frequency at that use (wsa, static); the eviction victim is the lowest rank
    outside the protected slots, ties going to the lower slot.
  - ``heat[key]``: decayed use frequency.  Decay is lazy: a use adds the current ``unit`` and every
    clock step multiplies ``unit`` by 1/decay, so older uses weigh decay^age relative to new ones
    without touching every key per step; before ``unit`` overflows, every heat value and ``unit`` are
    divided by 1e100 together (ratios, hence decisions, are unchanged).
  - ``fill``: slots [fill, nslots) have never been used; a miss takes the lowest of them before any
    eviction (slots only become free again through ``resized``).

Decisions -- which slot a key gets, what is evicted, hit/miss/eviction counts -- are those of the
reference policy (wisp/cache_core.py:15-149); ``tests/test_cache_core.py`` replays operation traces
recorded from the reference against this class.  No torch here: the host logic runs on CPU.
"""

from __future__ import annotations

import numpy as np

_RENORM = 1e100


class CacheCore:
    def __init__(self, nslots, policy="lru", decay=0.9995, n_static=0, admit_after=2.0):
        if policy not in ("lru", "wsa", "static"):
            raise AssertionError(policy)
        if not 0 <= n_static <= nslots:
            raise AssertionError("n_static must be within [0, nslots]")
        self.nslots, self.policy, self.decay = int(nslots), policy, float(decay)
        self.n_static, self.admit_after = int(n_static), float(admit_after)
        self.owner = np.full(self.nslots, -1, dtype=np.int64)  # key held by each slot, -1 = empty
        self.rank = np.zeros(self.nslots)  # eviction rank of each slot (see module docstring)
        self.slot_of = np.full(0, -1, dtype=np.int64)  # key -> slot (-1: not resident), grown on demand
        self.heat = np.zeros(0)  # key -> decayed use frequency, in units of `unit`
        self.fill = self.n_static  # first never-used dynamic slot
        self.tick, self.unit = 0, 1.0
        self.stats = dict(hits=0, misses=0, evictions=0, calls=0)
        self.last_evicted = None  # key the last acquire() evicted (None: it took a never-used slot)

    # ---- key space ----------------------------------------------------------------------------------
    def _grow(self, top):
        """Make key `top` addressable."""
        if top < self.slot_of.size:
            return
        n = max(top + 1, 2 * self.slot_of.size, 64)
        so = np.full(n, -1, dtype=np.int64)
        so[: self.slot_of.size] = self.slot_of
        he = np.zeros(n)
        he[: self.heat.size] = self.heat
        self.slot_of, self.heat = so, he

    def _keys(self, keys):
        ks = np.asarray(keys, dtype=np.int64).reshape(-1)
        if ks.size:
            if ks.min() < 0:
                raise AssertionError("keys must be non-negative")
            self._grow(int(ks.max()))
        return ks

    def _use_rank(self, key):
        return float(self.tick) if self.policy == "lru" else float(self.heat[key])

    # ---- clock and frequency ------------------------------------------------------------------------
    def step(self):
        """One routing decision: advance the clock (frequencies age by one decay factor)."""
        self.tick += 1
        self.unit /= self.decay
        if self.unit > _RENORM:
            self.heat /= _RENORM
            if self.policy != "lru":
                self.rank /= _RENORM
            self.unit /= _RENORM

    def note(self, keys):
        """Record one use of each key (a key listed twice counts twice); resident keys' slots move up
        in the eviction order."""
        ks = self._keys(keys)
        if not ks.size:
            return
        np.add.at(self.heat, ks, self.unit)
        s = self.slot_of[ks]
        live = s >= 0
        if live.any():
            if self.policy == "lru":
                self.rank[s[live]] = float(self.tick)
            else:
                self.rank[s[live]] = self.heat[ks[live]]

    def norm_freq(self, k):
        return float(self.heat[k]) / self.unit if 0 <= k < self.heat.size else 0.0

    def should_admit(self, k):
        return self.norm_freq(k) >= self.admit_after

    # ---- residency -----------------------------------------------------------------------------------
    def lookup(self, k):
        if 0 <= k < self.slot_of.size:
            s = int(self.slot_of[k])
            return s if s >= 0 else None
        return None

    @property
    def key2slot(self):
        """Resident keys as a {key: slot} dict (a snapshot)."""
        ks = np.flatnonzero(self.slot_of >= 0)
        return {int(k): int(self.slot_of[k]) for k in ks}

    @property
    def free(self):
        """Never-used slots, in the order a list's pop() would hand them out (the last one first)."""
        return list(range(self.nslots - 1, self.fill - 1, -1))

    def table(self, size=None):
        """The residency table key -> slot (-1: not resident) as int32, ``size`` keys long (the layout
        of the device slot table)."""
        n = self.slot_of.size if size is None else int(size)
        t = np.full(n, -1, dtype=np.int32)
        m = min(n, self.slot_of.size)
        t[:m] = self.slot_of[:m]
        return t

    def _place(self, key, s):
        self.owner[s] = key
        self.slot_of[key] = s
        self.rank[s] = self._use_rank(key)

    def preload(self, keys):
        """Pin ``keys`` into the static region, in order; returns the (key, slot) copies to issue."""
        if len(keys) > self.n_static:
            raise AssertionError("more preload keys than static slots")
        self._keys(keys)
        out = []
        for s, k in enumerate(keys):
            k = int(k)
            self.owner[s] = k
            self.slot_of[k] = s
            out.append((k, s))
        return out

    def victim(self, protected):
        """The slot ``acquire`` would take next and the key it would evict from it: (slot, -1) while
        never-used slots remain, None when every dynamic slot is protected."""
        if self.fill < self.nslots:
            return self.fill, -1
        lo = self.n_static
        cand = self.rank[lo:].copy()
        p = np.fromiter((q - lo for q in protected if lo <= q < self.nslots), dtype=np.int64)
        cand[p] = np.inf
        if not cand.size:
            return None
        j = int(np.argmin(cand))
        if not np.isfinite(cand[j]):
            return None
        return lo + j, int(self.owner[lo + j])

    def acquire(self, key, protected):
        """A slot for ``key``: the lowest never-used slot, else the dynamic slot ranked lowest by the
        policy outside ``protected`` (slots the current request already uses)."""
        key = int(key)
        self._grow(key)
        self.last_evicted = None
        if self.fill < self.nslots:
            s = self.fill
            self.fill += 1
        else:
            lo = self.n_static
            cand = self.rank[lo:].copy()
            p = np.fromiter((q - lo for q in protected if lo <= q < self.nslots), dtype=np.int64)
            cand[p] = np.inf
            j = int(np.argmin(cand)) if cand.size else 0
            if not cand.size or not np.isfinite(cand[j]):
                raise RuntimeError("no evictable slot: dynamic region smaller than the working request")
            s = lo + j
            victim = int(self.owner[s])
            self.slot_of[victim] = -1
            self.last_evicted = victim
            self.stats["evictions"] += 1
        self._place(key, s)
        return s

    # ---- policies ------------------------------------------------------------------------------------
    def ensure(self, keys):
        """Transfer policy: every key becomes resident.  Returns (slots aligned with keys, [(key, slot)]
        copies to issue for the misses)."""
        self.step()
        self.note(keys)
        self.stats["calls"] += 1
        ks = self._keys(keys)
        got = self.slot_of[ks].copy()
        hit = got >= 0
        self.stats["hits"] += int(hit.sum())
        busy = set(int(s) for s in got[hit])
        loads = []
        for i in np.flatnonzero(~hit):
            k = int(ks[i])
            s = self.lookup(k)  # a key listed twice: the first listing made it resident
            if s is None:
                s = self.acquire(k, busy)
                loads.append((k, s))
                self.stats["misses"] += 1
            busy.add(s)
            got[i] = s
        return [int(s) for s in got], loads

    def split(self, keys):
        """Hybrid policy: (hit keys, hit slots, miss keys); nothing is loaded."""
        self.step()
        self.note(keys)
        self.stats["calls"] += 1
        ks = self._keys(keys)
        got = self.slot_of[ks]
        hit = got >= 0
        self.stats["hits"] += int(hit.sum())
        self.stats["misses"] += int((~hit).sum())
        return [int(k) for k in ks[hit]], [int(s) for s in got[hit]], [int(k) for k in ks[~hit]]

    def admit(self, key, protected):
        """Bring a key served elsewhere into the cache once it is hot enough; slot or None."""
        if self.lookup(key) is not None or not self.should_admit(key):
            return None
        try:
            return self.acquire(key, protected)
        except RuntimeError:
            return None

    def resized(self, nslots):
        """A new core of ``nslots`` keeping the highest-ranked resident keys (lru: most recently used,
        wsa: most frequent; equal ranks keep slot order).  Returns (core, [(key, new_slot)]) -- the
        copies into the new pool, in new-slot order."""
        if self.n_static:
            raise AssertionError("resize is not supported with a static region")
        nc = CacheCore(nslots, self.policy, self.decay, 0, self.admit_after)
        nc.tick, nc.unit, nc.stats = self.tick, self.unit, self.stats
        nc.slot_of = np.full(self.slot_of.size, -1, dtype=np.int64)
        nc.heat = self.heat  # the frequency history carries over
        live = np.flatnonzero(self.owner >= 0)
        order = live[np.argsort(-self.rank[live], kind="stable")][: nc.nslots]
        loads = []
        for ns, s in enumerate(order):
            k = int(self.owner[s])
            nc.owner[ns] = k
            nc.slot_of[k] = ns
            nc.rank[ns] = self.rank[s]
            loads.append((k, ns))
        nc.fill = len(order)
        return nc, loads
