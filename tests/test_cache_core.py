"""Host logic of the expert cache (CPU): the slot policies of the reference CacheCore
(wisp/cache_core.py) -- hits, misses, LRU and frequency eviction, protection of the current request,
the static region, admission, resize."""

import numpy as np
import pytest

from wisp.cache_core import CacheCore


def test_ensure_hits_misses_and_lru_eviction():
    c = CacheCore(4)
    slots, loads = c.ensure([10, 11])
    assert slots == [0, 1] and loads == [(10, 0), (11, 1)]
    slots, loads = c.ensure([10, 12])
    assert slots == [0, 2] and loads == [(12, 2)]
    c.ensure([13])
    assert sorted(c.key2slot) == [10, 11, 12, 13]
    # full: the least recently used (11, last used at tick 1) goes
    slots, loads = c.ensure([14])
    assert loads == [(14, 1)] and 11 not in c.key2slot
    assert c.stats == dict(hits=1, misses=5, evictions=1, calls=4)


def test_current_request_is_protected():
    c = CacheCore(3)
    c.ensure([1, 2, 3])
    slots, loads = c.ensure([1, 4, 5])  # 1 is a hit and must not be evicted for 4 or 5
    assert 1 in c.key2slot and slots[0] == c.key2slot[1]
    assert len(set(slots)) == 3
    with pytest.raises(RuntimeError):
        c.ensure([6, 7, 8, 9])  # more keys than slots


def test_wsa_keeps_frequent_keys():
    c = CacheCore(2, policy="wsa", decay=0.99)
    for _ in range(5):
        c.ensure([1])
    c.ensure([2])
    c.ensure([3])  # evicts 2 (seen once) rather than 1 (seen five times, decayed)
    assert 1 in c.key2slot and 2 not in c.key2slot


def test_static_region_never_evicted():
    c = CacheCore(3, policy="static", n_static=2)
    assert c.preload([7, 8]) == [(7, 0), (8, 1)]
    for k in (20, 21, 22):
        slots, _ = c.ensure([k])
        assert slots == [2]
    assert c.key2slot[7] == 0 and c.key2slot[8] == 1


def test_split_and_admit():
    c = CacheCore(2, admit_after=2.0)
    c.ensure([1])
    hk, hs, mk = c.split([1, 2])
    assert hk == [1] and hs == [c.key2slot[1]] and mk == [2]
    assert c.admit(2, set()) is None or c.norm_freq(2) >= 2.0
    c.split([2])
    c.split([2])
    s = c.admit(2, {c.key2slot[1]})
    assert s is not None and c.key2slot[2] == s


def test_resized_keeps_hottest():
    c = CacheCore(4)
    for k in (1, 2, 3, 4):
        c.ensure([k])
    c.ensure([2])
    nc, loads = c.resized(2)
    assert [k for k, _ in loads] == [2, 4] and [s for _, s in loads] == [0, 1]
    assert nc.free == [] and nc.key2slot == {2: 0, 4: 1}
    nc2, loads2 = c.resized(6)
    assert len(loads2) == 4 and nc2.free == [5, 4]


def _tokens(n, L, E, k, seed):
    rng = np.random.default_rng(seed)
    return [[list(rng.choice(E, k, replace=False)) for _ in range(L)] for _ in range(n)]


@pytest.mark.parametrize("policy", ["lru"])
def test_plan_token_follows_per_layer_ensure(policy):
    """With nothing in flight, the token-level plan makes the same decisions as the reference's
    per-layer ensure under LRU: same hits, misses, evictions and final residency.  (Under wsa the
    plan may differ: a page-in issued for an earlier layer of the same token is still in flight, so it
    is never the victim, while the reference could evict a just-loaded, rarely used key.)"""
    from wisp.cache import plan_token

    L, E, k = 3, 8, 2
    a, b = CacheCore(10, policy), CacheCore(10, policy)
    for rows in _tokens(40, L, E, k, seed=1):
        evicted, loads = plan_token(a, rows, E, set())
        want_loads = []
        for l, row in enumerate(rows):
            _, ld = b.ensure([l * E + int(e) for e in row])
            want_loads += ld
        assert loads == want_loads
        assert len(evicted) <= len(loads)
        assert a.key2slot == b.key2slot
    assert a.stats == b.stats


def test_plan_token_never_evicts_busy_slots():
    from wisp.cache import plan_token

    L, E, k = 2, 16, 4
    core = CacheCore(8)
    busy = set()
    plan_token(core, [[0, 1, 2, 3], [0, 1, 2, 3]], E, busy)
    assert busy == set(range(8))  # every page-in is in flight
    before = dict(core.key2slot)
    evicted, loads = plan_token(core, [[4, 5, 6, 7], [4, 5, 6, 7]], E, busy)
    assert evicted == [] and loads == []  # nothing admitted, the misses stay host-served
    assert core.key2slot == before
    assert core.stats["misses"] == 16
    busy.clear()
    evicted, loads = plan_token(core, [[4, 5, 6, 7], [0, 1, 2, 3]], E, busy)
    assert sorted(k for k, _ in loads) == [4, 5, 6, 7]
    assert len(evicted) == 4 and all(e < E for e in evicted)  # layer 0's old keys went


def test_plan_token_hot_admission():
    from wisp.cache import plan_token

    core = CacheCore(4, decay=1.0, admit_after=2.0)
    _, loads = plan_token(core, [[1]], 8, set(), admit="hot")
    assert loads == []  # seen once
    _, loads = plan_token(core, [[1]], 8, set(), admit="hot")
    assert loads == [(1, 0)]  # seen twice: admitted


def _replay(case, ops):
    core = CacheCore(case["nslots"], case["policy"], case["decay"], case["n_static"], case["admit_after"])
    for i, op in enumerate(ops):
        kind, where = op["op"], f"{case['name']} op {i} ({op['op']})"
        if kind == "preload":
            assert [list(p) for p in core.preload(op["keys"])] == op["res"], where
        elif kind == "ensure":
            slots, loads = core.ensure(op["keys"])
            assert [slots, [list(p) for p in loads]] == op["res"], where
        elif kind == "split":
            assert [list(r) for r in core.split(op["keys"])] == op["res"], where
        elif kind == "admit":
            s = core.admit(op["keys"][0], set(op["prot"]))
            assert (-1 if s is None else s) == op["res"], where
        elif kind == "acquire":
            assert core.lookup(op["keys"][0]) is None, where
            assert core.acquire(op["keys"][0], set(op["prot"])) == op["res"], where
        elif kind == "lookup":
            assert core.lookup(op["keys"][0]) == op["res"], where
        elif kind == "resized":
            core, loads = core.resized(op["n"])
            assert [list(p) for p in loads] == op["res"], where
        elif kind == "error":
            with pytest.raises(RuntimeError):
                core.ensure(op["keys"])
            return core
        if "resident" in op:  # recorded after every operation but the initial preload
            assert sorted([k, s] for k, s in core.key2slot.items()) == op["resident"], where
            assert core.stats == op["stats"], where
    return core


def test_decisions_equal_reference_traces(golden):
    """Seeded operation sequences recorded from the reference CacheCore (tests/golden/make_golden.py,
    gen_cache_trace): lru, wsa, wsa with the frequency renormalisation crossed (decay 0.5), static with
    a pinned region, and a tight lru pool; ensure / split / admit / acquire / resized.  Every returned
    slot and page-in, the residency after each operation and the statistics must be equal."""
    import json

    trace = json.loads(str(golden("cache_trace")["trace"]))
    assert {t["case"]["name"] for t in trace} == {"lru", "wsa", "wsa_renorm", "static", "lru_tight"}
    for t in trace:
        core = _replay(t["case"], t["ops"])
        if t["case"]["name"] == "wsa_renorm":
            assert core.tick > 400  # 2**tick passed 1e100: the renormalisation ran


def test_table_is_the_device_layout():
    c = CacheCore(3)
    c.ensure([5, 9])
    t = c.table(12)
    assert t.dtype == np.int32 and t.shape == (12,)
    assert t[5] == 0 and t[9] == 1 and (np.delete(t, [5, 9]) == -1).all()


def test_victim_matches_acquire():
    c = CacheCore(3)
    assert c.victim(set()) == (0, -1)
    c.ensure([1, 2, 3])
    c.ensure([2])
    c.ensure([3])
    s, k = c.victim(set())
    assert (s, k) == (c.key2slot[1], 1)  # least recently used
    assert c.victim({0, 1, 2}) is None
    assert c.acquire(9, set()) == s and 1 not in c.key2slot


def test_plan_token_lfu_and_none_admission():
    from wisp.cache import plan_token

    core = CacheCore(2, decay=1.0)
    plan_token(core, [[0, 1]], 8, set(), admit="all")  # keys 0, 1 resident, used once
    for _ in range(3):
        plan_token(core, [[0]], 8, set(), admit="all")  # key 0 used 4 times
    _, loads = plan_token(core, [[5]], 8, set(), admit="lfu")  # 5 (used once) would evict 1 (once): no
    assert loads == []
    for _ in range(2):
        plan_token(core, [[5]], 8, set(), admit="none")  # still served from the host
    assert 5 not in core.key2slot
    _, loads = plan_token(core, [[5]], 8, set(), admit="lfu")  # 4 uses against 1: admitted over key 1
    assert loads == [(5, core.key2slot[5])] and 1 not in core.key2slot and 0 in core.key2slot
