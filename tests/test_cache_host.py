"""Expert-cache host logic on CPU.

The device planner (stblarge_b200/csrc/cache.cu, cache_plan_kernel) does not keep the reference's LRU
list: it gives every slot a logical last-use clock and takes, for a call's misses, the slots with the
smallest clocks among those the call has not touched (ties: the lower slot).  Here that rule,
restated in numpy exactly as the kernel applies it, is run against the reference's list algorithm
(oracle.LruExpertCache, stbl/model.cu:347-422, 503-520) on long random call sequences: both must
place every expert in the same slot and count the same hits and misses.  Also checks the configs[4]
route generator's properties."""

import numpy as np
import pytest

from oracle import oracle as O
from stblarge_b200.streamed import route_trace


class ClockPlanner:
    """The device planner's decisions, restated (one call = the kernel's phases in order).  flag: 1 =
    filled by a prefetch and not yet routed to, 2 = freed by a cancelled prefetch; state: the prefetch
    job's claim word (0 landed or no job, 1 queued)."""

    def __init__(self, n_layers, n_experts, slots):
        self.E, self.S = n_experts, slots
        self.map = np.full((n_layers, n_experts), -1, np.int64)
        self.owner = np.full(slots, -1, np.int64)
        self.ts = np.zeros(slots, np.int64)
        self.flag = np.zeros(slots, np.int8)
        self.state = np.zeros(slots, np.int8)
        self.clock = self.last_base = 0
        self.hits = self.misses = self.prefetched = self.pf_landed = self.cancelled = self.taken = 0

    def _place(self, layer, e, t, guard):
        """The victim search: key (class, slot), freed 0, never used 1, else last use + 1; slots a
        prefetch is still filling are skipped.  None when the best has a use newer than `guard`."""
        sl = np.arange(self.S)
        key = (self.ts + 1) * (1 << 20) + sl
        key[self.flag == 2] = sl[self.flag == 2]
        key[(self.flag == 1) & (self.state != 0)] = np.iinfo(np.int64).max
        s = int(np.argmin(key))
        if key[s] >> 20 > guard + 1:
            return None
        if self.owner[s] >= 0:
            self.map.reshape(-1)[self.owner[s]] = -1
        self.owner[s] = layer * self.E + e
        self.map[layer, e] = s
        self.ts[s] = t
        return s

    def call(self, layer, ids, pending="landed"):
        if pending == "landed":
            self.state[:] = 0
        u = list(dict.fromkeys(int(e) for e in np.asarray(ids).reshape(-1)))
        nu, base = len(u), self.clock
        row = self.map[layer]
        for s in range(self.S):  # cancel this layer's unrouted queued guesses, forget older landed ones
            if self.flag[s] != 1:
                continue
            l, e = divmod(int(self.owner[s]), self.E)
            if l == layer and e not in u:
                if self.state[s] == 1:
                    self.state[s] = 0
                    row[e] = -1
                    self.owner[s], self.ts[s], self.flag[s] = -1, 0, 2
                    self.cancelled += 1
            elif l < layer and self.state[s] == 0:
                self.flag[s] = 0
        for i, e in enumerate(u):
            s = row[e]
            if s < 0:
                continue
            self.ts[s] = base + 1 + nu + i
            if self.flag[s] != 1:
                self.hits += 1
                continue
            self.flag[s] = 0
            if self.state[s] == 1:  # taken over: this call copies it
                self.state[s] = 0
                self.taken += 1
                self.misses += 1
            else:
                self.hits += 1
                self.pf_landed += 1
        for i, e in enumerate(u):
            if row[e] >= 0:
                continue
            s = self._place(layer, e, base + 1 + nu + i, base)
            assert s is not None, "every slot is in use by this call"
            self.flag[s] = 0
            self.misses += 1
        self.clock = base + 1 + 2 * nu
        self.last_base = base

    def prefetch(self, layer, ids, consider):
        """the planner's prefetch mode: cached guesses untouched, no slot newer than the last call's
        start; the earlier prefetch copy has ended"""
        self.state[:] = 0
        u = list(dict.fromkeys(int(e) for e in np.asarray(ids).reshape(-1)))[:consider]
        base = self.clock
        for i, e in enumerate(u):
            if self.map[layer, e] >= 0:
                continue
            s = self._place(layer, e, base + 1 + i, self.last_base)
            if s is None:
                break
            self.flag[s], self.state[s] = 1, 1
            self.prefetched += 1
        self.clock = base + 1 + len(u)


@pytest.mark.parametrize("slots,T", [(8, 1), (12, 2), (40, 4), (64, 1)])
def test_clock_planner_equals_reference_lru(slots, T):
    L, E, K = 5, 32, 4
    rng = np.random.default_rng(slots * 10 + T)
    ref, dev = O.LruExpertCache(slots), ClockPlanner(L, E, slots)
    for call in range(400):
        layer = int(rng.integers(L))
        # skewed popularity so that calls both hit and evict
        ids = np.stack([rng.choice(E, K, replace=False, p=np.linspace(2.0, 0.2, E) / np.linspace(2.0, 0.2, E).sum())
                        for _ in range(T)])
        ref.call(layer, ids)
        dev.call(layer, ids)
        m, owner = ref.state(L, E)
        assert np.array_equal(m, dev.map), f"call {call}: residency differs"
        assert np.array_equal(owner, dev.owner), f"call {call}: slot owners differ"
        assert (ref.hits, ref.misses) == (dev.hits, dev.misses)
    assert ref.hits > 0 and ref.misses > slots


@pytest.mark.parametrize("pending", ["landed", "queued", "mixed"])
@pytest.mark.parametrize("slots,T,consider", [(8, 1, 3), (12, 2, 4), (40, 4, 8), (6, 1, 8)])
def test_clock_planner_with_prefetch_equals_reference_lru(slots, T, consider, pending):
    # the shadow next-layer prefetch between calls: guesses for the next layer, some right, some wrong;
    # the next call plans after the prefetch copy ("landed") or before it started ("queued": its
    # unrouted guesses are cancelled, its routed ones taken over)
    L, E, K = 4, 32, 4
    rng = np.random.default_rng(slots * 7 + T + consider + len(pending))
    ref, dev = O.LruExpertCache(slots), ClockPlanner(L, E, slots)
    p = np.linspace(2.0, 0.2, E)
    p /= p.sum()
    nxt = None
    for call in range(400):
        layer = call % L
        if nxt is not None and rng.random() < 0.7:
            ids = nxt  # the guess was right (the first tokens' experts)
        else:
            ids = np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(T)])
        st = pending if pending != "mixed" else ("landed", "queued")[int(rng.integers(2))]
        placed = ref.call(layer, ids, st)
        dev.call(layer, ids, st)
        nxt = np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(T)])
        guess = np.concatenate([nxt.reshape(-1), rng.choice(E, 3)])
        ref.prefetch((layer + 1) % L, guess, consider)
        dev.prefetch((layer + 1) % L, guess, consider)
        m, owner = ref.state(L, E)
        assert np.array_equal(m, dev.map), f"call {call}: residency differs"
        assert np.array_equal(owner, dev.owner), f"call {call}: slot owners differ"
        assert (ref.hits, ref.misses, ref.prefetched, ref.pf_landed, ref.cancelled, ref.taken) == \
            (dev.hits, dev.misses, dev.prefetched, dev.pf_landed, dev.cancelled, dev.taken)
        assert all(owner[s] == layer * E + e for s, e in placed)
    assert ref.prefetched > 0
    if pending != "queued":
        assert ref.pf_landed > 0
    if pending != "landed":
        assert ref.cancelled > 0 and ref.taken > 0


def test_reference_cancel_and_take_over():
    # a prefetch of layer 1 guesses 7, 8, 9; layer 1 then routes to 8 before the copy starts: 7 and 9
    # are cancelled (slots freed, lowest first to the next misses), 8 is taken over (a miss into its slot)
    c = O.LruExpertCache(6)
    c.call(0, [1, 2])
    assert c.prefetch(1, [7, 8, 9], 3) == [(2, 7), (3, 8), (4, 9)]
    assert c.call(1, [8, 3], pending="queued") == [(3, 8), (2, 3)]
    assert (c.cancelled, c.taken, c.pf_used, c.hits, c.misses) == (2, 1, 0, 0, 4)
    assert c.free == [4]
    assert c.call(1, [5]) == [(4, 5)]
    # landed guesses: routed ones are hits counted as used; a later layer's call forgets the others
    c.prefetch(2, [10, 11], 2)
    c.call(2, [10])
    assert c.pf_landed == 1 and (2, 11) in c.jobs
    c.call(3, [12])
    assert (2, 11) not in c.jobs
    c.call(2, [11])
    assert c.pf_landed == 1


def test_reference_lru_fills_slots_in_order_then_evicts_least_recent():
    c = O.LruExpertCache(3)
    assert c.call(0, [5, 6]) == [(0, 5), (1, 6)]
    assert c.call(0, [7]) == [(2, 7)]
    c.call(0, [5])                       # 5 becomes the most recent; 6 is now the least recent
    assert c.call(1, [5]) == [(1, 5)]    # layer 1's expert 5 takes 6's slot
    assert c.hits == 1 and c.misses == 4


def test_route_trace_properties():
    E, K, L, steps = 256, 8, 6, 200
    tr = route_trace(E, K, L, steps)
    assert tr.shape == (steps, L, K)
    assert all(len(set(tr[t, l])) == K for t in range(steps) for l in range(L)), "experts repeat within a token"
    reuse = np.mean([len(set(tr[t, l]) & set(tr[t - 1, l])) / K for t in range(1, steps) for l in range(L)])
    assert 0.55 < reuse < 0.8, reuse  # 0.6 by design, plus Zipf draws that land on last step's experts
    assert np.array_equal(tr, route_trace(E, K, L, steps)), "the generator is seeded"
