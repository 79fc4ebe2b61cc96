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
    """The device planner's decisions, restated (one call = the kernel's phases in order)."""

    def __init__(self, n_layers, n_experts, slots):
        self.E, self.S = n_experts, slots
        self.map = np.full((n_layers, n_experts), -1, np.int64)
        self.owner = np.full(slots, -1, np.int64)
        self.ts = np.zeros(slots, np.int64)
        self.clock = 0
        self.hits = self.misses = 0

    def call(self, layer, ids):
        u = list(dict.fromkeys(int(e) for e in np.asarray(ids).reshape(-1)))
        nu, base = len(u), self.clock
        row = self.map[layer]
        for i, e in enumerate(u):
            if row[e] >= 0:
                self.ts[row[e]] = base + 1 + nu + i
                self.hits += 1
        for i, e in enumerate(u):
            if row[e] >= 0:
                continue
            key = self.ts * (1 << 20) + np.arange(self.S)
            s = int(np.argmin(key))
            assert self.ts[s] <= base, "every slot is in use by this call"
            if self.owner[s] >= 0:
                self.map.reshape(-1)[self.owner[s]] = -1
            self.owner[s] = layer * self.E + e
            row[e] = s
            self.ts[s] = base + 1 + nu + i
            self.misses += 1
        self.clock = base + 1 + 2 * nu


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
