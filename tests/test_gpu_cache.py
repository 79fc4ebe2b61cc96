"""GPU expert cache (stbl_cache_*) and forced routes (stbl_moe_forward_routed), through the C ABI.

Cached layers must give the same bits as layers holding every expert in device memory (same
kernels, same weights, read from the cache's slots), and the cache's decisions (which slot holds
which expert, hits, misses) must equal the reference's LRU bookkeeping restated in the oracle
(oracle.LruExpertCache, stbl/model.cu:347-422, 503-520) after every call.  Forced routes are checked
against the oracle layer with the same routes."""

import ctypes
import threading
import time

import numpy as np
import pytest
import torch

from oracle import oracle as O
from stblarge_b200 import synth
from stblarge_b200.cache import ExpertCache, host_store
from stblarge_b200.config import CFG1, CFG1_FP4
from stblarge_b200.moe import MoELayer
from tests.test_gpu_layer import TOL, compare_y, oracle_weights_from_device

pytestmark = pytest.mark.gpu


def _x(cfg, T, seed):
    return torch.from_numpy(synth.make_x(cfg.hidden, T, seed=seed).view(np.int16)).cuda()


@pytest.mark.parametrize("cfg", [CFG1, CFG1_FP4], ids=["fp8", "mxfp4"])
def test_cached_layers_match_resident_layers_and_reference_lru(cfg):
    L, S, Tmax, E = 3, 8, 2, cfg.n_experts
    store = host_store(cfg, L)
    cache = ExpertCache(cfg, L, S, store)
    resident = [synth.device_layer(cfg, seed_base=1000 + l * E) for l in range(L)]
    plain = [MoELayer(cfg, resident[l], max_tokens=Tmax) for l in range(L)]
    cached = [MoELayer(cfg, resident[l], max_tokens=Tmax, cache=(cache, l)) for l in range(L)]
    lru = O.LruExpertCache(S)
    rng = np.random.default_rng(11)
    for call in range(16):
        l, T = int(rng.integers(L)), int(rng.integers(1, Tmax + 1))
        x = _x(cfg, T, 500 + call)
        y_plain, y = plain[l](x), cached[l](x)
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), y_plain.view(torch.int16)), f"call {call}: cached layer differs"
        lru.call(l, cached[l].last_route()["idx"])
        mp, owner = cache.state()
        emp, eowner = lru.state(L, E)
        assert np.array_equal(mp, emp), f"call {call}: residency map differs"
        assert np.array_equal(owner, eowner), f"call {call}: slot owners differ"
        st = cache.stats()
        assert (st["hits"], st["misses"]) == (lru.hits, lru.misses)
    assert lru.misses > S and lru.hits > 0, "the sequence must both evict and hit"
    assert cache.stats()["bytes"] == lru.misses * sum(
        t[0].numel() * t.element_size() for t in store["w"] + store["s"])
    for layer in cached + plain:
        assert layer.status() == 0
        layer.close()
    cache.close()


@pytest.mark.parametrize("cfg", [CFG1, CFG1_FP4], ids=["fp8", "mxfp4"])
def test_forward_routed_matches_oracle(cfg):
    dev = synth.device_layer(cfg)
    layer = MoELayer(cfg, dev, max_tokens=8)
    rng = np.random.default_rng(3)
    for T in (1, 5):
        x_bits = synth.make_x(cfg.hidden, T, seed=40 + T)
        forced = np.stack([rng.permutation(cfg.n_experts)[:cfg.topk] for _ in range(T)]).astype(np.int32)
        y = layer.forward_routed(torch.from_numpy(x_bits.view(np.int16)).cuda(), torch.from_numpy(forced).cuda())
        torch.cuda.synchronize()
        route = layer.last_route()
        assert np.array_equal(route["idx"], forced)
        W = oracle_weights_from_device(cfg, dev, forced.reshape(-1))
        y_ref, idx_ref, w_ref = O.moe_forward(cfg.as_dict(), W, x_bits, forced=forced)
        assert np.array_equal(route["weights"].view(np.uint32), w_ref.view(np.uint32)), "routing weights differ"
        counts, offsets, perm = O.dispatch(forced, cfg.n_experts)
        assert np.array_equal(route["perm"], perm)
        rel, same, ulps = compare_y(y.view(torch.int16).cpu().numpy().view(np.uint16), y_ref)
        assert rel <= TOL, f"max-abs-rel {rel:.3e} ({ulps:.1f} bf16 ulps)"
    assert layer.status() == 0
    # a row that repeats an expert is replaced by experts 0..topk-1 and flagged
    bad = np.zeros((1, cfg.topk), np.int32)
    layer.forward_routed(_x(cfg, 1, 9), torch.from_numpy(bad).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(layer.last_route()["idx"][0], np.arange(cfg.topk))
    assert layer.status() == 2
    layer.close()


def test_cache_sized_from_free_memory():
    # slots = 0: the library sizes the cache; a small store fits entirely (one slot per expert)
    cfg, L = CFG1_FP4, 2
    store = host_store(cfg, L)
    cache = ExpertCache(cfg, L, 0, store)
    assert cache.slots == L * cfg.n_experts
    assert cache.slot_bytes >= sum(t[0].numel() * t.element_size() for t in store["w"] + store["s"])
    resident = synth.device_layer(cfg, seed_base=1000 + cfg.n_experts)
    plain = MoELayer(cfg, resident, max_tokens=2)
    cached = MoELayer(cfg, resident, max_tokens=2, cache=(cache, 1))
    seen, routed = set(), 0
    for call in range(3):
        x = _x(cfg, 2, 700 + call)
        assert torch.equal(cached(x).view(torch.int16), plain(x).view(torch.int16))
        ids = set(int(e) for e in cached.last_route()["idx"].reshape(-1))
        routed += len(ids)
        seen |= ids
    st = cache.stats()
    # every slot is free or holds its expert for good: each distinct expert misses exactly once
    assert st["misses"] == len(seen) and st["hits"] == routed - len(seen)
    for layer in (cached, plain):
        assert layer.status() == 0
        layer.close()
    cache.close()


@pytest.mark.parametrize("cfg", [CFG1, CFG1_FP4], ids=["fp8", "mxfp4"])
def test_cached_layer_with_forced_routes(cfg):
    # the streamed-decode combination: routes given, experts brought in by the cache
    L, S, E = 2, 6, cfg.n_experts
    store = host_store(cfg, L)
    cache = ExpertCache(cfg, L, S, store)
    resident = [synth.device_layer(cfg, seed_base=1000 + l * E) for l in range(L)]
    plain = [MoELayer(cfg, resident[l], max_tokens=1) for l in range(L)]
    cached = [MoELayer(cfg, resident[l], max_tokens=1, cache=(cache, l)) for l in range(L)]
    lru = O.LruExpertCache(S)
    rng = np.random.default_rng(21)
    for call in range(12):
        l = call % L
        idx = torch.from_numpy(rng.permutation(E)[:cfg.topk].astype(np.int32).reshape(1, -1)).cuda()
        x = _x(cfg, 1, 800 + call)
        y_plain, y = plain[l].forward_routed(x, idx), cached[l].forward_routed(x, idx)
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), y_plain.view(torch.int16)), f"call {call}"
        lru.call(l, idx.cpu().numpy())
        assert (cache.stats()["hits"], cache.stats()["misses"]) == (lru.hits, lru.misses)
    for layer in cached + plain:
        assert layer.status() == 0
        layer.close()
    cache.close()


@pytest.mark.parametrize("cfg,S", [(CFG1, 12), (CFG1_FP4, 12), (CFG1_FP4, 8)], ids=["fp8", "mxfp4", "mxfp4_small"])
def test_shadow_prefetch_matches_resident_layers_and_reference_lru(cfg, S):
    # layer l runs layer l+1's router on its own input and prefetches the top guesses for l+1, copied on
    # a second stream beside l's experts (stbl_moe_attach_prefetch); the next call waits for that copy
    L, E, T, n_predict, consider = 3, cfg.n_experts, 2, 4, 3
    store = host_store(cfg, L)
    cache = ExpertCache(cfg, L, S, store)
    resident = [synth.device_layer(cfg, seed_base=1000 + l * E) for l in range(L)]
    plain = [MoELayer(cfg, resident[l], max_tokens=T) for l in range(L)]
    cached = [MoELayer(cfg, resident[l], max_tokens=T, cache=(cache, l)) for l in range(L)]
    side = torch.cuda.Stream()
    for l in range(L - 1):
        cached[l].attach_prefetch(cached[l + 1], n_predict, consider, side)
    lru = O.LruExpertCache(S)
    for step in range(6):
        x_bits = synth.make_x(cfg.hidden, T, seed=900 + step)
        x = torch.from_numpy(x_bits.view(np.int16)).cuda()
        for l in range(L):  # the same input for every layer: the next layer's guesses are its routes
            y_plain, y = plain[l](x), cached[l](x)
            torch.cuda.synchronize()
            assert torch.equal(y.view(torch.int16), y_plain.view(torch.int16)), f"step {step} layer {l}"
            lru.call(l, cached[l].last_route()["idx"])
            if l + 1 < L:
                nw = resident[l + 1]
                lg = O.router_logits(nw["router_w"].cpu().numpy(), x_bits)
                _, guess, _ = O.router_select(lg, nw["router_bias"].cpu().numpy(), n_predict, cfg.n_groups, cfg.topk_groups,
                                              cfg.score_fn, cfg.route_scale)
                lru.prefetch(l + 1, guess, consider)
            mp, owner = cache.state()
            emp, eowner = lru.state(L, E)
            assert np.array_equal(mp, emp), f"step {step} layer {l}: residency map differs"
            assert np.array_equal(owner, eowner), f"step {step} layer {l}: slot owners differ"
            st, pf = cache.stats(), cache.prefetch_stats()
            assert (st["hits"], st["misses"]) == (lru.hits, lru.misses)
            assert (pf["prefetched"], pf["used"]) == (lru.prefetched, lru.pf_used)
    assert lru.prefetched > 0 and lru.pf_used > 0
    # every call plans after the prefetch copy has landed: nothing is read late or cancelled
    assert cache.prefetch_counters() == [lru.prefetched, lru.pf_landed, 0, 0]
    for layer in cached + plain:
        assert layer.status() == 0
        layer.close()
    cache.close()


def _cu():
    cu = ctypes.CDLL("libcuda.so.1")
    cu.cuLaunchHostFunc.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    cu.cuStreamCreate.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_uint]
    cu.cuStreamDestroy_v2.argtypes = [ctypes.c_void_p]
    return cu


def _nonblocking_stream():
    """A stream that does not synchronise with the legacy default stream (CU_STREAM_NON_BLOCKING), so
    the cache's counters can be read with cudaMemcpy while work on it waits."""
    h = ctypes.c_void_p()
    assert _cu().cuStreamCreate(ctypes.byref(h), 1) == 0
    return torch.cuda.ExternalStream(h.value), h


class _StreamGate:
    """Holds a stream at a host function until open() is called (or 60 s pass): the work queued on
    the stream behind it does not start before then."""
    _CB = ctypes.CFUNCTYPE(None, ctypes.c_void_p)

    def __init__(self, stream):
        self._ev = threading.Event()
        self._cb = self._CB(lambda _: self._ev.wait(60))
        assert _cu().cuLaunchHostFunc(ctypes.c_void_p(stream.cuda_stream), ctypes.cast(self._cb, ctypes.c_void_p), None) == 0

    def open(self):
        self._ev.set()


@pytest.mark.parametrize("cfg", [CFG1, CFG1_FP4], ids=["fp8", "mxfp4"])
def test_prefetch_cancelled_and_taken_over_before_its_copy_starts(cfg):
    # the reference's cancellation (stbl/model.cu:397-414, 478-494): a call that plans before the
    # prefetch copy for its layer has started cancels the guesses it does not route to and takes over
    # the ones it does.  The copy stream is held by a host function until the call's planner has run
    # (its hit/miss counts moved); every third step lets the copy land first.  Routes are forced, one
    # token routed to one guess of the prefetch, so both cases occur; outputs must equal resident layers,
    # decisions and counters the reference's bookkeeping (oracle.LruExpertCache with the job states).
    L, S, T, E, K, n_predict, consider = 3, 12, 2, cfg.n_experts, cfg.topk, 4, 4
    torch.cuda.init()
    store = host_store(cfg, L)
    cache = ExpertCache(cfg, L, S, store)
    resident = [synth.device_layer(cfg, seed_base=1000 + l * E) for l in range(L)]
    plain = [MoELayer(cfg, resident[l], max_tokens=T) for l in range(L)]
    cached = [MoELayer(cfg, resident[l], max_tokens=T, cache=(cache, l)) for l in range(L)]
    main, hm = _nonblocking_stream()
    side, hs = _nonblocking_stream()
    for l in range(L - 1):
        cached[l].attach_prefetch(cached[l + 1], n_predict, consider, side)
    lru = O.LruExpertCache(S)
    rng = np.random.default_rng(5)
    gates = []
    try:
        with torch.cuda.stream(main):
            for step in range(6):
                gated = step % 3 != 2
                placed, held = [], None
                for l in range(L):
                    x_bits = synth.make_x(cfg.hidden, T, seed=1200 + 10 * step + l)
                    guessed = [e for _, e in placed]
                    keep = guessed[:1]
                    others = [int(e) for e in rng.permutation(E) if e not in guessed]
                    rows = np.array([keep + others[:K - len(keep)], others[K - len(keep):2 * K - len(keep)]], np.int32)
                    x = torch.from_numpy(x_bits.view(np.int16)).cuda()
                    idx = torch.from_numpy(rows).cuda()
                    y_plain = plain[l].forward_routed(x, idx)
                    nxt = _StreamGate(side) if gated and l + 1 < L else None  # holds this call's prefetch copy
                    if nxt is not None:
                        gates.append(nxt)
                    st0 = cache.stats()
                    y = cached[l].forward_routed(x, idx)
                    if held is not None:
                        t0 = time.time()
                        while sum(cache.stats()[k] for k in ("hits", "misses")) == st0["hits"] + st0["misses"]:
                            assert time.time() - t0 < 30, "the call's planner did not run"
                            time.sleep(0.002)
                        held.open()
                    main.synchronize()
                    if nxt is None:
                        torch.cuda.synchronize()  # the prefetch copy (if any) lands before the next call
                    assert torch.equal(y.view(torch.int16), y_plain.view(torch.int16)), f"step {step} layer {l}"
                    lru.call(l, rows, pending="queued" if held is not None else "landed")
                    held, placed = nxt, []
                    if l + 1 < L:
                        nw = resident[l + 1]
                        lg = O.router_logits(nw["router_w"].cpu().numpy(), x_bits)
                        _, guess, _ = O.router_select(lg, nw["router_bias"].cpu().numpy(), n_predict, cfg.n_groups,
                                                      cfg.topk_groups, cfg.score_fn, cfg.route_scale)
                        placed = lru.prefetch(l + 1, guess, consider)
                    mp, owner = cache.state()
                    emp, eowner = lru.state(L, E)
                    assert np.array_equal(mp, emp), f"step {step} layer {l}: residency map differs"
                    assert np.array_equal(owner, eowner), f"step {step} layer {l}: slot owners differ"
                    st = cache.stats()
                    assert (st["hits"], st["misses"]) == (lru.hits, lru.misses), f"step {step} layer {l}"
                    assert cache.prefetch_counters() == [lru.prefetched, lru.pf_landed, 0, lru.cancelled]
        torch.cuda.synchronize()
    finally:
        for g in gates:
            g.open()
    assert lru.cancelled > 0 and lru.taken > 0 and lru.pf_landed > 0
    st, pf = cache.stats(), cache.prefetch_stats()
    # bytes: the demand copies (misses, taken-over guesses included) and the prefetch copies that ran
    assert pf["bytes"] * lru.misses == st["bytes"] * (lru.prefetched - lru.cancelled - lru.taken)
    for layer in cached + plain:
        assert layer.status() == 0
        layer.close()
    cache.close()
    _cu().cuStreamDestroy_v2(hm)
    _cu().cuStreamDestroy_v2(hs)
