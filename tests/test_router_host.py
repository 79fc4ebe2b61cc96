"""Routing rules of the oracle on hand-made scores: ties go to the lower expert (and group) id,
group-limited selection keeps the best groups by the sum of their two best biased scores, weights
are the unbiased scores normalised in selection order, and the dispatch permutation is expert-major
and token-ordered (stbl/model.cu:444-451, 527-530).  A brute-force Python restatement is the check."""

import numpy as np
import pytest

from oracle import oracle as O


def brute_select(scores, bias, topk, G, KG, route_scale):
    T, E = scores.shape
    gsz = E // G
    idx = np.zeros((T, topk), np.int32)
    w = np.zeros((T, topk), np.float32)
    for t in range(T):
        b = (scores[t] + bias).astype(np.float32)
        keep = np.ones(E, bool)
        if G > 1 and KG < G:
            gs = []
            for g in range(G):
                order = sorted(range(g * gsz, (g + 1) * gsz), key=lambda e: (-b[e], e))
                gs.append(np.float32(b[order[0]] + b[order[1]]))
            gorder = sorted(range(G), key=lambda g: (-gs[g], g))[:KG]
            keep[:] = False
            for g in gorder:
                keep[g * gsz:(g + 1) * gsz] = True
        cand = sorted([e for e in range(E) if keep[e]], key=lambda e: (-b[e], e))[:topk]
        idx[t] = cand
        s = np.float32(0)
        for e in cand:
            s = np.float32(s + scores[t, e])
        for i, e in enumerate(cand):
            w[t, i] = np.float32(np.float32(scores[t, e] / np.float32(s + np.float32(1e-20))) * np.float32(route_scale))
    return idx, w


def logits_for(scores):
    """logits whose sigmoid (evaluated in double, rounded to fp32) gives back exactly `scores`."""
    lg = np.log(scores.astype(np.float64) / (1 - scores.astype(np.float64))).astype(np.float32)
    return lg


def sig(lg):
    return (1.0 / (1.0 + np.exp(-lg.astype(np.float64)))).astype(np.float32)


@pytest.mark.parametrize("E,topk,G,KG", [(16, 4, 4, 2), (256, 8, 8, 4), (64, 6, 1, 1), (32, 4, 8, 8)])
def test_selection_matches_brute_force(E, topk, G, KG):
    rng = np.random.default_rng(E + topk)
    lg = rng.standard_normal((12, E)).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    scores, idx, w = O.router_select(lg, bias, topk, G, KG, O.SCORE_SIGMOID, 2.5)
    assert np.array_equal(scores, sig(lg))
    bidx, bw = brute_select(scores, bias, topk, G, KG, 2.5)
    assert np.array_equal(idx, bidx)
    assert np.array_equal(w, bw)


def test_ties_go_to_the_lower_expert_id():
    E = 16
    lg = np.zeros((3, E), np.float32)          # every score 0.5
    bias = np.zeros(E, np.float32)
    bias[[3, 9, 12]] = 0.25                      # three clear winners, the rest tied
    _, idx, w = O.router_select(lg, bias, 6, 1, 1, O.SCORE_SIGMOID, 1.0)
    assert idx[0].tolist() == [3, 9, 12, 0, 1, 2]
    assert np.allclose(w.sum(1), 1.0, atol=1e-6)


def test_group_ties_go_to_the_lower_group_id():
    E, G = 16, 4
    lg = np.zeros((1, E), np.float32)
    bias = np.zeros(E, np.float32)               # all four groups score the same
    _, idx, _ = O.router_select(lg, bias, 4, G, 2, O.SCORE_SIGMOID, 1.0)
    assert sorted(idx[0].tolist()) == [0, 1, 2, 3]  # groups 0 and 1 kept, lowest ids first
    bias[12] = 1.0                                  # group 3 now has the best pair sum? only one high member
    bias[13] = 1.0
    _, idx, _ = O.router_select(lg, bias, 4, G, 2, O.SCORE_SIGMOID, 1.0)
    assert idx[0].tolist()[:2] == [12, 13] and set(idx[0].tolist()[2:]) <= {0, 1, 2, 3}


def test_group_limit_excludes_experts_of_dropped_groups():
    E, G = 16, 4
    lg = np.zeros((1, E), np.float32)
    bias = np.full(E, 0.0, np.float32)
    bias[0] = 5.0                                # group 0 has one huge expert but a weak second
    bias[4:8] = 1.0                              # group 1 strong pair
    bias[8:12] = 0.9                             # group 2 strong pair
    _, idx, _ = O.router_select(lg, bias, 2, G, 2, O.SCORE_SIGMOID, 1.0)
    # group sums: g0 = 5 + 0 (+0.5 scores), g1 = 2.0, g2 = 1.8 -> keep g0 and g1
    assert idx[0].tolist() == [0, 4]


def test_sqrt_softplus_scores():
    lg = np.array([[-30.0, -1.0, 0.0, 1.0, 19.9, 20.0, 20.5, 40.0]], np.float32)
    s, _, _ = O.router_select(lg, np.zeros(8, np.float32), 2, 1, 1, O.SCORE_SQRT_SOFTPLUS, 1.0)
    x = lg.astype(np.float64)
    want = np.where(lg > 20, x, np.log1p(np.exp(x)))
    assert np.array_equal(s, np.sqrt(want).astype(np.float32))


def test_dispatch_permutation_is_expert_major_and_stable():
    rng = np.random.default_rng(3)
    T, E, k = 37, 16, 4
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    counts, offsets, perm = O.dispatch(idx, E)
    assert counts.sum() == T * k and offsets[-1] == T * k
    assert np.array_equal(np.sort(perm), np.arange(T * k))       # a permutation
    for e in range(E):
        seg = perm[offsets[e]:offsets[e + 1]]
        assert np.all(idx.reshape(-1)[seg] == e)                  # bucket holds expert e only
        assert np.all(np.diff(seg // k) > 0)                      # tokens ascending


def test_router_logits_split_order_is_deterministic():
    """The restated GPU order (4 hidden slices, lane-strided fused multiply-adds, butterfly) is close to
    a float64 dot product and independent of thread count."""
    rng = np.random.default_rng(5)
    W = rng.standard_normal((8, 1024)).astype(np.float32) * 0.02
    x = (rng.standard_normal((3, 1024)).astype(np.float32).view(np.uint32) & 0xFFFF0000).view(np.float32)
    bits = (x.view(np.uint32) >> 16).astype(np.uint16)
    got = O.router_logits(W, bits)
    want = x.astype(np.float64) @ W.T.astype(np.float64)
    assert np.allclose(got, want, rtol=1e-5, atol=1e-5)
    assert np.array_equal(got, O.router_logits(W, bits))
