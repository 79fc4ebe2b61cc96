"""The oracle's Q8 activation numerics (oracle.q8_codes, oracle.gemv_mxfp4_q8) against the reference's
own emulation (ref/emulate_ds4.py q8_codes :23-30, the FP4 branch of linear :69-77) run on the same
inputs (tests/golden/q8.npz, written by tests/golden/make_q8_golden.py).  Codes and scales bit-exact;
the FP4 linear within fp32 summation noise (the emulation sums in torch's order, the oracle exactly)."""

import os

import numpy as np

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "q8.npz")


def test_q8_codes_match_the_reference_emulation():
    g = np.load(GOLDEN)
    q, d = O.q8_codes(g["x"])
    assert np.array_equal(q, g["q"])
    assert np.array_equal(d.view(np.uint32), g["d"].view(np.uint32))
    values = (q.astype(np.float32).reshape(q.shape[0], -1, 32) * d[..., None]).reshape(q.shape)
    assert np.array_equal(values.view(np.uint32), g["values"].view(np.uint32))
    # the inputs exercise an all-zero block (d = 0) and round-half-to-even ties
    assert (d == 0).any()
    t = g["x"].reshape(-1, 32) / np.where(d.reshape(-1, 1) > 0, d.reshape(-1, 1), 1)
    assert (np.abs(t - np.trunc(t)) == 0.5).any()


def test_fp4_linear_with_q8_activations_matches_the_reference_emulation():
    g = np.load(GOLDEN)
    q, d = O.q8_codes(g["x"])
    y = O.gemv_mxfp4_q8(g["codes"], g["scales"], q, d)
    ref = g["y"]
    assert y.shape == ref.shape
    err = np.abs(y - ref).max() / np.abs(ref).max()
    assert err <= 1e-6, err
