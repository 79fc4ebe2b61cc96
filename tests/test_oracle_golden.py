"""The CPU oracle against golden vectors made by the reference's own torch stand-ins
(ref/kernel.py, via tests/golden/make_golden.py).  Quantizers and formats are bit-exact; GEMMs
match within fp32 summation-order noise; the whole small layer matches the reference composition
(expert ids exactly, output within the 1e-2 bf16 tolerance, in practice at most one bf16 ulp)."""

import dataclasses
import hashlib
import os
import sys

import numpy as np
import pytest

from oracle import oracle as O
from stblarge_b200 import synth
from stblarge_b200.config import CFG1, CFG1_FP4


def test_pow2_ceil(golden):
    g = golden("scalars")
    assert np.array_equal(O.pow2_ceil(g["pow2_in"]), g["pow2_out"])


def test_fp4_rounding_and_codes(golden):
    g = golden("scalars")
    codes = O.e2m1_encode(g["fp4_in"])
    assert np.array_equal(codes, g["fp4_codes"])
    vals = O.FP4_TABLE[codes]
    assert np.array_equal(vals.view(np.uint32), g["fp4_round"].view(np.uint32))  # signed zeros too


def test_e4m3_encode_matches_torch_cast(golden):
    g = golden("scalars")
    assert np.array_equal(O.e4m3_encode(g["e4m3_in"]), g["e4m3_codes"])


def test_e4m3_values_roundtrip():
    vals = O.e4m3_values()
    finite = np.isfinite(vals)
    codes = np.arange(256, dtype=np.uint8)[finite]
    back = O.e4m3_encode(vals[finite])
    # +0 and -0 keep their sign bit; every finite code maps to itself
    assert np.array_equal(back, codes)


def test_act_quant_128_fp32(golden):
    g = golden("quant")
    x = O.bf16_bits_to_f32(g["aq_x"])
    c, s = O.act_quant(x, 128, False)
    assert np.array_equal(c, g["aq128_codes"]) and np.array_equal(s, g["aq128_scales"])


def test_act_quant_32_pow2(golden):
    g = golden("quant")
    x = O.bf16_bits_to_f32(g["aq_x"])
    c, s = O.act_quant(x, 32, True)
    assert np.array_equal(c, g["aq32_codes"]) and np.array_equal(s, g["aq32_scales"])


def test_reference_inplace_act_quant(golden):
    """stbl/kernels.cu:56-63 (in-place, bf16 result) equals act_quant(..., inplace=True) bit for bit,
    the reference's own tol-0 check (stbl/test_kernels.py:63-69)."""
    g = golden("quant")
    x = O.bf16_bits_to_f32(g["aq_x"]).reshape(-1)
    got = O.ref_act_quant_fp8(x)
    assert np.array_equal(O.f32_to_bf16_bits(got), g["aq32_inplace"].reshape(-1))


def test_mxfp4_weight_quant(golden):
    g = golden("quant")
    p, s = O.quant_mxfp4(g["fp4w_in"])
    assert np.array_equal(p, g["fp4w_packed"]) and np.array_equal(s, g["fp4w_scales"])


def test_fp8_b128_weight_quant(golden):
    g = golden("quant")
    c, s = O.quant_fp8_b128(g["fp8w_in"])
    assert np.array_equal(c, g["fp8w_codes"]) and np.array_equal(s, g["fp8w_scales"])


def test_fp8_gemm(golden):
    g = golden("gemm")
    y = O.gemv_fp8_b128(g["g8_w"], g["g8_ws"], g["g8_aq"], g["g8_as"], 128)
    np.testing.assert_allclose(y, g["g8_y"], rtol=1e-5, atol=1e-5 * np.abs(g["g8_y"]).max())


def test_fp4_gemm(golden):
    g = golden("gemm")
    y = O.gemv_mxfp4(g["g4_w"], g["g4_ws"], g["g4_aq"], g["g4_as"], 32)
    np.testing.assert_allclose(y, g["g4_y"], rtol=1e-5, atol=1e-5 * np.abs(g["g4_y"]).max())


def _digest(W):
    h = hashlib.sha256()
    for m in range(3):
        for e in range(len(W["routed"][0])):
            for i in range(2):
                h.update(np.ascontiguousarray(W["routed"][m][e][i]).tobytes())
    for m in range(3):
        for i in range(2):
            h.update(np.ascontiguousarray(W["shared"][m][i]).tobytes())
    return h.hexdigest()


def _oracle_quantized_layer(cfg):
    """The layer's weights re-quantized by the oracle's own C quantizers from the seeded floats."""
    routed = [[None] * cfg.n_experts for _ in range(3)]
    q = O.quant_fp8_b128 if cfg.routed_fmt == O.FMT_FP8_B128 else O.quant_mxfp4
    for e in range(cfg.n_experts):
        for m, w in enumerate(synth.expert_floats(cfg, 1000 + e)):
            routed[m][e] = q(w)
    shared = [O.quant_fp8_b128(w) for w in synth.expert_floats(cfg, 3)]
    return {"router_w": synth.router_w(cfg), "router_bias": synth.router_bias(cfg), "routed": routed, "shared": shared}


@pytest.mark.parametrize("cfg,name", [(CFG1, "layer_cfg1"), (CFG1_FP4, "layer_cfg1_fp4")])
def test_layer_matches_reference_composition(golden, cfg, name):
    g = golden(name)
    W = _oracle_quantized_layer(cfg)
    assert _digest(W) == str(g["weights_sha256"]), "oracle quantizers rebuilt different weight bytes"
    logits = O.router_logits(W["router_w"], g["x"])
    np.testing.assert_allclose(logits, g["logits"], rtol=1e-5, atol=1e-5)
    y, idx, w = O.moe_forward(cfg.as_dict(), W, g["x"])
    assert np.array_equal(idx, g["idx"])
    np.testing.assert_allclose(w, g["w"], rtol=1e-6)
    yf, ref = O.bf16_bits_to_f32(y), O.bf16_bits_to_f32(g["y"])
    err = np.abs(yf - ref).max()
    assert err <= 1e-2 * np.abs(ref).max(), err
    # in practice the oracle and the reference composition differ by at most one bf16 ulp
    ulp = np.abs(ref) * 2.0 ** -7 + 1e-30
    assert np.all(np.abs(yf - ref) <= ulp * 1.01)


@pytest.mark.parametrize("rule", ["v3", "sp"])
def test_oracle_full_size_routes_match_reference_composition(golden, rule):
    """The oracle's router (it restates the GPU's exact logits order, so the GPU equals it bit for bit)
    against the reference-style torch composition of the full-size router on 256 tokens
    (tests/golden/route_cfg2.npz): v3 group-limited sigmoid top-8 and the reference engine's
    sqrt(softplus) flat top-8.  Every mismatch is reported with the reference's selection margin (as
    stbl/test_layers.py:105 does) and allowed only below 1e-5, what fp32 summation order can move."""
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    from make_route_golden import inputs

    from stblarge_b200.config import CFG2, SCORE_SQRT_SOFTPLUS
    g = golden("route_cfg2")
    W, b, x, digest = inputs()
    assert digest == str(g["inputs_sha256"]), "synth no longer regenerates the fixture's inputs"
    cfg = CFG2 if rule == "v3" else dataclasses.replace(CFG2, score_fn=SCORE_SQRT_SOFTPLUS, n_groups=1, topk_groups=1)
    lg = O.router_logits(W, x)
    _, idx, w = O.router_select(lg, b, cfg.topk, cfg.n_groups, cfg.topk_groups, cfg.score_fn, cfg.route_scale)
    want, margin = g["idx_" + rule], g["margin_" + rule]
    flips = [(t, float(margin[t]), sorted(set(idx[t].tolist()) ^ set(want[t].tolist())))
             for t in range(len(want)) if set(idx[t].tolist()) != set(want[t].tolist())]
    print(f"\n{rule}: route mismatches {len(flips)}/{len(want)} (token, ref margin, differing ids): {flips}")
    assert all(m < 1e-5 for _, m, _ in flips), flips
    same = [t for t in range(len(want)) if set(idx[t].tolist()) == set(want[t].tolist())]
    assert np.array_equal(idx[same], want[same])
    np.testing.assert_allclose(w[same], g["w_" + rule][same], rtol=1e-5)
