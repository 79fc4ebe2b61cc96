"""Parity of the B200 MoE layer (libstbl_moe.so through its C ABI) with the CPU oracle.

Bar: router logits, scores, expert ids, routing weights and the dispatch permutation bit-exact;
the layer's own activation quantizations (x per token, h per dispatch position and per shared-expert
token, as the expert kernels read them) bit-exact against the reference's act_quant rule (tolerance
0, as stbl/test_kernels.py:63-69); layer output within max-abs 1e-2 of max |reference| in bf16
(BASELINE tolerance), reported in bf16 ulps as well.  Small layers run the oracle on every expert;
full-size layers hand the oracle only the experts the GPU chose (it fails if it would route
elsewhere).  Full-size routes are also compared with the reference-style torch composition of the
router (tests/golden/route_cfg2.npz), every mismatch reported with its selection margin."""

import dataclasses

import numpy as np
import pytest
import torch

from oracle import oracle as O
from stblarge_b200 import synth
from stblarge_b200.config import CFG1, CFG1_FP4, CFG2, CFG3, CFG3_Q8, FMT_FP8_B128, FMT_NONE, SCORE_SQRT_SOFTPLUS
from stblarge_b200.moe import MoELayer, host_weights_to_device

pytestmark = pytest.mark.gpu

TOL = 1e-2


def compare_y(y_bits, ref_bits):
    y, ref = O.bf16_bits_to_f32(y_bits), O.bf16_bits_to_f32(ref_bits)
    err = np.abs(y - ref).max()
    scale = np.abs(ref).max()
    ulps = np.abs(y - ref) / np.maximum(np.abs(ref) * 2.0 ** -8, 1e-30)
    return err / scale, float(np.mean(y_bits == ref_bits)), float(ulps.max())


def oracle_weights_from_device(cfg, dev, experts):
    W = {"router_w": dev["router_w"].cpu().numpy(), "router_bias": dev["router_bias"].cpu().numpy(),
         "routed": [[None] * cfg.n_experts for _ in range(3)], "shared": None}
    for e in sorted(set(int(v) for v in experts)):
        for m in range(3):
            W["routed"][m][e] = (dev["routed_w"][m][e].cpu().numpy(), dev["routed_s"][m][e].cpu().numpy())
    if cfg.shared_fmt != FMT_NONE:
        W["shared"] = [(dev["shared_w"][m].cpu().numpy(), dev["shared_s"][m].cpu().numpy()) for m in range(3)]
    return W


def run_and_check(cfg, layer, dev_w, host_W, x_bits):
    x = torch.from_numpy(x_bits.view(np.int16)).cuda()
    y = layer(x)
    torch.cuda.synchronize()
    y_bits = y.view(torch.int16).cpu().numpy().view(np.uint16)
    route = layer.last_route()
    scores = layer.last_scores()
    if host_W is None:
        host_W = oracle_weights_from_device(cfg, dev_w, route["idx"].reshape(-1))
    # router: logits order restated exactly in the oracle -> scores, ids, weights, dispatch bit-exact
    lg = O.router_logits(host_W["router_w"], x_bits)
    s_ref, idx_ref, w_ref = O.router_select(lg, host_W["router_bias"], cfg.topk, cfg.n_groups, cfg.topk_groups,
                                            cfg.score_fn, cfg.route_scale)
    assert np.array_equal(scores.view(np.uint32), s_ref.view(np.uint32)), "router scores differ"
    assert np.array_equal(route["idx"], idx_ref), "expert ids differ"
    assert np.array_equal(route["weights"].view(np.uint32), w_ref.view(np.uint32)), "routing weights differ"
    counts, offsets, perm = O.dispatch(idx_ref, cfg.n_experts)
    assert np.array_equal(route["counts"], counts)
    assert np.array_equal(route["offsets"], offsets)
    assert np.array_equal(route["perm"], perm), "dispatch permutation differs"
    y_ref, idx2, _ = O.moe_forward(cfg.as_dict(), host_W, x_bits)
    assert np.array_equal(idx2, idx_ref)
    rel, same, ulps = compare_y(y_bits, y_ref)
    assert rel <= TOL, f"max-abs-rel {rel:.3e} (bit-identical fraction {same:.4f}, max {ulps:.1f} bf16 ulps)"
    check_quantizers(cfg, layer, x_bits)
    assert layer.status() == 0
    return rel, same


def check_quantizers(cfg, layer, x_bits):
    """The layer's act_quant steps, read back as the expert kernels consume them, equal the oracle's
    act_quant (pinned bit-exact to ref/kernel.py by tests/test_oracle_golden.py) applied to the same
    input: x per token for the routed and the shared experts; h (the bf16 values the up kernels
    produced, read back too) per dispatch position and per shared-expert token.  Codes and scales
    bit for bit: per-128 fp32 amax/448 for FP8 128x128 weights, per-32 power-of-two for MXFP4 and
    FP8-e8m0 weights."""
    xf = O.bf16_bits_to_f32(x_bits)
    kinds = [(MoELayer.ACTS_X_ROUTED, cfg.routed_fmt), (MoELayer.ACTS_H_ROUTED, cfg.routed_fmt)]
    if cfg.shared_fmt != FMT_NONE:
        kinds += [(MoELayer.ACTS_X_SHARED, cfg.shared_fmt), (MoELayer.ACTS_H_SHARED, cfg.shared_fmt)]
    for which, fmt in kinds:
        a = layer.last_acts(which)
        if "h" in a:
            src = O.bf16_bits_to_f32(a["h"])
            assert np.any(a["h"] != 0), f"acts {which}: h was not written"
        else:
            src = xf
        if a["rule"] == "q8":
            # the Q8 rule (ref/emulate_ds4.py:23-30): int8 codes, fp32 scale amax / 127 per 32
            q, scales = O.q8_codes(src)
            codes = q.view(np.uint8)
        else:
            codes, scales = O.act_quant(src, a["blk"], fmt != FMT_FP8_B128)
        assert np.array_equal(a["codes"], codes), f"acts {which}: codes differ at {np.argwhere(a['codes'] != codes)[:4]}"
        assert np.array_equal(a["scales"].view(np.uint32), scales.view(np.uint32)), f"acts {which}: scales differ"


@pytest.fixture(scope="module")
def small_layers():
    out = {}
    for cfg in (CFG1, CFG1_FP4):
        W = synth.host_layer(cfg)
        dev = host_weights_to_device(cfg, W)
        out[cfg.name] = (W, dev, MoELayer(cfg, dev, max_tokens=64))
    return out


@pytest.mark.parametrize("name", ["cfg1", "cfg1_fp4"])
@pytest.mark.parametrize("T", [1, 4, 5, 16, 17, 40, 64])  # 17, 40: ragged 32-token chunks (MXFP4)
def test_small_layer_parity(small_layers, name, T):
    W, dev, layer = small_layers[name]
    cfg = layer.cfg
    run_and_check(cfg, layer, dev, W, synth.make_x(cfg.hidden, T, seed=100 + T))


@pytest.mark.parametrize("name,golden_name", [("cfg1", "layer_cfg1"), ("cfg1_fp4", "layer_cfg1_fp4")])
def test_small_layer_matches_reference_golden(small_layers, golden, name, golden_name):
    """The GPU layer against the reference's own torch composition (fixture from ref/kernel.py)."""
    W, dev, layer = small_layers[name]
    g = golden(golden_name)
    x = torch.from_numpy(g["x"].view(np.int16)).cuda()
    y = layer(x)
    torch.cuda.synchronize()
    route = layer.last_route()
    assert np.array_equal(route["idx"], g["idx"])
    np.testing.assert_allclose(route["weights"], g["w"], rtol=1e-6)
    rel, _, _ = compare_y(y.view(torch.int16).cpu().numpy().view(np.uint16), g["y"])
    assert rel <= TOL


def test_repeat_is_bitwise_deterministic(small_layers):
    W, dev, layer = small_layers["cfg1"]
    x = torch.from_numpy(synth.make_x(1024, 16, seed=7).view(np.int16)).cuda()
    a = layer(x).clone()
    b = layer(x).clone()
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_forward_host_matches_device(small_layers):
    W, dev, layer = small_layers["cfg1"]
    xb = synth.make_x(1024, 8, seed=9)
    y_host = layer.forward_host(xb)
    y_dev = layer(torch.from_numpy(xb.view(np.int16)).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(y_host, y_dev.view(torch.int16).cpu().numpy().view(np.uint16))


def test_planted_router_ties(small_layers):
    """Identical router rows give identical logits: ties must go to the lower expert id, as in the
    reference's partial_sort comparator (stbl/model.cu:444-449)."""
    W, dev, _ = small_layers["cfg1"]
    cfg = CFG1
    W2 = dict(W)
    rw = W["router_w"].copy()
    rw[5] = rw[2]
    rw[9] = rw[2]
    rw[13] = rw[1]
    W2["router_w"] = rw
    W2["router_bias"] = np.zeros_like(W["router_bias"])
    dev2 = dict(dev)
    dev2["router_w"] = torch.from_numpy(rw).cuda()
    dev2["router_bias"] = torch.zeros_like(dev["router_bias"])
    layer = MoELayer(cfg, dev2, max_tokens=16)
    run_and_check(cfg, layer, dev2, W2, synth.make_x(1024, 16, seed=11))
    layer.close()


@pytest.fixture(scope="module")
def cfg2_layer():
    dev = synth.device_layer(CFG2)
    layer = MoELayer(CFG2, dev, max_tokens=256)
    yield dev, layer
    layer.close()
    del dev
    torch.cuda.empty_cache()


@pytest.mark.parametrize("T", [1, 4, 16, 64])  # 64: gathered activations, experts with several chunks
def test_full_size_fp8_layer(cfg2_layer, T):
    dev, layer = cfg2_layer
    run_and_check(CFG2, layer, dev, None, synth.make_x(CFG2.hidden, T, seed=200 + T))


@pytest.mark.parametrize("zipf", [0.0, 1.2])
def test_full_size_cfg4_single_gpu(cfg2_layer, zipf):
    """configs[3] on one GPU: the full-size FP8 layer at T = 256 (gathered activations; under
    Zipf(1.2) popular experts hold many 16-token chunks), uniform routing (bias 0) and Zipf(1.2)."""
    dev, _ = cfg2_layer
    cfg = dataclasses.replace(CFG2, name="cfg4", bias_std=0.0, zipf_s=zipf)
    dev4 = dict(dev)
    dev4["router_bias"] = torch.from_numpy(synth.router_bias(cfg)).cuda()
    layer = MoELayer(cfg, dev4, max_tokens=256)
    run_and_check(cfg, layer, dev4, None, synth.make_x(cfg.hidden, 256, seed=400 + int(10 * zipf)))
    layer.close()


def route_report(got_idx, want_idx, margin):
    """Route mismatches as stbl/test_layers.py:105 reports them: (token, reference margin, ids in one
    route but not the other), compared as sets of ids."""
    flips = []
    for t in range(want_idx.shape[0]):
        a, b = set(got_idx[t].tolist()), set(want_idx[t].tolist())
        if a != b:
            flips.append((t, float(margin[t]), sorted(a ^ b)))
    return flips


@pytest.mark.parametrize("rule", ["v3", "sp"])
def test_full_size_routes_match_reference_composition(cfg2_layer, golden, rule):
    """The full-size router against the routes of the torch composition the reference's harness uses
    (fp32 x @ W^T, score, + bias, top-k; tests/golden/make_route_golden.py), 256 tokens: v3 = the
    group-limited sigmoid gate, sp = the reference engine's sqrt(softplus) flat top-8.  A mismatch is
    allowed only where the reference's own selection margin is below what fp32 summation order can
    move (1e-5); the report lists every mismatch with its margin."""
    dev, _ = cfg2_layer
    g = golden("route_cfg2")
    cfg = CFG2 if rule == "v3" else dataclasses.replace(CFG2, name="cfg2_sp", score_fn=SCORE_SQRT_SOFTPLUS,
                                                         n_groups=1, topk_groups=1)
    T = int(g["T"])
    xb = synth.make_x(cfg.hidden, T, seed=int(g["x_seed"]))
    layer = MoELayer(cfg, dev, max_tokens=T) if rule == "sp" else cfg2_layer[1]
    layer(torch.from_numpy(xb.view(np.int16)).cuda())
    route = layer.last_route()
    want, margin = g["idx_" + rule], g["margin_" + rule]
    flips = route_report(route["idx"], want, margin)
    print(f"\n{rule}: route mismatches {len(flips)}/{T} (token, ref margin, differing ids): {flips}")
    assert all(m < 1e-5 for _, m, _ in flips), flips
    same = [t for t in range(T) if set(route["idx"][t].tolist()) == set(want[t].tolist())]
    assert np.array_equal(route["idx"][same], want[same]), "same experts in a different order"
    np.testing.assert_allclose(route["weights"][same], g["w_" + rule][same], rtol=1e-5)
    assert layer.status() == 0
    if rule == "sp":
        layer.close()


def test_full_size_fp8_device_quantization_matches_oracle(cfg2_layer):
    """The GPU-side synthetic quantizer (torch on the device) agrees byte for byte with the oracle's."""
    dev, _ = cfg2_layer
    g = torch.Generator(device="cuda")
    g.manual_seed(1234)
    w = torch.randn(256, 1024, generator=g, device="cuda") * 0.02
    c, s = synth.quant_fp8_b128(w)
    oc, os_ = O.quant_fp8_b128(w.cpu().numpy())
    assert np.array_equal(c.cpu().numpy(), oc) and np.array_equal(s.cpu().numpy(), os_)


@pytest.fixture(scope="module")
def cfg3_layer():
    dev = synth.device_layer(CFG3)
    layer = MoELayer(CFG3, dev, max_tokens=64)
    yield dev, layer
    layer.close()
    del dev
    torch.cuda.empty_cache()


@pytest.mark.parametrize("T", [1, 4, 16, 64])
def test_full_size_fp4_layer(cfg3_layer, T):
    dev, layer = cfg3_layer
    run_and_check(CFG3, layer, dev, None, synth.make_x(CFG3.hidden, T, seed=300 + T))


@pytest.mark.parametrize("T", [1, 16, 64])
def test_full_size_fp4_layer_q8_activations(cfg3_layer, T):
    """configs[2]'s layer (the same MXFP4 experts) with Q8 activations for the routed experts
    (ref/emulate_ds4.py: int8 per 32, scale amax/127; CUDA-core kernels), FP8 shared expert."""
    dev, _ = cfg3_layer
    layer = MoELayer(CFG3_Q8, dev, max_tokens=64)
    run_and_check(CFG3_Q8, layer, dev, None, synth.make_x(CFG3_Q8.hidden, T, seed=500 + T))
    layer.close()


@pytest.mark.parametrize("name", ["cfg1", "cfg1_fp4"])
def test_expert_slots_repoint_experts(small_layers, name):
    """An expert cache re-points experts at other slots of the expert arrays: with experts 0..15
    reading slots 15..0, the layer must equal the oracle whose expert e has slot 15 - e's weights."""
    W, dev, _ = small_layers[name]
    cfg = CFG1 if name == "cfg1" else CFG1_FP4
    layer = MoELayer(cfg, dev, max_tokens=16)
    E = cfg.n_experts
    for e in range(E):
        layer.set_expert_slot(e, E - 1 - e)
    W2 = dict(W)
    W2["routed"] = [[W["routed"][m][E - 1 - e] for e in range(E)] for m in range(3)]
    run_and_check(cfg, layer, dev, W2, synth.make_x(cfg.hidden, 16, seed=77))
    layer.close()


def test_layer_rejects_bad_calls(small_layers):
    """Calls outside the layer's limits (no tokens, more than max_tokens, unaligned x, no output)
    return -1 with a message and launch nothing; the layer then still computes the same bits as
    before them, with a clean status word."""
    import ctypes

    W, dev, layer = small_layers["cfg1"]
    x = torch.from_numpy(synth.make_x(1024, 16, seed=31).view(np.int16)).cuda()
    y0 = layer(x).clone()
    torch.cuda.synchronize()
    lib, h = layer.lib, layer.handle
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    y = torch.empty_like(y0)
    xp, yp = ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr())
    cases = [
        (xp, 0, yp, b"max_tokens"),                               # no tokens
        (xp, 65, yp, b"max_tokens"),                              # beyond the layer's sizing (64)
        (ctypes.c_void_p(x.data_ptr() + 2), 4, yp, b"aligned"),  # x not on a 16-byte boundary
        (xp, 4, ctypes.c_void_p(0), b"null"),                     # no output
    ]
    for xa, T, ya, msg in cases:
        assert lib.stbl_moe_forward(h, xa, T, ya, st) == -1, (T, msg)
        assert msg in lib.stbl_moe_error(h), lib.stbl_moe_error(h)
    y1 = layer(x)
    torch.cuda.synchronize()
    assert torch.equal(y0.view(torch.int16), y1.view(torch.int16))
    assert layer.status() == 0


@pytest.mark.parametrize("base", ["cfg1", "cfg1_fp4"])
@pytest.mark.parametrize("T", [1, 16, 40])  # 40: 32-token chunks (MXFP4) / the width chosen on the device (FP8)
def test_layer_without_shared_expert(base, T):
    """A layer with no shared expert (shared format none): no shared chunks, the routed experts alone
    in the expert launches, and a combine of the routed rows only, against the oracle's layer."""
    cfg = dataclasses.replace(CFG1 if base == "cfg1" else CFG1_FP4, name=base + "_noshared", shared_fmt=FMT_NONE)
    W = synth.host_layer(cfg)
    dev = host_weights_to_device(cfg, W)
    layer = MoELayer(cfg, dev, max_tokens=64)
    run_and_check(cfg, layer, dev, W, synth.make_x(cfg.hidden, T, seed=300 + T))
    assert layer.status() == 0
    layer.close()
