"""The reference engine's weight formats in the oracle (CPU): the GGUF MXFP4 17-byte blocks against the
reference converter's own output (tests/golden/gguf_mxfp4.npz, made by make_gguf_golden.py with
tools/convert_official.py), and FP8 with e8m0 32x32 block scales (quantizer and GEMV)."""

import os

import numpy as np
import torch

from oracle import oracle as O
from stblarge_b200 import synth
from stblarge_b200.config import CFG1_E8, CFG1_REF

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "gguf_mxfp4.npz")


def test_gguf_blocks_match_the_reference_converter():
    g = np.load(GOLDEN)
    assert np.array_equal(O.mxfp4_to_gguf(g["codes"], g["scales"]), g["blocks"])
    codes, scales = O.mxfp4_from_gguf(g["blocks"])
    assert np.array_equal(codes, g["codes"]) and np.array_equal(scales, g["scales"])


def test_fp8_e8m0_quantizer_device_generator_equals_oracle():
    rng = np.random.default_rng(5)
    for rows, k in ((96, 512), (70, 256)):  # 70: a last 32-row block that is partly empty
        w = (rng.standard_normal((rows, k)) * 0.02).astype(np.float32)
        c, s = synth.quant_fp8_e8m0(torch.from_numpy(w))
        oc, os_ = O.quant_fp8_e8m0(w)
        assert np.array_equal(c.numpy(), oc) and np.array_equal(s.numpy(), os_)


def test_fp8_e8m0_gemv_equals_dequantized_product():
    rng = np.random.default_rng(6)
    rows, k, T = 64, 256, 3
    codes, scales = O.quant_fp8_e8m0((rng.standard_normal((rows, k)) * 0.02).astype(np.float32))
    xc, xs = O.act_quant(rng.standard_normal((T, k)).astype(np.float32), 32, True)
    y = O.gemv_fp8_e8m0(codes, scales, xc, xs, 32)
    lut = O.e4m3_values().astype(np.float64)
    W = lut[codes] * np.repeat(np.repeat(2.0 ** (scales.astype(np.float64) - 127), 32, 0)[:rows], 32, 1)
    X = lut[xc] * np.repeat(xs.astype(np.float64), 32, 1)
    assert np.allclose(y, X @ W.T, rtol=1e-5, atol=1e-6)


def test_reference_format_layers_run_on_the_oracle():
    for cfg in (CFG1_REF, CFG1_E8):
        W = synth.host_layer(cfg)
        y, idx, w = O.moe_forward(cfg.as_dict(), W, synth.make_x(cfg.hidden, 2, seed=7))
        assert y.shape == (2, cfg.hidden) and idx.shape == (2, cfg.topk) and np.isfinite(O.bf16_bits_to_f32(y)).all()
