"""Layers in the reference engine's own weight formats, through the C ABI on the GPU.

The reference (DeepSeek-V4.1 engine) keeps routed experts as MXFP4 in GGUF 17-byte blocks and the shared
expert as FP8 with e8m0 32x32 block scales, quantizes activations per 32 with power-of-two scales and
routes by sqrt(softplus) scores without a group limit.  Layers built that way (cfg1_ref, cfg3_ref) and
with FP8-e8m0 routed experts too (cfg1_e8) must match the oracle: ids, weights and dispatch bit-exact,
outputs within the tolerance.  GGUF blocks load through stbl_mxfp4_from_gguf, checked against the
reference converter's own output (tests/golden/gguf_mxfp4.npz) and end to end: a layer loaded from the
blocks gives the same bits as one loaded from the official layout."""

import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from stblarge_b200 import lib as L
from stblarge_b200 import synth
from stblarge_b200.config import CFG1_E8, CFG1_REF, CFG3_REF
from stblarge_b200.moe import MoELayer, host_weights_to_device
from tests.test_gpu_layer import run_and_check

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "gguf_mxfp4.npz")
CFGS = {c.name: c for c in (CFG1_REF, CFG1_E8)}


@pytest.fixture(scope="module")
def ref_layers():
    out = {}
    for cfg in CFGS.values():
        W = synth.host_layer(cfg)
        dev = host_weights_to_device(cfg, W)
        out[cfg.name] = (W, dev, MoELayer(cfg, dev, max_tokens=64))
    yield out
    for _, _, layer in out.values():
        layer.close()


@pytest.mark.parametrize("name", list(CFGS))
@pytest.mark.parametrize("T", [1, 4, 16, 17, 40, 64])  # > 16: chunks of up to 32 tokens, shared expert's too
def test_reference_format_layer_parity(ref_layers, name, T):
    W, dev, layer = ref_layers[name]
    run_and_check(CFGS[name], layer, dev, W, synth.make_x(CFGS[name].hidden, T, seed=600 + T))


@pytest.mark.parametrize("T", [1, 16])
def test_full_size_reference_format_layer(T):
    dev = synth.device_layer(CFG3_REF)
    layer = MoELayer(CFG3_REF, dev, max_tokens=16)
    run_and_check(CFG3_REF, layer, dev, None, synth.make_x(CFG3_REF.hidden, T, seed=650 + T))
    layer.close()
    del dev
    torch.cuda.empty_cache()


def _from_gguf(blocks_dev, rows, k):
    codes = torch.empty(rows, k // 2, dtype=torch.uint8, device="cuda")
    scales = torch.empty(rows, k // 32, dtype=torch.uint8, device="cuda")
    rc = L.load().stbl_mxfp4_from_gguf(ctypes.c_void_p(blocks_dev.data_ptr()), rows, k, ctypes.c_void_p(codes.data_ptr()),
                                       ctypes.c_void_p(scales.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    return codes, scales


def test_gguf_conversion_matches_reference_converter():
    g = np.load(GOLDEN)
    rows, k = g["codes"].shape[0], g["codes"].shape[1] * 2
    codes, scales = _from_gguf(torch.from_numpy(g["blocks"]).cuda(), rows, k)
    torch.cuda.synchronize()
    assert np.array_equal(codes.cpu().numpy(), g["codes"]) and np.array_equal(scales.cpu().numpy(), g["scales"])


def test_layer_loaded_from_gguf_blocks_is_bit_identical(ref_layers):
    cfg = CFG1_REF
    W, dev, layer = ref_layers[cfg.name]
    # the routed experts as the reference engine stores them, then loaded through the converter
    dev2 = dict(dev)
    dev2["routed_w"], dev2["routed_s"] = [], []
    for m in range(3):
        rows, k = W["routed"][m][0][0].shape[0], W["routed"][m][0][0].shape[1] * 2
        blocks = np.stack([O.mxfp4_to_gguf(*W["routed"][m][e]) for e in range(cfg.n_experts)])  # [E][rows][k/32][17]
        codes, scales = _from_gguf(torch.from_numpy(blocks.reshape(cfg.n_experts * rows, k // 32, 17)).cuda(),
                                   cfg.n_experts * rows, k)
        dev2["routed_w"].append(codes.view(cfg.n_experts, rows, k // 2))
        dev2["routed_s"].append(scales.view(cfg.n_experts, rows, k // 32))
    layer2 = MoELayer(cfg, dev2, max_tokens=4)
    x = torch.from_numpy(synth.make_x(cfg.hidden, 4, seed=77).view(np.int16)).cuda()
    y1, y2 = layer(x), layer2(x)
    torch.cuda.synchronize()
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))
    assert layer2.status() == 0
    layer2.close()
