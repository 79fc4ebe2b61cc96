"""A layer loaded from a GGUF checkpoint (stblarge_b200/gguf.py: load_moe_layer) is the layer built from
the same weights directly: same device tensors after the on-device MXFP4 block conversion, same
routes and bit-identical outputs, and within tolerance of the oracle.  The file is written in the
reference converter's names and types (tools/convert_official.py:116-126) with the reference
engine's SwiGLU clamp set, for a layer in its own formats (MXFP4 routed, FP8-e8m0 shared)."""

import dataclasses

import numpy as np
import pytest
import torch

from oracle import oracle as O
from stblarge_b200 import gguf as G
from stblarge_b200 import synth
from stblarge_b200.config import CFG1_REF
from stblarge_b200.moe import MoELayer
from tests.test_gpu_layer import TOL, compare_y, oracle_weights_from_device

pytestmark = pytest.mark.gpu


def write_layer_file(path, cfg, dev, layers=2):
    tensors = []
    for layer in range(layers):
        experts = []
        for m in range(3):
            codes, scales = dev["routed_w"][m].cpu().numpy(), dev["routed_s"][m].cpu().numpy()
            E, rows, kh = codes.shape
            experts.append(O.mxfp4_to_gguf(codes.reshape(E * rows, kh), scales.reshape(E * rows, -1)).reshape(E, rows, -1))
        shared = [(dev["shared_w"][m].cpu().numpy(), dev["shared_s"][m].cpu().numpy()) for m in range(3)]
        bias = dev["router_bias"].cpu().numpy() + np.float32(layer)  # layers differ
        tensors += G.moe_layer_tensors(layer, dev["router_w"].cpu().numpy(), bias, shared, experts)
    G.write_gguf(path, G.moe_metadata(cfg, layers), tensors)


def test_layer_from_gguf_equals_layer_from_its_tensors(tmp_path):
    cfg = dataclasses.replace(CFG1_REF, swiglu_limit=10.0)
    dev = synth.device_layer(cfg)
    path = tmp_path / "layer.gguf"
    write_layer_file(path, cfg, dev)
    with G.GgufFile(path) as g:
        cfg_g, w = G.load_moe_layer(g, 0)
        _, w1 = G.load_moe_layer(g, 1)
    for f in ("hidden", "inter", "n_experts", "topk", "n_groups", "topk_groups", "score_fn", "route_scale",
              "swiglu_limit", "routed_fmt", "shared_fmt"):
        assert getattr(cfg_g, f) == getattr(cfg, f), f
    for m in range(3):
        for key in ("routed_w", "routed_s", "shared_w", "shared_s"):
            assert torch.equal(w[key][m], dev[key][m]), (key, m)
    assert torch.equal(w["router_w"], dev["router_w"]) and torch.equal(w["router_bias"], dev["router_bias"])
    assert torch.equal(w1["router_bias"], dev["router_bias"] + 1)
    direct, loaded = MoELayer(cfg, dev, max_tokens=8), MoELayer(cfg_g, w, max_tokens=8)
    for T in (1, 5):
        x_bits = synth.make_x(cfg.hidden, T, seed=60 + T)
        x = torch.from_numpy(x_bits.view(np.int16)).cuda()
        y_d, y_l = direct(x), loaded(x)
        torch.cuda.synchronize()
        assert torch.equal(y_l.view(torch.int16), y_d.view(torch.int16))
        route = loaded.last_route()
        W = oracle_weights_from_device(cfg, dev, route["idx"].reshape(-1))
        y_ref, idx_ref, _ = O.moe_forward(cfg.as_dict(), W, x_bits)
        assert np.array_equal(route["idx"], idx_ref)
        rel, _, ulps = compare_y(y_l.view(torch.int16).cpu().numpy().view(np.uint16), y_ref)
        assert rel <= TOL, f"max-abs-rel {rel:.3e} ({ulps:.1f} bf16 ulps)"
    for layer in (direct, loaded):
        assert layer.status() == 0
        layer.close()
