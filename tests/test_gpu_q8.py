"""The Q8 activation variant on the GPU (routed MXFP4 experts x int8 activations per 32, the
reference's ds4 numerics, ref/emulate_ds4.py): the linear alone (stbl_gemv_mxfp4_q8) against the
reference's own emulation run on the same inputs (tests/golden/q8.npz) and against the oracle's exact
restatement; and the whole small act_q8 layer against the oracle layer, with the layer's own x and h
quantizations read back and checked bit for bit against the Q8 rule."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from stblarge_b200 import lib as L
from stblarge_b200 import synth
from stblarge_b200.config import CFG1_Q8
from stblarge_b200.moe import MoELayer, host_weights_to_device

from test_gpu_layer import run_and_check

pytestmark = pytest.mark.gpu


def gemv_q8(w, ws, q, d):
    lib = L.load()
    rows, k = w.shape[0], w.shape[1] * 2
    T = q.shape[0]
    tw, ts = torch.from_numpy(w).cuda(), torch.from_numpy(ws).cuda()
    tq, td = torch.from_numpy(q).cuda(), torch.from_numpy(d).cuda()
    y = torch.empty(T, rows, dtype=torch.float32, device="cuda")
    rc = lib.stbl_gemv_mxfp4_q8(y.data_ptr(), tw.data_ptr(), ts.data_ptr(), tq.data_ptr(), td.data_ptr(), rows, k, T,
                                torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    return y.cpu().numpy()


def test_gemv_q8_matches_reference_emulation(golden):
    g = golden("q8")
    q, d = O.q8_codes(g["x"])
    assert np.array_equal(q, g["q"])  # the codes the reference's emulation made
    y = gemv_q8(g["codes"], g["scales"], q, d)
    ref = g["y"]
    assert np.abs(y - ref).max() / np.abs(ref).max() <= 1e-6
    orc = O.gemv_mxfp4_q8(g["codes"], g["scales"], q, d)
    assert np.abs(y - orc).max() / np.abs(orc).max() <= 1e-6


@pytest.mark.parametrize("T", [1, 9, 16])
def test_gemv_q8_full_size_rows_against_oracle(T):
    """A full-size gate matrix (2048 x 7168) and tokens in several groups of eight."""
    rng = np.random.default_rng(90 + T)
    w = rng.integers(0, 256, (2048, 7168 // 2), dtype=np.uint8)
    ws = rng.integers(118, 124, (2048, 7168 // 32), dtype=np.uint8)
    q, d = O.q8_codes(rng.standard_normal((T, 7168)).astype(np.float32))
    y = gemv_q8(w, ws, q, d)
    orc = O.gemv_mxfp4_q8(w, ws, q, d)
    assert np.abs(y - orc).max() / np.abs(orc).max() <= 1e-6


@pytest.fixture(scope="module")
def q8_layer():
    W = synth.host_layer(CFG1_Q8)
    dev = host_weights_to_device(CFG1_Q8, W)
    layer = MoELayer(CFG1_Q8, dev, max_tokens=64)
    yield W, dev, layer
    layer.close()


@pytest.mark.parametrize("T", [1, 4, 5, 16, 64])
def test_small_layer_q8_parity(q8_layer, T):
    W, dev, layer = q8_layer
    run_and_check(CFG1_Q8, layer, dev, W, synth.make_x(CFG1_Q8.hidden, T, seed=600 + T))


def test_q8_layer_differs_from_fp8_activations(q8_layer):
    """The act_q8 switch changes the routed numerics (it is not silently the FP8 rule)."""
    W, dev, layer = q8_layer
    import dataclasses
    cfg_fp8 = dataclasses.replace(CFG1_Q8, act_q8=0)
    other = MoELayer(cfg_fp8, dev, max_tokens=16)
    x = torch.from_numpy(synth.make_x(CFG1_Q8.hidden, 16, seed=77).view(np.int16)).cuda()
    a, b = layer(x), other(x)
    torch.cuda.synchronize()
    assert not torch.equal(a.view(torch.int16), b.view(torch.int16))
    other.close()
