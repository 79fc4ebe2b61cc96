"""stbl_route_noalloc: routing for callers that cannot allocate device memory (an engine with its
own fixed memory pool, a runtime without an allocator).  Its working
memory is a fixed array inside the library; this test calls it through the C ABI and checks, on two
calls in a row, that it returns exactly the routing of the regular layer entry point
(stbl_moe_forward + stbl_moe_last_route): expert ids, weights, counts, offsets and the dispatch
permutation, bit for bit, which is the tolerance the routing tests use; that the status word the
router kernels raise reads 0 after each call (stbl_route_noalloc_status); that the full-size router
(256 experts, hidden 7168) at the array's token limit (64) equals the CPU oracle bit for bit; and
that sizes beyond the array's limit are refused.  Collected last so that a failure here leaves every
other test already run; it needs nothing from the other test files."""

import ctypes

import numpy as np
import pytest
import torch

from stblarge_b200 import lib as L
from stblarge_b200 import synth
from oracle import oracle as O
from stblarge_b200.config import CFG1, CFG2
from stblarge_b200.moe import MoELayer, host_weights_to_device

pytestmark = pytest.mark.gpu


def route_noalloc(lib, cfg, dev, x):
    T = x.shape[0]
    idx = torch.empty(T, cfg.topk, dtype=torch.int32, device="cuda")
    w = torch.empty(T, cfg.topk, dtype=torch.float32, device="cuda")
    counts = torch.empty(cfg.n_experts, dtype=torch.int32, device="cuda")
    offsets = torch.empty(cfg.n_experts + 1, dtype=torch.int32, device="cuda")
    perm = torch.empty(T * cfg.topk, dtype=torch.int32, device="cuda")
    err = ctypes.create_string_buffer(256)
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.stbl_route_noalloc(dev["router_w"].data_ptr(), dev["router_bias"].data_ptr(), x.data_ptr(), T,
                                cfg.n_experts, cfg.hidden, cfg.topk, cfg.n_groups, cfg.topk_groups, cfg.score_fn,
                                cfg.route_scale, idx.data_ptr(), w.data_ptr(), counts.data_ptr(), offsets.data_ptr(),
                                perm.data_ptr(), st, err, 256)
    assert rc == 0, err.value.decode()
    status = ctypes.c_uint32(123)
    assert lib.stbl_route_noalloc_status(ctypes.byref(status)) == 0
    assert status.value == 0, f"router status bits {status.value:#x}"
    return {"idx": idx.cpu().numpy(), "weights": w.cpu().numpy(), "counts": counts.cpu().numpy(),
            "offsets": offsets.cpu().numpy(), "perm": perm.cpu().numpy()}


def test_noalloc_routing_matches_layer_on_two_calls():
    lib = L.load()
    cfg = CFG1
    dev = host_weights_to_device(cfg, synth.host_layer(cfg))
    layer = MoELayer(cfg, dev, max_tokens=64)
    for call, (T, seed) in enumerate(((16, 501), (5, 502))):
        x = torch.from_numpy(synth.make_x(cfg.hidden, T, seed=seed).view(np.int16)).cuda()
        layer(x)
        want = layer.last_route()
        got = route_noalloc(lib, cfg, dev, x)
        for k in ("idx", "counts", "offsets", "perm"):
            assert np.array_equal(got[k], want[k]), (call, k)
        assert np.array_equal(got["weights"].view(np.uint32), want["weights"].view(np.uint32)), call
    layer.close()


def test_noalloc_full_size_at_its_token_limit_matches_oracle():
    """The full-size router (configs[1]: 256 experts, hidden 7168, top-8 of 8 groups keeping 4) at
    T = 64, the array's limit, on two calls in a row, against the CPU oracle's restatement of the
    router (logits order, scores, selection, weights, dispatch) bit for bit."""
    lib = L.load()
    cfg = CFG2
    dev = {"router_w": torch.from_numpy(synth.router_w(cfg)).cuda(),
           "router_bias": torch.from_numpy(synth.router_bias(cfg)).cuda()}
    for call, seed in enumerate((611, 612)):
        xb = synth.make_x(cfg.hidden, 64, seed=seed)
        got = route_noalloc(lib, cfg, dev, torch.from_numpy(xb.view(np.int16)).cuda())
        lg = O.router_logits(synth.router_w(cfg), xb)
        _, idx, w = O.router_select(lg, synth.router_bias(cfg), cfg.topk, cfg.n_groups, cfg.topk_groups,
                                    cfg.score_fn, cfg.route_scale)
        counts, offsets, perm = O.dispatch(idx, cfg.n_experts)
        assert np.array_equal(got["idx"], idx), call
        assert np.array_equal(got["weights"].view(np.uint32), w.view(np.uint32)), call
        assert np.array_equal(got["counts"], counts) and np.array_equal(got["offsets"], offsets), call
        assert np.array_equal(got["perm"], perm), call


def test_noalloc_rejects_sizes_beyond_its_array():
    lib = L.load()
    cfg = CFG1
    dev = host_weights_to_device(cfg, synth.host_layer(cfg))
    x = torch.zeros(65, cfg.hidden, dtype=torch.int16, device="cuda")
    out = torch.empty(65 * 16, dtype=torch.int32, device="cuda")
    err = ctypes.create_string_buffer(256)
    rc = lib.stbl_route_noalloc(dev["router_w"].data_ptr(), dev["router_bias"].data_ptr(), x.data_ptr(), 65,
                                cfg.n_experts, cfg.hidden, cfg.topk, cfg.n_groups, cfg.topk_groups, cfg.score_fn,
                                cfg.route_scale, out.data_ptr(), out.data_ptr(), out.data_ptr(), out.data_ptr(),
                                out.data_ptr(), torch.cuda.current_stream().cuda_stream, err, 256)
    assert rc == -1 and b"T must be" in err.value
