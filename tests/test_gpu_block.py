"""The layer inside its transformer block (stbl_moe_forward_block): RMSNorm fused into the router
kernel, the hyper-connection post into the combine kernel.  The result must be bit-identical to the
unfused sequence the reference runs (stbl/model.cu:803-805) -- the reference's own k_rms_norm, this
layer on its bf16 output, the reference's own k_hc_post per token -- with the reference's kernels
built from its sources into oracle/_ref; without them, against the oracle's restatements (the norm
within one bf16 step, see tests/test_oracle_block.py)."""

import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from stblarge_b200 import synth
from stblarge_b200.config import CFG1, CFG1_REF
from stblarge_b200.moe import MoELayer

pytestmark = pytest.mark.gpu

REF_SO = os.path.join(os.path.dirname(O.HERE), "oracle", "_ref", "libstbl_ref_kernels.so")
P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def block_inputs(cfg, T, hc, seed):
    g = torch.Generator().manual_seed(seed)
    x_pre = (torch.randn(T, cfg.hidden, generator=g) * 3.0).bfloat16().float()  # hc_pre outputs are bf16 values
    norm_w = 1.0 + 0.1 * torch.randn(cfg.hidden, generator=g)
    res = torch.randn(T, hc, cfg.hidden, generator=g).bfloat16().float()
    post = torch.rand(T, hc, generator=g) * 2.0
    comb = torch.rand(T, hc, hc, generator=g)
    return [t.cuda() for t in (x_pre, norm_w, res, post, comb)]


@pytest.mark.parametrize("cfg", [CFG1_REF, CFG1], ids=["mxfp4_e8m0", "fp8"])
def test_fused_block_equals_the_reference_sequence(cfg):
    dev = synth.device_layer(cfg)
    layer = MoELayer(cfg, dev, max_tokens=64)
    eps, hc = 1e-6, 4
    ref = ctypes.CDLL(REF_SO) if os.path.exists(REF_SO) else None
    for T, seed in ((1, 1), (5, 2), (16, 3), (40, 4)):  # 40: the router stages its normalized rows in two rounds
        x_pre, norm_w, res, post, comb = block_inputs(cfg, T, hc, seed)
        h = layer.forward_block(x_pre, norm_w, eps, res, post, comb)
        torch.cuda.synchronize()
        # the unfused sequence: norm -> layer (bf16 in and out) -> hc_post per token
        if ref is not None:
            xn = torch.empty_like(x_pre)
            ref.stbl_rms_norm(P(xn.data_ptr()), P(x_pre.data_ptr()), P(norm_w.data_ptr()), I(T), I(cfg.hidden), F(eps), P(0))
            torch.cuda.synchronize()
        else:
            xn = torch.from_numpy(O.ref_rms_norm(x_pre.cpu().numpy(), norm_w.cpu().numpy(), eps)).cuda()
        y = layer(xn.bfloat16())
        torch.cuda.synchronize()
        yf = y.float()
        if ref is not None:
            want = torch.empty_like(h)
            for t in range(T):
                ref.stbl_hc_post(P(want[t].data_ptr()), P(yf[t].data_ptr()), P(res[t].data_ptr()), P(post[t].data_ptr()),
                                 P(comb[t].data_ptr()), I(hc), I(cfg.hidden), P(0))
            torch.cuda.synchronize()
            assert torch.equal(h.view(torch.int32), want.view(torch.int32)), f"T={T}: fused block differs from the reference's sequence"
        else:
            want = np.stack([O.ref_hc_post(yf[t].cpu().numpy(), res[t].cpu().numpy(), post[t].cpu().numpy(),
                                           comb[t].cpu().numpy()) for t in range(T)])
            np.testing.assert_allclose(h.cpu().numpy(), want, rtol=2 ** -7, atol=1e-3)
        # the routes of the fused call are those of the unfused call's layer input
        assert layer.status() == 0
    layer.close()


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="the unfused sequence uses the reference's kernels (oracle/_ref)")
@pytest.mark.parametrize("T", [1, 16])
def test_fused_block_saves_the_separate_launches(T, capsys):
    """Device time per block call, L2 flushed: the fused call against the reference's sequence of separate
    launches around this layer (k_rms_norm, the bf16 conversion the layer's interface takes, the layer,
    the fp32 conversion, k_hc_post per token), on a full-shape FP8 layer with 16 experts."""
    import dataclasses

    from stblarge_b200.config import CFG2
    cfg = dataclasses.replace(CFG2, n_experts=16, n_groups=4, topk_groups=2)
    layer = MoELayer(cfg, synth.device_layer(cfg), max_tokens=16)
    ref = ctypes.CDLL(REF_SO)
    hc, eps = 4, 1e-6
    x_pre, norm_w, res, post, comb = block_inputs(cfg, T, hc, 7)
    xn, h = torch.empty_like(x_pre), torch.empty(T, hc, cfg.hidden, device="cuda")
    xb = torch.empty(T, cfg.hidden, dtype=torch.bfloat16, device="cuda")
    y = torch.empty_like(xb)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    st = P(torch.cuda.current_stream().cuda_stream)

    def unfused():
        ref.stbl_rms_norm(P(xn.data_ptr()), P(x_pre.data_ptr()), P(norm_w.data_ptr()), I(T), I(cfg.hidden), F(eps), st)
        xb.copy_(xn)
        layer(xb, y)
        yf = y.float()
        for t in range(T):
            ref.stbl_hc_post(P(h[t].data_ptr()), P(yf[t].data_ptr()), P(res[t].data_ptr()), P(post[t].data_ptr()),
                             P(comb[t].data_ptr()), I(hc), I(cfg.hidden), st)

    def fused():
        layer.forward_block(x_pre, norm_w, eps, res, post, comb, out=h)

    def timed(fn, n=20):
        for _ in range(3):
            fn()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for a, b in ev:
            flush.zero_()
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        return float(np.mean([a.elapsed_time(b) for a, b in ev])) * 1e3

    t_unfused, t_fused = timed(unfused), timed(fused)
    with capsys.disabled():
        print(f"\nblock call, FP8 16 experts, T={T}: unfused {t_unfused:.1f} us, fused {t_fused:.1f} us")
    assert t_fused < t_unfused
    assert layer.status() == 0
    layer.close()


def test_fused_block_on_cached_layers_with_prefetch():
    # the block form on layers whose experts live in a cache fed from a host store, with the shadow
    # next-layer prefetch attached: the same bits as the block form on resident layers
    from stblarge_b200.cache import ExpertCache, host_store
    cfg, L, S, T, hc, eps = CFG1_REF, 2, 10, 2, 4, 1e-6
    E = cfg.n_experts
    store = host_store(cfg, L)
    cache = ExpertCache(cfg, L, S, store)
    resident = [synth.device_layer(cfg, seed_base=1000 + l * E) for l in range(L)]
    plain = [MoELayer(cfg, resident[l], max_tokens=T) for l in range(L)]
    cached = [MoELayer(cfg, resident[l], max_tokens=T, cache=(cache, l)) for l in range(L)]
    side = torch.cuda.Stream()
    cached[0].attach_prefetch(cached[1], 4, 3, side)
    for step in range(4):
        x_pre, norm_w, res, post, comb = block_inputs(cfg, T, hc, 50 + step)
        for l in range(L):
            want = plain[l].forward_block(x_pre, norm_w, eps, res, post, comb)
            got = cached[l].forward_block(x_pre, norm_w, eps, res, post, comb)
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int32), want.view(torch.int32)), f"step {step} layer {l}"
    assert cache.prefetch_stats()["prefetched"] > 0
    for layer in cached + plain:
        assert layer.status() == 0
        layer.close()
    cache.close()
