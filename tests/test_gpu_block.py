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
    layer = MoELayer(cfg, dev, max_tokens=16)
    eps, hc = 1e-6, 4
    ref = ctypes.CDLL(REF_SO) if os.path.exists(REF_SO) else None
    for T, seed in ((1, 1), (5, 2), (16, 3)):
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
