"""Generate the golden vectors that pin the CPU oracle to the reference.

Run where the reference tree is present (it imports ref/kernel.py, the reference's own torch
stand-ins for its quantizers and GEMMs):

    python tests/golden/make_golden.py [--reference <reference tree>]   (default: STBL_REFERENCE, else ../reference)

Writes small .npz fixtures next to this file.  The tests read only the fixtures; nothing at test
time touches the reference tree.  Layer weights are not stored: they are regenerated from fixed
seeds by stblarge_b200.synth.host_layer, and a SHA-256 of the quantized bytes is stored so the test
can prove it rebuilt exactly the bytes used here.
"""

import argparse
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from stblarge_b200 import synth  # noqa: E402
from stblarge_b200.config import CFG1, CFG1_FP4, FMT_FP8_B128  # noqa: E402


def load_reference(path):
    sys.path.insert(0, os.path.join(path, "ref"))
    import kernel as K  # the reference's ref/kernel.py
    return K


def sha(arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def layer_digest(W):
    arrays = [W["routed"][m][e][i] for m in range(3) for e in range(len(W["routed"][0])) for i in range(2)]
    arrays += [W["shared"][m][i] for m in range(3) for i in range(2)]
    return sha(arrays)


def scalar_cases(K):
    out = {}
    rng = np.random.default_rng(7)
    # pow2_ceil: the reference test's values (ref/test_kernel.py:12-15) plus a random sweep
    t = np.concatenate([np.array([1e-6, 0.25, 0.3, 1.0, 1.0000001, 3.0, 448.0, 1000.0], np.float32),
                        (10.0 ** rng.uniform(-30, 30, 4000)).astype(np.float32),
                        (2.0 ** np.arange(-60, 60)).astype(np.float32)])
    out["pow2_in"] = t
    out["pow2_out"] = K._pow2_ceil(torch.from_numpy(t)).numpy()
    # fp4 rounding on the reference test's grid plus ties and random values (ref/test_kernel.py:18-23)
    v = np.concatenate([np.linspace(-6, 6, 4801, dtype=np.float32),
                        np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -0.0, 0.0], np.float32),
                        rng.uniform(-6, 6, 4000).astype(np.float32)])
    out["fp4_in"] = v
    q = K._round_fp4(torch.from_numpy(v))
    out["fp4_round"] = q.numpy()
    out["fp4_codes"] = K._fp4_codes(q).numpy().astype(np.uint8)
    # e4m3 casts of values within [-448, 448] (the only inputs ref/kernel.py:41 gives the cast):
    # every bf16 value in range, random fp32 values, and the exact midpoints between e4m3 neighbours
    bf = (np.arange(0, 1 << 16, dtype=np.uint32) << 16).view(np.float32)
    bf = bf[np.isfinite(bf) & (np.abs(bf) <= 448)]
    vals = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    grid = np.unique(np.abs(vals[np.isfinite(vals)])).astype(np.float32)
    mids = ((grid[1:] + grid[:-1]) / 2).astype(np.float32)
    e4 = np.concatenate([bf, rng.uniform(-448, 448, 20000).astype(np.float32),
                         np.clip(rng.standard_normal(20000) * 10.0 ** rng.uniform(-4, 2, 20000), -448, 448).astype(np.float32),
                         mids, -mids]).astype(np.float32)
    out["e4m3_in"] = e4
    out["e4m3_codes"] = torch.from_numpy(e4).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return out


def quant_cases(K):
    out = {}
    torch.manual_seed(0)
    # the shape of ref/test_kernel.py:26-35, wider
    x = (torch.randn(6, 1024) * torch.logspace(-3, 3, 1024)).to(torch.bfloat16)
    out["aq_x"] = x.view(torch.int16).numpy().view(np.uint16)
    y, s = K.act_quant(x, 128, None, torch.float32)
    out["aq128_codes"], out["aq128_scales"] = y.view(torch.uint8).numpy(), s.numpy()
    y, s = K.act_quant(x, 32, "ue8m0", torch.float32)
    out["aq32_codes"], out["aq32_scales"] = y.view(torch.uint8).numpy(), s.numpy()
    z = x.clone()
    K.act_quant(z, 32, "ue8m0", torch.float8_e8m0fnu, True)
    out["aq32_inplace"] = z.view(torch.int16).numpy().view(np.uint16)
    # MXFP4 weight quantization (E8M0 branch); the synthetic generator must agree byte for byte
    w = torch.randn(64, 512) * 0.02
    out["fp4w_in"] = w.numpy()
    packed, s = K.fp4_act_quant(w, 32, False, torch.float8_e8m0fnu)
    out["fp4w_packed"], out["fp4w_scales"] = packed.view(torch.uint8).numpy(), s.view(torch.uint8).numpy()
    p2, s2 = synth.quant_mxfp4(w)
    assert np.array_equal(p2.numpy(), out["fp4w_packed"]) and np.array_equal(s2.numpy(), out["fp4w_scales"])
    # FP8 128x128 weight quantization = act_quant's rule (block 128, fp32 scale) on 2-D blocks: check the
    # synthetic generator against act_quant on a [128 x k] slab whose rows share one block row
    w8 = torch.randn(128, 512) * 0.02
    c8, s8 = synth.quant_fp8_b128(w8)
    for j in range(4):
        blk = w8[:, j * 128:(j + 1) * 128].reshape(1, -1)
        yq, ys = K.act_quant(blk, blk.numel(), None, torch.float32)
        assert np.array_equal(yq.view(torch.uint8).numpy().reshape(128, 128), c8[:, j * 128:(j + 1) * 128].numpy())
        assert float(ys.reshape(-1)[0]) == float(s8[0, j])
    out["fp8w_in"], out["fp8w_codes"], out["fp8w_scales"] = w8.numpy(), c8.numpy(), s8.numpy()
    return out


def gemm_cases(K):
    out = {}
    rng = np.random.default_rng(11)
    # fp8_gemm with 128-blocks and fp32 scales (the BASELINE weight format)
    a = torch.from_numpy(rng.standard_normal((5, 1024)).astype(np.float32)).to(torch.bfloat16)
    aq, as_ = K.act_quant(a, 128, None, torch.float32)
    wc, ws = synth.quant_fp8_b128(torch.from_numpy(rng.standard_normal((320, 1024)).astype(np.float32) * 0.02))
    c = K.fp8_gemm(aq, as_, wc.view(torch.float8_e4m3fn), ws, torch.float32, 128).float()
    out.update(g8_w=wc.numpy(), g8_ws=ws.numpy(), g8_aq=aq.view(torch.uint8).numpy(), g8_as=as_.numpy(),
               g8_y=c.numpy())
    # fp4_gemm with per-32 pow2 activation scales (the reference engine's rule for MXFP4 experts)
    aq, as_ = K.act_quant(a, 32, "ue8m0", torch.float32)
    w4 = torch.from_numpy(rng.standard_normal((256, 1024)).astype(np.float32) * 0.02)
    packed, s4 = K.fp4_act_quant(w4, 32, False, torch.float8_e8m0fnu)
    c = K.fp4_gemm(aq, as_, packed, s4, torch.float32, 32).float()
    out.update(g4_w=packed.view(torch.uint8).numpy(), g4_ws=s4.view(torch.uint8).numpy(),
               g4_aq=aq.view(torch.uint8).numpy(), g4_as=as_.numpy(), g4_y=c.numpy())
    return out


def v3_gate(logits, bias, topk, n_groups, topk_groups, route_scale):
    """DeepSeek-V3 group-limited sigmoid gate, restated from the public V3 inference code (the
    reference engine routes V4.1 style, so this rule has no source in the reference)."""
    scores = logits.sigmoid()
    original = scores
    scores = scores + bias
    if n_groups > 1:
        g = scores.view(scores.size(0), n_groups, -1).topk(2, dim=-1)[0].sum(dim=-1)
        keep = g.topk(topk_groups, dim=-1)[1]
        mask = torch.ones_like(g, dtype=torch.bool).scatter_(1, keep, False)
        scores = scores.view(scores.size(0), n_groups, -1).masked_fill(mask.unsqueeze(-1), float("-inf")).flatten(1)
    idx = scores.topk(topk, dim=-1)[1]
    w = original.gather(1, idx)
    w = w / (w.sum(dim=-1, keepdim=True) + 1e-20)
    return idx, w * route_scale


def layer_case(K, cfg, T, seed_x):
    """The MoE layer composed as stbl/model.cu:426-594 does, on the reference's torch stand-ins:
    routed experts gate/up -> SwiGLU with the routing weight folded in -> act_quant -> down; shared
    expert; fp32 sum in top-k order, plus shared, one bf16 rounding."""
    W = synth.host_layer(cfg)
    x = synth.make_x(cfg.hidden, T, seed_x)
    xb = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16)
    logits = xb.float() @ torch.from_numpy(W["router_w"]).t()
    idx, wts = v3_gate(logits, torch.from_numpy(W["router_bias"]), cfg.topk, cfg.n_groups, cfg.topk_groups,
                       cfg.route_scale)
    torch.set_default_dtype(torch.bfloat16)  # the GEMMs return the model dtype, as in the reference harness

    def gemm(fmt, a, w):
        c, s = torch.from_numpy(w[0]), torch.from_numpy(w[1])
        if fmt == FMT_FP8_B128:
            aq, as_ = K.act_quant(a, 128, None, torch.float32)
            return K.fp8_gemm(aq, as_, c.view(torch.float8_e4m3fn), s, torch.float32, 128)
        aq, as_ = K.act_quant(a, 32, "ue8m0", torch.float32)
        return K.fp4_gemm(aq, as_, c.view(torch.float4_e2m1fn_x2), s.view(torch.float8_e8m0fnu), torch.float32, 32)

    def expert(fmt, ws, a, wt):
        g = gemm(fmt, a, ws[0]).float()
        u = gemm(fmt, a, ws[1]).float()
        h = (g / (1 + torch.exp(-g)) * u * wt[:, None]).to(torch.bfloat16)
        return gemm(fmt, h, ws[2]).float()

    acc = torch.zeros(T, cfg.hidden, dtype=torch.float32)
    for s in range(cfg.topk):
        for t in range(T):
            e = int(idx[t, s])
            ws = [W["routed"][m][e] for m in range(3)]
            acc[t] = acc[t] + expert(cfg.routed_fmt, ws, xb[t:t + 1], wts[t:t + 1, s].float())[0]
    sh = expert(cfg.shared_fmt, W["shared"], xb, torch.ones(T))
    y = (acc + sh).to(torch.bfloat16)
    torch.set_default_dtype(torch.float32)
    return dict(x=x, logits=logits.numpy(), idx=idx.numpy().astype(np.int32), w=wts.float().numpy(),
                y=y.view(torch.int16).numpy().view(np.uint16), weights_sha256=np.array(layer_digest(W)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("STBL_REFERENCE", os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "..", "reference")))
    args = ap.parse_args()
    K = load_reference(args.reference)
    torch.set_num_threads(1)  # reproducible summation inside the torch GEMMs
    np.savez_compressed(os.path.join(HERE, "scalars.npz"), **scalar_cases(K))
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **quant_cases(K))
    np.savez_compressed(os.path.join(HERE, "gemm.npz"), **gemm_cases(K))
    for name, cfg in (("layer_cfg1", CFG1), ("layer_cfg1_fp4", CFG1_FP4)):
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **layer_case(K, cfg, 4, 4))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
