"""Generate the full-size routing fixture (tests/golden/route_cfg2.npz).

    python tests/golden/make_route_golden.py

The routes of 256 decode tokens through the full-size router (256 experts, hidden 7168), computed by
torch on the CPU the way the reference's own harness composes routing (stbl/test_layers.py:64-66:
fp32 logits x @ W^T, score function, + bias, top-k), for both rules the layer implements:

  * v3: sigmoid scores, group-limited top-8 (8 groups, 4 kept), the DeepSeek-V3 gate restated in
    make_golden.v3_gate (the reference engine routes V4.1 style, so this rule has no source there);
  * sp: the reference engine's rule (stbl/model.cu:430-452): sqrt(softplus(logit)) + bias, flat top-8.

For every token it also stores the selection margin the reference reports beside each route
mismatch (stbl/test_layers.py:65-66, 105): the k-th minus the (k+1)-th biased score among the
eligible experts, and for v3 the margin of the group selection (the topk_groups-th minus the next
group score).  Inputs are not stored: the router weights, bias and tokens are regenerated from
their seeds by stblarge_b200.synth, and a SHA-256 of them is stored so the test proves it rebuilt the
same bytes.  The fixture needs no reference tree (no reference function computes these rules on the
CPU beyond the composition restated here).
"""

import hashlib
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)
from make_golden import v3_gate  # noqa: E402

from stblarge_b200 import synth  # noqa: E402
from stblarge_b200.config import CFG2  # noqa: E402

T = 256
X_SEED = 4242


def inputs():
    cfg = CFG2
    W, b = synth.router_w(cfg), synth.router_bias(cfg)
    x = synth.make_x(cfg.hidden, T, seed=X_SEED)
    h = hashlib.sha256()
    for a in (W, b, x):
        h.update(np.ascontiguousarray(a).tobytes())
    return W, b, x, h.hexdigest()


def main():
    torch.set_num_threads(1)  # one fixed summation order for the fp32 logits
    cfg = CFG2
    W, b, x, digest = inputs()
    xb = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16)
    logits = xb.float() @ torch.from_numpy(W).t()
    bias = torch.from_numpy(b)
    k = cfg.topk

    # v3: group-limited sigmoid gate
    idx_v3, w_v3 = v3_gate(logits, bias, k, cfg.n_groups, cfg.topk_groups, cfg.route_scale)
    s = logits.sigmoid() + bias
    gs = s.view(T, cfg.n_groups, -1).topk(2, dim=-1)[0].sum(dim=-1)
    gsorted = gs.sort(dim=-1, descending=True)[0]
    gmargin = gsorted[:, cfg.topk_groups - 1] - gsorted[:, cfg.topk_groups]
    keep = gs.topk(cfg.topk_groups, dim=-1)[1]
    mask = torch.ones_like(gs, dtype=torch.bool).scatter_(1, keep, False)
    sm = s.view(T, cfg.n_groups, -1).masked_fill(mask.unsqueeze(-1), float("-inf")).flatten(1)
    top = sm.topk(k + 1, dim=-1)[0]
    margin_v3 = top[:, k - 1] - top[:, k]

    # sp: the reference engine's sqrt(softplus) + bias, flat top-k, unbiased renormalised weights
    sc = F.softplus(logits).sqrt()
    top_sp = (sc + bias).topk(k + 1, dim=-1)
    idx_sp = top_sp[1][:, :k]
    margin_sp = top_sp[0][:, k - 1] - top_sp[0][:, k]
    w_sp = sc.gather(1, idx_sp)
    w_sp = w_sp / (w_sp.sum(dim=-1, keepdim=True) + 1e-20) * cfg.route_scale

    np.savez_compressed(os.path.join(HERE, "route_cfg2.npz"),
                        inputs_sha256=np.array(digest), x_seed=np.int64(X_SEED), T=np.int64(T),
                        idx_v3=idx_v3.numpy().astype(np.int32), w_v3=w_v3.float().numpy(),
                        margin_v3=margin_v3.numpy(), gmargin_v3=gmargin.numpy(),
                        idx_sp=idx_sp.numpy().astype(np.int32), w_sp=w_sp.float().numpy(),
                        margin_sp=margin_sp.numpy())
    print("route_cfg2.npz written; smallest margins v3 %.2e (groups %.2e), sp %.2e"
          % (float(margin_v3.min()), float(gmargin.min()), float(margin_sp.min())))


if __name__ == "__main__":
    main()
