"""A small, profiler-friendly case of the MoE layer: full-size expert shapes (hidden 7168,
moe_intermediate 2048, FP8 128x128 or MXFP4) but only a few routed experts resident, so that a
capture under ncu holds under 2 GB of device memory and ends in seconds.

    python -m stblarge_b200.profile_case [--experts 16] [--tokens 1] [--calls 3] [--fmt fp8|fp4]

Each call is preceded by a 256 MB write that flushes L2.  Prints the per-kernel device times.
"""

import argparse
import dataclasses

import numpy as np
import torch

from . import synth
from .config import CFG2, CFG3
from .moe import MoELayer


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--experts", type=int, default=16)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--fmt", default="fp8", choices=["fp8", "fp4"])
    a = ap.parse_args()
    base = CFG2 if a.fmt == "fp8" else CFG3
    E = a.experts
    groups = 8 if E % 8 == 0 and E // 8 >= 2 else 1
    cfg = dataclasses.replace(base, name=f"{base.name}_E{E}", n_experts=E, n_groups=groups,
                              topk_groups=min(4, groups) if groups > 1 else 1)
    dev = synth.device_layer(cfg)
    layer = MoELayer(cfg, dev, max_tokens=max(a.tokens, 1))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    xs = [torch.from_numpy(synth.make_x(cfg.hidden, a.tokens, seed=90 + i).view(np.int16)).cuda()
          for i in range(a.warmup + a.calls)]
    for i in range(a.warmup):
        flush.zero_()
        layer(xs[i])
    torch.cuda.synchronize()
    layer.timing()
    layer.set_timing(True)
    for i in range(a.calls):
        flush.zero_()
        layer(xs[a.warmup + i])
    torch.cuda.synchronize()
    t = layer.timing()
    n = max(t["calls"], 1)
    print(f"{cfg.name} T={a.tokens}: router {t['router'] / n * 1e3:.4f} ms, up {t['up'] / n * 1e3:.4f} ms, "
          f"down {t['down'] / n * 1e3:.4f} ms per call, status {layer.status()}")
    layer.close()


if __name__ == "__main__":
    main()
