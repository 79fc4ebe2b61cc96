"""A small, profiler-friendly case of the MoE layer: full-size expert shapes (hidden 7168,
moe_intermediate 2048, FP8 128x128, MXFP4, or the reference engine's formats: MXFP4 routed and
FP8-e8m0 shared, sqrt(softplus) scores) but only a few routed experts resident, so that a
capture under ncu holds under 2 GB of device memory and ends in seconds.

    python -m stblarge_b200.profile_case [--experts 16] [--tokens 1] [--calls 3] [--fmt fp8|fp4|ref]
    python -m stblarge_b200.profile_case --router-only [--experts 256] [--tokens 16]

Each call is preceded by a 256 MB write that flushes L2.  Prints the per-kernel device times.
--router-only runs just the router kernel (through stbl_route_noalloc) on the full-size router
(7168 x E fp32), holding about 10 MB of device memory.
"""

import argparse
import ctypes
import dataclasses

import numpy as np
import torch

from . import lib as L
from . import synth
from .config import CFG2, CFG3, CFG3_REF
from .moe import MoELayer


def router_only(a):
    cfg = dataclasses.replace(CFG2, n_experts=a.experts, n_groups=8 if a.experts % 8 == 0 and a.experts >= 16 else 1,
                              topk_groups=4 if a.experts % 8 == 0 and a.experts >= 16 else 1)
    lib = L.load()
    w = torch.from_numpy(synth.router_w(cfg)).cuda()
    b = torch.from_numpy(synth.router_bias(cfg)).cuda()
    T = a.tokens
    idx = torch.empty(T * cfg.topk, dtype=torch.int32, device="cuda")
    wt = torch.empty(T * cfg.topk, dtype=torch.float32, device="cuda")
    counts = torch.empty(cfg.n_experts + 1, dtype=torch.int32, device="cuda")
    offsets = torch.empty(cfg.n_experts + 1, dtype=torch.int32, device="cuda")
    perm = torch.empty(T * cfg.topk, dtype=torch.int32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    err = ctypes.create_string_buffer(256)
    xs = [torch.from_numpy(synth.make_x(cfg.hidden, T, seed=90 + i).view(np.int16)).cuda()
          for i in range(a.warmup + a.calls)]
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in xs]
    st = torch.cuda.current_stream().cuda_stream
    for x, (e0, e1) in zip(xs, ev):
        flush.zero_()
        e0.record()
        rc = lib.stbl_route_noalloc(w.data_ptr(), b.data_ptr(), x.data_ptr(), T, cfg.n_experts, cfg.hidden, cfg.topk,
                                    cfg.n_groups, cfg.topk_groups, cfg.score_fn, cfg.route_scale, idx.data_ptr(),
                                    wt.data_ptr(), counts.data_ptr(), offsets.data_ptr(), perm.data_ptr(), st, err, 256)
        e1.record()
        assert rc == 0, err.value.decode()
    torch.cuda.synchronize()
    ms = [e0.elapsed_time(e1) for e0, e1 in ev[a.warmup:]]
    print(f"router E={cfg.n_experts} T={T}: {np.mean(ms) * 1e3:.1f} us per call (event-timed, L2 flushed)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--experts", type=int, default=16)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--fmt", default="fp8", choices=["fp8", "fp4", "ref"])
    ap.add_argument("--router-only", action="store_true")
    a = ap.parse_args()
    if a.router_only:
        router_only(a)
        return
    base = {"fp8": CFG2, "fp4": CFG3, "ref": CFG3_REF}[a.fmt]
    E = a.experts
    groups = 8 if E % 8 == 0 and E // 8 >= 2 and base.n_groups > 1 else 1
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
    distinct = len(np.unique(layer.last_route()["idx"]))
    print(f"{cfg.name} T={a.tokens}: router {t['router'] / n * 1e3:.4f} ms, up {t['up'] / n * 1e3:.4f} ms, "
          f"down {t['down'] / n * 1e3:.4f} ms per call, status {layer.status()}, "
          f"distinct routed experts in the last call {distinct} (+ the shared expert)")
    layer.close()


if __name__ == "__main__":
    main()
