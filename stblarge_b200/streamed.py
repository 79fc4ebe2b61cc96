"""Multi-layer streamed decode: batch-1 decode through a stack of full-size MoE layers
(MXFP4 routed experts, FP8 shared expert) whose routed experts live in pinned host memory and are
brought into a GPU expert cache (stbl_cache_*) on demand, the reference's SSD/host-streamed mode
(stbl/model.cu:269-345, 347-422, 503-520).

Routes are forced from a generator (stbl_moe_forward_routed), temporally correlated as configs[4]
specifies: at every step each of a layer's topk slots reuses, with probability 0.6, one of that
layer's experts of the previous step (not already taken), and otherwise draws an expert from a
Zipf(1.0) popularity (a seeded permutation of ranks per layer) without replacement.  A step is one
token through every layer; tokens/s = steps / device time, hit rate = cache hits / routed experts.

    python -m stblarge_b200.streamed [--layers 58] [--cache-gb 40] [--store-experts 1024] [--steps 64]
"""

import argparse
import json
import time

import numpy as np

from . import synth
from .config import CFG3


def route_trace(E, K, L, steps, reuse=0.6, zipf_s=1.0, seed=5):
    """int32 [steps][L][K] expert ids."""
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, E + 1, dtype=np.float64) ** zipf_s
    pe = [p[rng.permutation(E)] for _ in range(L)]  # expert e of layer l has the popularity of its rank
    out = np.empty((steps, L, K), np.int32)
    prev = [None] * L
    for t in range(steps):
        for l in range(L):
            chosen = []
            for _ in range(K):
                if prev[l] is not None and rng.random() < reuse:
                    cand = [e for e in prev[l] if e not in chosen]
                    if cand:
                        chosen.append(int(cand[rng.integers(len(cand))]))
                        continue
                q = pe[l].copy()
                q[chosen] = 0.0
                chosen.append(int(rng.choice(E, p=q / q.sum())))
            out[t, l] = chosen
            prev[l] = chosen
    return out


def run(layers=58, cache_gb=40.0, store_experts=1024, steps=64, warmup=3, seed=5, log=print, on_timed=None):
    """on_timed(True / False): called right before the timed steps are enqueued and after they finished
    (a clock sampler's start and stop)."""
    import torch

    from .cache import ExpertCache, host_store
    from .moe import MoELayer

    cfg = CFG3
    E, K = cfg.n_experts, cfg.topk
    t0 = time.time()
    store = host_store(cfg, layers, physical=store_experts)
    t_store = time.time() - t0
    slot_bytes = sum(((t[0].numel() * t.element_size() + 1023) // 1024) * 1024 for t in store["w"] + store["s"])
    slots = int(cache_gb * 1e9 // slot_bytes)
    cache = ExpertCache(cfg, layers, slots, store)
    stack = []
    for l in range(layers):
        w = synth.device_layer(cfg, experts=range(0))  # router + this layer's own shared expert
        stack.append(MoELayer(cfg, w, max_tokens=1, cache=(cache, l)))
    trace = route_trace(E, K, layers, warmup + steps, seed=seed)
    idx = torch.from_numpy(trace).cuda().view(warmup + steps, layers, 1, K)
    xs = [torch.from_numpy(synth.make_x(cfg.hidden, 1, seed=4 + t).view(np.int16)).cuda() for t in range(warmup + steps)]
    log(f"store {store['rows']} experts pinned in {t_store:.0f} s; cache {slots} slots ({slots * slot_bytes / 1e9:.1f} GB)")

    def token(t):
        x = xs[t]
        for l in range(layers):
            x = stack[l].forward_routed(x, idx[t, l])
        return x

    for t in range(warmup):
        token(t)
    torch.cuda.synchronize()
    s0 = cache.stats()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    if on_timed:
        on_timed(True)
    for i in range(steps):
        ev[i][0].record()
        token(warmup + i)
        ev[i][1].record()
    torch.cuda.synchronize()
    if on_timed:
        on_timed(False)
    s1 = cache.stats()
    ms = [a.elapsed_time(b) for a, b in ev]
    total_s = sum(ms) / 1e3
    hits, misses = s1["hits"] - s0["hits"], s1["misses"] - s0["misses"]
    status = max(layer.status() for layer in stack)
    res = {
        "tokens_per_s": steps / total_s, "ms_per_token": 1e3 * total_s / steps,
        "hit_rate": hits / max(hits + misses, 1), "misses_per_token": misses / steps,
        "host_to_device_gbs": (s1["bytes"] - s0["bytes"]) / total_s / 1e9,
        "layers": layers, "slots": slots, "cache_gb": slots * slot_bytes / 1e9, "store_experts": store["rows"],
        "steps": steps, "warmup": warmup, "device_status": status,
    }
    for layer in stack:
        layer.close()
    cache.close()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=58)
    ap.add_argument("--cache-gb", type=float, default=40.0)
    ap.add_argument("--store-experts", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    print(json.dumps(run(a.layers, a.cache_gb, a.store_experts, a.steps, a.warmup)), flush=True)


if __name__ == "__main__":
    main()
