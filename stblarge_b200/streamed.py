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

With --source file the experts are streamed from a GGUF checkpoint instead (the reference's reads from
the file, stbl/model.cu:269-308; stbl_cache_create_file): a file of --file-experts full-size MXFP4
experts (the same expert repeated; every layer reads the same tensors) is written to --file-dir, and
each token's missing experts are read from it by the cache's reader threads (O_DIRECT where the file
system takes it) and converted on the device.  Reported besides tokens/s: bytes read per second of
read time and whether O_DIRECT was in use.

    python -m stblarge_b200.streamed --source file [--layers 8] [--file-experts 32] [--slots 16] [--steps 12]

With --routes router the layers route the token themselves instead (each layer its own router weights
and a per-layer permutation of the Zipf(1.0) bias), and a layer's input is the previous layer's input
plus its output (a residual stream), so that the next layer's router on this layer's input can guess
its routes: the workload of the reference's shadow next-layer prefetch (stbl/model.cu:432-475,
555-586).  --prefetch N,C attaches it (the next layer's top N per token, the first C distinct ones);
--ab runs the same tokens without and with it on one host store.

    python -m stblarge_b200.streamed --routes router --ab --prefetch 8,8 [--layers 58] [--steps 24]
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


def layer_router(cfg, l, device="cuda"):
    """Router of layer l in the router-routed mode: fresh N(0, router_std) weights (seed 50 + l) and the
    configured bias with its experts permuted per layer (seed 500 + l)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(50 + l)
    w = torch.randn(cfg.n_experts, cfg.hidden, generator=g, device=device, dtype=torch.float32) * cfg.router_std
    perm = np.random.default_rng(500 + l).permutation(cfg.n_experts)
    return w.contiguous(), torch.from_numpy(np.ascontiguousarray(synth.router_bias(cfg)[perm])).to(device)


def run_routed(layers=58, cache_gb=40.0, store_experts=1024, steps=24, warmup=32, prefetch=None, store=None,
               update_scale=1.0, log=print):
    """Batch-1 decode through `layers` MXFP4 layers whose routes come from their own routers, on a
    residual stream (x of layer l + 1 = x of layer l + update_scale * its output: smaller scales make
    consecutive layers' inputs, and so the next layer's routes, easier to guess), experts streamed from
    a pinned host store into a GPU expert cache.  prefetch: None, or (n_predict, consider) for the
    shadow next-layer prefetch (stbl_moe_attach_prefetch) on a second stream.  store: a host_store() to
    reuse.  The warm-up tokens bring the cache to its steady state before the timed ones."""
    import torch

    from .cache import ExpertCache, host_store
    from .moe import MoELayer

    cfg = CFG3
    if store is None:
        t0 = time.time()
        store = host_store(cfg, layers, physical=store_experts)
        log(f"store {store['rows']} experts pinned in {time.time() - t0:.0f} s")
    slot_bytes = sum(((t[0].numel() * t.element_size() + 1023) // 1024) * 1024 for t in store["w"] + store["s"])
    slots = int(cache_gb * 1e9 // slot_bytes)
    cache = ExpertCache(cfg, layers, slots, store)
    stack = []
    for l in range(layers):
        w = synth.device_layer(cfg, experts=range(0))  # shared expert; the router is the layer's own
        w["router_w"], w["router_bias"] = layer_router(cfg, l)
        stack.append(MoELayer(cfg, w, max_tokens=1, cache=(cache, l)))
    side = torch.cuda.Stream()
    if prefetch:
        for l in range(layers - 1):
            stack[l].attach_prefetch(stack[l + 1], prefetch[0], prefetch[1], side)
    xs = [torch.from_numpy(synth.make_x(cfg.hidden, 1, seed=4 + t).view(np.int16)).cuda().view(torch.bfloat16)
          for t in range(warmup + steps)]

    def token(t):
        x = xs[t]
        for l in range(layers):
            x = x + stack[l](x) if update_scale == 1.0 else x + update_scale * stack[l](x)
        return x

    for t in range(warmup):
        token(t)
    torch.cuda.synchronize()
    s0, p0 = cache.stats(), cache.prefetch_counters()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        ev[i][0].record()
        token(warmup + i)
        ev[i][1].record()
    torch.cuda.synchronize()
    s1, p1, pb = cache.stats(), cache.prefetch_counters(), cache.prefetch_stats()
    total_s = sum(a.elapsed_time(b) for a, b in ev) / 1e3
    hits, misses = s1["hits"] - s0["hits"], s1["misses"] - s0["misses"]
    pf = [b - a for a, b in zip(p0, p1)]
    res = {
        "prefetch": list(prefetch) if prefetch else None, "update_scale": update_scale,
        "tokens_per_s": steps / total_s, "ms_per_token": 1e3 * total_s / steps,
        "hit_rate": hits / max(hits + misses, 1), "misses_per_token": misses / steps,
        "demand_gbs": (s1["bytes"] - s0["bytes"]) / total_s / 1e9,
        # the reference's stbl_prefetch counters per token: issued, routed after landing, routed while
        # being copied, cancelled
        "prefetch_per_token": {k: v / steps for k, v in zip(("issued", "landed", "reading", "cancelled"), pf)},
        "prefetch_bytes_total": pb["bytes"],
        "layers": layers, "slots": slots, "cache_gb": slots * slot_bytes / 1e9, "store_experts": store["rows"],
        "steps": steps, "warmup": warmup, "device_status": max(layer.status() for layer in stack),
    }
    for layer in stack:
        layer.close()
    cache.close()
    return res


def run_file(layers=8, file_experts=32, slots=16, steps=12, warmup=3, readers=8, direct=1, stage_experts=2,
             file_dir=None, seed=5, log=print):
    import dataclasses
    import os
    import tempfile

    import torch

    from . import gguf as G
    from .moe import MoELayer

    cfg = dataclasses.replace(CFG3, name="cfg3_file", n_experts=file_experts, n_groups=1, topk_groups=1)
    E, K, H, I = cfg.n_experts, cfg.topk, cfg.hidden, cfg.inter
    fd, path = tempfile.mkstemp(suffix=".gguf", dir=file_dir)
    os.close(fd)
    try:
        t0 = time.time()
        w, s = synth.routed_expert(cfg, 1000)
        tensors = []
        for m, part in enumerate(("gate", "up", "down")):
            rows, k = (I, H) if m < 2 else (H, I)
            blocks = G.mxfp4_to_blocks(w[m].cpu().numpy(), s[m].cpu().numpy())
            tensors.append((f"blk.0.ffn_{part}_exps.weight", G.T_MXFP4, (k, rows, E), G.Repeated(blocks.tobytes(), E)))
        G.write_gguf(path, [], tensors)
        file_gb = os.path.getsize(path) / 1e9
        with G.GgufFile(path) as g:
            offsets = G.expert_offsets(g, [0]) * layers  # every layer reads the same expert tensors
        t_write = time.time() - t0
        from .cache import ExpertCache
        cache = ExpertCache(cfg, layers, slots, file={"path": path, "offsets": offsets, "readers": readers,
                                                        "direct": direct, "stage_experts": stage_experts})
        stack = []
        for l in range(layers):
            wl = synth.device_layer(cfg, experts=range(0))
            stack.append(MoELayer(cfg, wl, max_tokens=1, cache=(cache, l)))
        trace = route_trace(E, K, layers, warmup + steps, seed=seed)
        idx = torch.from_numpy(trace).cuda().view(warmup + steps, layers, 1, K)
        xs = [torch.from_numpy(synth.make_x(H, 1, seed=4 + t).view(np.int16)).cuda() for t in range(warmup + steps)]
        log(f"file {file_gb:.2f} GB written in {t_write:.1f} s; cache {slots} slots")

        def token(t):
            x = xs[t]
            for l in range(layers):
                x = stack[l].forward_routed(x, idx[t, l])
            return x

        for t in range(warmup):
            token(t)
        torch.cuda.synchronize()
        s0, f0 = cache.stats(), cache.file_stats()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            ev[i][0].record()
            token(warmup + i)
            ev[i][1].record()
        torch.cuda.synchronize()
        s1, f1 = cache.stats(), cache.file_stats()
        total_s = sum(a.elapsed_time(b) for a, b in ev) / 1e3
        hits, misses = s1["hits"] - s0["hits"], s1["misses"] - s0["misses"]
        read_b, read_s = f1["bytes"] - f0["bytes"], f1["seconds"] - f0["seconds"]
        res = {
            "tokens_per_s": steps / total_s, "ms_per_token": 1e3 * total_s / steps,
            "hit_rate": hits / max(hits + misses, 1), "misses_per_token": misses / steps,
            "read_gbs": read_b / max(read_s, 1e-9) / 1e9, "read_share_of_time": read_s / total_s,
            "bytes_read_per_token": read_b / steps, "direct": f1["direct"], "failed_rounds": f1["failed_rounds"],
            "layers": layers, "slots": slots, "file_experts": E, "file_gb": file_gb, "readers": readers,
            "stage_experts": stage_experts, "steps": steps, "warmup": warmup,
            "device_status": max(layer.status() for layer in stack),
        }
        for layer in stack:
            layer.close()
        cache.close()
        return res
    finally:
        os.unlink(path)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--source", choices=("host", "file"), default="host")
    ap.add_argument("--file-experts", type=int, default=32)
    ap.add_argument("--slots", type=int, default=16)
    ap.add_argument("--readers", type=int, default=8)
    ap.add_argument("--direct", type=int, default=1)
    ap.add_argument("--stage-experts", type=int, default=2)
    ap.add_argument("--file-dir", default=None)
    ap.add_argument("--layers", type=int, default=58)
    ap.add_argument("--cache-gb", type=float, default=40.0)
    ap.add_argument("--store-experts", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--routes", choices=("forced", "router"), default="forced")
    ap.add_argument("--prefetch", default=None, help="n_predict,consider (with --routes router)")
    ap.add_argument("--ab", action="store_true", help="with --routes router: without, then with the prefetch")
    ap.add_argument("--update-scale", type=float, default=1.0, help="with --routes router: residual update scale")
    a = ap.parse_args()
    if a.routes == "router":
        import torch

        from .cache import host_store
        pf = tuple(int(v) for v in a.prefetch.split(",")) if a.prefetch else None
        t0 = time.time()
        store = host_store(CFG3, a.layers, physical=a.store_experts)
        print(f"store {store['rows']} experts pinned in {time.time() - t0:.0f} s", flush=True)
        for p in ([None, pf] if a.ab else [pf]):
            print(json.dumps(run_routed(a.layers, a.cache_gb, a.store_experts, a.steps, a.warmup, p, store,
                                        a.update_scale)), flush=True)
            torch.cuda.empty_cache()
    elif a.source == "file":
        print(json.dumps(run_file(a.layers, a.file_experts, a.slots, a.steps, a.warmup, a.readers, a.direct,
                                  a.stage_experts, a.file_dir)), flush=True)
    else:
        print(json.dumps(run(a.layers, a.cache_gb, a.store_experts, a.steps, a.warmup)), flush=True)


if __name__ == "__main__":
    main()
