"""MoE-layer decode benchmark (BASELINE.json metric: decode tokens/s and achieved HBM GB/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl b200|reference] [--workload ...]

A step is one call of a full-size DeepSeek-V3-shaped MoE layer (hidden 7168, moe_intermediate 2048,
256 routed experts + 1 shared, top-8 of 8 groups keeping 4), weights resident in HBM.  Every step
gets fresh tokens (different routing), and L2 is flushed before each step; each step is timed with
CUDA events on the launching stream.  `e2e` is the same metric through the host-buffer entry point
(stbl_moe_forward_host: H2D of x, layer, D2H of y, inside the timed region).

Default workload:
  * one GPU: configs[1] (cfg2, FP8 128x128 weights) at T = 16 decode tokens, the headline; the line
    also carries `sweep` (configs[1] at T = 1, 4, 16), `cfg3_sweep` (configs[2]: MXFP4 routed experts,
    FP8 shared, Zipf(1.0) bias, T = 1, 4, 16, 64), `cfg3q8_sweep` (the same layer with Q8 activations
    for the routed experts, the reference's ds4 numerics), `cfg4_n1` (configs[3]'s 256 tokens on this one
    GPU: the N = 1 point of the strong-scaling curve) and `cfg4_n1_zipf` (the same with Zipf(1.2) routing);
  * N > 1 GPUs: configs[3] (cfg4), 256 tokens in all split over the ranks (strong scaling), expert
    parallelism: rank r holds routed experts [r 256/N, (r+1) 256/N) (router and shared expert
    replicated), every rank routes its own tokens and the layer's kernels dispatch them to the owning
    ranks and bring the outputs back through NVLink peer memory.  The line also carries `weak_cfg2`
    (configs[1] with 16 tokens per rank).  Time = max over ranks of the device time.
--workload cfg2|cfg3|cfg3ref|cfg3q8|cfg4|cfg5 picks one explicitly (--zipf: Zipf(1.2) routing for cfg4).

--impl reference: the reference's CPU path (the CPU oracle restating stbl/model.cu:426-594 on the
numerics of ref/kernel.py) on the host cores, the same workload, config and metric; rank 0 only.
"""

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from stblarge_b200 import synth  # noqa: E402
from stblarge_b200.config import CFG2, CFG3, CFG3_Q8, CFG3_REF, FMT_FP8_E8M0, FMT_MXFP4  # noqa: E402

METRIC = "MoE-layer decode tokens/s (full-size FP8 layer)"
UNIT = "tokens/s"
HBM_NOMINAL_GBS = 8000.0


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def layer_bytes(cfg, n_distinct, T):
    """Algorithmic bytes of one layer call: distinct routed experts + shared expert (codes and scales),
    router weights + bias, x in, y out (per-token intermediates excluded)."""
    return (n_distinct * cfg.bytes_per_expert() + cfg.bytes_per_expert(cfg.shared_fmt) + cfg.n_experts * cfg.hidden * 4
            + cfg.n_experts * 4 + 2 * T * cfg.hidden * 2)


def up_bytes(cfg, n_distinct):
    """Algorithmic bytes of one expert-up launch: gate + up codes and scales of the distinct experts and
    the shared expert (activations in and h out are under 0.1% and left out)."""
    H, I = cfg.hidden, cfg.inter

    def mat(fmt):
        if fmt == FMT_MXFP4:
            return I * H // 2 + I * (H // 32)
        if fmt == FMT_FP8_E8M0:
            return I * H + ((I + 31) // 32) * (H // 32)
        return I * H + 4 * ((I + 127) // 128) * ((H + 127) // 128)
    return 2 * (n_distinct * mat(cfg.routed_fmt) + mat(cfg.shared_fmt))


class NvmlClockSampler:
    """SM clock and clock-event (throttle) reasons of the GPU, read through NVML from a thread every
    `period` seconds while the timed region runs (the region can be a few tens of milliseconds, shorter
    than nvidia-smi's start-up).  Reads only; nothing on the GPU is changed.  start() returns once the
    first sample is taken."""

    def __init__(self, cuda_index, period=0.002):
        import threading

        import pynvml
        self.nv = pynvml
        pynvml.nvmlInit()
        # the CUDA device's NVML handle (CUDA_VISIBLE_DEVICES may renumber): by UUID, else by index
        self.h = None
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(cuda_index).uuid)
            self.h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
        except Exception:
            self.h = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
        self.period = period
        self.samples, self.reasons = [], 0
        self.stop_ev, self.first = threading.Event(), threading.Event()
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self.nv
        while not self.stop_ev.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            self.first.set()
            time.sleep(self.period)

    def start(self):
        self.thread.start()
        self.first.wait(timeout=5)

    def stop(self):
        self.stop_ev.set()
        self.thread.join(timeout=5)
        nv = self.nv
        try:
            mx = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
        except Exception:
            mx = None
        names = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                 "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                 "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                 "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
        reasons = sorted(n for n, bit in names.items() if self.reasons & bit)
        sm = [float(v) for v in self.samples]
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": reasons, "source": "nvml"}


def clock_sampler(cuda_index):
    """NVML sampling in-process when the bindings load, else the nvidia-smi subprocess."""
    try:
        return NvmlClockSampler(cuda_index)
    except Exception:
        return ClockSampler(cuda_index)


class ClockSampler:
    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.12)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [v.strip() for v in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


def cpu_oracle_layer(cfg, W_host, x_bits, nthreads):
    from oracle import oracle as O
    t0 = time.perf_counter()
    O.moe_forward(cfg.as_dict(), W_host, x_bits, nthreads=nthreads)
    return time.perf_counter() - t0


def workload_of(args, world):
    """(name, cfg, tokens per rank).  Default: configs[1] (cfg2, T tokens) on one GPU; configs[3]
    (cfg4, 256 tokens split over the ranks, expert parallelism) on more than one."""
    import dataclasses
    wl = args.workload or ("cfg2" if world == 1 else "cfg4")
    if wl == "cfg4":
        if 256 % world:
            raise SystemExit("cfg4 splits 256 tokens over the ranks: --gpus must divide 256")
        return wl, dataclasses.replace(CFG2, name="cfg4", bias_std=0.0, zipf_s=1.2 if args.zipf else 0.0), 256 // world
    if wl == "cfg3":
        return wl, CFG3, args.tokens
    if wl == "cfg3ref":
        return wl, CFG3_REF, args.tokens
    if wl == "cfg3q8":
        return wl, CFG3_Q8, args.tokens
    return wl, CFG2, args.tokens


def config_of(args, wl, T, world):
    """The `config` object of the JSON line: the same for the b200 arm and the reference arm."""
    E_loc = 256 // world
    return {"workload": (f"cfg4 expert-parallel full-size FP8 MoE layer, 256 tokens split over {world} GPU(s), "
                         f"{'Zipf(1.2)' if args.zipf else 'uniform'} routing"
                         if wl == "cfg4" else
                         "cfg3 full-size layer, MXFP4 routed experts (FP8 shared), Zipf(1.0) routing"
                         if wl == "cfg3" else
                         "cfg3q8 full-size layer, MXFP4 routed experts with Q8 activations (int8 per 32), FP8 shared, "
                         "Zipf(1.0) routing"
                         if wl == "cfg3q8" else
                         "cfg3ref full-size layer in the reference engine's formats and routing: MXFP4 routed "
                         "experts, FP8 shared expert with e8m0 32x32 block scales, sqrt(softplus) top-8 of 256"
                         if wl == "cfg3ref" else
                         "cfg2 full-size FP8 MoE layer (7168/2048, 256+1 experts, top-8, 8 groups keep 4)")
                        + f", T={T} decode tokens per rank", "tokens_per_rank": T,
            "parallelism": "single GPU" if world == 1 else
            f"ep{world}: expert parallelism, {E_loc} routed experts per GPU, dispatch/combine through NVLink peer memory",
            "l2": "flushed (256 MB write) before every timed step; fresh tokens each step"}


def step_tokens(cfg, T, world, step):
    """The tokens of one step of the whole job (every rank's, rank-major), bf16 bits [world * T, H]."""
    return np.concatenate([synth.make_x(cfg.hidden, T, seed=1_000_000 * (r + 1) + step) for r in range(world)])


def run_reference(args, rank, world):
    """The reference's CPU path (the oracle restating stbl/model.cu:426-594 on the numerics of
    ref/kernel.py) on this host's cores, on the b200 arm's workload and config: each step is one layer
    call on the whole job's tokens of that step (every rank's), rank 0 only."""
    if rank != 0:
        return
    import torch
    wl, cfg, T = workload_of(args, world)
    if cfg.routed_fmt != CFG2.routed_fmt:
        raise SystemExit("the reference arm times the FP8 workloads (cfg2, cfg4)")
    cores = os.cpu_count()
    torch.set_num_threads(cores)
    # 8 generated experts; each of the 256 ids holds its own copy of one of them with every code row
    # rotated by a per-id amount, so the oracle streams 256 distinct experts' bytes (the real working
    # set) with the value distribution of the generated weights
    g = torch.Generator().manual_seed(1000)
    pool = []
    for _ in range(8):
        ws = []
        for (r, k) in synth.mat_shapes(cfg):
            c, s_ = synth.quant_fp8_b128(torch.randn(r, k, generator=g) * cfg.weight_std)
            ws.append((c.numpy(), s_.numpy()))
        pool.append(ws)
    routed = [[(np.roll(pool[e % 8][m][0], 1 + e // 8, axis=1), pool[e % 8][m][1]) for e in range(cfg.n_experts)]
              for m in range(3)]
    W = {"router_w": synth.router_w(cfg), "router_bias": synth.router_bias(cfg), "routed": routed, "shared": pool[0]}
    Tj = T * world
    for i in range(args.warmup):
        cpu_oracle_layer(cfg, W, step_tokens(cfg, T, world, i), cores)
    total = 0.0
    for i in range(args.steps):
        total += cpu_oracle_layer(cfg, W, step_tokens(cfg, T, world, args.warmup + i), cores)
    value = Tj * args.steps / total
    sample = (f"{args.steps} full layer calls of {Tj} tokens each (the whole job's tokens of a step) on the CPU "
              f"oracle with {cores} threads; the 256 experts are distinct in memory (8 generated experts, "
              f"code rows rotated per id)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "strong" if wl == "cfg4" else "weak", "vs_baseline": None,
            "dtype": "fp8-e4m3 weights and activations, fp32 accumulate, bf16 io",
            "data": "synthetic (seeded ~N(0,0.02) weights quantized to FP8 128x128; bf16 ~N(0,1) tokens)",
            "config": config_of(args, wl, T, world),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_streamed(args, rank, world):
    """batch-1 decode through 58 MXFP4 layers with host-streamed experts and a 40 GB GPU
    expert cache (stblarge_b200/streamed.py); one GPU, rank 0."""
    if rank != 0:
        return
    from stblarge_b200 import streamed
    clocks = clock_sampler(0)
    ck = {}

    def on_timed(begin):  # sample the clocks over the timed steps only (the store build leaves the GPU idle)
        if begin:
            clocks.start()
        else:
            ck.update(clocks.stop())
    r = streamed.run(layers=58, cache_gb=40.0, store_experts=1024, steps=args.steps, warmup=args.warmup,
                     log=lambda m: print(m, file=sys.stderr, flush=True), on_timed=on_timed)
    line = {
        "metric": "streamed decode tokens/s (58 MXFP4 layers, host-streamed experts, 40 GB GPU expert cache)",
        "value": r["tokens_per_s"], "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["ms_per_token"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e2m1 routed / e4m3 shared weights, e4m3 activations, fp32 accumulate, bf16 io",
        "data": "synthetic (seeded weights; a pinned store of 1024 distinct experts repeated over the 58 x 256)",
        "config": {"workload": "cfg5 streamed decode: 58 layers, batch 1, forced routes (reuse 0.6, Zipf 1.0)",
                   "parallelism": "single GPU", "cache_slots": r["slots"], "cache_gb": r["cache_gb"]},
        "hit_rate": r["hit_rate"], "misses_per_token": r["misses_per_token"],
        "host_to_device_gbs": r["host_to_device_gbs"], "clocks": ck, "device_status": r["device_status"],
    }
    print(json.dumps(line), flush=True)


def sweep_layer(layer, cfg, token_counts, distinct_of, timed_steps, peak, seed0):
    """Device time per call and per kernel at each decode batch size in token_counts (20 timed calls
    each, L2 flushed before every call, fresh tokens), with the HBM fraction of the layer and of its
    up kernel."""
    import torch
    out = []
    dev = torch.device("cuda", torch.cuda.current_device())
    for Ts in token_counts:
        xs2 = [torch.from_numpy(synth.make_x(cfg.hidden, Ts, seed=seed0 + 100 * Ts + i).view(np.int16)).to(dev)
               for i in range(23)]
        for i in range(3):
            layer(xs2[i])
        torch.cuda.synchronize()
        # the call time without the library's per-kernel events (an event between two chained kernels
        # keeps the second from starting while the first drains), then the per-kernel times with them
        ms = timed_steps(layer, xs2[3:])
        base = layer.timing()
        layer.set_timing(True)
        timed_steps(layer, xs2[3:])
        layer.set_timing(False)
        k2 = layer.timing()
        n2 = max(k2["calls"] - base["calls"], 1)
        dd = [distinct_of(layer, x) for x in xs2[3:]]
        mean_ms = float(np.mean(ms))
        gbs = np.mean([layer_bytes(cfg, d, Ts) for d in dd]) / (mean_ms / 1e3) / 1e9
        kms = {k: (k2[k] - base[k]) / n2 * 1e3 for k in ("router", "up", "down")}
        up_gbs = np.mean([up_bytes(cfg, d) for d in dd]) / (kms["up"] / 1e3) / 1e9
        out.append({"tokens": Ts, "tokens_per_s": Ts / (mean_ms / 1e3), "ms_per_call": mean_ms,
                    "distinct_experts": float(np.mean(dd)), "hbm_gbs": float(gbs), "hbm_frac_of_measured": float(gbs / peak),
                    "kernel_ms": kms, "up_gbs": float(up_gbs), "up_frac_of_measured": float(up_gbs / peak)})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=16)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--workload", default=None, choices=["cfg2", "cfg3", "cfg3ref", "cfg3q8", "cfg4", "cfg5"],
                    help="default: cfg2 on one GPU, cfg4 on more")
    ap.add_argument("--zipf", action="store_true", help="cfg4: Zipf(1.2) expert popularity instead of uniform")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.workload == "cfg5":
        run_streamed(args, rank, world)
        return

    import dataclasses

    import torch
    import torch.distributed as dist
    from stblarge_b200.moe import MoELayer

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    wl, cfg, T = workload_of(args, world)
    E_loc = cfg.n_experts // world
    shard = range(rank * E_loc, (rank + 1) * E_loc)
    weights = synth.device_layer(cfg, device=dev, experts=shard)
    layer = MoELayer(cfg, weights, max_tokens=max(T, 64 if wl in ("cfg3", "cfg3ref", "cfg3q8") else 16),
                     ep=(rank, world, None) if world > 1 else None)
    n_steps = args.warmup + args.steps
    xs = torch.stack([torch.from_numpy(synth.make_x(cfg.hidden, T, seed=1_000_000 * (rank + 1) + i).view(np.int16))
                      for i in range(n_steps)]).to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 256 MB > 126 MB L2

    def distinct_of(lay, x):
        """Distinct routed experts of this rank's shard that the step streams: the experts that any
        rank's tokens are routed to (untimed pass, every rank in step; routes read back)."""
        lay(x)
        ids = lay.last_route()["idx"]
        if world > 1:
            allids = [None] * world
            dist.all_gather_object(allids, ids)
            ids = np.concatenate([a.reshape(-1) for a in allids])
        ids = np.unique(ids)
        return int(np.sum((ids >= shard.start) & (ids < shard.stop)))

    def timed_steps(lay, inputs):
        """Device time of each call, L2 flushed before each; nothing synchronises inside the loop, so
        the host runs ahead and the GPU executes flush, layer, flush, layer ... back to back."""
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in inputs]
        for x, (a, b) in zip(inputs, evs):
            flush.zero_()
            a.record()
            lay(x)
            b.record()
        torch.cuda.synchronize()
        return [a.elapsed_time(b) for a, b in evs]

    def max_over_ranks(v):
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(args.warmup):
        layer(xs[i])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = clock_sampler(local)
    sampler.start()
    step_ms = timed_steps(layer, [xs[args.warmup + i] for i in range(args.steps)])
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    # per-kernel device times (router, up, down) from a second pass over the same steps with the
    # library's timing events on; the headline pass above runs without them (an event between two
    # chained kernels keeps the second from starting while the first drains)
    layer.timing()
    layer.set_timing(True)
    timed_steps(layer, [xs[args.warmup + i] for i in range(args.steps)])
    layer.set_timing(False)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    kt = layer.timing()
    distinct = [distinct_of(layer, xs[args.warmup + i]) for i in range(args.steps)]
    total_s = sum(step_ms) / 1e3
    total_max = max_over_ranks(total_s)
    value = world * T * args.steps / total_max
    bytes_steps = [layer_bytes(cfg, d, T) for d in distinct]
    hbm_gbs = sum(bytes_steps) / total_s / 1e9
    peak, peak_kind = peaks()
    up_alg = sum(up_bytes(cfg, d) for d in distinct) / args.steps
    up_ms = kt["up"] / max(kt["calls"], 1) * 1e3
    up_gbs = up_alg / (up_ms / 1e3) / 1e9
    launches = layer.stats()["launches_per_call"]

    # end to end through the host-buffer entry point (pinned host memory)
    xh = [xs[args.warmup + i].cpu().pin_memory() for i in range(args.steps)]
    yh = torch.empty_like(xh[0]).pin_memory()
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    stream = torch.cuda.current_stream()
    for i in range(2):
        layer.forward_host(xh[i], yh)
    for i in range(args.steps):
        flush.zero_()
        e2e_ev[i][0].record(stream)
        layer.forward_host(xh[i], yh)
        e2e_ev[i][1].record(stream)
    torch.cuda.synchronize()
    e2e_s = sum(a.elapsed_time(b) for a, b in e2e_ev) / 1e3
    e2e_value = world * T * args.steps / max_over_ranks(e2e_s)

    extra = {}
    sweep = []
    if not args.no_sweep and world == 1 and wl in ("cfg2", "cfg3", "cfg3ref", "cfg3q8"):
        # batch sizes of the workload's config: configs[1] 1, 4, 16; configs[2] 1, 4, 16, 64
        sweep = sweep_layer(layer, cfg, (1, 4, 16) if wl == "cfg2" else (1, 4, 16, 64), distinct_of, timed_steps,
                            peak, 7_000_000)
    status = layer.status()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import oracle as O  # noqa: F401  (the CPU baseline is the oracle)
        xb = xs[args.warmup].cpu().numpy().view(np.uint16)
        layer(xs[args.warmup])
        r = layer.last_route()
        W = {"router_w": weights["router_w"].cpu().numpy(), "router_bias": weights["router_bias"].cpu().numpy(),
             "routed": [[None] * cfg.n_experts for _ in range(3)],
             "shared": [(weights["shared_w"][m].cpu().numpy(), weights["shared_s"][m].cpu().numpy()) for m in range(3)]}
        for e in np.unique(r["idx"]):
            for m in range(3):
                W["routed"][m][int(e)] = (weights["routed_w"][m][e].cpu().numpy(), weights["routed_s"][m][e].cpu().numpy())
        cores = os.cpu_count()
        dt = cpu_oracle_layer(cfg, W, xb, cores)
        cpu = {"value": T / dt, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"1 layer call of the T={T} workload (the first timed step's tokens) on the CPU oracle"}

    if not args.no_sweep and world == 1 and wl == "cfg2":
        # configs[3] on this one GPU (256 tokens, the same FP8 experts with bias 0): the N = 1 point of
        # the strong-scaling curve that `--gpus N` (default workload cfg4) measures at N > 1
        cfg4 = dataclasses.replace(CFG2, name="cfg4", bias_std=0.0, zipf_s=0.0)
        w4 = dict(weights)
        w4["router_bias"] = torch.from_numpy(synth.router_bias(cfg4)).to(dev)
        l4 = MoELayer(cfg4, w4, max_tokens=256)
        x4 = [torch.from_numpy(synth.make_x(cfg4.hidden, 256, seed=1_000_000 + i).view(np.int16)).to(dev)
              for i in range(args.warmup + 20)]
        for i in range(args.warmup):
            l4(x4[i])
        ms4 = timed_steps(l4, x4[args.warmup:])
        extra["cfg4_n1"] = {"workload": "cfg4 (configs[3]) on one GPU: 256 tokens, uniform routing, full-size FP8",
                            "tokens_per_s": 256 * len(ms4) / (sum(ms4) / 1e3), "ms_per_step": float(np.mean(ms4)),
                            "steps": len(ms4), "device_status": l4.status()}
        l4.close()
        # the same with configs[3]'s Zipf(1.2) routing (hot experts: the 32-token items)
        cfg4z = dataclasses.replace(CFG2, name="cfg4", bias_std=0.0, zipf_s=1.2)
        w4["router_bias"] = torch.from_numpy(synth.router_bias(cfg4z)).to(dev)
        l4 = MoELayer(cfg4z, w4, max_tokens=256)
        for i in range(args.warmup):
            l4(x4[i])
        ms4 = timed_steps(l4, x4[args.warmup:])
        extra["cfg4_n1_zipf"] = {"workload": "cfg4 (configs[3]) on one GPU: 256 tokens, Zipf(1.2) routing, full-size FP8",
                                 "tokens_per_s": 256 * len(ms4) / (sum(ms4) / 1e3), "ms_per_step": float(np.mean(ms4)),
                                 "steps": len(ms4), "device_status": l4.status()}
        l4.close()
        del w4, l4
        # configs[2] (MXFP4 routed experts, FP8 shared, Zipf(1.0)) at T = 1, 4, 16, 64 on this GPU
        layer.close()
        del weights, layer
        torch.cuda.empty_cache()
        w3 = synth.device_layer(CFG3, device=dev)
        l3 = MoELayer(CFG3, w3, max_tokens=64)
        extra["cfg3_sweep"] = sweep_layer(l3, CFG3, (1, 4, 16, 64), distinct_of, timed_steps, peak, 8_000_000)
        extra["cfg3_device_status"] = l3.status()
        l3.close()
        # the same experts with Q8 activations for the routed experts (CUDA-core kernels)
        lq = MoELayer(CFG3_Q8, w3, max_tokens=64)
        extra["cfg3q8_sweep"] = sweep_layer(lq, CFG3_Q8, (1, 4, 16, 64), distinct_of, timed_steps, peak, 8_000_000)
        extra["cfg3q8_device_status"] = lq.status()
        lq.close()
        layer = None

    if world > 1 and not args.no_sweep and wl == "cfg4":
        # weak scaling beside it: configs[1] with 16 tokens per rank (the same shard, configs[1]'s bias)
        w2 = dict(weights)
        w2["router_bias"] = torch.from_numpy(synth.router_bias(CFG2)).to(dev)
        l2 = MoELayer(CFG2, w2, max_tokens=16, ep=(rank, world, None))
        x2 = [torch.from_numpy(synth.make_x(CFG2.hidden, 16, seed=2_000_000 * (rank + 1) + i).view(np.int16)).to(dev)
              for i in range(args.warmup + 20)]
        for i in range(args.warmup):
            l2(x2[i])
        torch.cuda.synchronize()
        dist.barrier()
        ms2 = timed_steps(l2, x2[args.warmup:])
        t2 = max_over_ranks(sum(ms2) / 1e3)
        extra["weak_cfg2"] = {"workload": "cfg2 (configs[1]) with 16 tokens per rank, expert parallelism",
                              "tokens_per_s": world * 16 * len(ms2) / t2, "ms_per_step": 1e3 * t2 / len(ms2),
                              "steps": len(ms2), "device_status": l2.status()}
        l2.close()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * total_max / args.steps, "higher_is_better": True,
            "scaling": "strong" if wl == "cfg4" else "weak", "vs_baseline": None,
            "dtype": ("fp8-e4m3 weights and activations, fp32 accumulate, bf16 io" if cfg.routed_fmt != FMT_MXFP4 else
                      "e2m1 routed / e4m3 shared weights, int8 routed / e4m3 shared activations, exact integer "
                      "block sums + fp32 accumulate, bf16 io" if cfg.act_q8 else
                      "e2m1 routed / e4m3 shared weights, e4m3 activations, fp32 accumulate, bf16 io"),
            "data": ("synthetic (seeded ~N(0,0.02) weights quantized to "
                     + {"cfg3": "MXFP4 routed / FP8 128x128 shared", "cfg3q8": "MXFP4 routed / FP8 128x128 shared",
                        "cfg3ref": "MXFP4 routed / FP8 e8m0-32x32 shared"}.get(wl, "FP8 128x128")
                     + "; bf16 ~N(0,1) tokens)"),
            "config": config_of(args, wl, T, world),
            "hbm_gbs": hbm_gbs, "hbm_frac_of_measured": hbm_gbs / peak, "hbm_frac_of_8tbs": hbm_gbs / HBM_NOMINAL_GBS,
            "hbm_note": "per GPU (rank 0): its shard's distinct routed experts + shared expert + router + x/y, over its device time",
            "distinct_experts_per_step": float(np.mean(distinct)),
            "kernel_ms_per_step": {"router": kt["router"] / max(kt["calls"], 1) * 1e3, "up": up_ms,
                                   "down": kt["down"] / max(kt["calls"], 1) * 1e3},
            "roofline": {"bound": "hbm", "kernel": ("expert_q8_kernel<up> (CUDA-core MXFP4 x Q8 routed gate+up, SwiGLU) "
                                                    "after expert_tc_kernel<up> (FP8 shared)" if cfg.act_q8 else
                                                    "expert_tc4_kernel<up> (tcgen05 MXFP4 routed + FP8 shared gate+up, SwiGLU)"
                                                    if cfg.routed_fmt == FMT_MXFP4 else
                                                    "expert_tc_kernel<up> (tcgen05 FP8 gate+up, SwiGLU)"),
                         "achieved": up_gbs, "peak": peak, "unit": "GB/s", "frac": up_gbs / peak, "peak_kind": peak_kind,
                         "traffic": traffic_from_profile(cfg, float(np.mean(distinct)) + 1.0, up_alg),
                         "traffic_note": ("ncu DRAM read+write over algorithmic bytes of one MXFP4 up launch "
                                          "(profiles/traffic.json) x this step's algorithmic up bytes"
                                          if cfg.routed_fmt == FMT_MXFP4 else
                                          "ncu DRAM read+write bytes per expert of one up launch (profiles/traffic.json) "
                                          "x the step's mean distinct routed experts + the shared expert")},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": T * cfg.hidden * 2,
                    "d2h_bytes_per_step": T * cfg.hidden * 2},
            "gpu_launches": launches * args.steps,
            "clocks": clocks, "sweep": sweep, "device_status": status,
            "cpu_baseline": cpu,
            **extra,
        }
        print(json.dumps(line), flush=True)
    if layer is not None:
        layer.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def traffic_from_profile(cfg, experts_per_launch, up_alg):
    """DRAM bytes per launch of the up kernel from the committed ncu captures of smaller cases, where
    traffic grows in proportion to the experts streamed: FP8, the figure per expert times the experts
    one launch streams; MXFP4 (a mixed launch), the captured DRAM / algorithmic ratio times this
    launch's algorithmic bytes.  None when there is no committed figure."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            t = json.load(f)
    except Exception:
        return None
    if cfg.routed_fmt == FMT_MXFP4:
        r = t.get("expert_up_mxfp4_dram_over_algorithmic")
        return None if r is None else r * up_alg
    per_expert = t.get("expert_up_fp8_dram_bytes_per_expert")
    return None if per_expert is None else per_expert * experts_per_launch


if __name__ == "__main__":
    main()
