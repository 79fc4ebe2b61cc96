"""Per-rank body of the expert-parallel GPU tests (tests/test_gpu_ep.py), run in spawned processes,
one per GPU: gloo carries only the exchange-region handles and the host-side barriers.  Test
infrastructure only."""

import datetime
import traceback

import numpy as np
import torch
import torch.distributed as dist

from oracle import oracle as O
from stblarge_b200 import synth
from stblarge_b200.config import CFG1
from stblarge_b200.moe import MoELayer, host_weights_to_device

TOL = 1e-2


def _rel(y_bits, ref_bits):
    y, ref = O.bf16_bits_to_f32(y_bits), O.bf16_bits_to_f32(ref_bits)
    return float(np.abs(y - ref).max() / np.abs(ref).max())


def parity(rank, n, port, q):
    """cfg1 (16 experts) sharded over n ranks: every rank's outputs and routes against the oracle
    over the full layer, for three calls with different token counts on each rank."""
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=n,
                                timeout=datetime.timedelta(seconds=60))
        cfg = CFG1
        W = synth.host_layer(cfg)
        E_loc = cfg.n_experts // n
        dev = host_weights_to_device(cfg, W, experts=range(rank * E_loc, (rank + 1) * E_loc))
        layer = MoELayer(cfg, dev, max_tokens=16, ep=(rank, n, None))
        report = []
        for call, T in enumerate((4 + rank, 16, 1 + 2 * rank)):
            x_bits = synth.make_x(cfg.hidden, T, seed=700 + 10 * call + rank)
            y = layer(torch.from_numpy(x_bits.view(np.int16)).cuda())
            torch.cuda.synchronize()
            y_bits = y.view(torch.int16).cpu().numpy().view(np.uint16)
            route = layer.last_route()
            y_ref, idx_ref, w_ref = O.moe_forward(cfg.as_dict(), W, x_bits)
            report.append({"T": T, "idx": bool(np.array_equal(route["idx"], idx_ref)),
                           "w": bool(np.array_equal(route["weights"].view(np.uint32), w_ref.view(np.uint32))),
                           "rel": _rel(y_bits, y_ref), "status": layer.status()})
        dist.barrier()
        layer.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, report, None))
    except Exception:
        q.put((rank, None, traceback.format_exc()))


def _parity_full(rank, n, port, q, zipf):
    """the full-size FP8 layer (256 experts, hidden 7168) sharded over n ranks, 256 tokens
    in all (256 / n per rank, the strong-scaling split), uniform routing (bias 0) or Zipf(1.2).  Each
    rank checks its routes and outputs against the single-device oracle layer, whose weights it
    regenerates from the same seeds (synth builds expert e from seed 1000 + e on any device)."""
    try:
        import dataclasses

        from stblarge_b200.config import CFG2
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=n,
                                timeout=datetime.timedelta(seconds=600))
        cfg = dataclasses.replace(CFG2, name="cfg4", bias_std=0.0, zipf_s=zipf)
        E_loc = cfg.n_experts // n
        dev = synth.device_layer(cfg, experts=range(rank * E_loc, (rank + 1) * E_loc))
        T = 256 // n
        layer = MoELayer(cfg, dev, max_tokens=T, ep=(rank, n, None))
        report = []
        for call in range(2):
            x_bits = synth.make_x(cfg.hidden, T, seed=900 + 10 * call + rank)
            y = layer(torch.from_numpy(x_bits.view(np.int16)).cuda())
            torch.cuda.synchronize()
            report.append({"y": y.view(torch.int16).cpu().numpy().view(np.uint16), "x": x_bits,
                           "route": layer.last_route(), "status": layer.status()})
        dist.barrier()
        layer.close()
        del dev
        torch.cuda.empty_cache()
        dist.barrier()
        dist.destroy_process_group()
        # the oracle over the whole layer: every expert this rank's tokens chose, rebuilt from its seed
        out = []
        shared = synth.device_layer(cfg, experts=range(0))  # the shared expert and router only
        shared = [(shared["shared_w"][m].cpu().numpy(), shared["shared_s"][m].cpu().numpy()) for m in range(3)]
        for r in report:
            idx = r["route"]["idx"]
            W = {"router_w": synth.router_w(cfg), "router_bias": synth.router_bias(cfg),
                 "routed": [[None] * cfg.n_experts for _ in range(3)], "shared": shared}
            for e in np.unique(idx):
                ws, ss = synth.routed_expert(cfg, 1000 + int(e), device="cuda")
                for m in range(3):
                    W["routed"][m][int(e)] = (ws[m].cpu().numpy(), ss[m].cpu().numpy())
            y_ref, idx_ref, w_ref = O.moe_forward(cfg.as_dict(), W, r["x"])
            out.append({"T": T, "idx": bool(np.array_equal(idx, idx_ref)),
                        "w": bool(np.array_equal(r["route"]["weights"].view(np.uint32), w_ref.view(np.uint32))),
                        "rel": _rel(r["y"], y_ref), "status": r["status"], "distinct": int(len(np.unique(idx)))})
        q.put((rank, out, None))
    except Exception:
        q.put((rank, None, traceback.format_exc()))


def parity_full_uniform(rank, n, port, q):
    _parity_full(rank, n, port, q, 0.0)


def parity_full_zipf(rank, n, port, q):
    _parity_full(rank, n, port, q, 1.2)


def skipped_call(rank, n, port, q):
    """Rank 1 skips one call: rank 0's waits on it run out (about 1 s each) and its status reports a
    timed-out wait; nothing faults.  Both ranks then meet at a host barrier before freeing anything."""
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=n,
                                timeout=datetime.timedelta(seconds=120))
        cfg = CFG1
        W = synth.host_layer(cfg)
        E_loc = cfg.n_experts // n
        dev = host_weights_to_device(cfg, W, experts=range(rank * E_loc, (rank + 1) * E_loc))
        layer = MoELayer(cfg, dev, max_tokens=16, ep=(rank, n, None))
        x = torch.from_numpy(synth.make_x(cfg.hidden, 4, seed=31 + rank).view(np.int16)).cuda()
        layer(x)
        torch.cuda.synchronize()
        first = layer.status()
        dist.barrier()
        second = None
        if rank == 0:
            layer(x)  # the other ranks do not take part in this call
            torch.cuda.synchronize()
            second = layer.status()
        dist.barrier()
        layer.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, {"first": first, "second": second}, None))
    except Exception:
        q.put((rank, None, traceback.format_exc()))
