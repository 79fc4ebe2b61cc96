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
