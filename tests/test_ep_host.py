"""Expert-parallel host logic on CPU, as two gloo ranks: every rank routes its own tokens with the
oracle, the ranks exchange their choices through torch.distributed, and each checks that the
device's closed-form receive-row rule (tests/ep_mirror.py: counts_rule) places its assignments
exactly where the explicit layout (expert-major, then source rank, then token order) puts them,
and that every owner's rows are filled once each."""

import socket

import numpy as np
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from stblarge_b200 import synth
from stblarge_b200.config import CFG1, CFG2
from tests.ep_mirror import counts_rule, receive_rows


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _route(cfg, W, b, T, seed):
    x = synth.make_x(cfg.hidden, T, seed=seed)
    lg = O.router_logits(W, x)
    _, idx, _ = O.router_select(lg, b, cfg.topk, cfg.n_groups, cfg.topk_groups, cfg.score_fn, cfg.route_scale)
    return idx


def _layout_worker(rank, n, port, q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=n)
        out = []
        for cfg, T in ((CFG1, 4 + rank), (CFG2, 16)):
            W, b = synth.router_w(cfg), synth.router_bias(cfg)
            idx = _route(cfg, W, b, T, seed=900 + rank)
            allidx = [None] * n
            dist.all_gather_object(allidx, idx)
            a_dst, rows = receive_rows(allidx, cfg.n_experts, n)
            mine = counts_rule(allidx, cfg.n_experts, n, rank)
            ok = np.array_equal(mine, a_dst[rank])
            # every owner's rows are distinct and contiguous from 0
            filled = all(sorted(r for s in range(n) for a, r in enumerate(a_dst[s]) if allidx[s].reshape(-1)[a] // (cfg.n_experts // n) == d)
                         == list(range(len(rows[d]))) for d in range(n))
            out.append((cfg.name, bool(ok), bool(filled)))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, out, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))


def test_receive_rows_rule_matches_layout_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_layout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    for rank, out, err in res:
        assert err is None, f"rank {rank}: {err}"
        for name, ok, filled in out:
            assert ok, f"rank {rank} {name}: closed-form rows differ from the layout"
            assert filled, f"rank {rank} {name}: receive rows not filled exactly once"
