"""Host mirror of the expert-parallel receive-row layout (the rule ep_counts_kernel applies on the
device, stblarge_b200/csrc/ep.cu): rank d owns routed experts [d E/n, (d+1) E/n); its receive rows
hold every source rank's assignments to those experts, expert-major, then by source rank, then in
the source's token order.  Test infrastructure only."""

import numpy as np


def receive_rows(idx_by_rank, E, n):
    """idx_by_rank[s]: int [T_s, topk] global expert ids chosen by source rank s.
    Returns (a_dst, rows): a_dst[s] int [T_s topk], the receive row of each of s's assignments at its
    owner; rows[d]: list of (source rank, assignment) in receive-row order."""
    E_loc = E // n
    flat = [np.asarray(i, np.int64).reshape(-1) for i in idx_by_rank]
    rows = [[] for _ in range(n)]
    for d in range(n):
        for e in range(d * E_loc, (d + 1) * E_loc):
            for s in range(n):
                for a in np.nonzero(flat[s] == e)[0]:
                    rows[d].append((s, int(a)))
    a_dst = [np.full(f.size, -1, np.int64) for f in flat]
    for d in range(n):
        for r, (s, a) in enumerate(rows[d]):
            a_dst[s][a] = r
    return a_dst, rows


def counts_rule(idx_by_rank, E, n, s):
    """The device's closed form for source s: row of expert e's first assignment from s at its owner
    = rows of the owner's earlier experts + the assignments to e from ranks below s."""
    E_loc = E // n
    C = np.stack([np.bincount(np.asarray(i).reshape(-1), minlength=E) for i in idx_by_rank])
    tot = C.sum(0)
    dst_off = np.zeros(E, np.int64)
    for e in range(E):
        seg = (e // E_loc) * E_loc
        dst_off[e] = tot[seg:e].sum() + C[:s, e].sum()
    flat = np.asarray(idx_by_rank[s]).reshape(-1)
    a_dst = np.empty(flat.size, np.int64)
    seen = np.zeros(E, np.int64)
    for a in range(flat.size):  # token order = the bucketed permutation's order within an expert
        e = flat[a]
        a_dst[a] = dst_off[e] + seen[e]
        seen[e] += 1
    return a_dst
