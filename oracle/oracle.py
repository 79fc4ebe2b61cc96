"""ctypes front end of the CPU oracle (liboracle.so).  TEST INFRASTRUCTURE ONLY.

Used by tests/, __graft_entry__.smoke() and bench.py's CPU legs as the checker and the CPU baseline;
the product package never imports it.  See moe_oracle.h for what each function restates.
"""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

FMT_NONE, FMT_FP8_B128, FMT_MXFP4 = 0, 1, 2
SCORE_SIGMOID, SCORE_SQRT_SOFTPLUS = 0, 1

_lib = None
P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        for name in ("orc_bf16_round", "orc_pow2_ceil", "orc_e4m3_value"):
            getattr(_lib, name).restype = ctypes.c_float
        _lib.orc_bf16_round.argtypes = [F]
        _lib.orc_pow2_ceil.argtypes = [F]
        _lib.orc_e4m3_value.argtypes = [ctypes.c_uint8]
        _lib.orc_e4m3_encode.restype = ctypes.c_uint8
        _lib.orc_e4m3_encode.argtypes = [F]
    return _lib


def ptr(a):
    return P(a.ctypes.data) if a is not None else P(0)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- scalar formats, vectorised ---------------------------------------------------------------

def bf16_round(x):
    x = _f32(x)
    out = np.empty_like(x)
    lib().orc_bf16_round_n(ptr(x), I(x.size), ptr(out))
    return out


def pow2_ceil(x):
    x = _f32(x)
    out = np.empty_like(x)
    lib().orc_pow2_ceil_n(ptr(x), I(x.size), ptr(out))
    return out


def e4m3_encode(x):
    x = _f32(x)
    out = np.empty(x.shape, np.uint8)
    lib().orc_e4m3_encode_n(ptr(x), I(x.size), ptr(out))
    return out


def e2m1_encode(x):
    x = _f32(x)
    out = np.empty(x.shape, np.uint8)
    lib().orc_e2m1_encode_n(ptr(x), I(x.size), ptr(out))
    return out


def e4m3_values():
    return np.array([lib().orc_e4m3_value(c) for c in range(256)], np.float32)


FP4_TABLE = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], np.float32)


def bf16_bits_to_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x):
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


# ---- quantizers ---------------------------------------------------------------------------------

def act_quant(x, block, pow2):
    x = _f32(x)
    rows, k = x.reshape(-1, x.shape[-1]).shape
    codes = np.empty((rows, k), np.uint8)
    scales = np.empty((rows, k // block), np.float32)
    lib().orc_act_quant(ptr(x), I(rows), I(k), I(block), I(int(pow2)), ptr(codes), ptr(scales))
    return codes, scales


def quant_fp8_b128(w):
    w = _f32(w)
    rows, k = w.shape
    codes = np.empty((rows, k), np.uint8)
    scales = np.empty(((rows + 127) // 128, (k + 127) // 128), np.float32)
    lib().orc_quant_fp8_b128(ptr(w), I(rows), I(k), ptr(codes), ptr(scales))
    return codes, scales


def quant_mxfp4(w):
    w = _f32(w)
    rows, k = w.shape
    packed = np.empty((rows, k // 2), np.uint8)
    scales = np.empty((rows, k // 32), np.uint8)
    lib().orc_quant_mxfp4(ptr(w), I(rows), I(k), ptr(packed), ptr(scales))
    return packed, scales


def quant_fp8_e8m0(w):
    w = _f32(w)
    rows, k = w.shape
    codes = np.empty((rows, k), np.uint8)
    scales = np.empty(((rows + 31) // 32, k // 32), np.uint8)
    lib().orc_quant_fp8_e8m0(ptr(w), I(rows), I(k), ptr(codes), ptr(scales))
    return codes, scales


def mxfp4_to_gguf(codes, scales):
    """Official MXFP4 (codes [rows][k/2], e8m0 [rows][k/32]) -> GGUF 17-byte blocks [rows][k/32][17]."""
    codes, scales = np.ascontiguousarray(codes, np.uint8), np.ascontiguousarray(scales, np.uint8)
    rows, k = codes.shape[0], codes.shape[1] * 2
    blocks = np.empty((rows, k // 32, 17), np.uint8)
    lib().orc_mxfp4_to_gguf(ptr(codes), ptr(scales), I(rows), I(k), ptr(blocks))
    return blocks


def mxfp4_from_gguf(blocks):
    blocks = np.ascontiguousarray(blocks, np.uint8)
    rows, k = blocks.shape[0], blocks.shape[1] * 32
    codes = np.empty((rows, k // 2), np.uint8)
    scales = np.empty((rows, k // 32), np.uint8)
    lib().orc_mxfp4_from_gguf(ptr(blocks), I(rows), I(k), ptr(codes), ptr(scales))
    return codes, scales


def gemv_fp8_b128(w, ws, xc, xs, act_block):
    rows, k = w.shape
    n = xc.shape[0]
    y = np.empty((n, rows), np.float32)
    lib().orc_gemv_fp8_b128(ptr(np.ascontiguousarray(w)), ptr(_f32(ws)), I(rows), I(k), ptr(np.ascontiguousarray(xc)),
                            ptr(_f32(xs)), I(act_block), I(n), ptr(y))
    return y


def gemv_fp8_e8m0(w, ws, xc, xs, act_block):
    rows, k = w.shape
    n = xc.shape[0]
    y = np.empty((n, rows), np.float32)
    lib().orc_gemv_fp8_e8m0(ptr(np.ascontiguousarray(w)), ptr(np.ascontiguousarray(ws)), I(rows), I(k),
                            ptr(np.ascontiguousarray(xc)), ptr(_f32(xs)), I(act_block), I(n), ptr(y))
    return y


def gemv_mxfp4(w, ws, xc, xs, act_block):
    rows = w.shape[0]
    k = w.shape[1] * 2
    n = xc.shape[0]
    y = np.empty((n, rows), np.float32)
    lib().orc_gemv_mxfp4(ptr(np.ascontiguousarray(w)), ptr(np.ascontiguousarray(ws)), I(rows), I(k),
                         ptr(np.ascontiguousarray(xc)), ptr(_f32(xs)), I(act_block), I(n), ptr(y))
    return y


# ---- router / dispatch ----------------------------------------------------------------------------

def q8_codes(x):
    """int8 codes and fp32 scales per 32 along the last axis (ref/emulate_ds4.py:23-30, activations)."""
    x = np.ascontiguousarray(x, np.float32)
    nb = x.size // 32
    q = np.empty(x.shape, np.int8)
    d = np.empty(x.shape[:-1] + (x.shape[-1] // 32,), np.float32)
    lib().orc_q8_codes(ptr(x), I(nb), ptr(q), ptr(d))
    return q, d


def gemv_mxfp4_q8(w, ws, q, d):
    """FP4 expert linear with Q8 activations (ref/emulate_ds4.py:69-77): w codes [rows][k/2], ws e8m0
    [rows][k/32], q int8 [T][k], d fp32 [T][k/32] -> fp32 [T][rows]."""
    w, ws = np.ascontiguousarray(w, np.uint8), np.ascontiguousarray(ws, np.uint8)
    q, d = np.ascontiguousarray(q, np.int8), np.ascontiguousarray(d, np.float32)
    rows, k = w.shape[0], w.shape[1] * 2
    T = q.shape[0]
    y = np.empty((T, rows), np.float32)
    lib().orc_gemv_mxfp4_q8(ptr(w), ptr(ws), I(rows), I(k), ptr(q), ptr(d), I(T), ptr(y))
    return y


def router_logits(W, x_bits):
    W = _f32(W)
    x_bits = np.ascontiguousarray(x_bits, np.uint16)
    E, H = W.shape
    T = x_bits.shape[0]
    out = np.empty((T, E), np.float32)
    lib().orc_router_logits(ptr(W), ptr(x_bits), I(T), I(E), I(H), ptr(out))
    return out


def router_select(logits, bias, topk, n_groups, topk_groups, score_fn, route_scale):
    logits = _f32(logits)
    T, E = logits.shape
    scores = np.empty((T, E), np.float32)
    idx = np.empty((T, topk), np.int32)
    w = np.empty((T, topk), np.float32)
    rc = lib().orc_router_select(ptr(logits), ptr(_f32(bias)), I(T), I(E), I(topk), I(n_groups), I(topk_groups),
                                 I(score_fn), F(route_scale), ptr(scores), ptr(idx), ptr(w))
    if rc:
        raise ValueError("router_select: bad group configuration")
    return scores, idx, w


def dispatch(idx, E):
    idx = np.ascontiguousarray(idx, np.int32)
    T, k = idx.shape
    counts = np.empty(E, np.int32)
    offsets = np.empty(E + 1, np.int32)
    perm = np.empty(T * k, np.int32)
    lib().orc_dispatch(ptr(idx), I(T), I(E), I(k), ptr(counts), ptr(offsets), ptr(perm))
    return counts, offsets, perm


# ---- whole layer ----------------------------------------------------------------------------------

class _Desc(ctypes.Structure):
    _fields_ = [
        ("hidden", I), ("inter", I), ("n_experts", I), ("topk", I), ("n_groups", I), ("topk_groups", I),
        ("score_fn", I), ("route_scale", F), ("swiglu_limit", F), ("routed_fmt", I), ("shared_fmt", I),
        ("router_w", P), ("router_bias", P), ("routed_w", P), ("routed_s", P),
        ("shared_w", P * 3), ("shared_s", P * 3), ("act_q8", I),
    ]


def moe_forward(cfg, weights, x_bits, nthreads=0, forced=None):
    """cfg: dict of layer shapes / routing (see stblarge_b200.config.MoEConfig.as_dict); weights: host
    numpy weights as produced by stblarge_b200.synth (routed[m][e] = (codes, scales) or None,
    shared[m] = (codes, scales) or None).  forced: int [T][topk] routed experts given instead of
    selected (weights from the router's scores of those experts).  Returns (y_bits [T][H] uint16,
    idx, weights)."""
    E = cfg["n_experts"]
    keep = []

    def p(a):
        if a is None:
            return None
        a = np.ascontiguousarray(a)
        keep.append(a)
        return a.ctypes.data

    rw = (P * (3 * E))()
    rs = (P * (3 * E))()
    for m in range(3):
        for e in range(E):
            item = weights["routed"][m][e]
            if item is not None:
                rw[m * E + e] = p(item[0])
                rs[m * E + e] = p(item[1])
    d = _Desc()
    d.hidden, d.inter, d.n_experts, d.topk = cfg["hidden"], cfg["inter"], E, cfg["topk"]
    d.n_groups, d.topk_groups, d.score_fn = cfg["n_groups"], cfg["topk_groups"], cfg["score_fn"]
    d.route_scale, d.swiglu_limit = cfg["route_scale"], cfg["swiglu_limit"]
    d.routed_fmt, d.shared_fmt = cfg["routed_fmt"], cfg["shared_fmt"]
    d.act_q8 = int(cfg.get("act_q8", 0))
    d.router_w = p(_f32(weights["router_w"]))
    d.router_bias = p(_f32(weights["router_bias"]))
    d.routed_w = ctypes.cast(rw, P)
    d.routed_s = ctypes.cast(rs, P)
    if cfg["shared_fmt"] != FMT_NONE:
        for m in range(3):
            d.shared_w[m] = p(weights["shared"][m][0])
            d.shared_s[m] = p(weights["shared"][m][1])
    x_bits = np.ascontiguousarray(x_bits, np.uint16)
    T = x_bits.shape[0]
    y = np.empty((T, cfg["hidden"]), np.uint16)
    idx = np.empty((T, cfg["topk"]), np.int32)
    w = np.empty((T, cfg["topk"]), np.float32)
    if forced is None:
        rc = lib().orc_moe_forward(ctypes.byref(d), ptr(x_bits), I(T), ptr(y), ptr(idx), ptr(w), I(nthreads))
    else:
        f = np.ascontiguousarray(forced, np.int32).reshape(T, cfg["topk"])
        rc = lib().orc_moe_forward_routed(ctypes.byref(d), ptr(x_bits), I(T), ptr(f), ptr(y), ptr(idx), ptr(w), I(nthreads))
    if rc:
        raise ValueError("oracle moe_forward: a routed expert's weights are absent")
    return y, idx, w


# ---- the reference's kernels (stbl/kernels.cu semantics) -------------------------------------------

def ref_act_quant_fp8(x):
    x = _f32(x).copy()
    lib().orc_ref_act_quant_fp8(ptr(x), I(x.size))
    return x


def ref_gemv_fp8(w, scale, x, round_out):
    rows, k = w.shape
    y = np.empty(rows, np.float32)
    lib().orc_ref_gemv_fp8(ptr(y), ptr(np.ascontiguousarray(w)), ptr(np.ascontiguousarray(scale)), ptr(_f32(x)),
                           I(rows), I(k), I(int(round_out)))
    return y


def ref_gemv_mxfp4(w17, x, rows, k):
    y = np.empty(rows, np.float32)
    lib().orc_ref_gemv_mxfp4(ptr(y), ptr(np.ascontiguousarray(w17)), ptr(_f32(x)), I(rows), I(k))
    return y


def ref_gemv_f32(w, x, round_out):
    rows, k = w.shape
    y = np.empty(rows, np.float32)
    lib().orc_ref_gemv_f32(ptr(y), ptr(_f32(w)), ptr(_f32(x)), I(rows), I(k), I(int(round_out)))
    return y


def ref_sqrt_softplus(s):
    s = _f32(s).copy()
    lib().orc_ref_sqrt_softplus(ptr(s), I(s.size))
    return s


def ref_swiglu(g, u, weights, limit, n):
    g, u, weights = _f32(g), _f32(u), _f32(weights)
    out = np.empty(len(weights) * n, np.float32)
    lib().orc_ref_swiglu(ptr(out), ptr(g), ptr(u), ptr(weights), I(len(weights)), F(limit), I(n))
    return out


def ref_axpy(y, x, a):
    y = _f32(y).copy()
    lib().orc_ref_axpy(ptr(y), ptr(_f32(x)), F(a), I(y.size))
    return y


def ref_rms_norm(x, w, eps):
    """k_rms_norm per row of x [rows][dim] (r from a correctly rounded 1/sqrt; see moe_oracle.c)."""
    x, w = _f32(x), _f32(w)
    rows, dim = x.shape
    out = np.empty_like(x)
    lib().orc_ref_rms_norm(ptr(out), ptr(x), ptr(w), I(rows), I(dim), F(eps))
    return out


def ref_hc_post(y, res, post, comb):
    """k_hc_post of one token: y [dim], res [hc][dim], post [hc], comb [hc][hc] -> [hc][dim]."""
    y, res, post, comb = _f32(y), _f32(res), _f32(post), _f32(comb)
    hc, dim = res.shape
    out = np.empty((hc, dim), np.float32)
    lib().orc_ref_hc_post(ptr(out), ptr(y), ptr(res), ptr(post), ptr(comb), I(hc), I(dim))
    return out


# ---- expert cache bookkeeping ---------------------------------------------------------------------

class LruExpertCache:
    """The reference's expert cache decisions (stbl/model.cu:99-106 ExpertCache,
    347-372 take_slot, 386-422 expert(), 478-494 the cancel pass and 503-520 the touch order in moe()):
    an LRU list of (layer, expert) keys, most recent first.  A call first moves its cached experts to
    the front in order, then walks its experts in order: a hit moves to the front again, a miss takes a
    slot freed by a cancelled prefetch, else the next never-used slot (slots are used in order), else
    the slot of the list's last key that no prefetch is still filling, and goes to the front.  A call
    with several tokens walks its distinct experts in order of first appearance (token-major, top-k
    order), the single-token rule applied to the token batch.

    Prefetch jobs (stbl/model.cu:92-97 PfJob) are "queued" or "landed" when a call plans (`pending`
    says which, for all of them: the copy has not started, or it has finished).  A call cancels its own
    layer's queued guesses it does not route to (their slots are freed), takes over the queued ones it
    routes to (a miss, copied into the same slot) and forgets landed guesses of earlier layers.  The
    reference's freed-slot stack is kept in ascending slot order (its cancel pass walks a hash map,
    whose order is unspecified).  Test infrastructure only."""

    def __init__(self, slots):
        self.slots = slots
        self.where = {}      # (layer, expert) -> slot
        self.lru = []        # keys, most recent first
        self.next_slot = 0
        self.free = []       # slots freed by cancelled prefetches
        self.hits = self.misses = 0
        self.last = set()    # keys of the last call (still being read while a prefetch is planned)
        self.jobs = {}       # prefetched keys no call has routed to yet -> "queued" | "landed"
        self.prefetched = self.pf_landed = self.pf_reading = self.cancelled = self.taken = 0

    @property
    def pf_used(self):
        return self.pf_landed + self.pf_reading

    def _front(self, key):
        self.lru.remove(key)
        self.lru.insert(0, key)

    def _victim(self):
        """The key take_slot would evict (the list's last key no prefetch is still filling)."""
        for key in reversed(self.lru):
            if self.jobs.get(key) != "queued":
                return key
        raise RuntimeError("every expert cache slot is being filled")

    def _take_slot(self):
        if self.free:
            s = min(self.free)
            self.free.remove(s)
            return s
        if self.next_slot < self.slots:
            self.next_slot += 1
            return self.next_slot - 1
        key = self._victim()
        self.lru.remove(key)
        self.jobs.pop(key, None)
        return self.where.pop(key)

    def prefetch(self, layer, ids, consider):
        """The reference's prefetch issue (stbl/model.cu:555-569): of the first `consider` distinct ids,
        the ones not cached take a slot (take_slot) and go to the front as queued jobs; cached ones are
        not touched.  Every earlier prefetch copy has ended when a prefetch plans (its jobs that no call
        cancelled or took over have landed).  A slot of the last call's experts is never taken (they may
        still be read): the prefetch stops there.  Returns the placed (slot, expert)."""
        for k in self.jobs:
            self.jobs[k] = "landed"
        order = list(dict.fromkeys(int(e) for e in np.asarray(ids).reshape(-1)))[:consider]
        placed = []
        for e in order:
            key = (layer, e)
            if key in self.where:
                continue
            if not self.free and self.next_slot >= self.slots and self._victim() in self.last:
                break
            s = self._take_slot()
            self.where[key] = s
            self.lru.insert(0, key)
            self.jobs[key] = "queued"
            self.prefetched += 1
            placed.append((s, e))
        return placed

    def call(self, layer, ids, pending="landed"):
        """ids: the call's routed expert ids, token-major.  pending: the state of the prefetch jobs when
        the call plans, "landed" (copied) or "queued" (not started).  Returns the copies of the call
        as (slot, expert): guesses taken over, then misses, each in order."""
        assert pending in ("landed", "queued")
        order = list(dict.fromkeys(int(e) for e in np.asarray(ids).reshape(-1)))
        if pending == "landed":
            for k in self.jobs:
                self.jobs[k] = "landed"
        routed = set(order)
        for key, st in list(self.jobs.items()):
            if key[0] == layer and key[1] not in routed and st == "queued":
                self.free.append(self.where.pop(key))
                self.lru.remove(key)
                del self.jobs[key]
                self.cancelled += 1
            elif key[0] < layer and st == "landed":
                del self.jobs[key]
        for e in order:
            if (layer, e) in self.where:
                self._front((layer, e))
        taken, placed = [], []
        for e in order:
            key = (layer, e)
            if key in self.where:
                self._front(key)
                st = self.jobs.pop(key, None)
                if st == "queued":
                    self.misses += 1
                    self.taken += 1
                    taken.append((self.where[key], e))
                    continue
                self.hits += 1
                if st == "landed":
                    self.pf_landed += 1
            else:
                self.misses += 1
                s = self._take_slot()
                self.where[key] = s
                self.lru.insert(0, key)
                placed.append((s, e))
        self.last = {(layer, e) for e in order}
        return taken + placed

    def state(self, n_layers, n_experts):
        """(map [n_layers][n_experts] slot or -1, owner [slots] layer * n_experts + expert or -1)"""
        m = np.full((n_layers, n_experts), -1, np.int32)
        owner = np.full(self.slots, -1, np.int32)
        for (l, e), s in self.where.items():
            m[l, e] = s
            owner[s] = l * n_experts + e
        return m, owner
