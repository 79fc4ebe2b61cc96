"""Host-side mirror of the MoE layer: a thin Python object over the stbl_moe C ABI.

    layer = MoELayer(cfg, weights, max_tokens=16)   # weights: device tensors (see synth.device_layer)
    y = layer(x)                                     # x: cuda bf16 [T, hidden] -> y: cuda bf16 [T, hidden]
    route = layer.last_route()                       # expert ids, weights, dispatch permutation

The layer call enqueues three kernels on the current torch stream (router + dispatch, expert
up + SwiGLU, expert down + combine) and never synchronises.  `forward_host` is the end-to-end form
(host buffers in and out, as the reference's stbl_block_test stage 4).
"""

import ctypes

import numpy as np
import torch

from . import lib as L
from .config import FMT_FP8_B128, FMT_NONE, MoEConfig


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


EP_HANDLE_BYTES = 64


class MoELayer:
    """ep: (rank, n_ranks, process_group) for expert parallelism: `weights` then holds this rank's
    routed experts [rank E/n, (rank+1) E/n) (synth.device_layer(cfg, experts=range(...))) and the
    full router; the layers of all ranks connect through their exchange regions (handles gathered
    with torch.distributed over the group), and every rank must then call forward in lockstep."""

    def __init__(self, cfg: MoEConfig, weights: dict, max_tokens: int = 16, ep=None, cache=None):
        """cache: (ExpertCache, layer index): the routed experts live in the cache (weights then needs
        only 'router_w', 'router_bias' and the shared expert)."""
        self.lib = L.load()
        self.cfg = cfg
        self.weights = weights  # keeps the device tensors alive
        self.max_tokens = max_tokens
        d = L.MoEDesc()
        d.hidden, d.inter, d.n_experts, d.topk = cfg.hidden, cfg.inter, cfg.n_experts, cfg.topk
        d.n_groups, d.topk_groups, d.score_fn = cfg.n_groups, cfg.topk_groups, cfg.score_fn
        d.route_scale, d.swiglu_limit = cfg.route_scale, cfg.swiglu_limit
        d.routed_fmt, d.shared_fmt, d.max_tokens = cfg.routed_fmt, cfg.shared_fmt, max_tokens
        d.act_q8 = cfg.act_q8
        d.router_w = weights["router_w"].data_ptr()
        d.router_bias = weights["router_bias"].data_ptr()
        if cache is not None:
            cache[0].layer_desc(d)
        for m in range(3):
            if cache is None:
                w, s = weights["routed_w"][m], weights["routed_s"][m]
                d.routed_w[m], d.routed_s[m] = w.data_ptr(), s.data_ptr()
                d.routed_w_stride[m] = w.stride(0) * w.element_size()
                d.routed_s_stride[m] = s.stride(0) * s.element_size()
            if cfg.shared_fmt != FMT_NONE:
                d.shared_w[m] = weights["shared_w"][m].data_ptr()
                d.shared_s[m] = weights["shared_s"][m].data_ptr()
        err = ctypes.create_string_buffer(512)
        h = ctypes.c_void_p()
        rank, n_ranks, group = ep if ep is not None else (0, 1, None)
        if self.lib.stbl_moe_create_ep(ctypes.byref(d), rank, n_ranks, ctypes.byref(h), err, 512) != 0:
            raise RuntimeError("stbl_moe_create_ep: " + err.value.decode())
        self.handle = h
        self._desc = d
        self.ep = (rank, n_ranks)
        self.cache = cache
        if cache is not None:
            self._check(self.lib.stbl_moe_attach_cache(self.handle, cache[0].handle, cache[1]), "stbl_moe_attach_cache")
        if n_ranks > 1:
            import torch.distributed as dist
            mine = ctypes.create_string_buffer(EP_HANDLE_BYTES)
            self._check(self.lib.stbl_moe_ep_handle(self.handle, mine), "stbl_moe_ep_handle")
            allh = [None] * n_ranks
            dist.all_gather_object(allh, bytes(mine.raw), group=group)
            blob = ctypes.create_string_buffer(b"".join(allh), EP_HANDLE_BYTES * n_ranks)
            self._check(self.lib.stbl_moe_ep_connect(self.handle, blob), "stbl_moe_ep_connect")

    def _check(self, rc, what):
        if rc < 0:
            raise RuntimeError(f"{what}: {self.lib.stbl_moe_error(self.handle).decode()}")
        return rc

    def __call__(self, x, out=None, stream=None):
        return self.forward(x, out, stream)

    def forward(self, x, out=None, stream=None):
        """x: cuda [T, hidden] bfloat16 (or int16/uint16 bf16 bits)."""
        assert x.is_cuda and x.dim() == 2 and x.shape[1] == self.cfg.hidden and x.element_size() == 2
        x = x.contiguous()
        if out is None:
            out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
        st = stream if stream is not None else torch.cuda.current_stream(x.device)
        self._check(self.lib.stbl_moe_forward(self.handle, _ptr(x), x.shape[0], _ptr(out), ctypes.c_void_p(st.cuda_stream)),
                    "stbl_moe_forward")
        return out

    def forward_routed(self, x, idx, out=None, stream=None):
        """The layer with its routed experts given: idx cuda int32 [T, topk] (distinct per token)."""
        assert x.is_cuda and x.dim() == 2 and x.shape[1] == self.cfg.hidden and x.element_size() == 2
        assert idx.is_cuda and idx.dtype == torch.int32 and tuple(idx.shape) == (x.shape[0], self.cfg.topk)
        x, idx = x.contiguous(), idx.contiguous()
        if out is None:
            out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
        st = stream if stream is not None else torch.cuda.current_stream(x.device)
        self._check(self.lib.stbl_moe_forward_routed(self.handle, _ptr(x), x.shape[0], _ptr(idx), _ptr(out),
                                                     ctypes.c_void_p(st.cuda_stream)), "stbl_moe_forward_routed")
        return out

    def attach_prefetch(self, next_layer, n_predict, consider, copy_stream):
        """Each call also runs next_layer's router on this call's input and prefetches its top n_predict
        experts per token (the first `consider` distinct ones) into the shared expert cache, copied on
        copy_stream (a torch.cuda.Stream) beside this call's experts (stbl_moe_attach_prefetch).
        next_layer None stops it."""
        self._pf = (next_layer, copy_stream)  # keep both alive while attached
        self._check(self.lib.stbl_moe_attach_prefetch(self.handle, next_layer.handle if next_layer is not None else None,
                                                      n_predict, consider,
                                                      ctypes.c_void_p(copy_stream.cuda_stream if copy_stream is not None else 0)),
                    "stbl_moe_attach_prefetch")

    def forward_block(self, x_pre, norm_w, eps, res, post, comb, out=None, stream=None):
        """The layer inside its block (stbl_moe_forward_block; stbl/model.cu:803-805): RMSNorm of x_pre
        (cuda float32 [T, hidden]) with norm_w (float32 [hidden]) and eps before it, the hyper-connection
        post after it: res float32 [T, hc, hidden], post [T, hc], comb [T, hc, hc] -> float32 [T, hc, hidden]."""
        T, H = x_pre.shape
        hc = res.shape[1]
        assert H == self.cfg.hidden and tuple(res.shape) == (T, hc, H) and tuple(post.shape) == (T, hc)
        assert tuple(comb.shape) == (T, hc, hc) and tuple(norm_w.shape) == (H,)
        ts = [t.contiguous() for t in (x_pre, norm_w, res, post, comb)]
        assert all(t.is_cuda and t.dtype == torch.float32 for t in ts)
        if out is None:
            out = torch.empty(T, hc, H, dtype=torch.float32, device=x_pre.device)
        st = stream if stream is not None else torch.cuda.current_stream(x_pre.device)
        x_pre, norm_w, res, post, comb = ts
        self._check(self.lib.stbl_moe_forward_block(self.handle, _ptr(x_pre), _ptr(norm_w), ctypes.c_float(eps), _ptr(res),
                                                    _ptr(post), _ptr(comb), hc, T, _ptr(out), ctypes.c_void_p(st.cuda_stream)),
                    "stbl_moe_forward_block")
        return out

    def forward_host(self, x_bits, y_bits=None, stream=None):
        """End to end with host buffers: x_bits uint16 [T, hidden] (numpy or pinned torch)."""
        if isinstance(x_bits, np.ndarray):
            x_bits = np.ascontiguousarray(x_bits, np.uint16)
            T = x_bits.shape[0]
            y = np.empty_like(x_bits) if y_bits is None else y_bits
            xp, yp = x_bits.ctypes.data, y.ctypes.data
        else:
            T = x_bits.shape[0]
            y = torch.empty_like(x_bits) if y_bits is None else y_bits
            xp, yp = x_bits.data_ptr(), y.data_ptr()
        st = stream if stream is not None else torch.cuda.current_stream()
        self._check(self.lib.stbl_moe_forward_host(self.handle, ctypes.c_void_p(xp), T, ctypes.c_void_p(yp),
                                                   ctypes.c_void_p(st.cuda_stream)), "stbl_moe_forward_host")
        return y

    def last_route(self):
        cfg = self.cfg
        T = self.max_tokens
        idx = np.empty((T, cfg.topk), np.int32)
        w = np.empty((T, cfg.topk), np.float32)
        counts = np.empty(cfg.n_experts, np.int32)
        offsets = np.empty(cfg.n_experts + 1, np.int32)
        perm = np.empty(T * cfg.topk, np.int32)
        T = self._check(self.lib.stbl_moe_last_route(self.handle, idx.ctypes.data, w.ctypes.data, counts.ctypes.data,
                                                     offsets.ctypes.data, perm.ctypes.data), "stbl_moe_last_route")
        return {"idx": idx[:T], "weights": w[:T], "counts": counts, "offsets": offsets, "perm": perm[:T * cfg.topk]}

    ACTS_X_ROUTED, ACTS_X_SHARED, ACTS_H_ROUTED, ACTS_H_SHARED = 0, 1, 2, 3

    def last_acts(self, which):
        """Quantized activations of the last call as the expert kernels read them
        (stbl_moe_last_acts): {'codes': uint8 [rows, width], 'scales': float32 [rows, width / blk],
        'blk': blk, 'h': bf16 bits uint16 [rows, width] for the h rows}.  x rows are tokens; h rows
        are dispatch positions (routed) or tokens (shared)."""
        cfg = self.cfg
        T = self.max_tokens
        x = which in (self.ACTS_X_ROUTED, self.ACTS_X_SHARED)
        shared = which in (self.ACTS_X_SHARED, self.ACTS_H_SHARED)
        fmt = cfg.shared_fmt if shared else cfg.routed_fmt
        blk = 128 if fmt == FMT_FP8_B128 else 32
        width = cfg.hidden if x else cfg.inter
        rows_max = T if (x or shared) else T * cfg.topk
        codes = np.empty((rows_max, width), np.uint8)
        scales = np.empty((rows_max, width // blk), np.float32)
        h = None if x else np.empty((rows_max, width), np.uint16)
        rows = self._check(self.lib.stbl_moe_last_acts(self.handle, which, h.ctypes.data if h is not None else None,
                                                       codes.ctypes.data, scales.ctypes.data), "stbl_moe_last_acts")
        out = {"codes": codes[:rows], "scales": scales[:rows], "blk": blk,
               "rule": "q8" if (cfg.act_q8 and not shared) else ("fp32" if blk == 128 else "pow2")}
        if h is not None:
            out["h"] = h[:rows]
        return out

    def last_scores(self):
        s = np.empty((self.max_tokens, self.cfg.n_experts), np.float32)
        T = self._check(self.lib.stbl_moe_last_scores(self.handle, s.ctypes.data), "stbl_moe_last_scores")
        return s[:T]

    def set_expert_slot(self, e, slot, stream=None):
        """Routed expert e reads slot `slot` of the layer's expert arrays from now on (an expert cache
        that keeps experts in a pool of slots re-points them this way)."""
        w = [self.weights["routed_w"][m][slot] for m in range(3)]
        s = [self.weights["routed_s"][m][slot] for m in range(3)]
        self.set_expert(e, w, s, stream)

    def set_expert(self, e, w, s, stream=None):
        """Point routed expert e at another slot of the layer's expert arrays (three codes, three
        scales, all of the same slot)."""
        wp = (ctypes.c_void_p * 3)(*[t.data_ptr() for t in w])
        sp = (ctypes.c_void_p * 3)(*[t.data_ptr() for t in s])
        st = stream if stream is not None else torch.cuda.current_stream()
        self._check(self.lib.stbl_moe_set_expert(self.handle, e, wp, sp, ctypes.c_void_p(st.cuda_stream)),
                    "stbl_moe_set_expert")

    def status(self):
        s = ctypes.c_uint32()
        self._check(self.lib.stbl_moe_status(self.handle, ctypes.byref(s)), "stbl_moe_status")
        return s.value

    def set_timing(self, enable=True):
        self._check(self.lib.stbl_moe_set_timing(self.handle, int(enable)), "stbl_moe_set_timing")

    def timing(self):
        """Per-kernel device seconds summed over the timed calls: router, up, down, calls."""
        sec = np.zeros(4, np.float64)
        self._check(self.lib.stbl_moe_timing(self.handle, sec.ctypes.data, 4), "stbl_moe_timing")
        return {"router": sec[0], "up": sec[1], "down": sec[2], "calls": int(sec[3])}

    def stats(self):
        calls, tokens, launches = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_int()
        self.lib.stbl_moe_stats(self.handle, ctypes.byref(calls), ctypes.byref(tokens), ctypes.byref(launches))
        return {"calls": calls.value, "tokens": tokens.value, "launches_per_call": launches.value}

    def close(self):
        if getattr(self, "handle", None):
            self.lib.stbl_moe_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def host_weights_to_device(cfg, W, device="cuda", experts=None):
    """Upload numpy weights made by synth.host_layer into the expert-major device layout (the routed
    experts in `experts`, e.g. an expert-parallel rank's shard; all by default)."""
    experts = range(cfg.n_experts) if experts is None else experts
    out = {"router_w": torch.from_numpy(W["router_w"]).to(device),
           "router_bias": torch.from_numpy(W["router_bias"]).to(device),
           "routed_w": [], "routed_s": [], "shared_w": None, "shared_s": None}
    for m in range(3):
        out["routed_w"].append(torch.from_numpy(np.stack([W["routed"][m][e][0] for e in experts])).to(device))
        out["routed_s"].append(torch.from_numpy(np.stack([W["routed"][m][e][1] for e in experts])).to(device))
    if cfg.shared_fmt != FMT_NONE:
        out["shared_w"] = [torch.from_numpy(W["shared"][m][0]).to(device) for m in range(3)]
        out["shared_s"] = [torch.from_numpy(W["shared"][m][1]).to(device) for m in range(3)]
    return out
