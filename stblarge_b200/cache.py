"""Host-side mirror of the GPU expert cache (stbl_cache_* C ABI, the reference's expert cache,
stbl/model.cu:99-106, 347-422).

    store = host_store(cfg, n_layers)                  # pinned host tensors, every expert of every layer
    cache = ExpertCache(cfg, n_layers, slots, store)   # `slots` experts in device memory
    layer = MoELayer(cfg, resident_weights, max_tokens=1, cache=(cache, l))
    y = layer(x)                                       # the call brings its experts into the cache
    cache.stats()                                      # hits, misses, bytes copied

The planning (hits, LRU victims) and the copies of missing experts run on the GPU inside the layer
call, ordered on its stream; nothing here synchronises except stats() / state().

A cache can also stream its experts from the GGUF checkpoint instead of a host store (the reference's
expert reads from the file, stbl/model.cu:269-308; stblarge_b200/gguf.py: file_cache):

    cache = ExpertCache(cfg, n_layers, slots, file={"path": p, "offsets": [[gate, up, down], ...]})
    cache.file_stats()                                 # pieces, bytes and seconds read, O_DIRECT or not
"""

import ctypes

import numpy as np
import torch

from . import lib as L
from . import synth
from .config import MoEConfig


def host_store(cfg: MoEConfig, n_layers: int, seed_of=None, physical=None):
    """Pinned host tensors holding the routed experts of n_layers layers, expert-major:
    'w'[m]: uint8 [n_layers * E, ...], 's'[m]: scales [n_layers * E, ...] (the layout of
    synth.device_layer's routed tensors, one layer after another).  Layer l's expert e gets the
    synthetic weights of seed seed_of(l, e) (default 1000 + l * E + e).  physical: hold only that many
    distinct experts and repeat them (store row r = physical row r % physical); the bytes each expert
    moves are the same, the host memory is smaller."""
    E = cfg.n_experts
    n = n_layers * E
    seed_of = seed_of or (lambda l, e: 1000 + l * E + e)
    rows = n if physical is None else min(physical, n)
    w0, s0 = synth.routed_expert(cfg, 0)
    w = [torch.empty((rows,) + tuple(t.shape), dtype=t.dtype, pin_memory=True) for t in w0]
    s = [torch.empty((rows,) + tuple(t.shape), dtype=t.dtype, pin_memory=True) for t in s0]
    for r in range(rows):
        l, e = divmod(r, E)
        ws, ss = synth.routed_expert(cfg, seed_of(l, e))
        for m in range(3):
            w[m][r].copy_(ws[m])
            s[m][r].copy_(ss[m])
    return {"w": w, "s": s, "rows": rows, "n": n}


class ExpertCache:
    def __init__(self, cfg: MoEConfig, n_layers: int, slots: int, store: dict = None, file: dict = None):
        """store: a host_store(); or file: {'path', 'offsets' ([n_layers][3] file offsets of the layers'
        gate / up / down expert tensors), optional 'readers', 'direct' (default 1), 'stage_experts'}."""
        if (store is None) == (file is None):
            raise ValueError("give exactly one of store and file")
        self.lib = L.load()
        self.cfg, self.n_layers, self.slots = cfg, n_layers, slots
        self.store = store  # keeps the pinned tensors alive
        d = L.CacheDesc()
        d.n_layers, d.n_experts, d.slots, d.fmt = n_layers, cfg.n_experts, slots, cfg.routed_fmt
        d.hidden, d.inter = cfg.hidden, cfg.inter
        err = ctypes.create_string_buffer(512)
        h = ctypes.c_void_p()
        if file is not None:
            offsets = np.ascontiguousarray(np.asarray(file["offsets"], np.uint64).reshape(n_layers, 3))
            f = L.CacheFileDesc()
            f.path = str(file["path"]).encode()
            f.offset = offsets.ctypes.data
            f.readers, f.direct = file.get("readers", 0), file.get("direct", 1)
            f.stage_experts = file.get("stage_experts", 0)
            if self.lib.stbl_cache_create_file(ctypes.byref(d), ctypes.byref(f), ctypes.byref(h), err, 512) != 0:
                raise RuntimeError("stbl_cache_create_file: " + err.value.decode())
        else:
            for m in range(3):
                w, s = store["w"][m], store["s"][m]
                d.host_w[m], d.host_s[m] = w.data_ptr(), s.data_ptr()
                d.host_w_stride[m] = w.stride(0) * w.element_size()
                d.host_s_stride[m] = s.stride(0) * s.element_size()
            d.host_rows = store["rows"]
            if self.lib.stbl_cache_create(ctypes.byref(d), ctypes.byref(h), err, 512) != 0:
                raise RuntimeError("stbl_cache_create: " + err.value.decode())
        self.handle = h
        self.file = file
        n, b = L.I(), L.U64()
        if self.lib.stbl_cache_info(self.handle, ctypes.byref(n), ctypes.byref(b)) != 0:
            raise RuntimeError("stbl_cache_info failed")
        self.slots, self.slot_bytes = n.value, b.value  # slots=0 asks the library to size the cache

    def layer_desc(self, desc):
        if self.lib.stbl_cache_layer_desc(self.handle, ctypes.byref(desc)) != 0:
            raise RuntimeError("stbl_cache_layer_desc failed")

    def stats(self):
        h, m, b = L.U64(), L.U64(), L.U64()
        if self.lib.stbl_cache_stats(self.handle, ctypes.byref(h), ctypes.byref(m), ctypes.byref(b)) != 0:
            raise RuntimeError("stbl_cache_stats failed")
        return {"hits": h.value, "misses": m.value, "bytes": b.value}

    def prefetch_stats(self):
        """Experts prefetched, prefetched experts a later call routed to (landed or being copied), bytes
        the prefetch copies wrote (cancelled and taken-over guesses are not copied by them)."""
        p, u, b = L.U64(), L.U64(), L.U64()
        if self.lib.stbl_cache_prefetch_stats(self.handle, ctypes.byref(p), ctypes.byref(u), ctypes.byref(b)) != 0:
            raise RuntimeError("stbl_cache_prefetch_stats failed")
        return {"prefetched": p.value, "used": u.value, "bytes": b.value}

    def prefetch_counters(self):
        """The reference's stbl_prefetch layout: issued, routed after landing, routed while being
        copied, cancelled."""
        out = (L.U64 * 4)()
        if self.lib.stbl_cache_prefetch_counters(self.handle, out) != 0:
            raise RuntimeError("stbl_cache_prefetch_counters failed")
        return [int(v) for v in out]

    def file_stats(self):
        """File-backed caches: pieces and bytes read, seconds the read steps took, whether reads go
        through O_DIRECT, read rounds that failed."""
        p, b, sec, di, fr = L.U64(), L.U64(), ctypes.c_double(), L.I(), L.U64()
        if self.lib.stbl_cache_file_stats(self.handle, ctypes.byref(p), ctypes.byref(b), ctypes.byref(sec), ctypes.byref(di),
                                          ctypes.byref(fr)) != 0:
            raise RuntimeError("stbl_cache_file_stats: not a file-backed cache")
        return {"pieces": p.value, "bytes": b.value, "seconds": sec.value, "direct": bool(di.value), "failed_rounds": fr.value}

    def inject_read_error(self, after, err_no):
        """Host-side fault injection (tests): read number `after` and every later one fail with err_no."""
        if self.lib.stbl_cache_inject_read_error(self.handle, after, err_no) != 0:
            raise RuntimeError("stbl_cache_inject_read_error failed")

    def error(self):
        return self.lib.stbl_cache_error(self.handle).decode()

    def state(self):
        mp = np.empty((self.n_layers, self.cfg.n_experts), np.int32)
        owner = np.empty(self.slots, np.int32)
        if self.lib.stbl_cache_state(self.handle, mp.ctypes.data, owner.ctypes.data) != 0:
            raise RuntimeError("stbl_cache_state failed")
        return mp, owner

    def close(self):
        if self.handle:
            self.lib.stbl_cache_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
