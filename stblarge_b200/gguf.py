"""GGUF checkpoints: the reference engine's on-disk format for the MoE layer's weights.

GgufFile wraps the library's reader (include/stbl_gguf.h: mmap, metadata and tensor tables; the
reference's GgufFile, stbl/gguf.h:17-31).  load_moe_layer builds one MoE layer's device tensors from
a file converted the reference's way (tools/convert_official.py:116-126; loaded by
stbl/model.cu:933-947):

    blk.N.ffn_gate_inp.weight     F32        dims (hidden, experts)      router W, [E][H]
    blk.N.exp_probs_b.bias        F32        dims (experts,)             correction bias
    blk.N.ffn_{gate,up,down}_shexp.weight   STBL_E4M3 (200)  dims (k, rows)    shared expert codes
    blk.N.ffn_{gate,up,down}_shexp.scale    STBL_E8M0 (201)  dims (k/32, rows/32)  its 32x32 block scales
    blk.N.ffn_{gate,up,down}_exps.weight    MXFP4 (39)  dims (k, rows, experts)  17-byte blocks

and the model's metadata under the `deepseek41.` prefix (hidden_size, moe_intermediate_size,
n_routed_experts, num_experts_per_tok, routed_scaling_factor, swiglu_limit; stbl/model.cu:842-867).
The expert blocks are converted on the device (stbl_mxfp4_from_gguf) into the layer's MXFP4 layout.

write_gguf writes a GGUF v3 file (the layout the reference's converter writes,
tools/convert_official.py:204-243): header, metadata records, tensor records, the data section at
the next multiple of the alignment, each tensor padded to the alignment.
"""

import ctypes
import struct

import numpy as np

from . import lib as L
from .config import FMT_FP8_E8M0, FMT_MXFP4, FMT_NONE, SCORE_SQRT_SOFTPLUS, MoEConfig

# GGUF metadata value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?", U64: "<Q",
           I64: "<q", F64: "<d"}

# tensor types (ggml ids and the reference's FP8 pair)
T_F32, T_F16, T_Q8_0, T_I8, T_BF16, T_MXFP4, T_STBL_E4M3, T_STBL_E8M0 = 0, 1, 8, 24, 30, 39, 200, 201
_BLOCK = {T_F32: (1, 4), T_F16: (1, 2), T_Q8_0: (32, 34), T_I8: (1, 1), T_BF16: (1, 2), T_MXFP4: (32, 17),
          T_STBL_E4M3: (1, 1), T_STBL_E8M0: (1, 1)}

PREFIX = "deepseek41."


def tensor_nbytes(ttype, dims):
    block, nb = _BLOCK[ttype]
    n = int(np.prod(dims, dtype=np.uint64)) if len(dims) else 1
    if n % block:
        raise ValueError(f"{n} elements are not a multiple of the type's {block}-element block")
    return n // block * nb


class GgufFile:
    """A GGUF file opened by the library's reader.  Tensor data are numpy views of the read-only
    mapping, valid until close()."""

    def __init__(self, path):
        self.lib = L.load()
        self.handle = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        if self.lib.stbl_gguf_open(str(path).encode(), ctypes.byref(self.handle), err, 512) != 0:
            raise ValueError(f"{path}: {err.value.decode()}")
        v, a, nkv, nt = L.U32(), L.U64(), L.U64(), L.U64()
        self.lib.stbl_gguf_info(self.handle, ctypes.byref(v), ctypes.byref(a), ctypes.byref(nkv), ctypes.byref(nt))
        self.version, self.alignment, self.n_kv, self.n_tensors = v.value, a.value, nkv.value, nt.value

    def close(self):
        if self.handle:
            self.lib.stbl_gguf_close(self.handle)
            self.handle = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @staticmethod
    def _info(t):
        return {"name": t.name.decode(), "type": t.type, "dims": tuple(t.dims[d] for d in range(t.n_dims)),
                "offset": t.offset, "nbytes": t.nbytes, "data": t.data}

    def tensors(self):
        out = []
        for i in range(self.n_tensors):
            t = L.GgufTensor()
            self.lib.stbl_gguf_tensor_at(self.handle, i, ctypes.byref(t))
            out.append(self._info(t))
        return out

    def tensor(self, name):
        """The tensor's record, or None when the file has no such tensor."""
        t = L.GgufTensor()
        if self.lib.stbl_gguf_find(self.handle, name.encode(), ctypes.byref(t)) != 0:
            return None
        return self._info(t)

    def bytes_of(self, name):
        """The tensor's data as a uint8 view of the mapping."""
        t = self.tensor(name)
        if t is None:
            raise KeyError(f"missing tensor {name}")
        if t["nbytes"] == 0:
            return np.zeros(0, np.uint8)
        buf = (ctypes.c_uint8 * t["nbytes"]).from_address(t["data"])
        return np.frombuffer(buf, dtype=np.uint8)

    def keys(self):
        out = []
        for i in range(self.n_kv):
            k, ty = ctypes.c_char_p(), L.U32()
            self.lib.stbl_gguf_kv_at(self.handle, i, ctypes.byref(k), ctypes.byref(ty))
            out.append((k.value.decode(), ty.value))
        return out

    def u32(self, key):
        v = L.U32()
        if self.lib.stbl_gguf_u32(self.handle, key.encode(), ctypes.byref(v)) != 0:
            raise KeyError(f"missing u32 {key}")
        return v.value

    def f32(self, key):
        v = ctypes.c_float()
        if self.lib.stbl_gguf_f32(self.handle, key.encode(), ctypes.byref(v)) != 0:
            raise KeyError(f"missing f32 {key}")
        return v.value

    def uints(self, key):
        n = self.lib.stbl_gguf_uints(self.handle, key.encode(), None, 0)
        if n < 0:
            raise KeyError(f"missing u32/u64 array {key}")
        v = (L.U64 * max(n, 1))()
        self.lib.stbl_gguf_uints(self.handle, key.encode(), v, n)
        return [int(v[i]) for i in range(n)]

    def string(self, key):
        n = self.lib.stbl_gguf_str(self.handle, key.encode(), None, 0)
        if n < 0:
            raise KeyError(f"missing string {key}")
        buf = ctypes.create_string_buffer(n + 1)
        self.lib.stbl_gguf_str(self.handle, key.encode(), buf, n + 1)
        return buf.raw[:n].decode()


# ---- writing ---------------------------------------------------------------------------------------

def _str(s):
    b = s.encode() if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


def _value(vtype, value):
    if vtype == STRING:
        return _str(value)
    if vtype == ARRAY:
        etype, items = value
        out = struct.pack("<IQ", etype, len(items))
        return out + b"".join(_value(etype, x) for x in items)
    return struct.pack(_SCALAR[vtype], value)


def kv(key, vtype, value):
    """One metadata record; for ARRAY the value is (element type, items)."""
    return _str(key) + struct.pack("<I", vtype) + _value(vtype, value)


class Repeated:
    """Tensor data given as `chunk` repeated `count` times (large synthetic checkpoints written without
    holding them in memory)."""

    def __init__(self, chunk, count):
        self.chunk, self.count = bytes(chunk), int(count)

    def __len__(self):
        return len(self.chunk) * self.count


def write_gguf(path, records, tensors, alignment=32):
    """records: metadata records (kv(...) bytes); tensors: (name, type, dims innermost first, bytes or
    Repeated).  The data offsets follow the tensors' order, each padded to the alignment."""
    infos, offset, payload = [], 0, []
    for name, ttype, dims, data in tensors:
        if not isinstance(data, Repeated):
            data = bytes(data)
        if len(data) != tensor_nbytes(ttype, dims):
            raise ValueError(f"{name}: {len(data)} bytes for a {ttype} tensor of dims {dims}")
        infos.append(_str(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
                     + struct.pack("<IQ", ttype, offset))
        pad = (-len(data)) % alignment
        payload.append((data, pad))
        offset += len(data) + pad
    header = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(records)) + b"".join(records) + b"".join(infos)
    header += bytes((-len(header)) % alignment)
    with open(path, "wb") as f:
        f.write(header)
        for data, pad in payload:
            if isinstance(data, Repeated):
                for _ in range(data.count):
                    f.write(data.chunk)
            else:
                f.write(data)
            f.write(bytes(pad))


def mxfp4_to_blocks(codes, scales):
    """The layer's MXFP4 layout (codes [rows][k/2], values 2j and 2j+1 in byte j, low nibble first; e8m0
    scales [rows][k/32]) -> GGUF blocks [rows][k/32 * 17] (per 32 values the scale, then values i and
    16 + i in the low and high nibble of byte i; the reference converter's layout,
    tools/convert_official.py:187-201); the inverse of stbl_mxfp4_from_gguf."""
    codes, scales = np.asarray(codes, np.uint8), np.asarray(scales, np.uint8)
    rows, nb = scales.shape
    c = codes.reshape(rows, nb, 16)
    v = np.stack([c & 15, c >> 4], -1).reshape(rows, nb, 32)  # values in order
    out = np.empty((rows, nb, 17), np.uint8)
    out[..., 0] = scales
    out[..., 1:] = v[..., :16] | (v[..., 16:] << 4)
    return out.reshape(rows, nb * 17)


def moe_layer_tensors(layer, router_w, router_bias, shared, experts):
    """The tensor records of one MoE layer in the reference's names and types.  router_w float32
    [E][H]; router_bias float32 [E]; shared: None or [(codes uint8 [rows][k], e8m0 scales uint8
    [ceil(rows/32)][ceil(k/32)])] x 3 (gate, up, down); experts: [GGUF MXFP4 blocks uint8
    [E][rows][k/32 * 17]] x 3."""
    b = f"blk.{layer}."
    E, H = router_w.shape
    out = [(b + "ffn_gate_inp.weight", T_F32, (H, E), np.ascontiguousarray(router_w, np.float32).tobytes()),
           (b + "exp_probs_b.bias", T_F32, (E,), np.ascontiguousarray(router_bias, np.float32).tobytes())]
    for m, part in enumerate(("gate", "up", "down")):
        if shared is not None:
            codes, scales = shared[m]
            rows, k = codes.shape
            out.append((b + f"ffn_{part}_shexp.weight", T_STBL_E4M3, (k, rows), np.ascontiguousarray(codes).tobytes()))
            out.append((b + f"ffn_{part}_shexp.scale", T_STBL_E8M0, (scales.shape[1], scales.shape[0]),
                        np.ascontiguousarray(scales).tobytes()))
        blocks = experts[m]
        ne, rows, nb = blocks.shape
        out.append((b + f"ffn_{part}_exps.weight", T_MXFP4, (nb // 17 * 32, rows, ne), np.ascontiguousarray(blocks).tobytes()))
    return out


def moe_metadata(cfg, n_layers=1):
    """The model metadata records load_moe_layer reads (the reference's key names)."""
    return [kv(PREFIX + "hidden_size", U32, cfg.hidden), kv(PREFIX + "moe_intermediate_size", U32, cfg.inter),
            kv(PREFIX + "n_routed_experts", U32, cfg.n_experts), kv(PREFIX + "num_experts_per_tok", U32, cfg.topk),
            kv(PREFIX + "num_hidden_layers", U32, n_layers), kv(PREFIX + "routed_scaling_factor", F32, cfg.route_scale),
            kv(PREFIX + "swiglu_limit", F32, cfg.swiglu_limit)]


# ---- loading a layer -------------------------------------------------------------------------------

def moe_config(g, layer=0, prefix=PREFIX):
    """The layer's MoEConfig from the file's metadata and tensor types: the reference engine's routing
    (sqrt(softplus) scores, top-k without group limit; stbl/model.cu:430-452), MXFP4 routed experts,
    the shared expert FP8-e8m0 when present."""
    b = f"blk.{layer}."
    shared = g.tensor(b + "ffn_gate_shexp.weight")
    if shared is not None and shared["type"] != T_STBL_E4M3:
        raise NotImplementedError(f"shared expert of type {shared['type']}: the layer takes FP8-e8m0 (STBL_E4M3 + E8M0)")
    return MoEConfig(f"gguf_blk{layer}", hidden=g.u32(prefix + "hidden_size"), inter=g.u32(prefix + "moe_intermediate_size"),
                     n_experts=g.u32(prefix + "n_routed_experts"), topk=g.u32(prefix + "num_experts_per_tok"),
                     n_groups=1, topk_groups=1, score_fn=SCORE_SQRT_SOFTPLUS,
                     route_scale=g.f32(prefix + "routed_scaling_factor"), swiglu_limit=g.f32(prefix + "swiglu_limit"),
                     routed_fmt=FMT_MXFP4, shared_fmt=FMT_FP8_E8M0 if shared is not None else FMT_NONE)


def expert_offsets(g, layers):
    """[[gate, up, down] file offsets] of the MXFP4 expert tensors of `layers` (ffn_*_exps.weight): where
    a file-backed expert cache reads them (the reference keeps the same file pointers,
    stbl/model.cu:940-949)."""
    out = []
    for layer in layers:
        row = []
        for part in ("gate", "up", "down"):
            t = g.tensor(f"blk.{layer}.ffn_{part}_exps.weight")
            if t is None:
                raise KeyError(f"missing tensor blk.{layer}.ffn_{part}_exps.weight")
            if t["type"] != T_MXFP4:
                raise ValueError(f"blk.{layer}.ffn_{part}_exps.weight has type {t['type']}, not MXFP4")
            row.append(t["offset"])
        out.append(row)
    return out


def file_cache(path, layers, slots, readers=0, direct=1, stage_experts=0, prefix=PREFIX):
    """An ExpertCache whose cache layer i streams model layer layers[i]'s routed experts from the GGUF
    file at `path` (read on demand, converted on the device).  Layers attached to it are loaded with
    load_moe_layer(g, layer, routed=False)."""
    from .cache import ExpertCache

    with GgufFile(path) as g:
        cfg = moe_config(g, layers[0], prefix)
        offsets = expert_offsets(g, layers)
    return ExpertCache(cfg, len(layers), slots, file={"path": str(path), "offsets": offsets, "readers": readers,
                                                       "direct": direct, "stage_experts": stage_experts})


def load_moe_layer(g, layer, prefix=PREFIX, device="cuda", routed=True):
    """(MoEConfig, device tensors in the layout MoELayer takes) for layer `layer` of an open GgufFile.
    The MXFP4 expert blocks are copied to the device and converted there (stbl_mxfp4_from_gguf).
    routed=False leaves the routed experts out (routed_w / routed_s empty): a layer attached to a
    file-backed expert cache reads them from the file."""
    import torch

    cfg = moe_config(g, layer, prefix)
    b = f"blk.{layer}."
    E, H, I = cfg.n_experts, cfg.hidden, cfg.inter

    def need(name, ttype, dims):
        t = g.tensor(name)
        if t is None:
            raise KeyError(f"missing tensor {name}")
        if t["type"] != ttype or tuple(t["dims"]) != tuple(dims):
            raise ValueError(f"{name}: type {t['type']} dims {t['dims']}, expected type {ttype} dims {tuple(dims)}")
        return torch.from_numpy(g.bytes_of(name).copy()).to(device)

    out = {"router_w": need(b + "ffn_gate_inp.weight", T_F32, (H, E)).view(torch.float32).view(E, H),
           "router_bias": need(b + "exp_probs_b.bias", T_F32, (E,)).view(torch.float32),
           "routed_w": [], "routed_s": [], "shared_w": None, "shared_s": None}
    shapes = ((I, H), (I, H), (H, I))
    lib = L.load()
    stream = torch.cuda.current_stream(device)
    for m, part in enumerate(("gate", "up", "down")):
        if not routed:
            break
        rows, k = shapes[m]
        blocks = need(b + f"ffn_{part}_exps.weight", T_MXFP4, (k, rows, E))
        codes = torch.empty(E, rows, k // 2, dtype=torch.uint8, device=device)
        scales = torch.empty(E, rows, k // 32, dtype=torch.uint8, device=device)
        rc = lib.stbl_mxfp4_from_gguf(blocks.data_ptr(), E * rows, k, codes.data_ptr(), scales.data_ptr(),
                                      ctypes.c_void_p(stream.cuda_stream))
        if rc != 0:
            raise RuntimeError(f"stbl_mxfp4_from_gguf failed for {part} ({rc})")
        out["routed_w"].append(codes)
        out["routed_s"].append(scales)
    if cfg.shared_fmt == FMT_FP8_E8M0:
        out["shared_w"], out["shared_s"] = [], []
        for m, part in enumerate(("gate", "up", "down")):
            rows, k = shapes[m]
            out["shared_w"].append(need(b + f"ffn_{part}_shexp.weight", T_STBL_E4M3, (k, rows)).view(rows, k))
            sr, sk = (rows + 31) // 32, (k + 31) // 32
            out["shared_s"].append(need(b + f"ffn_{part}_shexp.scale", T_STBL_E8M0, (sk, sr)).view(sr, sk))
    torch.cuda.synchronize(device)
    return cfg, out
