"""GGUF reader (include/stbl_gguf.h) and writer (stblarge_b200/gguf.py), on CPU.

Pinned to the reference three ways: tests/golden/gguf_moe_small.gguf was written by the reference's own
writing code (tests/golden/make_gguf_file.py) and is read back here; this module's writer reproduces
that file byte for byte from the same content; and, where oracle/_ref holds the reference's reader
(stbl/gguf.cpp, built by oracle/build_ref.sh), both readers must report the same tensor table and
metadata values for the golden file and for generated ones.  Malformed files must be refused with an
error, never read past the mapping."""

import ctypes
import os
import struct

import numpy as np
import pytest

from stblarge_b200 import gguf as G
from stblarge_b200.config import FMT_FP8_E8M0, FMT_MXFP4, SCORE_SQRT_SOFTPLUS
from tests.golden.make_gguf_file import FILE as GOLDEN, content

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libstbl_ref_gguf.so")


def our_records(meta):
    kinds = {"string": G.STRING, "u32": G.U32, "f32": G.F32, "bool": G.BOOL}
    out = []
    for key, kind, value in meta:
        if kind == "u32s":
            out.append(G.kv(key, G.ARRAY, (G.U32, value)))
        else:
            out.append(G.kv(key, kinds[kind], value))
    return out


def test_golden_file_reads_back():
    meta, tensors = content()
    with G.GgufFile(GOLDEN) as g:
        assert (g.version, g.alignment, g.n_kv, g.n_tensors) == (3, 32, len(meta), len(tensors))
        types = {"string": G.STRING, "u32": G.U32, "f32": G.F32, "bool": G.BOOL, "u32s": G.ARRAY}
        assert g.keys() == [(k, types[kind]) for k, kind, _ in meta]
        for key, kind, value in meta:
            if kind == "u32":
                assert g.u32(key) == value
            elif kind == "f32":
                assert g.f32(key) == np.float32(value)
            elif kind == "string":
                assert g.string(key) == value
            elif kind == "u32s":
                assert g.uints(key) == value
        table = g.tensors()
        assert [t["name"] for t in table] == [t[0] for t in tensors]
        for t, (name, ttype, dims, data) in zip(table, tensors):
            assert (t["type"], t["dims"], t["nbytes"]) == (ttype, tuple(dims), len(data))
            assert t["offset"] % 32 == 0
            assert g.bytes_of(name).tobytes() == data
        assert g.tensor("blk.9.ffn_up_exps.weight") is None
        with pytest.raises(KeyError):
            g.u32("deepseek41.routed_scaling_factor")  # an f32: the typed accessor refuses it


def test_writer_reproduces_the_reference_written_file(tmp_path):
    meta, tensors = content()
    out = tmp_path / "ours.gguf"
    G.write_gguf(out, our_records(meta), tensors)
    assert out.read_bytes() == open(GOLDEN, "rb").read()


def test_moe_config_from_metadata():
    with G.GgufFile(GOLDEN) as g:
        cfg = G.moe_config(g, 1)
    assert (cfg.hidden, cfg.inter, cfg.n_experts, cfg.topk) == (64, 32, 4, 2)
    assert (cfg.route_scale, cfg.swiglu_limit) == (2.5, 10.0)
    assert (cfg.score_fn, cfg.n_groups, cfg.routed_fmt, cfg.shared_fmt) == (SCORE_SQRT_SOFTPLUS, 1, FMT_MXFP4, FMT_FP8_E8M0)


class RefReader:
    """The reference's reader through oracle/_ref/libstbl_ref_gguf.so."""

    def __init__(self):
        self.lib = ctypes.CDLL(REF_LIB)
        self.lib.ref_gguf_open.restype = ctypes.c_void_p
        self.lib.ref_gguf_open.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
        self.lib.ref_gguf_close.argtypes = [ctypes.c_void_p]
        self.lib.ref_gguf_n_tensors.argtypes = [ctypes.c_void_p]
        self.lib.ref_gguf_tensor_at.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_int] + \
            [ctypes.POINTER(ctypes.c_uint32)] * 2 + [ctypes.POINTER(ctypes.c_uint64)] * 3
        self.lib.ref_gguf_u32.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32)]
        self.lib.ref_gguf_f32.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float)]

    def read(self, path, u32_keys=(), f32_keys=()):
        err = ctypes.create_string_buffer(256)
        h = self.lib.ref_gguf_open(str(path).encode(), err, 256)
        assert h, err.value
        table = {}
        for i in range(self.lib.ref_gguf_n_tensors(h)):
            name = ctypes.create_string_buffer(256)
            ty, nd = ctypes.c_uint32(), ctypes.c_uint32()
            dims, off, nb = (ctypes.c_uint64 * 4)(), ctypes.c_uint64(), ctypes.c_uint64()
            assert self.lib.ref_gguf_tensor_at(h, i, name, 256, ty, nd, dims, off, nb) == 0
            table[name.value.decode()] = (ty.value, tuple(dims[:nd.value]), off.value, nb.value)
        vals = {}
        for k in u32_keys:
            v = ctypes.c_uint32()
            assert self.lib.ref_gguf_u32(h, k.encode(), v) == 0
            vals[k] = v.value
        for k in f32_keys:
            v = ctypes.c_float()
            assert self.lib.ref_gguf_f32(h, k.encode(), v) == 0
            vals[k] = v.value
        self.lib.ref_gguf_close(h)
        return table, vals


def random_file(path, rng):
    """A file with every metadata value type (nested arrays and strings included), a chosen alignment
    and tensors of every type the reference's reader sizes."""
    align = int(rng.choice([32, 64, 256]))
    recs = [G.kv("general.alignment", G.U32, align), G.kv("a.u8", G.U8, 7), G.kv("a.i8", G.I8, -3),
            G.kv("a.u16", G.U16, 65000), G.kv("a.i16", G.I16, -2), G.kv("a.i32", G.I32, -9), G.kv("a.u64", G.U64, 1 << 40),
            G.kv("a.i64", G.I64, -(1 << 40)), G.kv("a.f64", G.F64, 0.25), G.kv("a.bool", G.BOOL, False),
            G.kv("a.strs", G.ARRAY, (G.STRING, ["x", "", "yz"])),
            G.kv("a.nested", G.ARRAY, (G.ARRAY, [(G.U8, [1, 2]), (G.STRING, ["q"])])),
            G.kv("a.u64s", G.ARRAY, (G.U64, [3, 1 << 33])), G.kv("m.u32", G.U32, int(rng.integers(1 << 31))),
            G.kv("m.f32", G.F32, float(np.float32(rng.standard_normal())))]
    tensors = []
    for i in range(int(rng.integers(1, 8))):
        ttype = int(rng.choice([G.T_F32, G.T_BF16, G.T_I8, G.T_MXFP4, G.T_STBL_E4M3, G.T_STBL_E8M0]))
        nd = int(rng.integers(1, 4))
        dims = [int(rng.integers(1, 5)) * (32 if d == 0 else 1) for d in range(nd)]
        data = rng.integers(0, 256, G.tensor_nbytes(ttype, dims), dtype=np.uint8).tobytes()
        tensors.append((f"t{i}.{ttype}", ttype, tuple(dims), data))
    G.write_gguf(path, recs, tensors, alignment=align)
    return tensors


@pytest.mark.skipif(not os.path.exists(REF_LIB), reason="the reference reader is built where the reference tree is")
def test_reader_matches_the_reference_reader(tmp_path):
    ref = RefReader()
    rng = np.random.default_rng(5)
    files = [GOLDEN] + [tmp_path / f"r{i}.gguf" for i in range(12)]
    for f in files[1:]:
        random_file(f, rng)
    for f in files:
        u32_keys = ["deepseek41.hidden_size"] if f == GOLDEN else ["m.u32", "general.alignment"]
        f32_keys = ["deepseek41.swiglu_limit"] if f == GOLDEN else ["m.f32"]
        table, vals = ref.read(f, u32_keys, f32_keys)
        with G.GgufFile(f) as g:
            ours = {t["name"]: (t["type"], t["dims"], t["offset"], t["nbytes"]) for t in g.tensors()}
            assert ours == table, f
            for k in u32_keys:
                assert g.u32(k) == vals[k]
            for k in f32_keys:
                assert g.f32(k) == np.float32(vals[k])


def test_metadata_types_round_trip(tmp_path):
    rng = np.random.default_rng(9)
    tensors = random_file(tmp_path / "m.gguf", rng)
    with G.GgufFile(tmp_path / "m.gguf") as g:
        keys = dict(g.keys())
        assert keys["a.nested"] == G.ARRAY and keys["a.strs"] == G.ARRAY and keys["a.f64"] == G.F64
        assert g.uints("a.u64s") == [3, 1 << 33]
        assert g.alignment == g.u32("general.alignment")
        for t, (name, ttype, dims, data) in zip(g.tensors(), tensors):
            assert t["name"] == name and t["offset"] % g.alignment == 0
            assert g.bytes_of(name).tobytes() == data


def _open_error(path):
    with pytest.raises(ValueError) as e:
        G.GgufFile(path)
    return str(e.value)


def test_malformed_files_are_refused(tmp_path):
    good = open(GOLDEN, "rb").read()
    meta, tensors = content()
    data_end = max(t["offset"] + t["nbytes"] for t in G.GgufFile(GOLDEN).tensors())
    # every truncation that cuts the header or a tensor's data
    for cut in list(range(0, 4096, 7)) + [data_end - 1]:
        p = tmp_path / "cut.gguf"
        p.write_bytes(good[:cut])
        _open_error(p)
    cases = {
        "magic": b"GGUX" + good[4:],
        "version1": good[:4] + struct.pack("<I", 1) + good[8:],
        "version4": good[:4] + struct.pack("<I", 4) + good[8:],
        "huge count": good[:8] + struct.pack("<Q", 1 << 60) + good[16:],
    }
    for what, blob in cases.items():
        p = tmp_path / f"{what}.gguf"
        p.write_bytes(blob)
        assert _open_error(p), what
    recs = our_records(meta)
    bad_tensors = {
        "unsupported type": [("x", 2, (32,), bytes(18))],      # Q4_1: not sized by this reader
        "five dims": [("x", G.T_I8, (1, 1, 1, 1, 2), bytes(2))],
        "duplicate": [("x", G.T_I8, (4,), bytes(4)), ("x", G.T_I8, (4,), bytes(4))],
    }
    for what, ts in bad_tensors.items():
        p = tmp_path / "bad.gguf"
        blob = b"GGUF" + struct.pack("<IQQ", 3, len(ts), len(recs)) + b"".join(recs)
        for name, ty, dims, data in ts:
            blob += G._str(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims) + struct.pack("<IQ", ty, 0)
        blob += bytes((-len(blob)) % 32) + b"".join(d + bytes((-len(d)) % 32) for *_, d in ts)
        p.write_bytes(blob)
        assert _open_error(p), what
    # an MXFP4 tensor whose element count is not a multiple of 32; an alignment of 0
    p = tmp_path / "block.gguf"
    blob = b"GGUF" + struct.pack("<IQQ", 3, 1, 0) + G._str("x") + struct.pack("<IQIQ", 1, 48, G.T_MXFP4, 0)
    p.write_bytes(blob + bytes((-len(blob)) % 32) + bytes(64))
    assert "multiple" in _open_error(p)
    p = tmp_path / "align.gguf"
    p.write_bytes(b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + G.kv("general.alignment", G.U32, 0))
    assert "alignment" in _open_error(p)
    assert "cannot open" in _open_error(tmp_path / "missing.gguf")


def test_mxfp4_blocks_writer_matches_the_oracle_converter():
    # the product's writer-side conversion (gguf.mxfp4_to_blocks) against the oracle's restatement of
    # the reference converter (tools/convert_official.py:187-201), itself pinned to golden vectors
    from oracle import oracle as O
    rng = np.random.default_rng(9)
    for rows, k in ((1, 32), (7, 64), (128, 1024)):
        codes = rng.integers(0, 256, (rows, k // 2), dtype=np.uint8)
        scales = rng.integers(0, 256, (rows, k // 32), dtype=np.uint8)
        assert np.array_equal(G.mxfp4_to_blocks(codes, scales), O.mxfp4_to_gguf(codes, scales).reshape(rows, -1))


def test_repeated_tensor_data_and_expert_offsets(tmp_path):
    # a checkpoint written from repeated chunks (no copy in memory) reads back chunk by chunk, and the
    # expert tensors' offsets are where a file-backed cache reads them
    H, I, E = 64, 32, 3
    rng = np.random.default_rng(4)
    chunk = {m: rng.integers(0, 256, (r * (k // 32) * 17,), dtype=np.uint8).tobytes()
             for m, (r, k) in enumerate(((I, H), (I, H), (H, I)))}
    tensors = [("blk.0.ffn_gate_inp.weight", G.T_F32, (H, E), bytes(H * E * 4))]
    for m, part in enumerate(("gate", "up", "down")):
        r, k = ((I, H), (I, H), (H, I))[m]
        tensors.append((f"blk.0.ffn_{part}_exps.weight", G.T_MXFP4, (k, r, E), G.Repeated(chunk[m], E)))
    path = tmp_path / "rep.gguf"
    G.write_gguf(path, [], tensors)
    raw = open(path, "rb").read()
    with G.GgufFile(path) as g:
        offs = G.expert_offsets(g, [0])[0]
        for m, part in enumerate(("gate", "up", "down")):
            t = g.tensor(f"blk.0.ffn_{part}_exps.weight")
            assert t["offset"] == offs[m] and t["offset"] % 32 == 0 and t["nbytes"] == E * len(chunk[m])
            for e in range(E):
                o = offs[m] + e * len(chunk[m])
                assert raw[o:o + len(chunk[m])] == chunk[m]
        with pytest.raises(KeyError):
            G.expert_offsets(g, [1])  # no such layer
