"""stbl_cache_create_file refuses a bad file description before it touches the device (no GPU needed):
the formats a file-backed cache holds, the required path and offsets, their 16-byte alignment and the
reader and staging counts."""

import ctypes

import numpy as np

from stblarge_b200 import lib as L
from stblarge_b200.config import FMT_FP8_B128, FMT_MXFP4


def _create(fmt=FMT_MXFP4, path=b"/nonexistent.gguf", offsets=(0, 64, 128), readers=0, stage=0, layers=1):
    lib = L.load()
    d = L.CacheDesc()
    d.n_layers, d.n_experts, d.slots, d.fmt, d.hidden, d.inter = layers, 8, 4, fmt, 512, 512
    off = np.array(list(offsets or ()) * layers, np.uint64)
    f = L.CacheFileDesc()
    f.path = path
    f.offset = off.ctypes.data if offsets is not None else None
    f.readers, f.direct, f.stage_experts = readers, 1, stage
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(256)
    rc = lib.stbl_cache_create_file(ctypes.byref(d), ctypes.byref(f), ctypes.byref(h), err, 256)
    return rc, err.value.decode()


def test_file_cache_holds_mxfp4_only():
    rc, msg = _create(fmt=FMT_FP8_B128)
    assert rc == -1 and "MXFP4" in msg


def test_path_and_offsets_are_required():
    assert _create(path=None)[1].startswith("file desc: path and offset")
    assert _create(offsets=None)[1].startswith("file desc: path and offset")


def test_offsets_must_be_16_byte_aligned():
    rc, msg = _create(offsets=(0, 64, 136), layers=2)
    assert rc == -1 and "multiples of 16" in msg


def test_counts_must_not_be_negative():
    assert ">= 0" in _create(readers=-1)[1]
    assert ">= 0" in _create(stage=-2)[1]
