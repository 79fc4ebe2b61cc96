"""The checkpoint reader (include/stbl_io.h), on the host: the reference's read_range / read_pieces
(stbl/model.cu:269-308) with O_DIRECT where the file system takes it.  Ranges come back byte-exact
wherever they start and end (unaligned offsets, 2 MiB piece boundaries, the file's last byte),
at the aligned place the header promises, with one or many threads; a range past the end of the file
and injected pread errors fail with a message and leave the reader usable.  No GPU."""

import ctypes
import errno

import numpy as np
import pytest

from stblarge_b200 import lib as L

PIECE, ALIGN = 2 << 20, 4096


@pytest.fixture(scope="module")
def data_file(tmp_path_factory):
    rng = np.random.default_rng(5)
    data = rng.integers(0, 256, 5 * PIECE + 12345, dtype=np.uint8)
    path = tmp_path_factory.mktemp("reader") / "blob.bin"
    data.tofile(path)
    return path, data


class Reader:
    def __init__(self, path, threads, direct):
        self.lib = L.load()
        self.h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(256)
        assert self.lib.stbl_reader_open(str(path).encode(), threads, direct, ctypes.byref(self.h), err, 256) == 0, err.value
        self.keep = []

    def region(self, nbytes):
        n = self.lib.stbl_reader_region_bytes(nbytes)
        assert n >= nbytes + (ALIGN - 1) and n % ALIGN == 0
        buf = np.zeros(n + ALIGN, np.uint8)
        a = (-buf.ctypes.data) % ALIGN
        self.keep.append(buf)
        return buf[a:a + n]

    def read(self, ranges):
        n = len(ranges)
        off = (ctypes.c_uint64 * max(n, 1))(*[o for o, _ in ranges])
        nb = (ctypes.c_uint64 * max(n, 1))(*[b for _, b in ranges])
        regions = [self.region(b) for _, b in ranges]
        ptrs = (ctypes.c_void_p * max(n, 1))(*[r.ctypes.data for r in regions])
        at = (ctypes.c_uint64 * max(n, 1))()
        rc = self.lib.stbl_reader_read(self.h, n, off, nb, ptrs, at)
        return rc, [r[at[i]:at[i] + ranges[i][1]] for i, r in enumerate(regions)], [at[i] for i in range(n)]

    def stats(self):
        p, b, s, d = L.U64(), L.U64(), ctypes.c_double(), L.I()
        assert self.lib.stbl_reader_stats(self.h, ctypes.byref(p), ctypes.byref(b), ctypes.byref(s), ctypes.byref(d)) == 0
        return p.value, b.value, s.value, d.value

    def error(self):
        return self.lib.stbl_reader_error(self.h).decode()

    def close(self):
        self.lib.stbl_reader_close(self.h)


@pytest.mark.parametrize("threads", [1, 4])
@pytest.mark.parametrize("direct", [0, 1])
def test_ranges_are_byte_exact(data_file, threads, direct):
    path, data = data_file
    size = len(data)
    r = Reader(path, threads, direct)
    rng = np.random.default_rng(threads * 10 + direct)
    ranges = [(0, 1), (17, 4096), (ALIGN - 3, 7), (PIECE - 100, 300), (PIECE, PIECE), (3, 2 * PIECE + 999),
              (size - 1, 1), (size - PIECE - 5, PIECE + 5), (12345, 0)]
    ranges += [(int(o), int(rng.integers(1, min(3 * PIECE, size - o) + 1))) for o in rng.integers(0, size - 1, 12)]
    rc, got, at = r.read(ranges)
    assert rc == 0, r.error()
    for (o, b), g, a in zip(ranges, got, at):
        assert a == o % ALIGN
        assert np.array_equal(g, data[o:o + b]), (o, b)
    pieces, nbytes, seconds, direct_on = r.stats()
    assert pieces >= len(ranges) - 1 and nbytes >= sum(b for _, b in ranges) and seconds > 0
    if not direct:
        assert direct_on == 0
    r.close()


def test_pieces_follow_the_2mib_split(data_file):
    path, _ = data_file
    r = Reader(path, 2, 0)
    rc, _, _ = r.read([(0, 2 * PIECE + 1), (ALIGN, PIECE)])  # 2 MiB pieces of the aligned supersets
    assert rc == 0
    pieces, nbytes, _, _ = r.stats()
    assert pieces == 3 + 1
    assert nbytes == (2 * PIECE + ALIGN) + PIECE
    r.close()


def test_range_past_the_end_fails_and_the_reader_recovers(data_file):
    path, data = data_file
    r = Reader(path, 3, 1)
    rc, _, _ = r.read([(len(data) - 10, 11)])
    assert rc == -1 and "file ends" in r.error()
    rc, got, _ = r.read([(len(data) - 10, 10)])
    assert rc == 0 and np.array_equal(got[0], data[-10:])
    r.close()


@pytest.mark.parametrize("after", [0, 3])
def test_injected_read_errors_fail_the_call_with_errno(data_file, after):
    path, data = data_file
    r = Reader(path, 1, 0)  # one thread: the failing read is the (after+1)-th of the call
    assert r.lib.stbl_reader_inject_error(r.h, after, errno.EIO) == 0
    rc, _, _ = r.read([(i * PIECE, PIECE) for i in range(5)])
    assert rc == -1 and "Input/output error" in r.error()
    pieces, _, _, _ = r.stats()
    assert pieces == after
    assert r.lib.stbl_reader_inject_error(r.h, 0, 0) == 0  # off again
    rc, got, _ = r.read([(5, 999)])
    assert rc == 0 and np.array_equal(got[0], data[5:1004])
    r.close()


def test_bad_arguments(data_file, tmp_path):
    path, _ = data_file
    lib = L.load()
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(256)
    assert lib.stbl_reader_open(str(tmp_path / "missing").encode(), 1, 0, ctypes.byref(h), err, 256) == -1
    assert b"cannot open" in err.value
    r = Reader(path, 1, 0)
    buf = np.zeros(3 * ALIGN, np.uint8)
    a = (-buf.ctypes.data) % ALIGN + 1  # misaligned region
    off, nb, at = (ctypes.c_uint64 * 1)(0), (ctypes.c_uint64 * 1)(10), (ctypes.c_uint64 * 1)()
    ptrs = (ctypes.c_void_p * 1)(buf.ctypes.data + a)
    assert lib.stbl_reader_read(r.h, 1, off, nb, ptrs, at) == -1 and "aligned" in r.error()
    assert lib.stbl_reader_read(r.h, 0, None, None, None, None) == 0
    r.close()
