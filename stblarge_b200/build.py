"""Build libstbl_moe.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed).

    python -m stblarge_b200.build [--force]

Objects go to stblarge_b200/_build/; the shared library to stblarge_b200/libstbl_moe.so, next to
this file, so that it travels with the source tree.  A hash of the sources, flags and compiler is
recorded in _build/libstbl_moe.sha256; the library is rebuilt when it differs.
"""

import argparse
import concurrent.futures
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libstbl_moe.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

SOURCES = ["router.cu", "combine.cu", "experts_tc.cu", "experts_tc4.cu", "experts_q8.cu", "moe.cu", "compat.cu", "noalloc.cu", "ep.cu", "cache.cu", "formats.cu", "gguf.cu", "reader.cu"]
NVCC = os.environ.get("NVCC", "nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
         "-I" + INCLUDE]


STAMP = os.path.join(BUILD, "libstbl_moe.sha256")


def _deps():
    return sorted([os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)])


def source_hash():
    """SHA-256 over every source and header (names and contents), the source list, the compiler
    flags and the compiler's version: the library is rebuilt whenever any of them differs from the
    build recorded beside it (file times are not trusted: a copied tree keeps no order of mtimes)."""
    h = hashlib.sha256()
    for d in _deps():
        h.update(os.path.relpath(d, HERE).encode() + b"\0")
        with open(d, "rb") as f:
            h.update(f.read())
    h.update(repr((SOURCES, FLAGS)).encode())
    try:
        h.update(subprocess.run([NVCC, "--version"], capture_output=True, check=True).stdout)
    except Exception:
        h.update(b"nvcc unavailable")
    return h.hexdigest()


def up_to_date():
    if not os.path.exists(LIB) or not os.path.exists(STAMP):
        return False
    with open(STAMP) as f:
        return f.read().strip() == source_hash()


def build(force=False, verbose=False):
    if not force and up_to_date():
        return LIB
    digest = source_hash()
    os.makedirs(BUILD, exist_ok=True)
    objs = [os.path.join(BUILD, src.replace(".cu", ".o")) for src in SOURCES]
    cmds = [[NVCC, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj] for src, obj in zip(SOURCES, objs)]
    if verbose:
        for cmd in cmds:
            print(" ".join(cmd), flush=True)
    # the translation units are independent: compile them side by side
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(len(cmds), os.cpu_count() or 1)) as ex:
        for r in list(ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), cmds)):
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise subprocess.CalledProcessError(r.returncode, r.args)
    tmp = LIB + ".tmp"
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", *objs, "-o", tmp]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    with open(STAMP, "w") as f:
        f.write(digest + "\n")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=True))
    sys.exit(0)
