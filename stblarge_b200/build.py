"""Build libstbl_moe.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed).

    python -m stblarge_b200.build [--force]

Objects go to stblarge_b200/_build/; the shared library to stblarge_b200/libstbl_moe.so, next to
this file, so that it travels with the source tree.
"""

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libstbl_moe.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

SOURCES = ["router.cu", "combine.cu", "experts_tc.cu", "experts_tc4.cu", "moe.cu", "compat.cu", "noalloc.cu", "ep.cu", "cache.cu", "formats.cu", "gguf.cu", "reader.cu"]
NVCC = os.environ.get("NVCC", "nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
         "-I" + INCLUDE]


def _deps():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in _deps())


def build(force=False, verbose=False):
    if not force and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = os.path.join(BUILD, src.replace(".cu", ".o"))
        cmd = [NVCC, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", *objs, "-o", tmp]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=True))
    sys.exit(0)
