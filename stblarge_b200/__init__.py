"""B200-native MoE decode hot path with the STBLarge C ABI.

The compute lives in libstbl_moe.so (hand-written sm_100a CUDA, built in-tree by
stblarge_b200/build.py); this package is the host-side mirror of the reference's Python driver
(ctypes, as stbl/run.py) plus synthetic-layer generation for tests and benchmarks.
"""
