"""Writes tests/golden/q8.npz: the reference's Q8 activation numerics (ref/emulate_ds4.py) run on seeded
inputs, for the oracle's restatement (oracle.q8_codes, oracle.gemv_mxfp4_q8) to be checked against.

emulate_ds4 imports DeepSeek's official `model` module, which the reference does not ship; it only
reads `model.linear` at import time, so a stub module stands in for it (nothing of the official model
runs).  Its FP4 branch takes ref/kernel.py's FP4_TABLE.

    python tests/golden/make_q8_golden.py        (needs the reference tree: STBL_REFERENCE, else ../reference)
"""

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
FILE = os.path.join(HERE, "q8.npz")


def inputs():
    """x fp32 [T][k] (one all-zero block, one block with a single nonzero value, ties at +-0.5 code
    steps), FP4 codes [rows][k/2] and e8m0 scales [rows][k/32] in a normal range."""
    rng = np.random.default_rng(8)
    T, rows, k = 3, 48, 256
    x = (rng.standard_normal((T, k)) * rng.choice([0.01, 1.0, 30.0], (T, k // 32)).repeat(32, 1)).astype(np.float32)
    x[0, :32] = 0.0
    x[1, 32:64] = 0.0
    x[1, 40] = -3.25
    x[2, 64:96] = np.arange(32, dtype=np.float32) - 15.5  # amax 127 below: d = 1, every value a .5 step
    x[2, 64] = 127.0
    codes = rng.integers(0, 256, (rows, k // 2), dtype=np.uint8)
    scales = rng.integers(118, 134, (rows, k // 32), dtype=np.uint8)
    return x, codes, scales


def main():
    ref = os.environ.get("STBL_REFERENCE", os.path.join(HERE, "..", "..", "..", "reference"))
    sys.path.insert(0, os.path.join(ref, "ref"))
    stub = types.ModuleType("model")
    stub.linear = lambda *a, **k: None
    sys.modules["model"] = stub
    import emulate_ds4 as D  # noqa: E402

    x, codes, scales = inputs()
    xt = torch.from_numpy(x)
    q, d = D.q8_codes(xt, False)
    values = D.q8_values(xt, False)
    weight = torch.from_numpy(codes).view(torch.float4_e2m1fn_x2)
    weight.scale = torch.from_numpy(scales).view(torch.float8_e8m0fnu)
    y = D.linear(xt, weight)
    np.savez_compressed(FILE, x=x, codes=codes, scales=scales, q=q.numpy().reshape(x.shape),
                        d=d.numpy().reshape(x.shape[0], -1), values=values.numpy(), y=y.float().numpy())
    print(f"wrote {FILE}", file=sys.stderr)


if __name__ == "__main__":
    main()
