"""Golden vectors for the GGUF MXFP4 conversion, made with the reference's own tools.

Run where the reference tree is present:

    python tests/golden/make_gguf_golden.py [--reference <reference tree>]   (default: STBL_REFERENCE, else ../reference)

Quantizes seeded weights to MXFP4 in the official layout with the reference's ref/kernel.py
(fp4_act_quant, E8M0 scales), then packs them into the reference engine's 17-byte GGUF blocks with
its converter (tools/convert_official.py: encode_expert), and writes gguf_mxfp4.npz next to this file:
official codes and scales and the blocks the converter produced.  Tests read only the fixture.
"""

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


class _Db:
    """The slice of the converter's safetensors reader that encode_expert uses."""

    def __init__(self, tensors):
        self.t = tensors

    def info(self, name):
        return {"shape": list(self.t[name].shape)}

    def read(self, name):
        return self.t[name].tobytes()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("STBL_REFERENCE", os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "..", "reference")))
    a = ap.parse_args()
    sys.path.insert(0, os.path.join(a.reference, "ref"))
    sys.path.insert(0, os.path.join(a.reference, "tools"))
    import convert_official as C  # the reference's converter
    import kernel as K  # the reference's ref/kernel.py
    rows, k = 96, 512
    g = torch.Generator().manual_seed(17)
    w = torch.randn(rows, k, generator=g) * 0.02
    packed, s = K.fp4_act_quant(w, 32)
    codes = packed.view(torch.uint8).numpy().reshape(rows, k // 2).copy()
    scales = s.view(torch.uint8).numpy().reshape(rows, k // 32).copy()
    name = "layers.0.ffn.experts.0.w1.weight"
    blocks = np.frombuffer(C.encode_expert(_Db({name: codes, C.scale_name(name): scales}), name), np.uint8)
    np.savez_compressed(os.path.join(HERE, "gguf_mxfp4.npz"), codes=codes, scales=scales,
                        blocks=blocks.reshape(rows, k // 32, 17))
    print("wrote gguf_mxfp4.npz", codes.shape, scales.shape, blocks.shape)


if __name__ == "__main__":
    main()
