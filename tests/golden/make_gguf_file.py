"""Writes tests/golden/gguf_moe_small.gguf with the reference's own GGUF writing code.

A two-layer MoE checkpoint in miniature (hidden 64, moe_intermediate 32, 4 routed experts, top-2), in
the reference converter's tensor names, types and order (tools/convert_official.py:116-126,
204-243): per layer the f32 router and bias, the FP8 shared expert (STBL_E4M3 codes + STBL_E8M0
scales) and the MXFP4 experts (17-byte blocks), plus metadata records of the types its helpers write
(u32, f32, string, bool, u32 array).  The header and data layout come from the reference's
tools/stbl_gguf.py helpers (pack_string, kv_*, tensor_header, align, qtype_nbytes), imported from the
reference tree; the content is seeded numpy and is rebuilt by `content()` without the reference,
which is what the tests compare the file with.

    python tests/golden/make_gguf_file.py        (needs the reference tree: STBL_REFERENCE, else ../reference)
"""

import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
FILE = os.path.join(HERE, "gguf_moe_small.gguf")

H, I, E, K, LAYERS = 64, 32, 4, 2, 2
T_F32, T_MXFP4, T_E4M3, T_E8M0 = 0, 39, 200, 201


def content():
    """(metadata [(key, kind, value)], tensors [(name, type, dims innermost first, bytes)])."""
    meta = [("general.architecture", "string", "deepseek41"),
            ("deepseek41.hidden_size", "u32", H), ("deepseek41.moe_intermediate_size", "u32", I),
            ("deepseek41.n_routed_experts", "u32", E), ("deepseek41.num_experts_per_tok", "u32", K),
            ("deepseek41.num_hidden_layers", "u32", LAYERS), ("deepseek41.routed_scaling_factor", "f32", 2.5),
            ("deepseek41.swiglu_limit", "f32", 10.0), ("deepseek41.compress_ratios", "u32s", [1, 4, 128, 4]),
            ("deepseek41.expert_weights_norm", "bool", True)]
    rng = np.random.default_rng(20)
    tensors = []
    shapes = {"gate": (I, H), "up": (I, H), "down": (H, I)}
    for layer in range(LAYERS):
        b = f"blk.{layer}."
        tensors.append((b + "ffn_gate_inp.weight", T_F32, (H, E), (rng.standard_normal((E, H)) * 0.02).astype(np.float32).tobytes()))
        tensors.append((b + "exp_probs_b.bias", T_F32, (E,), (rng.standard_normal(E) * 0.1).astype(np.float32).tobytes()))
        for part in ("gate", "up", "down"):
            rows, k = shapes[part]
            codes = rng.integers(0, 256, (rows, k), dtype=np.uint8)
            codes[(codes & 127) == 127] = 0  # no NaN codes (the converter refuses them)
            scales = rng.integers(118, 131, ((rows + 31) // 32, (k + 31) // 32), dtype=np.uint8)
            tensors.append((b + f"ffn_{part}_shexp.weight", T_E4M3, (k, rows), codes.tobytes()))
            tensors.append((b + f"ffn_{part}_shexp.scale", T_E8M0, (scales.shape[1], scales.shape[0]), scales.tobytes()))
            blocks = rng.integers(0, 256, (E, rows, k // 32, 17), dtype=np.uint8)
            blocks[..., 0] = rng.integers(118, 131, (E, rows, k // 32), dtype=np.uint8)
            tensors.append((b + f"ffn_{part}_exps.weight", T_MXFP4, (k, rows, E), blocks.tobytes()))
    return meta, tensors


def main():
    ref = os.environ.get("STBL_REFERENCE", os.path.join(HERE, "..", "..", "..", "reference"))
    spec = importlib.util.spec_from_file_location("stbl_gguf", os.path.join(ref, "tools", "stbl_gguf.py"))
    G = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(G)
    # the converter's additions for its FP8 pair (tools/convert_official.py:31-34)
    G.QTYPE_NAMES.update({T_E4M3: "STBL_E4M3", T_E8M0: "STBL_E8M0"})
    G.QTYPE_LAYOUT.update({T_E4M3: (1, 1), T_E8M0: (1, 1)})
    meta, tensors = content()
    records = []
    for key, kind, value in meta:
        if kind == "string":
            records.append(G.kv_string(key, value))
        elif kind == "u32":
            records.append(G.kv_u32(key, value))
        elif kind == "f32":
            records.append(G.kv_f32(key, value))
        elif kind == "bool":
            records.append(G.kv_bool(key, value))
        elif kind == "u32s":
            records.append(G.kv_u32_array(key, value))
    plan, offset = [], 0
    for name, qtype, dims, data in tensors:
        item = G.TensorPlan(name, tuple(dims), qtype, "test")
        item.offset = offset
        item.nbytes = G.qtype_nbytes(qtype, item.shape)
        assert item.nbytes == len(data), name
        offset += G.align(item.nbytes, G.GGUF_ALIGNMENT)
        plan.append(item)
    data_start, _ = G.print_plan(plan, records, [], G.GGUF_ALIGNMENT)
    header = b"GGUF" + G.struct.pack("<IQQ", 3, len(plan), len(records))
    header += b"".join(records) + b"".join(G.tensor_header(item) for item in plan)
    header += bytes(data_start - len(header))
    with open(FILE, "wb") as fp:
        fp.write(header)
        for item, (_, _, _, data) in zip(plan, tensors):
            assert fp.tell() == data_start + item.offset
            fp.write(data)
            fp.write(bytes(G.align(item.nbytes, G.GGUF_ALIGNMENT) - item.nbytes))
    print(f"wrote {FILE} ({os.path.getsize(FILE)} bytes)", file=sys.stderr)


if __name__ == "__main__":
    main()
