"""bench.py's output contract, on CPU: the reference arm (the CPU oracle timed on the host's cores) prints
one JSON line with the keys and meanings the driver reads, and the algorithmic byte counts behind the
roofline figures agree with the weight formats' definitions."""

import json
import os
import subprocess
import sys

import pytest

from stblarge_b200.config import CFG2, CFG3, CFG3_REF, FMT_FP8_B128, FMT_FP8_E8M0, FMT_MXFP4

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["steps"] == 1 and d["warmup"] >= 3
    assert "workload" in d["config"]
    # the same config object the b200 arm prints for this workload (the driver compares the two)
    import argparse

    import bench
    assert d["config"] == bench.config_of(argparse.Namespace(zipf=False), "cfg2", 16, 1)
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def mat_bytes(fmt, rows, k):
    """Stored bytes of one matrix: codes and scales, as the formats define them."""
    if fmt == FMT_FP8_B128:
        return rows * k + 4 * ((rows + 127) // 128) * ((k + 127) // 128)
    if fmt == FMT_MXFP4:
        return rows * k // 2 + rows * (k // 32)
    if fmt == FMT_FP8_E8M0:
        return rows * k + ((rows + 31) // 32) * (k // 32)
    raise ValueError(fmt)


@pytest.mark.parametrize("cfg", [CFG2, CFG3, CFG3_REF], ids=lambda c: c.name)
def test_algorithmic_bytes_follow_the_formats(cfg):
    import bench
    H, I = cfg.hidden, cfg.inter
    for fmt in {cfg.routed_fmt, cfg.shared_fmt}:
        assert cfg.bytes_per_expert(fmt) == 2 * mat_bytes(fmt, I, H) + mat_bytes(fmt, H, I)
    for n in (0, 1, 37):
        want_up = 2 * (n * mat_bytes(cfg.routed_fmt, I, H) + mat_bytes(cfg.shared_fmt, I, H))
        assert bench.up_bytes(cfg, n) == want_up
        want_layer = (n * cfg.bytes_per_expert() + cfg.bytes_per_expert(cfg.shared_fmt) + cfg.n_experts * H * 4
                      + cfg.n_experts * 4 + 2 * 16 * H * 2)
        assert bench.layer_bytes(cfg, n, 16) == want_layer
