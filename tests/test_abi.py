"""The C-ABI library loads and exports every symbol include/*.h declares (no GPU needed; nothing is
called that would touch the device)."""

import os
import re
import subprocess

import pytest

from stblarge_b200 import build, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in sorted(f for f in os.listdir(os.path.join(ROOT, "include")) if f.endswith(".h")):
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(stbl_\w+)\s*\(", text))
    return names


@pytest.fixture(scope="module")
def built():
    return build.build()


def test_headers_declare_the_expected_api():
    names = declared_symbols()
    for required in ("stbl_moe_create", "stbl_moe_forward", "stbl_moe_forward_host", "stbl_moe_last_route",
                     "stbl_moe_destroy", "stbl_gemv_fp8", "stbl_gemv_mxfp4_batch", "stbl_act_quant_fp8",
                     "stbl_gemv_f32", "stbl_swiglu_batch", "stbl_axpy", "stbl_round_bf16", "stbl_sqrt_softplus",
                     "stbl_gguf_open", "stbl_gguf_find", "stbl_gguf_u32"):
        assert required in names


def test_library_exports_every_declared_symbol(built):
    out = subprocess.run(["nm", "-D", "--defined-only", built], check=True, capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (stbl_\w+)", out))
    missing = declared_symbols() - exported
    assert not missing, missing


def test_ctypes_binds_every_symbol(built):
    L = lib.load()
    assert declared_symbols() <= set(lib.SIGNATURES)
    for name in declared_symbols():
        assert getattr(L, name) is not None


def test_kernels_are_sm100a_only(built):
    out = subprocess.run(["cuobjdump", "--list-elf", built], capture_output=True, text=True).stdout
    assert "sm_100a" in out
    assert "sm_90" not in out and "sm_80" not in out


def test_library_leaves_none_of_its_own_symbols_undefined(built):
    """Every translation unit is linked in: no function of the library's namespace or C ABI is left
    for the dynamic loader to find (a source missing from the build would show up here)."""
    out = subprocess.run(["nm", "-D", "--undefined-only", "-C", built], check=True, capture_output=True, text=True).stdout
    own = [l for l in out.splitlines() if "stbl" in l]
    assert not own, own
