"""kernels.h-compatible entry points (include/stbl_kernels.h) on the GPU.

Each is checked against the CPU oracle's restatement of the reference kernel (bit-exact where the
reference fixes the summation order, otherwise the reference test's own tolerance), and, when the
reference's kernels have been built from its sources into oracle/_ref (oracle/build_ref.sh), bit
for bit against them on the same inputs, 20 seeds, as stbl/cmp_kernels.py compares two builds."""

import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from stblarge_b200 import lib as L

pytestmark = pytest.mark.gpu

REF_SO = os.path.join(os.path.dirname(O.HERE), "oracle", "_ref", "libstbl_ref_kernels.so")
P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def p(t):
    return P(t.data_ptr())


@pytest.fixture(scope="module")
def lib():
    return L.load()


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_SO):
        pytest.skip("reference kernels not built (oracle/build_ref.sh needs the reference tree)")
    return ctypes.CDLL(REF_SO)


def bf16_vals(n, scale, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, generator=g) * scale).bfloat16().float()


def fp8_weight(rows, k, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randint(0, 256, (rows, k), generator=g, dtype=torch.uint8)
    w[(w & 0x7F) == 0x7F] = 0  # no NaN codes (stbl/cmp_kernels.py:39)
    s = torch.randint(110, 130, ((rows + 31) // 32, k // 32), generator=g, dtype=torch.uint8)
    return w, s


def mxfp4_gguf(rows, k, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randint(0, 256, (rows, k // 32 * 17), generator=g, dtype=torch.uint8)
    w[:, ::17] = torch.randint(110, 130, (rows, k // 32), generator=g, dtype=torch.uint8)
    return w


def test_act_quant_fp8_bit_exact(lib):
    x = bf16_vals(4 * 1024, 3.0, 0) * (10 ** torch.linspace(-3, 2, 4 * 1024))
    x = x.bfloat16().float()
    want = O.ref_act_quant_fp8(x.numpy())
    got = x.cuda()
    lib.stbl_act_quant_fp8(p(got), got.numel(), None)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("rows,k,round_out", [(1000, 1280, 1), (2048, 7168, 0), (7168, 2048, 1), (100, 32, 0)])
def test_gemv_fp8_bit_exact(lib, rows, k, round_out):
    w, s = fp8_weight(rows, k, rows + k)
    x = torch.from_numpy(O.ref_act_quant_fp8(bf16_vals(k, 1.0, k).numpy()))
    want = O.ref_gemv_fp8(w.numpy(), s.numpy(), x.numpy(), round_out)
    y = torch.empty(rows, device="cuda")
    wc, sc, xc = w.cuda(), s.cuda(), x.cuda()
    lib.stbl_gemv_fp8(p(y), p(wc), p(sc), p(xc), rows, k, round_out, None)
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("rows,k", [(2304, 5120), (5120, 2304), (2048, 7168), (7168, 2048)])
def test_gemv_mxfp4_bit_exact(lib, rows, k):
    w = mxfp4_gguf(rows, k, rows)
    x = torch.from_numpy(O.ref_act_quant_fp8(bf16_vals(k, 1.0, k).numpy()))
    want = O.ref_gemv_mxfp4(w.numpy(), x.numpy(), rows, k)
    y = torch.empty(rows, device="cuda")
    wc, xc = w.cuda(), x.cuda()
    lib.stbl_gemv_mxfp4(p(y), p(wc), p(xc), rows, k, None)
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_gemv_mxfp4_batch(lib):
    rows, k, n = 512, 2048, 5
    ws = [mxfp4_gguf(rows, k, 50 + j).cuda() for j in range(n)]
    xs = [torch.from_numpy(O.ref_act_quant_fp8(bf16_vals(k, 1.0, 60 + j).numpy())).cuda() for j in range(n)]
    ys = [torch.empty(rows, device="cuda") for _ in range(n)]
    arr = lambda ts: (P * n)(*[t.data_ptr() for t in ts])  # noqa: E731
    lib.stbl_gemv_mxfp4_batch(arr(ys), arr(ws), arr(xs), n, rows, k, None)
    torch.cuda.synchronize()
    for j in range(n):
        want = O.ref_gemv_mxfp4(ws[j].cpu().numpy(), xs[j].cpu().numpy(), rows, k)
        assert np.array_equal(ys[j].cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("round_out", [0, 1])
def test_gemv_f32_bit_exact(lib, round_out):
    rows, k = 777, 4096
    w = (torch.randn(rows, k) * 0.02).float()
    x = bf16_vals(k, 1.0, 3)
    want = O.ref_gemv_f32(w.numpy(), x.numpy(), round_out)
    y = torch.empty(rows, device="cuda")
    wc, xc = w.cuda(), x.cuda()
    lib.stbl_gemv_f32(p(y), p(wc), p(xc), rows, k, round_out, None)
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_swiglu_sqrt_softplus_axpy_round(lib):
    n = 2304
    g, u = bf16_vals(3 * n, 4.0, 1), bf16_vals(3 * n, 4.0, 2)
    wts = np.array([0.37, 1.0, 2.5], np.float32)
    for limit in (0.0, 10.0):
        out = torch.empty(3 * n, device="cuda")
        gc, uc = g.cuda(), u.cuda()
        lib.stbl_swiglu_batch(p(out), p(gc), p(uc), wts.ctypes.data, 3, F(limit), n, None)
        torch.cuda.synchronize()
        want = O.ref_swiglu(g.numpy(), u.numpy(), wts, limit, n)
        # expf differs between CUDA and the host libm by an ulp: the reference's own tolerance (1e-2)
        assert np.abs(out.cpu().numpy() - want).max() <= 1e-2 * np.abs(want).max()
    s = torch.randn(384) * 8
    sc = s.cuda()
    lib.stbl_sqrt_softplus(p(sc), 384, None)
    torch.cuda.synchronize()
    np.testing.assert_allclose(sc.cpu().numpy(), O.ref_sqrt_softplus(s.numpy()), rtol=1e-6)
    y, x = torch.randn(5000), torch.randn(5000)
    yc, xc = y.cuda(), x.cuda()
    lib.stbl_axpy(p(yc), p(xc), F(0.75), 5000, None)
    lib.stbl_round_bf16(p(yc), 5000, None)
    torch.cuda.synchronize()
    want = O.bf16_round(O.ref_axpy(y.numpy(), x.numpy(), 0.75))
    assert np.array_equal(yc.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_bitwise_against_reference_kernels(lib, ref):
    """stbl/cmp_kernels.py's A/B on the GEMV shapes it uses, 20 seeds: libstbl_moe.so against the
    reference's kernels.cu built from source."""
    bad = 0
    for seed in range(20):
        torch.manual_seed(seed)
        for rows, k in ((2304, 5120), (5120, 2304)):
            w = torch.randint(0, 256, (rows, k // 32 * 17), device="cuda", dtype=torch.uint8)
            w[:, ::17] = torch.randint(110, 130, (rows, k // 32), device="cuda", dtype=torch.uint8)
            x = torch.randn(k, device="cuda").bfloat16().float() * (10 ** torch.empty(k, device="cuda").uniform_(-2, 1))
            x2 = x.clone()
            lib.stbl_act_quant_fp8(p(x), k, None)
            ref.stbl_act_quant_fp8(p(x2), I(k), None)
            a, b = torch.empty(rows, device="cuda"), torch.empty(rows, device="cuda")
            lib.stbl_gemv_mxfp4(p(a), p(w), p(x), rows, k, None)
            ref.stbl_gemv_mxfp4(p(b), p(w), p(x), I(rows), I(k), None)
            torch.cuda.synchronize()
            bad += int((x != x2).sum()) + int((a != b).sum())
        for rows, k in ((32768, 1280), (5120, 8192), (512, 5120), (2304, 5120), (5120, 2304)):
            w = torch.randint(0, 256, (rows, k), device="cuda", dtype=torch.uint8)
            w[(w & 0x7F) == 0x7F] = 0
            sc = torch.randint(110, 130, ((rows + 31) // 32, k // 32), device="cuda", dtype=torch.uint8)
            x = torch.randn(k, device="cuda").bfloat16().float() * (10 ** torch.empty(k, device="cuda").uniform_(-2, 1))
            lib.stbl_act_quant_fp8(p(x), k, None)
            a, b = torch.empty(rows, device="cuda"), torch.empty(rows, device="cuda")
            lib.stbl_gemv_fp8(p(a), p(w), p(sc), p(x), rows, k, seed % 2, None)
            ref.stbl_gemv_fp8(p(b), p(w), p(sc), p(x), I(rows), I(k), I(seed % 2), None)
            torch.cuda.synchronize()
            bad += int((a != b).sum())
        rows, k = 256, 7168
        wf = torch.randn(rows, k, device="cuda") * 0.02
        x = torch.randn(k, device="cuda").bfloat16().float()
        a, b = torch.empty(rows, device="cuda"), torch.empty(rows, device="cuda")
        lib.stbl_gemv_f32(p(a), p(wf), p(x), rows, k, 0, None)
        ref.stbl_gemv_f32(p(b), p(wf), p(x), I(rows), I(k), I(0), None)
        s1 = torch.randn(256, device="cuda") * 8
        s2 = s1.clone()
        lib.stbl_sqrt_softplus(p(s1), 256, None)
        ref.stbl_sqrt_softplus(p(s2), I(256), None)
        g, u = torch.randn(2304 * 2, device="cuda") * 4, torch.randn(2304 * 2, device="cuda") * 4
        o1, o2 = torch.empty_like(g), torch.empty_like(g)
        wts = np.array([0.3, 1.7], np.float32)
        lib.stbl_swiglu_batch(p(o1), p(g), p(u), wts.ctypes.data, 2, F(10.0), 2304, None)
        ref.stbl_swiglu_batch(p(o2), p(g), p(u), P(wts.ctypes.data), I(2), F(10.0), I(2304), None)
        y1 = torch.randn(7168, device="cuda")
        y2 = y1.clone()
        xx = torch.randn(7168, device="cuda")
        lib.stbl_axpy(p(y1), p(xx), F(0.5), 7168, None)
        ref.stbl_axpy(p(y2), p(xx), F(0.5), I(7168), None)
        torch.cuda.synchronize()
        bad += int((a != b).sum()) + int((s1 != s2).sum()) + int((o1 != o2).sum()) + int((y1 != y2).sum())
    assert bad == 0, f"{bad} values differ from the reference kernels"
