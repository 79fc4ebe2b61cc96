"""The oracle's restatements of the reference's RMSNorm and hyper-connection post (the ops the fused
block, stbl_moe_forward_block, takes into the layer's kernels), on CPU.

hc_post (stbl/kernels.cu:328-338) is exact arithmetic in a fixed order: numpy float32 operations
(each rounded to nearest) restate it independently and must agree bit for bit.  rms_norm
(stbl/kernels.cu:217-236) calls CUDA's rsqrtf, which the oracle replaces by a correctly rounded
1/sqrt: its outputs must be within one bf16 step of the float64 norm (the GPU test compares the fused
kernels with the reference kernel itself, bit for bit)."""

import numpy as np

from oracle import oracle as O


def bf16(x):
    b = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) >> 16 << 16
    return b.astype(np.uint32).view(np.float32)


def test_hc_post_equals_stepwise_float32():
    rng = np.random.default_rng(4)
    for hc, dim in ((4, 64), (3, 40), (1, 8)):
        y = bf16(rng.standard_normal(dim))
        res = rng.standard_normal((hc, dim)).astype(np.float32)
        post = rng.standard_normal(hc).astype(np.float32)
        comb = rng.standard_normal((hc, hc)).astype(np.float32)
        want = np.empty((hc, dim), np.float32)
        for j in range(hc):
            s = np.zeros(dim, np.float32)
            for a in range(hc):
                s = (s + (comb[a, j] * res[a]).astype(np.float32)).astype(np.float32)
            want[j] = bf16((post[j] * y).astype(np.float32) + s)
        assert np.array_equal(O.ref_hc_post(y, res, post, comb).view(np.uint32), want.view(np.uint32))


def test_rms_norm_within_one_bf16_step_of_float64():
    rng = np.random.default_rng(6)
    for dim in (7168, 1024, 300):
        x = bf16(rng.standard_normal((3, dim)) * 2.0)
        w = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
        out = O.ref_rms_norm(x, w, 1e-6)
        x64 = x.astype(np.float64)
        exact = w * x64 / np.sqrt((x64 ** 2).mean(1, keepdims=True) + 1e-6)
        step = np.abs(exact) * 2.0 ** -8 + 1e-30
        assert np.all(np.abs(out - exact) <= step), np.max(np.abs(out - exact) / step)
        assert np.array_equal(out, bf16(out)), "outputs are bf16 values"
