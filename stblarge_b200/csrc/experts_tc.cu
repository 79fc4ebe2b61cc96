// FP8 128x128-block expert kernels (the body is tc8_body.cuh), the gather of x rows by position and
// the re-quantization of h between the up and down products.
#include "tc8_body.cuh"

namespace stbl {

template <bool UP, bool T2, int NTOK>
__global__ void __launch_bounds__(kTcThreads, 1) expert_tc_kernel(const __grid_constant__ TcMaps maps, TcParams p,
                                                                  int nst) {
    tc8_body<UP, T2, NTOK>(maps, p, nst, blockIdx.x, gridDim.x);
}

// x codes and scales of every position (routed assignments in dispatch order, then the shared
// expert's tokens), for the up kernel's activation tiles when T > 16
__global__ void __launch_bounds__(256) gather_kernel(GatherParams p) {
    pdl_launch_dependents();  // the next kernel may start its prologue; it waits for this one's end
    pdl_wait();
    const int pos = blockIdx.x;
    const int nrouted = p.T * p.topk;
    const int tok = pos < nrouted ? p.perm[pos] / p.topk : pos - nrouted;
    const uint4 *src = reinterpret_cast<const uint4 *>(p.xq + (size_t)tok * p.H);
    uint4 *dst = reinterpret_cast<uint4 *>(p.xq_pos + (size_t)pos * p.H);
    for (int i = threadIdx.x; i < p.H / 16; i += blockDim.x) dst[i] = __ldg(src + i);
    if (p.xe8) {
        for (int i = threadIdx.x; i < p.H / 128; i += blockDim.x)
            *reinterpret_cast<uint32_t *>(p.xe8_pos + ((size_t)i * p.xe8_pos_rows + pos) * 16) =
                __ldg(reinterpret_cast<const uint32_t *>(p.xe8 + ((size_t)i * p.xe8_rows + tok) * 16));
    } else {
        for (int i = threadIdx.x; i < p.H / 128; i += blockDim.x)
            p.xs_pos[(size_t)pos * (p.H / 128) + i] = __ldg(p.xs + (size_t)tok * p.xs_stride + i);
    }
}

// act_quant per 128 (ref/kernel.py:35-45, fp32 scale amax/448) of h for the down kernel: one warp per
// (position, 128-value block), four values a lane.
__global__ void __launch_bounds__(256) hquant_kernel(HquantParams p) {
    pdl_launch_dependents();  // the next kernel may start its prologue; it waits for this one's end
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int per_row = p.I / 128;
    const int nw = gridDim.x * (blockDim.x / 32);
    // rows: [0, n_pos), or under expert parallelism [0, routed rows received) and the shared rows
    const int n_head = p.n_routed_dev ? min(*p.n_routed_dev, p.n_pos) : p.n_pos;
    const int rows = n_head + (p.n_routed_dev ? p.n_tail : 0);
    const int items = rows * per_row;
    // two blocks per iteration, their loads issued together (a warp may have several blocks to do
    // when the grid is sized for the SMs rather than the rows, as under expert parallelism)
    for (int w0 = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); w0 < items; w0 += 2 * nw) {
      uint2 xin[2];
#pragma unroll
      for (int k = 0; k < 2; k++) {
        const int w = w0 + k * nw;
        if (w >= items) continue;
        int pos = w / per_row;
        if (pos >= n_head) pos = p.n_pos + (pos - n_head);
        xin[k] = __ldg(reinterpret_cast<const uint2 *>(p.h + (size_t)pos * p.I + (w % per_row) * 128 + 4 * lane));
      }
#pragma unroll
      for (int k = 0; k < 2; k++) {
        const int w = w0 + k * nw;
        if (w >= items) continue;
        int pos = w / per_row;
        const int g = w % per_row;
        if (pos >= n_head) pos = p.n_pos + (pos - n_head);
        const uint2 xv = xin[k];
        const float v[4] = {__uint_as_float(xv.x << 16), __uint_as_float(xv.x & 0xffff0000u), __uint_as_float(xv.y << 16),
                            __uint_as_float(xv.y & 0xffff0000u)};
        float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        // per-128: fp32 amax / 448 over the warp; per-32: power-of-two ceiling over 8 lanes
        for (int o = p.he8 ? 4 : 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        amax = fmaxf(amax, 1e-4f);
        const float tq = amax * (1.0f / 448.0f);
        const float s = p.he8 ? pow2_ceil(tq) : tq;
        uint32_t codes = 0;
#pragma unroll
        for (int u = 0; u < 4; u++) codes |= (uint32_t)e4m3_code(fminf(fmaxf(v[u] / s, -448.f), 448.f)) << (8 * u);
        *reinterpret_cast<uint32_t *>(p.hq + (size_t)pos * p.I + g * 128 + 4 * lane) = codes;
        if (p.he8) {
            if ((lane & 7) == 0) p.he8[(size_t)pos * (p.I / 32) + g * 4 + (lane >> 3)] = (uint8_t)(__float_as_uint(s) >> 23);
        } else if (lane == 0) {
            p.hs[(size_t)pos * per_row + g] = s;
        }
      }
    }
}

const void *hquant_kernel_ptr() { return (const void *)hquant_kernel; }

template __global__ void expert_tc_kernel<true, false, 16>(const __grid_constant__ TcMaps, TcParams, int);
template __global__ void expert_tc_kernel<true, true, 16>(const __grid_constant__ TcMaps, TcParams, int);
template __global__ void expert_tc_kernel<false, false, 16>(const __grid_constant__ TcMaps, TcParams, int);
template __global__ void expert_tc_kernel<false, true, 16>(const __grid_constant__ TcMaps, TcParams, int);
template __global__ void expert_tc_kernel<true, true, 32>(const __grid_constant__ TcMaps, TcParams, int);
template __global__ void expert_tc_kernel<false, true, 32>(const __grid_constant__ TcMaps, TcParams, int);

// two: items of two 128-row tiles (up: 128 gate + 128 up rows; down: 256 rows of W2); wide: items of
// up to 32 tokens (two-tile forms only)
const void *expert_tc_kernel_ptr(bool up, bool two, bool wide) {
    if (wide) return up ? (const void *)expert_tc_kernel<true, true, 32> : (const void *)expert_tc_kernel<false, true, 32>;
    if (up) return two ? (const void *)expert_tc_kernel<true, true, 16> : (const void *)expert_tc_kernel<true, false, 16>;
    return two ? (const void *)expert_tc_kernel<false, true, 16> : (const void *)expert_tc_kernel<false, false, 16>;
}

const void *gather_kernel_ptr() { return (const void *)gather_kernel; }

// dynamic shared-memory bytes of one launch (1 KB of it aligns the stages)
int expert_tc_smem_bytes(bool up, int H, int I, int nst, bool two, bool wide) {
    const int nkb = (up ? H : I) / 128;
    // the layout depends on the tile count and width only (up and down differ in nkb)
    if (wide) return Tc8<true, true, 32>::smem_bytes(nkb, nst);
    return two ? Tc8<true, true, 16>::smem_bytes(nkb, nst) : Tc8<true, false, 16>::smem_bytes(nkb, nst);
}

}  // namespace stbl
