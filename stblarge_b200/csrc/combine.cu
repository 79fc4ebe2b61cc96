// Ordered combine of the MoE layer: y = bf16(((0 + eo_0) + ... + eo_{k-1}) + shared), the sums in fp32
// in top-k order (stbl/model.cu:589-592, the reference's k_axpy chain + k_round_bf16), one thread per
// 8 outputs.  Under expert parallelism the routed rows were written by the owning GPUs; the kernel
// first waits for every rank's done flag (raised by the last CTA of that rank's down kernel).  With the fused
// hyper-connection post (CombineParams::hout) each thread also writes its 8 outputs of every stream j
// of the block's residual update (stbl/model.cu:805, k_hc_post, stbl/kernels.cu:328-338).
#include "layer.cuh"

namespace stbl {

__global__ void __launch_bounds__(256) combine_kernel(CombineParams p) {
    pdl_launch_dependents();  // the next kernel may start its prologue; it waits for this one's end
    pdl_wait();
    if (p.ep.n_ranks > 1) {
        // expert parallelism: every rank's down kernel has written its rows into this rank's eo rows
        // once that rank's done flag carries this call
        __shared__ int ok;
        if (threadIdx.x == 0) {
            ok = wait_flags_sys(reinterpret_cast<const unsigned int *>(p.ep.region[p.ep.rank] + p.ep.L.done_flag),
                                p.ep.n_ranks, p.ep.epoch);
            if (!ok) atomicOr(p.status, kErrWaitTimeout);
        }
        __syncthreads();
    }
    const int per_row = p.H / 8;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= p.T * per_row) return;
    const int t = i / per_row, c = (i % per_row) * 8;
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; q++) acc[q] = 0.f;
    for (int s = 0; s < p.topk; s++) {
        // L2 loads: under expert parallelism the rows were written by other GPUs during this call
        const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(p.eo + ((size_t)t * p.topk + s) * p.H + c));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            acc[2 * q] = acc[2 * q] + __uint_as_float(w[q] << 16);
            acc[2 * q + 1] = acc[2 * q + 1] + __uint_as_float(w[q] & 0xffff0000u);
        }
    }
    if (p.has_shared) {
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(p.sh + (size_t)t * p.H + c));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            acc[2 * q] = acc[2 * q] + __uint_as_float(w[q] << 16);
            acc[2 * q + 1] = acc[2 * q + 1] + __uint_as_float(w[q] & 0xffff0000u);
        }
    }
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; q++) o[q] = (uint32_t)f32_to_bf16_bits(acc[2 * q]) | ((uint32_t)f32_to_bf16_bits(acc[2 * q + 1]) << 16);
    if (p.y) *reinterpret_cast<uint4 *>(p.y + (size_t)t * p.H + c) = make_uint4(o[0], o[1], o[2], o[3]);
    if (p.hout) {
        // hout[t][j][d] = bf16(post[j] * y[d] + sum_a comb[a][j] * res[a][d]), y the bf16 output
        float yv[8];
#pragma unroll
        for (int q = 0; q < 4; q++) yv[2 * q] = __uint_as_float(o[q] << 16), yv[2 * q + 1] = __uint_as_float(o[q] & 0xffff0000u);
        const float *post = p.post + (size_t)t * p.hc, *comb = p.comb + (size_t)t * p.hc * p.hc;
        const float *res = p.res + (size_t)t * p.hc * p.H + c;
        for (int j = 0; j < p.hc; j++) {
            float sum[8];
#pragma unroll
            for (int q = 0; q < 8; q++) sum[q] = 0.f;
            for (int a = 0; a < p.hc; a++) {
                const float cj = __ldg(comb + a * p.hc + j);
                const float4 r0 = __ldg(reinterpret_cast<const float4 *>(res + (size_t)a * p.H));
                const float4 r1 = __ldg(reinterpret_cast<const float4 *>(res + (size_t)a * p.H + 4));
                const float rv[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
                for (int q = 0; q < 8; q++) sum[q] = __fadd_rn(sum[q], __fmul_rn(cj, rv[q]));
            }
            const float pj = __ldg(post + j);
            float hv[8];
#pragma unroll
            for (int q = 0; q < 8; q++) hv[q] = bf16r(__fadd_rn(__fmul_rn(pj, yv[q]), sum[q]));
            float4 *dst = reinterpret_cast<float4 *>(p.hout + ((size_t)t * p.hc + j) * p.H + c);
            dst[0] = make_float4(hv[0], hv[1], hv[2], hv[3]);
            dst[1] = make_float4(hv[4], hv[5], hv[6], hv[7]);
        }
    }
}

const void *combine_kernel_ptr() { return (const void *)combine_kernel; }

}  // namespace stbl
