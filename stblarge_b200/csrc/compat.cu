// kernels.h-compatible entry points of the MoE hot path (include/stbl_kernels.h).
//
// These accept the reference's storage formats (FP8 with E8M0 32x32 block scales, MXFP4 in 17-byte
// GGUF blocks, fp32 router weights) and reproduce its results bit for bit: the GEMVs keep the
// reference's summation order (products of a 32-block added by the halving tree, block sums
// added in block order: stbl/kernels.cu:94-97), written with explicit round-to-nearest intrinsics
// so that no multiply-add is fused where the reference rounds twice.  They serve callers of the
// reference's per-kernel ABI; the fused layer path (router.cu, experts.cu) is the fast path.
#include "../../include/stbl_kernels.h"
#include "common.cuh"

namespace stbl {
namespace {

constexpr int kRowsPerCta = 8;  // one warp per output row

__device__ __forceinline__ float tree32(float (&p)[32]) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < o; i++) p[i] = __fadd_rn(p[i], p[i + o]);
    return p[0];
}

__global__ void act_quant_fp8_kernel(float *x, int n_blocks) {
    const int b = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (b >= n_blocks) return;
    const float v = x[(size_t)b * 32 + lane];
    const float amax = fmaxf(warp_max(fabsf(v)), 1e-4f);
    const float s = pow2_ceil(amax * (1.0f / 448.0f));
    const float q = fminf(fmaxf(v / s, -448.f), 448.f);
    x[(size_t)b * 32 + lane] = bf16r(__fmul_rn(e4m3_value(e4m3_code(q)), s));
}

__global__ void round_bf16_kernel(float *x, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = bf16r(x[i]);
}

// FP8 rows with E8M0 32x32 scales: lane l takes block kb0 + l of its warp's row (two 16-byte loads).
__global__ void gemv_fp8_kernel(float *y, const uint8_t *w, const uint8_t *scale, const float *x, int rows, int k,
                                int round_out) {
    const int r = blockIdx.x * kRowsPerCta + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;
    const int nblk = k / 32;
    const uint8_t *wr = w + (size_t)r * k;
    const uint8_t *sr = scale + (size_t)(r / 32) * nblk;
    float acc = 0.f;
    for (int kb0 = 0; kb0 < nblk; kb0 += 32) {
        const int nb = min(32, nblk - kb0);
        float bs = 0.f;
        if (lane < nb) {
            const int kb = kb0 + lane;
            const uint4 q0 = __ldg(reinterpret_cast<const uint4 *>(wr + (size_t)kb * 32));
            const uint4 q1 = __ldg(reinterpret_cast<const uint4 *>(wr + (size_t)kb * 32 + 16));
            const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            const float4 *xv = reinterpret_cast<const float4 *>(x + (size_t)kb * 32);
            float p[32];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const float4 xq = __ldg(xv + q);
                p[4 * q + 0] = __fmul_rn(xq.x, e4m3_value(words[q] & 0xff));
                p[4 * q + 1] = __fmul_rn(xq.y, e4m3_value((words[q] >> 8) & 0xff));
                p[4 * q + 2] = __fmul_rn(xq.z, e4m3_value((words[q] >> 16) & 0xff));
                p[4 * q + 3] = __fmul_rn(xq.w, e4m3_value(words[q] >> 24));
            }
            bs = __fmul_rn(tree32(p), e8m0(sr[kb]));
        }
        for (int b = 0; b < nb; b++) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, bs, b));
    }
    if (lane == 0) y[r] = round_out ? bf16r(acc) : acc;
}

struct MxBatchArgs {
    float *y[kMxBatch];
    const uint8_t *w[kMxBatch];
    const float *x[kMxBatch];
};

__constant__ float kFp4Table[16] = {0.f, .5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f, -0.f, -.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

// MXFP4 GGUF rows: the warp stages 32 blocks (544 bytes) of its row in shared memory with 4-byte
// loads, then lane l sums block kb0 + l.  The value table sits in shared memory so that lanes
// indexing different codes do not serialise.
__global__ void gemv_mxfp4_kernel(MxBatchArgs b, int rows, int k) {
    __shared__ uint32_t stage[kRowsPerCta][136];
    __shared__ float table[16];
    if (threadIdx.x < 16) table[threadIdx.x] = kFp4Table[threadIdx.x];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = blockIdx.x * kRowsPerCta + warp;
    if (r >= rows) return;
    float *y = b.y[blockIdx.y];
    const uint8_t *w = b.w[blockIdx.y];
    const float *x = b.x[blockIdx.y];
    const int nblk = k / 32;
    const uint8_t *wr = w + (size_t)r * nblk * 17;
    const uint8_t *sb = reinterpret_cast<const uint8_t *>(stage[warp]);
    float acc = 0.f;
    for (int kb0 = 0; kb0 < nblk; kb0 += 32) {
        const int nb = min(32, nblk - kb0), words = nb * 17 / 4;
        const uint32_t *src = reinterpret_cast<const uint32_t *>(wr + (size_t)kb0 * 17);
        for (int i = lane; i < words; i += 32) stage[warp][i] = __ldg(src + i);
        __syncwarp();
        float bs = 0.f;
        if (lane < nb) {
            const uint8_t *blk = sb + lane * 17;
            const float4 *xv = reinterpret_cast<const float4 *>(x + (size_t)(kb0 + lane) * 32);
            float p[32];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float4 lo = __ldg(xv + q), hi = __ldg(xv + q + 4);
                const uint32_t c0 = blk[1 + 4 * q], c1 = blk[2 + 4 * q], c2 = blk[3 + 4 * q], c3 = blk[4 + 4 * q];
                p[4 * q + 0] = __fmul_rn(lo.x, table[c0 & 15]);
                p[4 * q + 1] = __fmul_rn(lo.y, table[c1 & 15]);
                p[4 * q + 2] = __fmul_rn(lo.z, table[c2 & 15]);
                p[4 * q + 3] = __fmul_rn(lo.w, table[c3 & 15]);
                p[16 + 4 * q + 0] = __fmul_rn(hi.x, table[c0 >> 4]);
                p[16 + 4 * q + 1] = __fmul_rn(hi.y, table[c1 >> 4]);
                p[16 + 4 * q + 2] = __fmul_rn(hi.z, table[c2 >> 4]);
                p[16 + 4 * q + 3] = __fmul_rn(hi.w, table[c3 >> 4]);
            }
            bs = __fmul_rn(tree32(p), e8m0(blk[0]));
        }
        for (int i = 0; i < nb; i++) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, bs, i));
        __syncwarp();
    }
    if (lane == 0) y[r] = bf16r(acc);
}

// fp32 GEMV: lane l accumulates x[i] * w[i] for i = l, l + 32, ... by fused multiply-add, then the
// xor butterfly adds the lane sums.
__global__ void gemv_f32_kernel(float *y, const float *w, const float *x, int rows, int k, int round_out) {
    const int r = blockIdx.x * kRowsPerCta + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;
    const float *wr = w + (size_t)r * k;
    float acc = 0.f;
    for (int i = lane; i < k; i += 32) acc = __fmaf_rn(__ldg(x + i), __ldg(wr + i), acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    if (lane == 0) y[r] = round_out ? bf16r(acc) : acc;
}

__global__ void sqrt_softplus_kernel(float *s, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = s[i];
    s[i] = sqrtf(v > 20.f ? v : log1pf(expf(v)));
}

struct SegWeights {
    float w[kMxBatch];
};

__global__ void swiglu_kernel(float *out, const float *g, const float *u, SegWeights ws, float limit, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const size_t at = (size_t)blockIdx.y * n + i;
    float gv = g[at], uv = u[at];
    if (limit > 0) {
        uv = fminf(fmaxf(uv, -limit), limit);
        gv = fminf(gv, limit);
    }
    out[at] = bf16r(__fmul_rn(__fmul_rn(__fdiv_rn(gv, __fadd_rn(1.f, expf(-gv))), uv), ws.w[blockIdx.y]));
}

__global__ void axpy_kernel(float *y, const float *x, float a, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fmaf_rn(a, x[i], y[i]);
}

inline int cdiv(int a, int b) { return (a + b - 1) / b; }

}  // namespace
}  // namespace stbl

using namespace stbl;

extern "C" {

void stbl_act_quant_fp8(float *x, int n, cudaStream_t st) {
    if (n < 32) return;
    act_quant_fp8_kernel<<<cdiv(n / 32, 8), 256, 0, st>>>(x, n / 32);
}

void stbl_round_bf16(float *x, int n, cudaStream_t st) {
    if (n < 1) return;
    round_bf16_kernel<<<cdiv(n, 256), 256, 0, st>>>(x, n);
}

void stbl_gemv_fp8(float *y, const void *w, const void *scale, const float *x, int rows, int k, int round_out,
                   cudaStream_t st) {
    if (rows < 1 || k < 32) return;
    gemv_fp8_kernel<<<cdiv(rows, kRowsPerCta), 32 * kRowsPerCta, 0, st>>>(y, static_cast<const uint8_t *>(w),
                                                                         static_cast<const uint8_t *>(scale), x, rows, k,
                                                                         round_out);
}

void stbl_gemv_mxfp4_batch(float *const *y, const void *const *w, const float *const *x, int n, int rows, int k,
                           cudaStream_t st) {
    if (n < 1 || n > kMxBatch || rows < 1 || k < 256) return;
    MxBatchArgs b{};
    for (int j = 0; j < n; j++) b.y[j] = y[j], b.w[j] = static_cast<const uint8_t *>(w[j]), b.x[j] = x[j];
    gemv_mxfp4_kernel<<<dim3(cdiv(rows, kRowsPerCta), n), 32 * kRowsPerCta, 0, st>>>(b, rows, k);
}

void stbl_gemv_mxfp4(float *y, const void *w, const float *x, int rows, int k, cudaStream_t st) {
    stbl_gemv_mxfp4_batch(&y, &w, &x, 1, rows, k, st);
}

void stbl_gemv_f32(float *y, const float *w, const float *x, int rows, int k, int round_out, cudaStream_t st) {
    if (rows < 1 || k < 1) return;
    gemv_f32_kernel<<<cdiv(rows, kRowsPerCta), 32 * kRowsPerCta, 0, st>>>(y, w, x, rows, k, round_out);
}

void stbl_sqrt_softplus(float *s, int n, cudaStream_t st) {
    if (n < 1) return;
    sqrt_softplus_kernel<<<cdiv(n, 256), 256, 0, st>>>(s, n);
}

void stbl_swiglu_batch(float *out, const float *g, const float *u, const float *weights, int count, float limit, int n,
                       cudaStream_t st) {
    if (count < 1 || count > kMxBatch || n < 1) return;
    SegWeights ws{};
    for (int j = 0; j < count; j++) ws.w[j] = weights[j];
    swiglu_kernel<<<dim3(cdiv(n, 256), count), 256, 0, st>>>(out, g, u, ws, limit, n);
}

void stbl_swiglu(float *out, const float *g, const float *u, float weight, float limit, int n, cudaStream_t st) {
    stbl_swiglu_batch(out, g, u, &weight, 1, limit, n, st);
}

void stbl_axpy(float *y, const float *x, float a, int n, cudaStream_t st) {
    if (n < 1) return;
    axpy_kernel<<<cdiv(n, 256), 256, 0, st>>>(y, x, a, n);
}

}  // extern "C"
