/* Kernel-level C ABI of the MoE hot path, compatible with the reference's stbl/kernels.h.
 *
 * Same names, signatures and semantics as the reference's launchers for the MoE path, so that a
 * caller of stbl/kernels.h (stbl/model.cu:236-248, 509-592; the ctypes tests stbl/test_kernels.py,
 * stbl/cmp_kernels.py, stbl/bench_gemv.py) can link libstbl_moe.so instead.  Activations are fp32
 * device buffers holding bf16-rounded values; weights are opaque device pointers in the reference's
 * storage formats; every launcher enqueues on `st` (NULL: the legacy stream), allocates nothing and
 * returns nothing, as in the reference.  The GEMVs keep the reference's summation orders, so their
 * results are bit-identical to the reference's kernels (checked on the GPU against the reference
 * built from its own sources).
 */
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* stbl/kernels.h:9 — in place, per 32 values: x = bf16(e4m3(x / s) * s), s = 2^ceil(log2(max(amax,1e-4)/448)) */
void stbl_act_quant_fp8(float *x, int n, cudaStream_t st);
/* stbl/kernels.h:11 — x = bf16(x), round to nearest even */
void stbl_round_bf16(float *x, int n, cudaStream_t st);
/* stbl/kernels.h:14-15 — y[r] = sum_k x[k] e4m3(w[r][k]) with E8M0 32x32 block scales; k % 32 == 0,
   16-byte aligned rows; round_out: bf16 output */
void stbl_gemv_fp8(float *y, const void *w, const void *scale, const float *x, int rows, int k, int round_out,
                   cudaStream_t st);
/* stbl/kernels.h:16 — MXFP4 rows of 17-byte GGUF blocks (E8M0 scale, values 0..15 low nibbles,
   16..31 high nibbles); k % 256 == 0, 8-byte aligned; bf16 output */
void stbl_gemv_mxfp4(float *y, const void *w, const float *x, int rows, int k, cudaStream_t st);
/* stbl/kernels.h:17-20 — n <= kMxBatch matrices of one shape in one launch */
enum { kMxBatch = 16 };
void stbl_gemv_mxfp4_batch(float *const *y, const void *const *w, const float *const *x, int n, int rows, int k,
                           cudaStream_t st);
/* stbl/kernels.h:23 — fp32 GEMV (the router) */
void stbl_gemv_f32(float *y, const float *w, const float *x, int rows, int k, int round_out, cudaStream_t st);
/* stbl/kernels.h:34 — s = sqrt(softplus(s)), softplus threshold 20 */
void stbl_sqrt_softplus(float *s, int n, cudaStream_t st);
/* stbl/kernels.h:35 — out = bf16(silu(min(g, limit)) * clamp(u, -limit, limit) * weight); limit 0: no clamps */
void stbl_swiglu(float *out, const float *g, const float *u, float weight, float limit, int n, cudaStream_t st);
/* stbl/kernels.h:36-38 — count <= kMxBatch consecutive n-long segments, segment j scaled by weights[j] */
void stbl_swiglu_batch(float *out, const float *g, const float *u, const float *weights, int count, float limit, int n,
                       cudaStream_t st);
/* stbl/kernels.h:39 — y += a * x */
void stbl_axpy(float *y, const float *x, float a, int n, cudaStream_t st);

#ifdef __cplusplus
}
#endif
