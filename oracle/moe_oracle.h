/* CPU oracle for the MoE decode hot path.  TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the reference's MoE layer (stbl/model.cu:426-594) and of the
 * numerics of its torch stand-ins (ref/kernel.py) and GPU kernels (stbl/kernels.cu).  It is used
 * by tests/, by __graft_entry__.smoke() and by bench.py's cpu_baseline / --impl reference legs as
 * the checker and the CPU baseline.  The product (stblarge_b200/) never links or calls it.
 *
 * Every function names the reference lines it restates.  Parity of this oracle against the
 * reference itself is pinned by tests/test_oracle_golden.py (golden vectors produced by importing
 * ref/kernel.py, script tests/golden/make_golden.py) and, on a GPU box, by bitwise A/B against
 * the reference's own kernels built from stbl/kernels.cu (oracle/build_ref.sh).
 */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* weight storage formats (same ids as include/stbl_moe.h) */
enum {
    ORC_FMT_NONE = 0,
    ORC_FMT_FP8_B128 = 1,    /* e4m3 codes [rows][k], fp32 scales [ceil(rows/128)][ceil(k/128)] */
    ORC_FMT_MXFP4 = 2,       /* e2m1 codes [rows][k/2] low nibble first, e8m0 scales [rows][k/32] */
    ORC_FMT_FP8_E8M0 = 3,    /* e4m3 codes [rows][k], e8m0 scales [ceil(rows/32)][k/32] (32x32 blocks) */
};

enum { ORC_SCORE_SIGMOID = 0, ORC_SCORE_SQRT_SOFTPLUS = 1 };

/* ---- scalar formats --------------------------------------------------------------------------- */
float orc_bf16_round(float x);               /* RNE to bf16, kernels.cu:13 */
float orc_pow2_ceil(float t);                /* ref/kernel.py:22-26, kernels.cu:26-30 */
float orc_e4m3_value(uint8_t code);          /* tools/convert_official.py:40-48 */
uint8_t orc_e4m3_encode(float v);            /* RNE, saturating to +-448 (torch .to(float8_e4m3fn) after clamp) */
float orc_e2m1_value(uint8_t nibble);        /* ref/kernel.py:14-16 */
uint8_t orc_e2m1_encode(float v);            /* ref/kernel.py:48-52 + 75-77, v already within [-6, 6] */
/* array forms of the above, for the Python tests */
void orc_bf16_round_n(const float *x, int n, float *out);
void orc_pow2_ceil_n(const float *x, int n, float *out);
void orc_e4m3_encode_n(const float *x, int n, uint8_t *out);
void orc_e2m1_encode_n(const float *x, int n, uint8_t *out);

/* ---- quantizers ------------------------------------------------------------------------------- */
/* act_quant(x, block, scale_fmt=pow2 ? "ue8m0" : None): ref/kernel.py:35-45, per row of k values. */
void orc_act_quant(const float *x, int rows, int k, int block, int pow2, uint8_t *codes, float *scales);
/* FP8 weight quantization with 128x128 fp32 block scales (act_quant's rule on 2-D blocks). */
void orc_quant_fp8_b128(const float *w, int rows, int k, uint8_t *codes, float *scales);
/* MXFP4 weight quantization, fp4_act_quant E8M0 branch: ref/kernel.py:55-72. */
void orc_quant_mxfp4(const float *w, int rows, int k, uint8_t *packed, uint8_t *scales);
void orc_quant_fp8_e8m0(const float *w, int rows, int k, uint8_t *codes, uint8_t *scales);
void orc_gemv_fp8_e8m0(const uint8_t *w, const uint8_t *ws, int rows, int k, const uint8_t *xc, const float *xs,
                       int act_block, int n_tok, float *y);
/* MXFP4 in the official layout -> the reference engine's GGUF 17-byte blocks, and back */
void orc_mxfp4_to_gguf(const uint8_t *codes, const uint8_t *scales, int rows, int k, uint8_t *blocks);
void orc_mxfp4_from_gguf(const uint8_t *blocks, int rows, int k, uint8_t *codes, uint8_t *scales);

/* ---- GEMVs over several tokens (fp8_gemm / fp4_gemm numerics, ref/kernel.py:85-102) ----------- */
/* y[t][r] = sum_k (code_x*sx) * (code_w*sw), fp32, no output rounding. xs: per-(token, act block). */
void orc_gemv_fp8_b128(const uint8_t *w, const float *ws, int rows, int k, const uint8_t *xc, const float *xs,
                       int act_block, int n_tok, float *y);
void orc_gemv_mxfp4(const uint8_t *w, const uint8_t *ws, int rows, int k, const uint8_t *xc, const float *xs,
                    int act_block, int n_tok, float *y);

/* ---- router (model.cu:430-452 composition, V3 group-limited or V4 flat selection) ------------- */
/* logits[t][e] = W[e] . x[t]; fp32 with the reduction order of the GPU router kernel: the hidden
 * dimension is cut into orc_router_ksplit(H) equal slices (4 when H % 512 == 0, else 1); in each, lane
 * l of 32 takes k = 128 i + 4 l + j (i ascending, j = 0..3) by fused multiply-add, then an xor
 * butterfly adds the 32 lane sums (16, 8, 4, 2, 1); the slice sums are added in slice order.
 * Needs H % 128 == 0. */
int orc_router_ksplit(int H);
void orc_router_logits(const float *W, const uint16_t *x_bf16, int T, int E, int H, float *logits);
/* scores, top-k ids in selection order (biased score descending, lower id first on ties) and
 * routing weights score / (sum + 1e-20) * route_scale (model.cu:444-451, 527-530). */
int orc_router_select(const float *logits, const float *bias, int T, int E, int topk, int n_groups, int topk_groups,
                      int score_fn, float route_scale, float *scores, int *idx, float *weights);
/* bucketed dispatch: counts[E], offsets[E+1], perm[T*topk] (expert-major, token then slot order);
 * perm holds t * topk + slot. */
void orc_dispatch(const int *idx, int T, int E, int topk, int *counts, int *offsets, int *perm);

/* ---- whole MoE layer -------------------------------------------------------------------------- */
typedef struct orc_moe_desc {
    int hidden, inter, n_experts, topk, n_groups, topk_groups, score_fn;
    float route_scale, swiglu_limit;
    int routed_fmt, shared_fmt;
    const float *router_w, *router_bias;
    /* routed expert e, matrix m (0 gate [inter][hidden], 1 up, 2 down [hidden][inter]) */
    const uint8_t *const *routed_w; /* [3 * n_experts], index m * n_experts + e; NULL = absent */
    const void *const *routed_s;    /* [3 * n_experts] */
    const uint8_t *shared_w[3];
    const void *shared_s[3];
    /* 1: routed MXFP4 experts take Q8 activations (int8 per 32, scale amax / 127) instead of FP8
     * (ref/emulate_ds4.py:23-30, 69-77); the shared expert keeps its FP8 rule */
    int act_q8;
} orc_moe_desc;

/* y = bf16(sum over top-k slots in order of the routed outputs, then + shared output).  Writes
 * idx / weights [T][topk] when non-NULL.  Returns 0, or -1 when a routed expert is absent. */
int orc_moe_forward(const orc_moe_desc *d, const uint16_t *x, int T, uint16_t *y, int *idx, float *weights,
                    int nthreads);
int orc_moe_forward_routed(const orc_moe_desc *d, const uint16_t *x, int T, const int *forced, uint16_t *y, int *idx,
                           float *weights, int nthreads);

/* ---- the reference's own kernel semantics (stbl/kernels.cu), exact summation orders ----------- */
void orc_ref_act_quant_fp8(float *x, int n);                                              /* :56-63 */
void orc_ref_round_bf16(float *x, int n);                                                 /* :86-89 */
void orc_ref_gemv_fp8(float *y, const uint8_t *w, const uint8_t *scale, const float *x, int rows, int k,
                      int round_out);                                                     /* :98-132 */
void orc_ref_gemv_mxfp4(float *y, const uint8_t *w, const float *x, int rows, int k);     /* :142-191 */
void orc_ref_gemv_f32(float *y, const float *w, const float *x, int rows, int k, int round_out); /* :206-214 */
void orc_ref_sqrt_softplus(float *s, int n);                                              /* :437-442 */
void orc_ref_swiglu(float *out, const float *g, const float *u, const float *weights, int count, float limit,
                    int n);                                                               /* :445-459 */
void orc_ref_axpy(float *y, const float *x, float a, int n);                              /* :461-464 */
void orc_ref_rms_norm(float *out, const float *x, const float *w, int rows, int dim, float eps); /* :217-236 */
void orc_ref_hc_post(float *out, const float *x, const float *res, const float *post, const float *comb, int hc,
                     int dim);                                                            /* :328-338 */

/* ---- Q8 activation variant (ref/emulate_ds4.py: q8_codes :23-30, the FP4 branch of linear :69-77) --------
 * Activations quantized per 32 values to int8 with scale d = amax / 127 (fp32, no fp16 rounding for
 * activations), codes round-half-even(x / d) clamped to [-128, 127] (d = 0: divided by 1).  The FP4
 * expert linear takes them instead of FP8 activations:
 *   y[t][r] = sum_b d[t][b] * 2^(s[r][b] - 127) * sum_i q[t][b][i] * e2m1(w[r][b][i])
 * with exact integer sums per block, the blocks added in double precision and the total rounded once
 * to fp32 (the emulation's fp32 matmul differs from it only by its own summation's rounding).  Codes in the layer's layout (values 2j, 2j + 1 in byte j, low nibble
 * first), e8m0 scales [rows][k/32] taken as 2^(s - 127). */
void orc_q8_codes(const float *x, int n_blocks, int8_t *q, float *d);
void orc_gemv_mxfp4_q8(const uint8_t *w, const uint8_t *ws, int rows, int k, const int8_t *q, const float *d, int n_tok,
                       float *y);

#ifdef __cplusplus
}
#endif
