/* CPU oracle for the MoE decode hot path.  TEST INFRASTRUCTURE ONLY (see moe_oracle.h).
 * Built with -ffp-contract=off so that every a*b+c below is two roundings unless fmaf is written. */
#include "moe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ---- scalar formats --------------------------------------------------------------------------- */

float orc_bf16_round(float x) {
    uint32_t b = f2u(x);
    if ((b & 0x7fffffffu) > 0x7f800000u) return x; /* NaN stays */
    b += 0x7fffu + ((b >> 16) & 1u);
    return u2f(b & 0xffff0000u);
}

static inline float bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }
static inline uint16_t f32_to_bf16_bits(float x) { return (uint16_t)(f2u(orc_bf16_round(x)) >> 16); }

/* ref/kernel.py:22-26: exponent of t, plus one when any mantissa bit is set. */
float orc_pow2_ceil(float t) {
    const uint32_t b = f2u(t);
    const int e = (int)((b >> 23) & 0xff) - 127 + ((b & 0x7fffffu) != 0);
    return u2f((uint32_t)(e + 127) << 23);
}

static float g_e4m3[256];
static int g_e4m3_ready = 0;

static void e4m3_init(void) {
    if (g_e4m3_ready) return;
    for (int c = 0; c < 256; c++) {
        const int e = (c >> 3) & 15, m = c & 7;
        float v = e == 0 ? (float)m / 8.0f * ldexpf(1.f, -6) : (1.0f + (float)m / 8.0f) * ldexpf(1.f, e - 7);
        if (e == 15 && m == 7) v = NAN;
        g_e4m3[c] = (c & 0x80) ? -v : v;
    }
    g_e4m3_ready = 1;
}

float orc_e4m3_value(uint8_t code) {
    e4m3_init();
    return g_e4m3[code];
}

/* Round to nearest even on the e4m3 grid (3 mantissa bits, subnormal quantum 2^-9), saturating to
 * the largest finite value 448.  The torch cast after clamp(-448, 448) (ref/kernel.py:41) and the
 * CUDA cast with saturation (kernels.cu:40-42) both land here. */
uint8_t orc_e4m3_encode(float v) {
    if (isnan(v)) return 0x7f;
    const uint8_t sign = signbit(v) ? 0x80 : 0;
    const float a = fabsf(v);
    if (a >= 448.f) return sign | 0x7e;
    int e;
    frexpf(a, &e); /* a = f * 2^e, f in [0.5, 1): a in [2^(e-1), 2^e) */
    int E = e - 1;
    if (a == 0.f || E < -6) E = -6;
    const float q = ldexpf(1.f, E - 3);
    const float r = rintf(a / q) * q; /* the division by a power of two is exact */
    if (r == 0.f) return sign;
    if (r >= 448.f) return sign | 0x7e;
    int e2;
    frexpf(r, &e2);
    const int E2 = e2 - 1;
    if (E2 < -6) return sign | (uint8_t)(int)(r * 512.f); /* subnormal: m * 2^-9 */
    const int m = (int)((r / ldexpf(1.f, E2) - 1.f) * 8.f);
    return sign | (uint8_t)(((E2 + 7) << 3) | m);
}

static const float kFp4[16] = {0.f, .5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f, -0.f, -.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

float orc_e2m1_value(uint8_t nibble) { return kFp4[nibble & 15]; }

/* ref/kernel.py:48-52 (_round_fp4: step 0.5 / 1 / 2, half to even) and :75-77 (_fp4_codes: index
 * on the magnitude grid, sign bit from signbit). */
uint8_t orc_e2m1_encode(float v) {
    const float a = fabsf(v);
    const float step = a < 2.f ? .5f : (a < 4.f ? 1.f : 2.f);
    const float q = rintf(a / step) * step;
    int mag = 0;
    while (mag < 7 && kFp4[mag] < q) mag++;
    return (uint8_t)(mag | (signbit(v) ? 8 : 0));
}

void orc_bf16_round_n(const float *x, int n, float *out) {
    for (int i = 0; i < n; i++) out[i] = orc_bf16_round(x[i]);
}
void orc_pow2_ceil_n(const float *x, int n, float *out) {
    for (int i = 0; i < n; i++) out[i] = orc_pow2_ceil(x[i]);
}
void orc_e4m3_encode_n(const float *x, int n, uint8_t *out) {
    for (int i = 0; i < n; i++) out[i] = orc_e4m3_encode(x[i]);
}
void orc_e2m1_encode_n(const float *x, int n, uint8_t *out) {
    for (int i = 0; i < n; i++) out[i] = orc_e2m1_encode(x[i]);
}

/* ---- quantizers ------------------------------------------------------------------------------- */

static const float kInv448 = (float)(1.0 / 448.0);
static const float kInv6 = (float)(1.0 / 6.0);

/* ref/kernel.py:35-45: amax over the block, clamp_min(1e-4), t = amax * fp32(1/448), the scale is t
 * or 2^ceil(log2 t); codes = e4m3(clamp(x / s, -448, 448)). */
void orc_act_quant(const float *x, int rows, int k, int block, int pow2, uint8_t *codes, float *scales) {
    const int nb = k / block;
    for (int r = 0; r < rows; r++)
        for (int b = 0; b < nb; b++) {
            const float *xb = x + (size_t)r * k + (size_t)b * block;
            float amax = 0.f;
            for (int i = 0; i < block; i++) amax = fmaxf(amax, fabsf(xb[i]));
            amax = fmaxf(amax, 1e-4f);
            const float t = amax * kInv448;
            const float s = pow2 ? orc_pow2_ceil(t) : t;
            for (int i = 0; i < block; i++) {
                float q = xb[i] / s;
                q = fminf(fmaxf(q, -448.f), 448.f);
                codes[(size_t)r * k + (size_t)b * block + i] = orc_e4m3_encode(q);
            }
            scales[(size_t)r * nb + b] = s;
        }
}

void orc_quant_fp8_b128(const float *w, int rows, int k, uint8_t *codes, float *scales) {
    const int rb = (rows + 127) / 128, kb = (k + 127) / 128;
    for (int bi = 0; bi < rb; bi++)
        for (int bj = 0; bj < kb; bj++) {
            float amax = 0.f;
            for (int r = bi * 128; r < rows && r < bi * 128 + 128; r++)
                for (int c = bj * 128; c < k && c < bj * 128 + 128; c++) amax = fmaxf(amax, fabsf(w[(size_t)r * k + c]));
            amax = fmaxf(amax, 1e-4f);
            const float s = amax * kInv448;
            for (int r = bi * 128; r < rows && r < bi * 128 + 128; r++)
                for (int c = bj * 128; c < k && c < bj * 128 + 128; c++) {
                    float q = w[(size_t)r * k + c] / s;
                    q = fminf(fmaxf(q, -448.f), 448.f);
                    codes[(size_t)r * k + c] = orc_e4m3_encode(q);
                }
            scales[(size_t)bi * kb + bj] = s;
        }
}

/* ref/kernel.py:55-72, E8M0 branch: amax clamp_min(6 * 2^-126), s = 2^ceil(log2(amax * fp32(1/6))),
 * q = round_fp4(clamp(w / s, -6, 6)); two codes per byte, the even index in the low nibble. */
void orc_quant_mxfp4(const float *w, int rows, int k, uint8_t *packed, uint8_t *scales) {
    const int nb = k / 32;
    for (int r = 0; r < rows; r++)
        for (int b = 0; b < nb; b++) {
            const float *wb = w + (size_t)r * k + (size_t)b * 32;
            float amax = 0.f;
            for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(wb[i]));
            amax = fmaxf(amax, 6.f * ldexpf(1.f, -126));
            const float s = orc_pow2_ceil(amax * kInv6);
            uint8_t c[32];
            for (int i = 0; i < 32; i++) {
                float q = wb[i] / s;
                q = fminf(fmaxf(q, -6.f), 6.f);
                c[i] = orc_e2m1_encode(q);
            }
            for (int i = 0; i < 16; i++) packed[(size_t)r * (k / 2) + (size_t)b * 16 + i] = (uint8_t)(c[2 * i] | (c[2 * i + 1] << 4));
            scales[(size_t)r * nb + b] = (uint8_t)(f2u(s) >> 23);
        }
}

/* FP8 weights with e8m0 scales per 32x32 block (the reference engine's format, kernels.cu:98-132,
 * tools/convert_official.py:74-81).  Synthetic weights only: the reference copies the checkpoint's
 * scales byte for byte; here a block's scale follows act_quant's power-of-two rule (ref/kernel.py:35-45
 * with scale_fmt): amax clamp_min(1e-4), s = 2^ceil(log2(amax / 448)), q = e4m3(clamp(w / s, +-448)). */
void orc_quant_fp8_e8m0(const float *w, int rows, int k, uint8_t *codes, uint8_t *scales) {
    const int rb = (rows + 31) / 32, kb = k / 32;
    for (int bi = 0; bi < rb; bi++)
        for (int bj = 0; bj < kb; bj++) {
            float amax = 0.f;
            for (int r = bi * 32; r < rows && r < bi * 32 + 32; r++)
                for (int c = bj * 32; c < bj * 32 + 32; c++) amax = fmaxf(amax, fabsf(w[(size_t)r * k + c]));
            amax = fmaxf(amax, 1e-4f);
            const float s = orc_pow2_ceil(amax * kInv448);
            for (int r = bi * 32; r < rows && r < bi * 32 + 32; r++)
                for (int c = bj * 32; c < bj * 32 + 32; c++) {
                    float q = w[(size_t)r * k + c] / s;
                    q = fminf(fmaxf(q, -448.f), 448.f);
                    codes[(size_t)r * k + c] = orc_e4m3_encode(q);
                }
            scales[(size_t)bi * kb + bj] = (uint8_t)(f2u(s) >> 23);
        }
}

/* GGUF MXFP4 block (kernels.cu:134-141, tools/convert_official.py:187-201): the scale byte, then 16
 * bytes with values 0..15 of the block in the low nibbles and 16..31 in the high nibbles. */
void orc_mxfp4_to_gguf(const uint8_t *codes, const uint8_t *scales, int rows, int k, uint8_t *blocks) {
    for (int r = 0; r < rows; r++)
        for (int b = 0; b < k / 32; b++) {
            const uint8_t *src = codes + (size_t)r * (k / 2) + (size_t)b * 16;
            uint8_t *dst = blocks + ((size_t)r * (k / 32) + b) * 17;
            uint8_t v[32];
            for (int i = 0; i < 16; i++) v[2 * i] = src[i] & 15, v[2 * i + 1] = src[i] >> 4;
            dst[0] = scales[(size_t)r * (k / 32) + b];
            for (int i = 0; i < 16; i++) dst[1 + i] = (uint8_t)(v[i] | (v[16 + i] << 4));
        }
}

void orc_mxfp4_from_gguf(const uint8_t *blocks, int rows, int k, uint8_t *codes, uint8_t *scales) {
    for (int r = 0; r < rows; r++)
        for (int b = 0; b < k / 32; b++) {
            const uint8_t *src = blocks + ((size_t)r * (k / 32) + b) * 17;
            uint8_t v[32];
            for (int i = 0; i < 16; i++) v[i] = src[1 + i] & 15, v[16 + i] = src[1 + i] >> 4;
            scales[(size_t)r * (k / 32) + b] = src[0];
            for (int i = 0; i < 16; i++) codes[(size_t)r * (k / 2) + (size_t)b * 16 + i] = (uint8_t)(v[2 * i] | (v[2 * i + 1] << 4));
        }
}

/* ---- GEMVs ------------------------------------------------------------------------------------ */

/* FP8 e4m3 with 32x32 e8m0 block scales: B = code * 2^(e8m0 - 127), dequantized products accumulated
 * in fp32, k ascending (the 32-block e8m0 variant of fp8_gemm, ref/kernel.py:85-91). */
void orc_gemv_fp8_e8m0(const uint8_t *w, const uint8_t *ws, int rows, int k, const uint8_t *xc, const float *xs,
                       int act_block, int n_tok, float *y) {
    e4m3_init();
    const int na = k / act_block;
    float *A = (float *)malloc(sizeof(float) * (size_t)n_tok * k);
    for (int t = 0; t < n_tok; t++)
        for (int c = 0; c < k; c++) A[(size_t)t * k + c] = g_e4m3[xc[(size_t)t * k + c]] * xs[(size_t)t * na + c / act_block];
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        const uint8_t *wr = w + (size_t)r * k;
        const uint8_t *sr = ws + (size_t)(r / 32) * (k / 32);
        /* tokens in groups of 64 (each token's sum is independent of the grouping) */
        for (int t0 = 0; t0 < n_tok; t0 += 64) {
        const int nt = n_tok - t0 < 64 ? n_tok - t0 : 64;
        float acc[64];
        for (int t = 0; t < nt; t++) acc[t] = 0.f;
        for (int c = 0; c < k; c++) {
            const float B = g_e4m3[wr[c]] * u2f((uint32_t)sr[c / 32] << 23);
            for (int t = 0; t < nt; t++) acc[t] = acc[t] + A[(size_t)(t0 + t) * k + c] * B;
        }
        for (int t = 0; t < nt; t++) y[(size_t)(t0 + t) * rows + r] = acc[t];
        }
    }
    free(A);
}

/* fp8_gemm (ref/kernel.py:85-91): A = code * a_s and B = code * b_s are each one fp32 product; the
 * dot product is accumulated in fp32, k ascending. */
void orc_gemv_fp8_b128(const uint8_t *w, const float *ws, int rows, int k, const uint8_t *xc, const float *xs,
                       int act_block, int n_tok, float *y) {
    e4m3_init();
    const int kb = (k + 127) / 128, na = k / act_block;
    float *A = (float *)malloc(sizeof(float) * (size_t)n_tok * k);
    for (int t = 0; t < n_tok; t++)
        for (int c = 0; c < k; c++) A[(size_t)t * k + c] = g_e4m3[xc[(size_t)t * k + c]] * xs[(size_t)t * na + c / act_block];
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        const uint8_t *wr = w + (size_t)r * k;
        const float *sr = ws + (size_t)(r / 128) * kb;
        /* tokens in groups of 64 (each token's sum is independent of the grouping) */
        for (int t0 = 0; t0 < n_tok; t0 += 64) {
        const int nt = n_tok - t0 < 64 ? n_tok - t0 : 64;
        float acc[64];
        for (int t = 0; t < nt; t++) acc[t] = 0.f;
        for (int c = 0; c < k; c++) {
            const float B = g_e4m3[wr[c]] * sr[c / 128];
            for (int t = 0; t < nt; t++) acc[t] = acc[t] + A[(size_t)(t0 + t) * k + c] * B;
        }
        for (int t = 0; t < nt; t++) y[(size_t)(t0 + t) * rows + r] = acc[t];
        }
    }
    free(A);
}

/* fp4_gemm (ref/kernel.py:94-102): B = table[nibble] * 2^(e8m0 - 127). */
void orc_gemv_mxfp4(const uint8_t *w, const uint8_t *ws, int rows, int k, const uint8_t *xc, const float *xs,
                    int act_block, int n_tok, float *y) {
    e4m3_init();
    const int na = k / act_block;
    float *A = (float *)malloc(sizeof(float) * (size_t)n_tok * k);
    for (int t = 0; t < n_tok; t++)
        for (int c = 0; c < k; c++) A[(size_t)t * k + c] = g_e4m3[xc[(size_t)t * k + c]] * xs[(size_t)t * na + c / act_block];
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        const uint8_t *wr = w + (size_t)r * (k / 2);
        const uint8_t *sr = ws + (size_t)r * (k / 32);
        /* tokens in groups of 64 (each token's sum is independent of the grouping) */
        for (int t0 = 0; t0 < n_tok; t0 += 64) {
        const int nt = n_tok - t0 < 64 ? n_tok - t0 : 64;
        float acc[64];
        for (int t = 0; t < nt; t++) acc[t] = 0.f;
        for (int c = 0; c < k; c++) {
            const uint8_t byte = wr[c / 2];
            const float B = kFp4[(c & 1) ? (byte >> 4) : (byte & 15)] * u2f((uint32_t)sr[c / 32] << 23);
            for (int t = 0; t < nt; t++) acc[t] = acc[t] + A[(size_t)(t0 + t) * k + c] * B;
        }
        for (int t = 0; t < nt; t++) y[(size_t)(t0 + t) * rows + r] = acc[t];
        }
    }
    free(A);
}

/* ---- router ----------------------------------------------------------------------------------- */

static void butterfly32(float *v) {
    float tmp[32];
    for (int o = 16; o > 0; o >>= 1) {
        for (int l = 0; l < 32; l++) tmp[l] = v[l] + v[l ^ o];
        memcpy(v, tmp, sizeof(tmp));
    }
}

int orc_router_ksplit(int H) { return (H % 512 == 0) ? 4 : 1; }

void orc_router_logits(const float *W, const uint16_t *x_bf16, int T, int E, int H, float *logits) {
    const int ks_n = orc_router_ksplit(H), slice = H / ks_n;
#pragma omp parallel for schedule(static)
    for (int e = 0; e < E; e++) {
        for (int t = 0; t < T; t++) {
            float total = 0.f;
            for (int ks = 0; ks < ks_n; ks++) {
                const float *w = W + (size_t)e * H + (size_t)ks * slice;
                const uint16_t *x = x_bf16 + (size_t)t * H + (size_t)ks * slice;
                float lane[32];
                for (int l = 0; l < 32; l++) {
                    float acc = 0.f;
                    for (int i = 0; i < slice / 128; i++)
                        for (int j = 0; j < 4; j++) {
                            const int c = 128 * i + 4 * l + j;
                            acc = fmaf(w[c], bf16_to_f32(x[c]), acc);
                        }
                    lane[l] = acc;
                }
                butterfly32(lane);
                total = ks == 0 ? lane[0] : total + lane[0];
            }
            logits[(size_t)t * E + e] = total;
        }
    }
}

/* Scores are evaluated in double and rounded once to fp32, so that the GPU and this CPU code agree
 * bit for bit (each library's double exp/log1p is within one double ulp).  sqrt-softplus keeps
 * torch's softplus threshold of 20 (kernels.cu:437-442). */
static float score_of(float logit, int fn) {
    if (fn == ORC_SCORE_SIGMOID) return (float)(1.0 / (1.0 + exp(-(double)logit)));
    const double sp = logit > 20.f ? (double)logit : log1p(exp((double)logit));
    return (float)sqrt(sp);
}

static inline int beats(float va, int a, float vb, int b) { return va > vb || (va == vb && a < b); }

int orc_router_select(const float *logits, const float *bias, int T, int E, int topk, int n_groups, int topk_groups,
                      int score_fn, float route_scale, float *scores, int *idx, float *weights) {
    if (n_groups < 1 || E % n_groups || topk > E || topk_groups > n_groups) return -1;
    const int gsz = E / n_groups;
    float *sc = (float *)malloc(sizeof(float) * E), *bs = (float *)malloc(sizeof(float) * E);
    float *gs = (float *)malloc(sizeof(float) * n_groups);
    char *keep = (char *)malloc(E), *gkeep = (char *)malloc(n_groups), *taken = (char *)malloc(E);
    for (int t = 0; t < T; t++) {
        for (int e = 0; e < E; e++) {
            sc[e] = score_of(logits[(size_t)t * E + e], score_fn);
            bs[e] = sc[e] + bias[e];
            if (scores) scores[(size_t)t * E + e] = sc[e];
        }
        /* group-limited selection (DeepSeek-V3 gate): group score = sum of its two best biased scores,
         * keep the topk_groups best groups (lower group id first on ties) */
        if (n_groups > 1 && topk_groups < n_groups) {
            for (int g = 0; g < n_groups; g++) {
                int b1 = -1, b2 = -1;
                for (int e = g * gsz; e < (g + 1) * gsz; e++) {
                    if (b1 < 0 || beats(bs[e], e, bs[b1], b1)) b2 = b1, b1 = e;
                    else if (b2 < 0 || beats(bs[e], e, bs[b2], b2)) b2 = e;
                }
                gs[g] = gsz > 1 ? bs[b1] + bs[b2] : bs[b1];
            }
            for (int g = 0; g < n_groups; g++) {
                int rank = 0;
                for (int h = 0; h < n_groups; h++) rank += beats(gs[h], h, gs[g], g);
                gkeep[g] = rank < topk_groups;
            }
            for (int e = 0; e < E; e++) keep[e] = gkeep[e / gsz];
        } else {
            memset(keep, 1, E);
        }
        /* top-k by biased score, descending, lower id first on ties (model.cu:444-449) */
        memset(taken, 0, E);
        for (int i = 0; i < topk; i++) {
            int best = -1;
            for (int e = 0; e < E; e++)
                if (keep[e] && !taken[e] && (best < 0 || beats(bs[e], e, bs[best], best))) best = e;
            taken[best] = 1;
            idx[(size_t)t * topk + i] = best;
        }
        /* unbiased weights, normalised in top-k order, then scaled (model.cu:450-451, 527-530) */
        float sum = 0.f;
        for (int i = 0; i < topk; i++) sum += sc[idx[(size_t)t * topk + i]];
        for (int i = 0; i < topk; i++) {
            float wt = sc[idx[(size_t)t * topk + i]];
            wt /= sum + 1e-20f;
            wt *= route_scale;
            weights[(size_t)t * topk + i] = wt;
        }
    }
    free(sc), free(bs), free(gs), free(keep), free(gkeep), free(taken);
    return 0;
}

void orc_dispatch(const int *idx, int T, int E, int topk, int *counts, int *offsets, int *perm) {
    memset(counts, 0, sizeof(int) * E);
    for (int a = 0; a < T * topk; a++) counts[idx[a]]++;
    offsets[0] = 0;
    for (int e = 0; e < E; e++) offsets[e + 1] = offsets[e] + counts[e];
    int *fill = (int *)calloc(E, sizeof(int));
    for (int t = 0; t < T; t++)
        for (int s = 0; s < topk; s++) {
            const int e = idx[t * topk + s];
            perm[offsets[e] + fill[e]++] = t * topk + s;
        }
    free(fill);
}

/* ---- whole layer ------------------------------------------------------------------------------ */

static int act_block_of(int fmt) { return fmt == ORC_FMT_FP8_B128 ? 128 : 32; }
static int act_pow2_of(int fmt) { return fmt == ORC_FMT_FP8_B128 ? 0 : 1; }

static void gemv_fmt(int fmt, const uint8_t *w, const void *s, int rows, int k, const uint8_t *xc, const float *xs,
                     int n_tok, float *y) {
    if (fmt == ORC_FMT_FP8_B128)
        orc_gemv_fp8_b128(w, (const float *)s, rows, k, xc, xs, act_block_of(fmt), n_tok, y);
    else if (fmt == ORC_FMT_FP8_E8M0)
        orc_gemv_fp8_e8m0(w, (const uint8_t *)s, rows, k, xc, xs, act_block_of(fmt), n_tok, y);
    else
        orc_gemv_mxfp4(w, (const uint8_t *)s, rows, k, xc, xs, act_block_of(fmt), n_tok, y);
}

/* One expert (routed or shared) on n_tok tokens: stbl/model.cu:516-547.
 * g, u = bf16(W1 xq), bf16(W3 xq); h = bf16(silu(g) * u * w) with the optional clamps
 * (kernels.cu:445-459); out = bf16(W2 act_quant(h)). */
static void expert_ffn(const orc_moe_desc *d, int fmt, const uint8_t *const w[3], const void *const s[3],
                       const float *xin, const float *wt, int n_tok, float *out) {
    const int H = d->hidden, I = d->inter, blk = act_block_of(fmt), p2 = act_pow2_of(fmt);
    uint8_t *xc = (uint8_t *)malloc((size_t)n_tok * (H > I ? H : I));
    float *xs = (float *)malloc(sizeof(float) * (size_t)n_tok * ((H > I ? H : I) / 32));
    float *g = (float *)malloc(sizeof(float) * (size_t)n_tok * I), *u = (float *)malloc(sizeof(float) * (size_t)n_tok * I);
    orc_act_quant(xin, n_tok, H, blk, p2, xc, xs);
    gemv_fmt(fmt, w[0], s[0], I, H, xc, xs, n_tok, g);
    gemv_fmt(fmt, w[1], s[1], I, H, xc, xs, n_tok, u);
    const float L = d->swiglu_limit;
    for (int t = 0; t < n_tok; t++)
        for (int j = 0; j < I; j++) {
            float gv = orc_bf16_round(g[(size_t)t * I + j]), uv = orc_bf16_round(u[(size_t)t * I + j]);
            if (L > 0) {
                uv = fminf(fmaxf(uv, -L), L);
                gv = fminf(gv, L);
            }
            g[(size_t)t * I + j] = orc_bf16_round(gv / (1.f + expf(-gv)) * uv * wt[t]);
        }
    orc_act_quant(g, n_tok, I, blk, p2, xc, xs);
    gemv_fmt(fmt, w[2], s[2], H, I, xc, xs, n_tok, out);
    for (size_t i = 0; i < (size_t)n_tok * H; i++) out[i] = orc_bf16_round(out[i]);
    free(xc), free(xs), free(g), free(u);
}

/* One routed MXFP4 expert with Q8 activations (ref/emulate_ds4.py:23-30, 69-77), composed as
 * expert_ffn: g, u = bf16(W1 q8(x)), bf16(W3 q8(x)); h = bf16(silu(g) * u * w) (clamps as above);
 * out = bf16(W2 q8(h)). */
static void expert_ffn_q8(const orc_moe_desc *d, const uint8_t *const w[3], const void *const s[3], const float *xin,
                          const float *wt, int n_tok, float *out) {
    const int H = d->hidden, I = d->inter, KM = H > I ? H : I;
    int8_t *q = (int8_t *)malloc((size_t)n_tok * KM);
    float *dq = (float *)malloc(sizeof(float) * (size_t)n_tok * (KM / 32));
    float *g = (float *)malloc(sizeof(float) * (size_t)n_tok * I), *u = (float *)malloc(sizeof(float) * (size_t)n_tok * I);
    orc_q8_codes(xin, n_tok * (H / 32), q, dq);
    orc_gemv_mxfp4_q8(w[0], (const uint8_t *)s[0], I, H, q, dq, n_tok, g);
    orc_gemv_mxfp4_q8(w[1], (const uint8_t *)s[1], I, H, q, dq, n_tok, u);
    const float L = d->swiglu_limit;
    for (int t = 0; t < n_tok; t++)
        for (int j = 0; j < I; j++) {
            float gv = orc_bf16_round(g[(size_t)t * I + j]), uv = orc_bf16_round(u[(size_t)t * I + j]);
            if (L > 0) {
                uv = fminf(fmaxf(uv, -L), L);
                gv = fminf(gv, L);
            }
            g[(size_t)t * I + j] = orc_bf16_round(gv / (1.f + expf(-gv)) * uv * wt[t]);
        }
    orc_q8_codes(g, n_tok * (I / 32), q, dq);
    orc_gemv_mxfp4_q8(w[2], (const uint8_t *)s[2], H, I, q, dq, n_tok, out);
    for (size_t i = 0; i < (size_t)n_tok * H; i++) out[i] = orc_bf16_round(out[i]);
    free(q), free(dq), free(g), free(u);
}

/* The layer with the routed experts given (forced routes): forced [T][topk], weights = unbiased
 * scores of the given experts normalised in the given order, times route_scale (the selection's
 * weight rule, model.cu:450-451, 527-530).  forced == NULL: the router selects. */
static int moe_forward_impl(const orc_moe_desc *d, const uint16_t *x, int T, const int *forced, uint16_t *y, int *idx_out,
                            float *w_out, int nthreads);

int orc_moe_forward(const orc_moe_desc *d, const uint16_t *x, int T, uint16_t *y, int *idx_out, float *w_out,
                    int nthreads) {
    return moe_forward_impl(d, x, T, NULL, y, idx_out, w_out, nthreads);
}

int orc_moe_forward_routed(const orc_moe_desc *d, const uint16_t *x, int T, const int *forced, uint16_t *y, int *idx_out,
                           float *w_out, int nthreads) {
    return moe_forward_impl(d, x, T, forced, y, idx_out, w_out, nthreads);
}

static int moe_forward_impl(const orc_moe_desc *d, const uint16_t *x, int T, const int *forced, uint16_t *y, int *idx_out,
                            float *w_out, int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
    const int H = d->hidden, E = d->n_experts, K = d->topk;
    float *logits = (float *)malloc(sizeof(float) * (size_t)T * E);
    int *idx = (int *)malloc(sizeof(int) * (size_t)T * K);
    float *wts = (float *)malloc(sizeof(float) * (size_t)T * K);
    orc_router_logits(d->router_w, x, T, E, H, logits);
    float *scores = (float *)malloc(sizeof(float) * (size_t)T * E);
    if (orc_router_select(logits, d->router_bias, T, E, K, d->n_groups, d->topk_groups, d->score_fn, d->route_scale,
                          scores, idx, wts)) {
        free(logits), free(idx), free(wts), free(scores);
        return -1;
    }
    if (forced) {
        for (int t = 0; t < T; t++) {
            float sum = 0.f;
            for (int i = 0; i < K; i++) {
                const int e = forced[t * K + i];
                if (e < 0 || e >= E) {
                    free(logits), free(idx), free(wts), free(scores);
                    return -1;
                }
                idx[t * K + i] = e;
                sum += scores[(size_t)t * E + e];
            }
            for (int i = 0; i < K; i++) {
                float wt = scores[(size_t)t * E + idx[t * K + i]];
                wt /= sum + 1e-20f;
                wt *= d->route_scale;
                wts[t * K + i] = wt;
            }
        }
    }
    free(scores);
    float *xf = (float *)malloc(sizeof(float) * (size_t)T * H);
    for (size_t i = 0; i < (size_t)T * H; i++) xf[i] = bf16_to_f32(x[i]);
    float *eo = (float *)calloc((size_t)T * K * H, sizeof(float));
    int rc = 0;
    /* routed experts: each distinct expert once, over its tokens in token order */
    float *xin = (float *)malloc(sizeof(float) * (size_t)T * H), *wt = (float *)malloc(sizeof(float) * T);
    float *out = (float *)malloc(sizeof(float) * (size_t)T * H);
    int *slot = (int *)malloc(sizeof(int) * T);
    for (int e = 0; e < E && !rc; e++) {
        int n = 0;
        for (int t = 0; t < T; t++)
            for (int s = 0; s < K; s++)
                if (idx[t * K + s] == e) {
                    memcpy(xin + (size_t)n * H, xf + (size_t)t * H, sizeof(float) * H);
                    wt[n] = wts[t * K + s];
                    slot[n++] = t * K + s;
                }
        if (!n) continue;
        const uint8_t *w[3];
        const void *sp[3];
        for (int m = 0; m < 3; m++) {
            w[m] = d->routed_w[m * E + e];
            sp[m] = d->routed_s[m * E + e];
            if (!w[m] || !sp[m]) rc = -1;
        }
        if (rc) break;
        if (d->act_q8 && d->routed_fmt == ORC_FMT_MXFP4)
            expert_ffn_q8(d, w, sp, xin, wt, n, out);
        else
            expert_ffn(d, d->routed_fmt, w, sp, xin, wt, n, out);
        for (int i = 0; i < n; i++) memcpy(eo + (size_t)slot[i] * H, out + (size_t)i * H, sizeof(float) * H);
    }
    float *sh = (float *)calloc((size_t)T * H, sizeof(float));
    if (!rc && d->shared_fmt != ORC_FMT_NONE) {
        for (int t = 0; t < T; t++) wt[t] = 1.f;
        expert_ffn(d, d->shared_fmt, d->shared_w, d->shared_s, xf, wt, T, sh);
    }
    /* combine: fp32 sum in top-k order, then the shared expert, then one bf16 rounding
     * (model.cu:589-592) */
    if (!rc)
        for (int t = 0; t < T; t++)
            for (int c = 0; c < H; c++) {
                float acc = 0.f;
                for (int s = 0; s < K; s++) acc = acc + eo[((size_t)t * K + s) * H + c];
                acc = acc + sh[(size_t)t * H + c];
                y[(size_t)t * H + c] = f32_to_bf16_bits(acc);
            }
    if (idx_out) memcpy(idx_out, idx, sizeof(int) * (size_t)T * K);
    if (w_out) memcpy(w_out, wts, sizeof(float) * (size_t)T * K);
    free(logits), free(idx), free(wts), free(xf), free(eo), free(xin), free(wt), free(out), free(slot), free(sh);
    return rc;
}

/* ---- the reference's kernels, exact orders (stbl/kernels.cu) ---------------------------------- */

/* :56-63 per 32 values: s = pow2_ceil(max(amax, 1e-4) / 448), x = bf16(e4m3(clamp(x / s)) * s) */
void orc_ref_act_quant_fp8(float *x, int n) {
    for (int b = 0; b < n / 32; b++) {
        float amax = 0.f;
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[b * 32 + i]));
        amax = fmaxf(amax, 1e-4f);
        const float s = orc_pow2_ceil(amax * (1.0f / 448.0f));
        for (int i = 0; i < 32; i++) {
            const float q = fminf(fmaxf(x[b * 32 + i] / s, -448.f), 448.f);
            x[b * 32 + i] = orc_bf16_round(orc_e4m3_value(orc_e4m3_encode(q)) * s);
        }
    }
}

void orc_ref_round_bf16(float *x, int n) {
    for (int i = 0; i < n; i++) x[i] = orc_bf16_round(x[i]);
}

static float tree32(float *p) {
    for (int o = 16; o > 0; o >>= 1)
        for (int i = 0; i < o; i++) p[i] = p[i] + p[i + o];
    return p[0];
}

/* :98-132: per 32-block the products x * e4m3(w) summed by the halving tree, times the block's
 * E8M0 scale (exact), block sums added in block order. */
void orc_ref_gemv_fp8(float *y, const uint8_t *w, const uint8_t *scale, const float *x, int rows, int k, int round_out) {
    e4m3_init();
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        const uint8_t *wr = w + (size_t)r * k;
        const uint8_t *sr = scale + (size_t)(r / 32) * (k / 32);
        float acc = 0.f;
        for (int kb = 0; kb < k / 32; kb++) {
            float p[32];
            for (int i = 0; i < 32; i++) p[i] = x[kb * 32 + i] * g_e4m3[wr[kb * 32 + i]];
            const float bs = tree32(p) * u2f((uint32_t)sr[kb] << 23);
            acc = acc + bs;
        }
        y[r] = round_out ? orc_bf16_round(acc) : acc;
    }
}

/* :142-191: GGUF MXFP4 blocks of 17 bytes (E8M0 scale, then values 0..15 in the low nibbles and
 * 16..31 in the high nibbles); same sum order as the FP8 GEMV; output rounded to bf16. */
void orc_ref_gemv_mxfp4(float *y, const uint8_t *w, const float *x, int rows, int k) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        const uint8_t *wr = w + (size_t)r * (k / 32) * 17;
        float acc = 0.f;
        for (int kb = 0; kb < k / 32; kb++) {
            const uint8_t *blk = wr + (size_t)kb * 17;
            float p[32];
            for (int i = 0; i < 16; i++) {
                p[i] = x[kb * 32 + i] * kFp4[blk[1 + i] & 15];
                p[16 + i] = x[kb * 32 + 16 + i] * kFp4[blk[1 + i] >> 4];
            }
            const float bs = tree32(p) * u2f((uint32_t)blk[0] << 23);
            acc = acc + bs;
        }
        y[r] = orc_bf16_round(acc);
    }
}

/* :206-214: lane l accumulates x[i] * w[i] for i = l, l + 32, ... by fused multiply-add, then the
 * xor butterfly of warp_sum (:15-18). */
void orc_ref_gemv_f32(float *y, const float *w, const float *x, int rows, int k, int round_out) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        float lane[32];
        for (int l = 0; l < 32; l++) {
            float acc = 0.f;
            for (int i = l; i < k; i += 32) acc = fmaf(x[i], w[(size_t)r * k + i], acc);
            lane[l] = acc;
        }
        butterfly32(lane);
        y[r] = round_out ? orc_bf16_round(lane[0]) : lane[0];
    }
}

void orc_ref_sqrt_softplus(float *s, int n) {
    for (int i = 0; i < n; i++) {
        const float x = s[i];
        s[i] = sqrtf(x > 20.f ? x : log1pf(expf(x)));
    }
}

void orc_ref_swiglu(float *out, const float *g, const float *u, const float *weights, int count, float limit, int n) {
    for (int j = 0; j < count; j++)
        for (int i = 0; i < n; i++) {
            float gv = g[(size_t)j * n + i], uv = u[(size_t)j * n + i];
            if (limit > 0) {
                uv = fminf(fmaxf(uv, -limit), limit);
                gv = fminf(gv, limit);
            }
            out[(size_t)j * n + i] = orc_bf16_round(gv / (1.f + expf(-gv)) * uv * weights[j]);
        }
}

void orc_ref_axpy(float *y, const float *x, float a, int n) {
    for (int i = 0; i < n; i++) y[i] = fmaf(a, x[i], y[i]);
}

/* k_rms_norm with its 256-thread launch (stbl/kernels.cu:217-236, 594-596), per row: the sum of squares
 * in the kernel's order (thread i: x[i], x[i + 256], ... by fused multiply-add; each warp's 32 sums by
 * the xor butterfly, lane 0's result; the 8 warp sums by the same butterfly), then
 * out = bf16(w * (x * r)).  r: the kernel calls CUDA's rsqrtf; here 1/sqrt correctly rounded from
 * double, which can differ from rsqrtf in the last bit of r (the GPU kernels are checked against the
 * reference kernel itself, bit for bit). */
static float warp_sum_xor32(const float *v32) {
    float v[32];
    for (int l = 0; l < 32; l++) v[l] = v32[l];
    for (int o = 16; o > 0; o >>= 1) {
        float n[32];
        for (int l = 0; l < 32; l++) n[l] = v[l] + v[l ^ o];
        for (int l = 0; l < 32; l++) v[l] = n[l];
    }
    return v[0];
}

void orc_ref_rms_norm(float *out, const float *x, const float *w, int rows, int dim, float eps) {
    for (int r = 0; r < rows; r++) {
        const float *xr = x + (size_t)r * dim;
        float part[32] = {0};
        for (int wp = 0; wp < 8; wp++) {
            float lanes[32];
            for (int l = 0; l < 32; l++) {
                float s = 0.f;
                for (int i = 32 * wp + l; i < dim; i += 256) s = fmaf(xr[i], xr[i], s);
                lanes[l] = s;
            }
            part[wp] = warp_sum_xor32(lanes);
        }
        const float total = warp_sum_xor32(part);
        const float rr = (float)(1.0 / sqrt((double)(total / (float)dim + eps)));
        for (int i = 0; i < dim; i++) out[(size_t)r * dim + i] = orc_bf16_round(w[i] * (xr[i] * rr));
    }
}

/* k_hc_post (stbl/kernels.cu:328-338): out[j][d] = bf16(post[j] * x[d] + sum_a comb[a][j] * res[a][d]),
 * each product and sum rounded in a's order (exact restatement). */
void orc_ref_hc_post(float *out, const float *x, const float *res, const float *post, const float *comb, int hc, int dim) {
    for (int j = 0; j < hc; j++)
        for (int d = 0; d < dim; d++) {
            float s = 0.f;
            for (int a = 0; a < hc; a++) s = s + comb[a * hc + j] * res[(size_t)a * dim + d];
            out[(size_t)j * dim + d] = orc_bf16_round(post[j] * x[d] + s);
        }
}

/* ---- Q8 activation variant ---------------------------------------------------------------------- */

void orc_q8_codes(const float *x, int n_blocks, int8_t *q, float *d) {
    for (int b = 0; b < n_blocks; b++) {
        const float *xb = x + (size_t)b * 32;
        float amax = 0.f;
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(xb[i]));
        const float db = amax / 127.0f;
        const float div = db > 0.f ? db : 1.0f;
        for (int i = 0; i < 32; i++) {
            float v = nearbyintf(xb[i] / div); /* round half to even (default rounding mode) */
            v = fminf(fmaxf(v, -128.f), 127.f);
            q[(size_t)b * 32 + i] = (int8_t)v;
        }
        d[b] = db;
    }
}

void orc_gemv_mxfp4_q8(const uint8_t *w, const uint8_t *ws, int rows, int k, const int8_t *q, const float *d, int n_tok,
                       float *y) {
    const int nb = k / 32;
    for (int t = 0; t < n_tok; t++)
#pragma omp parallel for schedule(static)
        for (int r = 0; r < rows; r++) {
            double acc = 0.0;
            for (int b = 0; b < nb; b++) {
                /* twice the e2m1 values are integers: the block's sum is exact in integers */
                long long s = 0;
                for (int i = 0; i < 32; i++) {
                    const uint8_t byte = w[(size_t)r * (k / 2) + b * 16 + i / 2];
                    const int nib = (i & 1) ? byte >> 4 : byte & 15;
                    s += (long long)q[(size_t)t * k + b * 32 + i] * (long long)(2.0f * kFp4[nib]);
                }
                acc += (double)s * 0.5 * (double)d[(size_t)t * nb + b] * ldexp(1.0, (int)ws[(size_t)r * nb + b] - 127);
            }
            y[(size_t)t * rows + r] = (float)acc;
        }
}
