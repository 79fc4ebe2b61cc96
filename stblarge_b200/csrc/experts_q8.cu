// Routed MXFP4 expert products with Q8 activations on the CUDA cores (the layer's act_q8 mode).
//
// The reference's ds4 numerics (ref/emulate_ds4.py:23-30, 69-77) feed the MXFP4 experts int8
// activations, quantized per 32 values with an fp32 scale d = amax / 127, instead of FP8.  There is
// no tensor-core form of that product: the block-scaled MMA kinds take e8m0 / ue4m3 scale factors,
// not an fp32 d per activation block, and kind::i8 has no per-block scaling (it would need one
// accumulator per 32-wide K block).  But twice every e2m1 value is an integer in [-12, 12], so a
// block's dot product is exact in integers:
//   y[t][r] = sum_b (d[t][b] * 2^(s[r][b] - 127) / 2) * sum_i q[t][b][i] * (2 w[r][b][i])
// Per 32-value block a lane loads the block's 16 code bytes with one 128-bit load, turns the nibbles
// into byte vectors with byte permutes (prmt against an 8-entry table of the magnitudes 2|w|; the
// nibble's sign bit, used as prmt's sign-replicate flag, zeroes the negative values in one vector
// and the positive ones in the other) and adds the block with dp4a: positive part minus negative
// part.  The block sum (|sum| < 2^16) is converted once and scaled in fp32.
//
// Work item: (chunk of <= 8 tokens of one expert, 32 output rows).  A CTA of 8 warps takes an item;
// warp w the output rows 4w .. 4w + 3 of its 32, lane l the K blocks l, l + 32, ...  Up: each output
// row reads its gate row and its up row, then h = bf16(silu(bf16 g) * bf16 u * w) (the reference's
// SwiGLU with the routing weight folded in, stbl/kernels.cu:445-459), and the CTA quantizes its 32
// h values per token to Q8 for the down product (one block: warp j takes token j).  Down: 4 output
// rows are read together (K = inter is short), outputs bf16 into the assignment's eo row.  Weights
// are read once per item; the tokens' codes come through L1.  Persistent grid, items taken in
// order by CTA (grid stride).
#include "../../include/stbl_moe.h"
#include "layer.cuh"
#include "tc_params.cuh"

namespace stbl {

constexpr int kQ8Threads = 256;  // 8 warps
constexpr int kQ8Tok = kQ8ChunkTokens;  // tokens per chunk (the router cuts routed chunks of this size)
constexpr int kQ8RowsPerWarp = 4;


__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// 2|e2m1| for magnitude codes 0..7: 0, 1, 2, 3, 4, 6, 8, 12 (bytes 0..3 and 4..7 of the table)
constexpr uint32_t kMagLo = 0x03020100u, kMagHi = 0x0C080604u;

// sum_i q_i * 2 w_i over one 32-value block: wv = 16 code bytes (value 2j in the low nibble of byte
// j), qa / qb = the 32 int8 codes
__device__ __forceinline__ int block_dot(const uint4 &wv, const uint4 &qa, const uint4 &qb) {
    const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
    const uint32_t qd[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    int pos = 0, neg = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        // word i holds values 8i .. 8i + 7 as nibbles 0..7; prmt reads the low 4 nibbles as selectors
        const uint32_t n = wd[i] ^ 0x88888888u;
        pos = __dp4a((int)prmt(kMagLo, kMagHi, wd[i]), (int)qd[2 * i], pos);
        pos = __dp4a((int)prmt(kMagLo, kMagHi, wd[i] >> 16), (int)qd[2 * i + 1], pos);
        neg = __dp4a((int)prmt(kMagLo, kMagHi, n), (int)qd[2 * i], neg);
        neg = __dp4a((int)prmt(kMagLo, kMagHi, n >> 16), (int)qd[2 * i + 1], neg);
    }
    return pos - neg;
}

__device__ __forceinline__ float e8m0_half(uint8_t s) {
    // 2^(s - 127) / 2 (the factor 1/2 undoes the doubled e2m1 values)
    return __uint_as_float((uint32_t)s << 23) * 0.5f;
}

// Signed bytes 2 w of one code word (8 values as nibbles 0..7, sign in each nibble's bit 3): lo gets
// values 0..3, hi values 4..7.  Two table lookups per half (magnitude and negated magnitude, prmt on
// the nibble's three index bits) and a third prmt picking between them by the sign bit.
__device__ __forceinline__ void expand_word(uint32_t wd, uint32_t &lo, uint32_t &hi) {
    constexpr uint32_t kNegLo = 0xFDFEFF00u, kNegHi = 0xF4F8FAFCu;  // 0, -1, -2, -3 | -4, -6, -8, -12
    const uint32_t idx = wd & 0x77777777u, sgn = wd & 0x88888888u;
    lo = prmt(prmt(kMagLo, kMagHi, idx), prmt(kNegLo, kNegHi, idx), (sgn >> 1) | 0x3210u);
    hi = prmt(prmt(kMagLo, kMagHi, idx >> 16), prmt(kNegLo, kNegHi, idx >> 16), (sgn >> 17) | 0x3210u);
}

// R weight rows (wr[j], their e8m0 scales sr[j]) against the chunk's n tokens: lane l takes the K
// blocks l + 32 i.  Per block each row's 16 code bytes become 32 signed bytes once; each token's 32
// codes are loaded once and meet all R rows (8 dp4a per row).  The next block's weights are loaded
// while this one is computed.  acc[j][t]: row j's lane partial for token t (reduced by the caller).
template <int NBL, int R>
__device__ __forceinline__ void q8_rows(const uint8_t *const (&wr)[R], const uint8_t *const (&sr)[R], int K, int nb, int n,
                                        const int *xrow, const Q8Params &p, int lane, float (&acc)[R][kQ8Tok]) {
#pragma unroll
    for (int j = 0; j < R; j++)
#pragma unroll
        for (int t = 0; t < kQ8Tok; t++) acc[j][t] = 0.f;
    uint4 wv[R];
    float sc[R];
    auto load = [&](int b) {
#pragma unroll
        for (int j = 0; j < R; j++) {
            wv[j] = __ldg(reinterpret_cast<const uint4 *>(wr[j] + (size_t)b * 16));
            sc[j] = e8m0_half(__ldg(sr[j] + b));
        }
    };
    if (lane < nb) load(lane);
#pragma unroll 1
    for (int i = 0; i < NBL; i++) {
        const int b = lane + 32 * i;
        if (b >= nb) break;  // a lane's blocks run out at its own count (nb need not be a multiple of 32)
        uint32_t sv[R][8];
        float s[R];
#pragma unroll
        for (int j = 0; j < R; j++) {
            const uint32_t wd[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
#pragma unroll
            for (int k = 0; k < 4; k++) expand_word(wd[k], sv[j][2 * k], sv[j][2 * k + 1]);
            s[j] = sc[j];
        }
        if (b + 32 < nb) load(b + 32);
#pragma unroll
        for (int t = 0; t < kQ8Tok; t++) {
            if (t >= n) break;
            const int8_t *xr = p.xq + (size_t)xrow[t] * K + (size_t)b * 32;
            const uint4 qa = __ldg(reinterpret_cast<const uint4 *>(xr));
            const uint4 qb = __ldg(reinterpret_cast<const uint4 *>(xr + 16));
            const float dx = __ldg(p.xd + (size_t)xrow[t] * p.xd_stride + b);
            const uint32_t qd[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
            for (int j = 0; j < R; j++) {
                int dot = 0;
#pragma unroll
                for (int k = 0; k < 8; k++) dot = __dp4a((int)sv[j][k], (int)qd[k], dot);
                acc[j][t] = fmaf((float)dot, s[j] * dx, acc[j][t]);
            }
        }
    }
}

template <bool UP, int NBL, int R>
__global__ void __launch_bounds__(kQ8Threads, 2) expert_q8_kernel(Q8Params p) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ float hs[kQ8Tok][32];
    __shared__ int xrow[kQ8Tok], dst[kQ8Tok];
    __shared__ float wt[kQ8Tok];
    const int K = UP ? p.H : p.I, rows_out = UP ? p.I : p.H, nb = K / 32, tiles = rows_out / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c0 = __ldg(p.n_chunks + 1), c1 = __ldg(p.n_chunks);
    const int n_items = max(0, c1 - c0) * tiles;
    const int n_routed = p.T * p.topk;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
        const int c = c0 + it / tiles, tile = it % tiles;
        const Chunk ch = p.chunks[c];
        if (ch.e < 0 || ch.e >= p.E || ch.n < 1 || ch.n > kQ8Tok || ch.pos0 < 0 || ch.pos0 + ch.n > n_routed) {
            if (threadIdx.x == 0) atomicOr(p.status, kErrBadTable);
            continue;
        }
        const int z = p.slot ? __ldg(p.slot + ch.e) : ch.e;
        // the chunk's columns: activation row (up: token, down: position), routing weight, output row
        if (threadIdx.x < kQ8Tok) {
            const int t = threadIdx.x;
            const int pos = ch.pos0 + min(t, ch.n - 1);
            const int a = __ldg(p.perm + pos);
            xrow[t] = UP ? a / p.topk : pos;
            wt[t] = UP ? __ldg(p.wts + a) : 1.f;
            dst[t] = UP ? pos : a;
        }
        __syncthreads();
        const int r0 = tile * 32 + warp * kQ8RowsPerWarp;
        if (UP) {
            // two output rows at a time: their gate rows and their up rows, then SwiGLU
#pragma unroll 1
            for (int j0 = 0; j0 < kQ8RowsPerWarp; j0 += 2) {
                const int r = r0 + j0;
                const uint8_t *g0 = p.w[0] + (size_t)z * p.w_stride[0] + (size_t)r * (K / 2);
                const uint8_t *u0 = p.w[1] + (size_t)z * p.w_stride[1] + (size_t)r * (K / 2);
                const uint8_t *gs = p.s[0] + (size_t)z * p.s_stride[0] + (size_t)r * nb;
                const uint8_t *us = p.s[1] + (size_t)z * p.s_stride[1] + (size_t)r * nb;
                const uint8_t *const wr[4] = {g0, u0, g0 + K / 2, u0 + K / 2};
                const uint8_t *const sr[4] = {gs, us, gs + nb, us + nb};
                float acc[4][kQ8Tok];
                q8_rows<NBL, 4>(wr, sr, K, nb, ch.n, xrow, p, lane, acc);
#pragma unroll
                for (int jj = 0; jj < 2; jj++)
#pragma unroll
                    for (int t = 0; t < kQ8Tok; t++) {
                        if (t >= ch.n) break;
                        float gv = bf16r(warp_sum(acc[2 * jj][t])), uv = bf16r(warp_sum(acc[2 * jj + 1][t]));
                        if (p.swiglu_limit > 0.f) {
                            gv = fminf(gv, p.swiglu_limit);
                            uv = fminf(fmaxf(uv, -p.swiglu_limit), p.swiglu_limit);
                        }
                        const float hv = bf16r(gv / (1.f + expf(-gv)) * uv * wt[t]);
                        if (lane == 0) {
                            hs[t][warp * kQ8RowsPerWarp + j0 + jj] = hv;
                            p.h[(size_t)dst[t] * p.I + r + jj] = f32_to_bf16_bits(hv);
                        }
                    }
            }
            __syncthreads();
            // Q8 of h for the down product: the 32 rows of this item are one block; warp t: token t
            if (warp < ch.n) {
                const float v = hs[warp][lane];
                float amax = fabsf(v);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                const float d = amax / 127.0f;
                const float div = d > 0.f ? d : 1.0f;
                const int q = (int)fminf(fmaxf(rintf(v / div), -128.f), 127.f);
                p.hq[(size_t)dst[warp] * p.I + tile * 32 + lane] = (int8_t)q;
                if (lane == 0) p.hd[(size_t)dst[warp] * (p.I / 32) + tile] = d;
            }
            __syncthreads();
        } else {
#pragma unroll 1
            for (int j0 = 0; j0 < kQ8RowsPerWarp; j0 += R) {
                const int r = r0 + j0;
                const uint8_t *w0 = p.w[0] + (size_t)z * p.w_stride[0] + (size_t)r * (K / 2);
                const uint8_t *s0 = p.s[0] + (size_t)z * p.s_stride[0] + (size_t)r * nb;
                uint8_t const *wr[R], *sr[R];
#pragma unroll
                for (int j = 0; j < R; j++) wr[j] = w0 + (size_t)j * (K / 2), sr[j] = s0 + (size_t)j * nb;
                float acc[R][kQ8Tok];
                q8_rows<NBL, R>(wr, sr, K, nb, ch.n, xrow, p, lane, acc);
#pragma unroll
                for (int j = 0; j < R; j++) {
                    // lane t stores token t's output of row r + j
                    float mine = 0.f;
                    int mdst = 0;
#pragma unroll
                    for (int t = 0; t < kQ8Tok; t++) {
                        if (t >= ch.n) break;
                        const float v = warp_sum(acc[j][t]);
                        if (lane == t) mine = v, mdst = dst[t];
                    }
                    if (lane < ch.n) p.eo[(size_t)mdst * p.H + r + j] = f32_to_bf16_bits(mine);
                }
            }
            __syncthreads();  // the next item rewrites the column table
        }
    }
}

template __global__ void expert_q8_kernel<true, 8, 4>(Q8Params);
template __global__ void expert_q8_kernel<false, 4, 4>(Q8Params);

}  // namespace stbl

namespace stbl {

// The two launches of the Q8 routed products (chunks [n_chunks[1], n_chunks[0]) of the router's
// table, chunks of <= 8 tokens): grid of two CTAs per SM, programmatic dependent launch.
cudaError_t launch_q8(bool up, const Q8Params &p, int sms, cudaStream_t st) {
    // blocks per lane: up K = hidden <= 8192 (8 x 32 blocks), down K = inter <= 4096 (4 x 32 blocks)
    const void *fn;
    if (up) {
        if (p.H > 32 * 32 * 8 || p.H % 32) return cudaErrorInvalidValue;
        fn = (const void *)expert_q8_kernel<true, 8, 4>;
    } else {
        if (p.I > 32 * 32 * 4 || p.I % 32) return cudaErrorInvalidValue;
        fn = (const void *)expert_q8_kernel<false, 4, 4>;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * sms);
    cfg.blockDim = dim3(kQ8Threads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q8Params q = p;
    void *args[] = {&q};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace stbl

namespace stbl {

// The Q8 linear alone (stbl_gemv_mxfp4_q8): a warp per weight row, lane l the blocks l, l + 32, ...,
// tokens eight at a time; the same block products as the layer's kernels.
__global__ void __launch_bounds__(256) gemv_mxfp4_q8_kernel(float *y, const uint8_t *w, const uint8_t *ws, const int8_t *q,
                                                            const float *d, int rows, int k, int n_tok) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int nb = k / 32;
    for (int t0 = 0; t0 < n_tok; t0 += kQ8Tok) {
        float acc[kQ8Tok];
#pragma unroll
        for (int t = 0; t < kQ8Tok; t++) acc[t] = 0.f;
        for (int b = lane; b < nb; b += 32) {
            const uint4 wv = __ldg(reinterpret_cast<const uint4 *>(w + (size_t)row * (k / 2) + (size_t)b * 16));
            const float sc = e8m0_half(__ldg(ws + (size_t)row * nb + b));
#pragma unroll
            for (int t = 0; t < kQ8Tok; t++) {
                if (t0 + t >= n_tok) break;
                const int8_t *xr = q + (size_t)(t0 + t) * k + (size_t)b * 32;
                const uint4 qa = __ldg(reinterpret_cast<const uint4 *>(xr));
                const uint4 qb = __ldg(reinterpret_cast<const uint4 *>(xr + 16));
                acc[t] = fmaf((float)block_dot(wv, qa, qb), sc * __ldg(d + (size_t)(t0 + t) * nb + b), acc[t]);
            }
        }
#pragma unroll
        for (int t = 0; t < kQ8Tok; t++) {
            const float v = warp_sum(acc[t]);
            if (lane == 0 && t0 + t < n_tok) y[(size_t)(t0 + t) * rows + row] = v;
        }
    }
}

}  // namespace stbl

extern "C" int stbl_gemv_mxfp4_q8(float *y, const void *w, const void *scales, const int8_t *q, const float *d, int rows, int k,
                                  int n_tok, cudaStream_t stream) {
    using namespace stbl;
    if (!y || !w || !scales || !q || !d || rows < 1 || n_tok < 1 || k < 32 || k % 32) return -1;
    if (((uintptr_t)w & 15) || ((uintptr_t)q & 15)) return -1;
    const int warps = 8;
    gemv_mxfp4_q8_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, stream>>>(
        y, static_cast<const uint8_t *>(w), static_cast<const uint8_t *>(scales), q, d, rows, k, n_tok);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
