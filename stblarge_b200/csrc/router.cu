// Router, top-k selection and bucketed dispatch of the MoE layer: one launch.
//
// Phase A (every CTA): router logits of a few experts (one warp per hidden slice, the slices combined
// in slice order in shared memory) and their scores, for all tokens at once; FP8 activation
// quantization of x for the expert kernels.  Phase B (the last CTA to finish phase A, by an atomic
// ticket): group-limited top-k, routing weights, and the bucketed permutation + chunk table.
//
// Replaces the reference's router GEMV, score kernel, blocking device->host copy and host
// partial_sort (stbl/model.cu:430-452, stbl/kernels.cu:206-214, 437-442): nothing leaves the GPU.
#include <limits.h>

#include "layer.cuh"

namespace stbl {

// ---- phase B helpers ------------------------------------------------------------------------------

__device__ __forceinline__ float router_score(float logit, int fn) {
    // double evaluation, one rounding to fp32: bit-identical to the CPU oracle's
    if (fn == kScoreSigmoid) return (float)(1.0 / (1.0 + exp(-(double)logit)));
    const double sp = logit > 20.f ? (double)logit : log1p(exp((double)logit));
    return (float)sqrt(sp);
}

__device__ __forceinline__ bool beats(float va, int a, float vb, int b) { return va > vb || (va == vb && a < b); }

// ---- phase A --------------------------------------------------------------------------------------

// One warp computes the slice ks of expert e's logits for tokens t0 .. t0+nt-1: lane l takes hidden
// positions base + 128 i + 4 l + j (i ascending, j = 0..3) by fused multiply-add, then the 32 lane
// sums are added by an xor butterfly.  oracle/moe_oracle.c restates exactly this order, so the logits
// agree bit for bit.  The weight loads of a slice are issued before any use (7 per lane in flight).
__device__ __forceinline__ void logits_slice(const RouterParams &p, int e, int ks, int t0, int nt, int lane,
                                             float *out /* [8] per token, lane 0 */) {
    const int slice = p.H / p.ksplit;
    const float *w = p.W + (size_t)e * p.H + (size_t)ks * slice;
    const uint16_t *x = p.x + (size_t)ks * slice;
    float acc[8];
#pragma unroll
    for (int t = 0; t < 8; t++) acc[t] = 0.f;
    const int n_it = slice / 128;
    for (int i0 = 0; i0 < n_it; i0 += 7) {
        float4 w4[7];
#pragma unroll
        for (int u = 0; u < 7; u++)
            if (i0 + u < n_it) w4[u] = __ldg(reinterpret_cast<const float4 *>(w + 128 * (i0 + u) + 4 * lane));
#pragma unroll
        for (int u = 0; u < 7; u++) {
            if (i0 + u < n_it) {
                const int k = 128 * (i0 + u) + 4 * lane;
#pragma unroll
                for (int t = 0; t < 8; t++) {
                    if (t < nt) {
                        const uint2 xv = __ldg(reinterpret_cast<const uint2 *>(x + (size_t)(t0 + t) * p.H + k));
                        acc[t] = fmaf(w4[u].x, __uint_as_float(xv.x << 16), acc[t]);
                        acc[t] = fmaf(w4[u].y, __uint_as_float(xv.x & 0xffff0000u), acc[t]);
                        acc[t] = fmaf(w4[u].z, __uint_as_float(xv.y << 16), acc[t]);
                        acc[t] = fmaf(w4[u].w, __uint_as_float(xv.y & 0xffff0000u), acc[t]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < 8; t++) {
        float v = acc[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = v + __shfl_xor_sync(0xffffffffu, v, o);
        out[t] = v;
    }
}

// act_quant (ref/kernel.py:35-45) of 128 consecutive values of one token: lane l takes 4 of them.
// blk 128: fp32 scale amax/448; blk 32: power-of-two scale per 32 (pow2 selects the rounding).
__device__ void quant_group(const uint16_t *x, int H, int t, int g, uint8_t *xq, float *xs, int blk, int pow2, int lane) {
    const int k = 128 * g + 4 * lane;
    const uint2 xv = __ldg(reinterpret_cast<const uint2 *>(x + (size_t)t * H + k));
    const float v[4] = {__uint_as_float(xv.x << 16), __uint_as_float(xv.x & 0xffff0000u), __uint_as_float(xv.y << 16),
                        __uint_as_float(xv.y & 0xffff0000u)};
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    for (int o = blk / 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    amax = fmaxf(amax, 1e-4f);
    const float tq = amax * (1.0f / 448.0f);
    const float s = pow2 ? pow2_ceil(tq) : tq;
    uint32_t codes = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float q = fminf(fmaxf(v[j] / s, -448.f), 448.f);
        codes |= (uint32_t)e4m3_code(q) << (8 * j);
    }
    *reinterpret_cast<uint32_t *>(xq + (size_t)t * H + k) = codes;
    if ((k % blk) == 0) xs[(size_t)t * (H / 32) + k / blk] = s;
}

// exclusive scan over n <= 2 * kRouterThreads values in smem (in place); returns the total
__device__ int block_exclusive_scan(int *v, int n, int *warp_tot) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int a = 2 * tid < n ? v[2 * tid] : 0, b = 2 * tid + 1 < n ? v[2 * tid + 1] : 0;
    int incl = a + b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = lane < kRouterThreads / 32 ? warp_tot[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < kRouterThreads / 32) warp_tot[lane] = w;  // inclusive per warp
    }
    __syncthreads();
    const int base = (warp ? warp_tot[warp - 1] : 0) + incl - (a + b);
    const int total = warp_tot[kRouterThreads / 32 - 1];
    __syncthreads();
    if (2 * tid < n) v[2 * tid] = base;
    if (2 * tid + 1 < n) v[2 * tid + 1] = base + a;
    __syncthreads();
    return total;
}

// ---- the kernel -----------------------------------------------------------------------------------

__global__ void __launch_bounds__(kRouterThreads) router_kernel(RouterParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps_grid = gridDim.x * (kRouterThreads / 32);
    const int gwarp = blockIdx.x * (kRouterThreads / 32) + warp;

    pdl_wait();  // x may come from the kernel before this one
    pdl_launch_dependents();

    // phase A: logits of experts_per_cta experts (ksplit warps each, slices combined in slice order
    // through shared memory), their scores, activation quantization of x
    __shared__ float part[kRouterThreads / 32][8];
    const int epc = (kRouterThreads / 32) / p.ksplit;  // experts per CTA
    const int e_loc = warp / p.ksplit, ks = warp % p.ksplit;
    const int e = blockIdx.x * epc + e_loc;
    for (int t0 = 0; t0 < p.T; t0 += 8) {
        const int nt = min(8, p.T - t0);
        float o[8];
        if (e < p.E) logits_slice(p, e, ks, t0, nt, lane, o);
        if (lane == 0 && e < p.E)
#pragma unroll
            for (int t = 0; t < 8; t++) part[warp][t] = o[t];
        __syncthreads();
        if (tid < epc * nt) {
            const int el = tid / nt, t = tid % nt, ee = blockIdx.x * epc + el;
            if (ee < p.E) {
                float logit = part[el * p.ksplit][t];
                for (int k2 = 1; k2 < p.ksplit; k2++) logit = logit + part[el * p.ksplit + k2][t];
                p.scores[(size_t)(t0 + t) * p.E + ee] = router_score(logit, p.score_fn);
            }
        }
        __syncthreads();
    }
    const int groups = p.T * (p.H / 128);
    for (int u = gwarp; u < groups; u += nwarps_grid) {
        quant_group(p.x, p.H, u / (p.H / 128), u % (p.H / 128), p.xq_a, p.xs_a, p.blk_a, p.pow2_a, lane);
        if (p.xq_b != p.xq_a)
            quant_group(p.x, p.H, u / (p.H / 128), u % (p.H / 128), p.xq_b, p.xs_b, p.blk_b, p.pow2_b, lane);
    }

    // last-CTA ticket
    __shared__ int is_last;
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        is_last = atomicAdd(p.done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();

    // phase B
    const int E = p.E, T = p.T, K = p.topk;
    const int TW = (T + 31) / 32;
    float *sb = reinterpret_cast<float *>(smem);                    // [8][E] biased scores
    float *sc = sb + (kRouterThreads / 32) * E;                      // [8][E] scores
    int *sidx = reinterpret_cast<int *>(sc + (kRouterThreads / 32) * E);  // [T][K]
    int *cnt = sidx + T * K;                                         // [E]
    int *off = cnt + E;                                              // [E]
    int *nch = off + E;                                              // [E]
    int *choff = nch + E;                                            // [E]
    uint32_t *bm = reinterpret_cast<uint32_t *>(choff + E);          // [E][TW]
    __shared__ int warp_tot[kRouterThreads / 32];

    const int EJ = (E + 31) / 32;
    const int gsz = E / p.n_groups;
    const bool grouped = p.n_groups > 1 && p.topk_groups < p.n_groups;
    for (int t = warp; t < T; t += kRouterThreads / 32) {
        float *wb = sb + warp * E, *ws = sc + warp * E;
        float bv[kMaxExperts / 32];
        uint32_t has = 0;
#pragma unroll
        for (int j = 0; j < kMaxExperts / 32; j++) {
            const int e = lane + 32 * j;
            bv[j] = 0.f;
            if (j < EJ && e < E) {
                const float s = __ldcg(p.scores + (size_t)t * E + e);
                const float b = s + __ldg(p.bias + e);
                wb[e] = b;
                ws[e] = s;
                bv[j] = b;
                has |= 1u << j;
            }
        }
        __syncwarp();
        uint32_t keepg = 0xffffffffu;
        if (grouped) {
            float gs = 0.f;
            if (lane < p.n_groups) {
                int b1 = -1, b2 = -1;
                for (int e = lane * gsz; e < (lane + 1) * gsz; e++) {
                    if (b1 < 0 || beats(wb[e], e, wb[b1], b1)) b2 = b1, b1 = e;
                    else if (b2 < 0 || beats(wb[e], e, wb[b2], b2)) b2 = e;
                }
                gs = gsz > 1 ? wb[b1] + wb[b2] : wb[b1];
            }
            int rank = 0;
            for (int h = 0; h < p.n_groups; h++) {
                const float gh = __shfl_sync(0xffffffffu, gs, h);
                rank += beats(gh, h, gs, lane);
            }
            keepg = __ballot_sync(0xffffffffu, lane < p.n_groups && rank < p.topk_groups);
        }
        uint32_t avail = 0;
#pragma unroll
        for (int j = 0; j < kMaxExperts / 32; j++) {
            const int e = lane + 32 * j;
            if (((has >> j) & 1u) && ((keepg >> (e / gsz)) & 1u)) avail |= 1u << j;
        }
        int mine = -1;
        for (int i = 0; i < K; i++) {
            int bj = -1;
            float bvv = 0.f;
#pragma unroll
            for (int j = 0; j < kMaxExperts / 32; j++)
                if (((avail >> j) & 1u) && (bj < 0 || bv[j] > bvv)) bj = j, bvv = bv[j];
            const uint32_t key = bj >= 0 ? float_key(bvv + 0.0f) : 0u;
            const uint32_t mk = __reduce_max_sync(0xffffffffu, key);
            const int cand = (bj >= 0 && key == mk) ? lane + 32 * bj : INT_MAX;
            int win = __reduce_min_sync(0xffffffffu, cand);
            if (win == INT_MAX) {  // fewer candidates than topk: cannot happen for a validated layer
                if (lane == 0) atomicOr(p.status, kErrBadTable);
                win = 0;
            }
            if (lane == (win & 31)) avail &= ~(1u << (win >> 5));
            if (lane == i) mine = win;
        }
        // weights: unbiased scores normalised in top-k order (stbl/model.cu:450-451, 527-530)
        const float s_mine = (lane < K) ? ws[mine] : 0.f;
        float sum = 0.f;
        for (int i = 0; i < K; i++) sum += __shfl_sync(0xffffffffu, s_mine, i);
        if (lane < K) {
            float wt = s_mine;
            wt /= sum + 1e-20f;
            wt *= p.route_scale;
            p.idx[t * K + lane] = mine;
            p.wts[t * K + lane] = wt;
            sidx[t * K + lane] = mine;
        }
        __syncwarp();
    }
    __syncthreads();

    // bucketed dispatch: counts, offsets, stable rank by token through a per-expert token bitmap
    for (int e = tid; e < E; e += kRouterThreads) cnt[e] = 0;
    for (int i = tid; i < E * TW; i += kRouterThreads) bm[i] = 0;
    __syncthreads();
    for (int a = tid; a < T * K; a += kRouterThreads) {
        const int e = sidx[a], t = a / K;
        atomicAdd(&cnt[e], 1);
        atomicOr(&bm[e * TW + (t >> 5)], 1u << (t & 31));
    }
    __syncthreads();
    for (int e = tid; e < E; e += kRouterThreads) {
        off[e] = cnt[e];
        nch[e] = (cnt[e] + p.nt_routed - 1) / p.nt_routed;
        choff[e] = nch[e];
    }
    __syncthreads();
    block_exclusive_scan(off, E, warp_tot);
    const int routed_chunks = block_exclusive_scan(choff, E, warp_tot);
    for (int a = tid; a < T * K; a += kRouterThreads) {
        const int e = sidx[a], t = a / K;
        int rank = __popc(bm[e * TW + (t >> 5)] & ((1u << (t & 31)) - 1u));
        for (int w = 0; w < (t >> 5); w++) rank += __popc(bm[e * TW + w]);
        p.perm[off[e] + rank] = a;
    }
    const int ns = p.has_shared ? (T + p.nt_shared - 1) / p.nt_shared : 0;
    for (int i = tid; i < ns; i += kRouterThreads)
        p.chunks[i] = Chunk{E, T * K + i * p.nt_shared, min(p.nt_shared, T - i * p.nt_shared), 0};
    for (int e = tid; e < E; e += kRouterThreads) {
        p.counts[e] = cnt[e];
        p.offsets[e] = off[e];
        for (int c = 0; c < nch[e]; c++)
            p.chunks[ns + choff[e] + c] = Chunk{e, off[e] + c * p.nt_routed, min(p.nt_routed, cnt[e] - c * p.nt_routed), 0};
    }
    if (tid == 0) {
        p.offsets[E] = T * K;
        p.n_chunks[0] = ns + routed_chunks;
        p.n_chunks[1] = ns;
        *p.done = 0;
    }
}

}  // namespace stbl
