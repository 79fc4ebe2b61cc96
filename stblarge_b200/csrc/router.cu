// Router, top-k selection and bucketed dispatch of the MoE layer: two launches.
//
// router_logits_kernel (many CTAs, clusters of ksplit): router logits and scores.  A CTA owns 8
// experts and one hidden slice; it streams its 8 weight rows and the tokens' x slices into shared
// memory with bulk copies (the weight copies start before the programmatic-launch wait, since the
// router weights never change), computes the slice partials of 4 experts x 8 tokens per warp from
// registers, and the ksplit CTAs of a cluster add their partials in slice order through distributed
// shared memory.  It also does the activation quantization of x for the expert kernels.
// router_select_kernel (a CTA of 512 threads per 16 tokens): group-limited top-k per token (a warp
// per token), routing weights; the last CTA builds the bucketed permutation + chunk table.
//
// Replaces the reference's router GEMV, score kernel, blocking device->host copy and host
// partial_sort (stbl/model.cu:430-452, stbl/kernels.cu:206-214, 437-442): nothing leaves the GPU.
#include <cooperative_groups.h>
#include <limits.h>

#include "layer.cuh"

namespace cg = cooperative_groups;

namespace stbl {

// ---- selection helpers -----------------------------------------------------------------------------

__device__ __forceinline__ float router_score(float logit, int fn) {
    // double evaluation, one rounding to fp32: bit-identical to the CPU oracle's
    if (fn == kScoreSigmoid) return (float)(1.0 / (1.0 + exp(-(double)logit)));
    const double sp = logit > 20.f ? (double)logit : log1p(exp((double)logit));
    return (float)sqrt(sp);
}

__device__ __forceinline__ bool beats(float va, int a, float vb, int b) { return va > vb || (va == vb && a < b); }

__device__ __forceinline__ float key_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// merge two (first, second) key pairs of disjoint sets into the pair of their union
__device__ __forceinline__ void top2_merge(uint32_t &a1, uint32_t &a2, uint32_t b1, uint32_t b2) {
    const uint32_t lo = min(a1, b1);
    a1 = max(a1, b1);
    a2 = max(lo, max(a2, b2));
}

// ---- fused RMSNorm (RouterParams::x_pre) ---------------------------------------------------------------

// the reference's warp_sum (stbl/kernels.cu:15-18): xor butterfly, lane 0's sum is the one used
__device__ __forceinline__ float warp_sum_xor(float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// The normalized input value: bf16(w * (x * r)), the two products rounded as written (k_rms_norm's
// output, stbl/kernels.cu:235), returned as the float of the bf16.
__device__ __forceinline__ float rms_value(float x, float w, float r) { return bf16r(w * (x * r)); }

// r = rsqrt(mean(x^2) + eps) of one token row, by all 256 threads of the CTA in the order of the
// reference's k_rms_norm with 256 threads (stbl/kernels.cu:217-234, launched by stbl_rms_norm with 256
// threads, kernels.cu:594-596): thread i sums x[i], x[i + 256], ... in index order, each warp's 32
// sums are added by the xor butterfly, then the 8 warp sums by the same butterfly in warp 0.  The
// result goes to *out (thread 0).  red: 8 floats of shared memory.
__device__ void rms_rsqrt(const float *xr, int H, float eps, float *red, float *out) {
    static_assert(kLgThreads == 256, "the reduction order is the reference's 256-thread one");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float s = 0.f;
    for (int i = tid; i < H; i += kLgThreads) s += xr[i] * xr[i];
    s = warp_sum_xor(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (warp == 0) {
        float v = lane < kLgThreads / 32 ? red[lane] : 0.f;
        v = warp_sum_xor(v);
        if (lane == 0) *out = rsqrtf(v / H + eps);
    }
    __syncthreads();
}

// act_quant (ref/kernel.py:35-45) of 128 consecutive values of one token: lane l takes 4 of them.
// blk 128: fp32 scale amax/448; blk 32: power-of-two scale per 32 (pow2 selects the rounding);
// pow2 == kActQ8 (blk 32): the Q8 rule instead, int8 codes with an fp32 scale amax/127.
// xe8 (optional): the scales as e8m0 bytes (per-32 power-of-two rule), laid out as the MXFP4 experts'
// tensor-core kernel copies them: [H/128][xe8_rows][16 B], row t's bytes 0..3 for the 128-K block.
// With the fused RMSNorm (nrm non-null) the values are normalized from x_pre first (rms_value).
__device__ void quant_group(const uint16_t *x, int H, int t, int g, uint8_t *xq, float *xs, int blk, int pow2, int lane,
                            uint8_t *xe8, int xe8_rows, const RouterParams *nrm = nullptr, float r = 0.f) {
    const int k = 128 * g + 4 * lane;
    float v[4];
    if (nrm) {
        const float4 xv = __ldg(reinterpret_cast<const float4 *>(nrm->x_pre + (size_t)t * H + k));
        const float4 wv = __ldg(reinterpret_cast<const float4 *>(nrm->norm_w + k));
        v[0] = rms_value(xv.x, wv.x, r), v[1] = rms_value(xv.y, wv.y, r), v[2] = rms_value(xv.z, wv.z, r),
        v[3] = rms_value(xv.w, wv.w, r);
    } else {
        const uint2 xv = __ldg(reinterpret_cast<const uint2 *>(x + (size_t)t * H + k));
        v[0] = __uint_as_float(xv.x << 16), v[1] = __uint_as_float(xv.x & 0xffff0000u), v[2] = __uint_as_float(xv.y << 16),
        v[3] = __uint_as_float(xv.y & 0xffff0000u);
    }
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    for (int o = blk / 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (pow2 == kActQ8) {
        // Q8 (ref/emulate_ds4.py:23-30): int8 codes round-half-even(x / d), d = amax / 127 (no floor;
        // d = 0 divides by 1), clamped to [-128, 127]; d kept as fp32 per 32 values
        const float d = amax / 127.0f;
        const float div = d > 0.f ? d : 1.0f;
        uint32_t codes = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int q = (int)fminf(fmaxf(rintf(v[j] / div), -128.f), 127.f);
            codes |= ((uint32_t)q & 0xffu) << (8 * j);
        }
        *reinterpret_cast<uint32_t *>(xq + (size_t)t * H + k) = codes;
        if ((k % 32) == 0) xs[(size_t)t * (H / 32) + k / 32] = d;
        return;
    }
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
    if ((k % blk) == 0) {
        xs[(size_t)t * (H / 32) + k / blk] = s;
        if (xe8) xe8[((size_t)(k / 128) * xe8_rows + t) * 16 + (k / 32) % 4] = (uint8_t)(__float_as_uint(s) >> 23);
    }
}

// ---- logits kernel -----------------------------------------------------------------------------------

// Shared memory of router_logits_kernel: weight rows [8][slice] f32 | x rows [min(T, 32)][slice] bf16 |
// slice partials [8][T] f32 | two mbarriers.
__host__ __device__ inline size_t router_logits_smem(int H, int T) {
    const int slice = H / router_ksplit(H), xr = T < kLgRound ? T : kLgRound;
    return (size_t)kLgExperts * slice * 4 + (size_t)xr * slice * 2 + (size_t)kLgExperts * T * 4 + 16;
}

// Slice partials of EPW experts x up to NT tokens by one warp, in the order router_logits_kernel
// states: lane l accumulates the products at positions 128 i + 4 l + j (i ascending, j = 0..3) by
// fused multiply-add, then the lane sums of each (expert, token) are added by the xor-butterfly tree
// (a reduce-scatter adds the same pairs).  w: the first expert's row of the slice in shared memory
// (rows slice floats apart); x: the first token's row (slice bf16 apart); the sums go to
// part[e * T + t0 + t] for e < ne, t < nt.
template <int EPW, int NT>
__device__ __forceinline__ void logits_tile(const float *w, const uint16_t *x, int slice, int n_it, int nt, int ne,
                                            int lane, float *part, int T, int t0) {
    constexpr int V = EPW * NT;
    float acc[V];
#pragma unroll
    for (int v = 0; v < V; v++) acc[v] = 0.f;
    const float *wl = w + 4 * lane;
    const uint16_t *xl = x + 4 * lane;
    for (int i = 0; i < n_it; i++) {
        float4 w4[EPW];
#pragma unroll
        for (int e = 0; e < EPW; e++) w4[e] = *reinterpret_cast<const float4 *>(wl + (size_t)e * slice + 128 * i);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            if (t < nt) {
                const uint2 xv = *reinterpret_cast<const uint2 *>(xl + (size_t)t * slice + 128 * i);
                const float x0 = __uint_as_float(xv.x << 16), x1 = __uint_as_float(xv.x & 0xffff0000u);
                const float x2 = __uint_as_float(xv.y << 16), x3 = __uint_as_float(xv.y & 0xffff0000u);
#pragma unroll
                for (int e = 0; e < EPW; e++) {
                    float a = acc[e * NT + t];
                    a = fmaf(w4[e].x, x0, a);
                    a = fmaf(w4[e].y, x1, a);
                    a = fmaf(w4[e].z, x2, a);
                    a = fmaf(w4[e].w, x3, a);
                    acc[e * NT + t] = a;
                }
            }
        }
    }
    const float sum = warp_reduce_scatter<V>(acc, lane);  // lane l: value l / (32 / V)
    constexpr int LPV = 32 / V;
    const int v = lane / LPV, e = v / NT, t = v % NT;
    if (lane % LPV == 0 && t < nt && e < ne) part[e * T + t0 + t] = sum;
}

// Logits of experts e0 .. e0+7 over hidden slice ks (= the CTA's rank in its cluster of ksplit).
// The 8 warps split the (expert, staged token) pairs by the number of tokens (logits_tile); lane l
// of a warp accumulates, for each of its (expert, token) pairs, the products at hidden positions
// base + 128 i + 4 l + j (i ascending, j = 0..3) by fused multiply-add, and the 32 lane sums of a
// pair are added by the xor-butterfly tree.  The cluster's CTAs then add their slice sums in slice
// order.  oracle/moe_oracle.c restates exactly this order,
// so the logits agree bit for bit.
__global__ void __launch_bounds__(kLgThreads) router_logits_kernel(RouterParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int abort_flag;
    // fused RMSNorm: r of the tokens this CTA reduces (t = its cluster rank mod ksplit), then of all
    __shared__ float r_own[kRouterMaxTokens], r_all[kRouterMaxTokens], red[kLgThreads / 32];
    const bool fused = p.x_pre != nullptr;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    cg::cluster_group cluster = cg::this_cluster();
    const int ks = (int)cluster.block_rank();
    const int eb = blockIdx.x / p.ksplit;
    const int slice = p.H / p.ksplit, n_it = slice / 128;
    const int e0 = eb * kLgExperts, ne = min(kLgExperts, p.E - e0);
    const int xr = min(p.T, kLgRound);
    float *w_s = reinterpret_cast<float *>(smem);
    uint16_t *x_s = reinterpret_cast<uint16_t *>(w_s + kLgExperts * slice);
    float *part = reinterpret_cast<float *>(x_s + (size_t)xr * slice);  // [8][T]
    uint64_t *bar_w = reinterpret_cast<uint64_t *>(part + kLgExperts * p.T);
    uint64_t *bar_x = bar_w + 1;

    if (tid == 0) {
        abort_flag = 0;
        mbar_init(bar_w, 1);
        mbar_init(bar_x, 1);
        fence_barrier_init();
    }
    __syncthreads();
    // the router weights are never written by a kernel: stream them before the programmatic wait
    if (warp == 0) {
        if (lane == 0) mbar_arrive_expect_tx(bar_w, (uint32_t)(ne * slice * 4));
        __syncwarp();
        if (lane < ne) bulk_g2s(w_s + lane * slice, p.W + (size_t)(e0 + lane) * p.H + (size_t)ks * slice, slice * 4, bar_w);
    }
    pdl_wait();  // x may come from the kernel before this one
    if (fused) {
        // the cluster's CTAs split the tokens' norms and share them through distributed shared memory
        for (int t = ks; t < p.T; t += p.ksplit) rms_rsqrt(p.x_pre + (size_t)t * p.H, p.H, p.norm_eps, red, &r_own[t]);
        cluster.sync();
        for (int t = tid; t < p.T; t += kLgThreads) r_all[t] = cluster.map_shared_rank(r_own, t % p.ksplit)[t];
        __syncthreads();
    }
    auto stage_x = [&](int r0, int nr) {
        if (fused) {
            // normalized rows of the slice, written by the threads (the round's barrier publishes them)
            const int base = ks * slice, q4 = slice / 4;
            for (int i = tid; i < nr * q4; i += kLgThreads) {
                const int t = i / q4, k = base + 4 * (i % q4);
                const float4 xv = __ldg(reinterpret_cast<const float4 *>(p.x_pre + (size_t)(r0 + t) * p.H + k));
                const float4 wv = __ldg(reinterpret_cast<const float4 *>(p.norm_w + k));
                const float r = r_all[r0 + t];
                const uint32_t lo = (uint32_t)f32_to_bf16_bits(rms_value(xv.x, wv.x, r)) |
                                    ((uint32_t)f32_to_bf16_bits(rms_value(xv.y, wv.y, r)) << 16);
                const uint32_t hi = (uint32_t)f32_to_bf16_bits(rms_value(xv.z, wv.z, r)) |
                                    ((uint32_t)f32_to_bf16_bits(rms_value(xv.w, wv.w, r)) << 16);
                *reinterpret_cast<uint2 *>(x_s + (size_t)t * slice + (k - base)) = make_uint2(lo, hi);
            }
            return;
        }
        if (warp == 0) {
            if (lane == 0) mbar_arrive_expect_tx(bar_x, (uint32_t)(nr * slice * 2));
            __syncwarp();
            for (int t = lane; t < nr; t += 32)
                bulk_g2s(x_s + (size_t)t * slice, p.x + (size_t)(r0 + t) * p.H + (size_t)ks * slice, slice * 2, bar_x);
        }
    };
    stage_x(0, xr);
    pdl_launch_dependents();
    if (blockIdx.x == 0) {  // the select kernel's global counts, token bitmaps and ticket start at zero
        const int TW = (p.T + 31) / 32;
        for (int i = tid; i < p.E; i += kLgThreads) p.sel_cnt[i] = 0;
        for (int i = tid; i < p.E * TW; i += kLgThreads) p.sel_bm[i] = 0;
        if (tid == 0) *p.sel_ticket = 0;
    }

    // activation quantization of x for the expert kernels, spread over every warp of the grid (none
    // when the caller routes only: xq_a null)
    if (p.xq_a) {
        const int nwarps_grid = gridDim.x * (kLgThreads / 32), gwarp = blockIdx.x * (kLgThreads / 32) + warp;
        const int groups = p.T * (p.H / 128);
        for (int u = gwarp; u < groups; u += nwarps_grid) {
            const int t = u / (p.H / 128), g = u % (p.H / 128);
            const RouterParams *nrm = fused ? &p : nullptr;
            const float r = fused ? r_all[t] : 0.f;
            quant_group(p.x, p.H, t, g, p.xq_a, p.xs_a, p.blk_a, p.pow2_a, lane, p.xe8_a, p.xe8_rows, nrm, r);
            if (p.xq_b != p.xq_a) quant_group(p.x, p.H, t, g, p.xq_b, p.xs_b, p.blk_b, p.pow2_b, lane, nullptr, 0, nrm, r);
        }
    }

    bool ok = mbar_wait(bar_w, 0, &abort_flag);
    int last_round = 0;  // the last round whose rows were requested
    for (int r0 = 0, round = 0; r0 < p.T; r0 += kLgRound, round++) {
        const int nr = min(kLgRound, p.T - r0);
        if (round > 0) {
            __syncthreads();  // every warp is done with the previous round's rows
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            stage_x(r0, nr);
            last_round = round;
        }
        if (!fused) ok = mbar_wait(bar_x, round & 1, &abort_flag) && ok;
        ok = __syncthreads_and(ok ? 1 : 0) != 0;  // uniform: every warp stops if one gave up
        if (!ok) break;
        // work split of the round by its token count: (experts, tokens) per warp
        if (nr <= 4) {  // a warp per expert
            if (warp < ne) {
                if (nr <= 2) logits_tile<1, 2>(w_s + (size_t)warp * slice, x_s, slice, n_it, nr, ne - warp, lane, part + warp * p.T, p.T, r0);
                else logits_tile<1, 4>(w_s + (size_t)warp * slice, x_s, slice, n_it, nr, ne - warp, lane, part + warp * p.T, p.T, r0);
            }
        } else if (nr <= 8) {  // 2 experts x half of the tokens
            const int e_lo = 2 * (warp & 3), tpg = (nr + 1) / 2, tb = (warp >> 2) * tpg, nt = min(tpg, nr - tb);
            if (e_lo < ne && nt > 0)
                logits_tile<2, 4>(w_s + (size_t)e_lo * slice, x_s + (size_t)tb * slice, slice, n_it, nt, ne - e_lo, lane,
                                  part + e_lo * p.T, p.T, r0 + tb);
        } else {  // 4 experts x a quarter of the tokens
            const int e_lo = 4 * (warp & 1), tpg = (nr + 3) / 4, tb = (warp >> 1) * tpg, nt = min(tpg, nr - tb);
            if (e_lo < ne && nt > 0) {
                if (nr <= 16)
                    logits_tile<4, 4>(w_s + (size_t)e_lo * slice, x_s + (size_t)tb * slice, slice, n_it, nt, ne - e_lo, lane,
                                      part + e_lo * p.T, p.T, r0 + tb);
                else
                    logits_tile<4, 8>(w_s + (size_t)e_lo * slice, x_s + (size_t)tb * slice, slice, n_it, nt, ne - e_lo, lane,
                                      part + e_lo * p.T, p.T, r0 + tb);
            }
        }
    }
    if (!ok && tid == 0) {
        atomicOr(p.status, kErrWaitTimeout);
        abort_flag = 1;
    }

    // slice partials of the cluster, added in slice order; scores
    cluster.sync();
    for (int u = ks + p.ksplit * tid; u < kLgExperts * p.T; u += p.ksplit * kLgThreads) {
        const int el = u / p.T, t = u % p.T;
        if (el < ne) {
            float logit = cluster.map_shared_rank(part, 0)[u];
            for (int k2 = 1; k2 < p.ksplit; k2++) logit = logit + cluster.map_shared_rank(part, k2)[u];
            p.scores[(size_t)t * p.E + e0 + el] = router_score(logit, p.score_fn);
        }
    }
    cluster.sync();  // the other CTAs have read this CTA's partials

    // a CTA that gave up waits (bounded) for its own copies before its shared memory is released
    if (abort_flag && tid == 0) {
        int dummy = 0;
        if (!mbar_wait(bar_w, 0, &dummy) || (!fused && !mbar_wait(bar_x, last_round & 1, &dummy)))
            atomicOr(p.status, kErrCopyTimeout);
    }
}

// ---- selection + dispatch kernel ---------------------------------------------------------------------


// Group-limited top-k of token t by one warp (stbl/model.cu:444-452 with the DeepSeek-V3 group limit):
// lane l holds experts l + 32 j (j < EJ) as keys of their biased scores (float_key order) and their
// unbiased scores.  The group score is the sum of the group's two largest biased scores; the
// topk_groups best groups are kept (ties to the lower group id), then the topk best experts of the
// kept groups are taken in order (ties to the lower expert id), and their unbiased scores,
// normalised in that order, times route_scale are the weights.  Written for latency: one token is
// a chain of warp collectives (about 25 cycles each), so independent collectives are issued
// unconditionally and the per-lane argmax is a tree.
template <int EJ>
__device__ __forceinline__ void select_token(const RouterParams &p, int t, int lane, int *sel_row, int *cnt, uint32_t *bm,
                                             int TW, int tb, bool live) {
    const int E = p.E, K = p.topk;
    const uint32_t lane_bit = 1u << lane;
    int mine = -1;
    float s_mine = 0.f;
    if (p.forced_idx) {
        // forced routes: the token's experts are given; a row that is out of range or repeats an
        // expert is replaced by experts 0..K-1 (and flagged), so the dispatch stays consistent
        int f = -1 - lane;  // distinct placeholders on lanes >= K
        if (lane < K) f = __ldg(p.forced_idx + (size_t)t * K + lane);
        const uint32_t same = __match_any_sync(0xffffffffu, f);
        const bool bad = lane < K && (f < 0 || f >= E || (same & (lane_bit - 1u)) != 0u);
        if (__any_sync(0xffffffffu, bad)) {
            if (lane == 0 && live) atomicOr(p.status, kErrBadTable);
            f = lane;
        }
        if (lane < K) mine = f, s_mine = __ldcg(p.scores + (size_t)t * E + f);
    } else {
        uint32_t key[EJ];
        float sv[EJ];
#pragma unroll
        for (int j = 0; j < EJ; j++) {
            const int e = lane + 32 * j;
            key[j] = 0u;  // below every float's key: not selectable
            sv[j] = 0.f;
            if (e < E) {
                const float s = __ldcg(p.scores + (size_t)t * E + e);
                sv[j] = s;
                key[j] = float_key(s + __ldg(p.bias + e) + 0.0f);
            }
        }
        if (p.n_groups > 1 && p.topk_groups < p.n_groups) {
            const int gsz = E / p.n_groups;
            const bool pow2 = (gsz & (gsz - 1)) == 0;
            // group score = top-1 + top-2 of the group's biased scores (values only); lane g ends with
            // group g's score
            float gs = 0.f;
            if (pow2 && gsz >= 32) {
                // a group is m whole registers: a tree of top-2 merges over them, then over the lanes
                const int m = gsz >> 5;
                uint32_t a1[EJ], a2[EJ];
#pragma unroll
                for (int j = 0; j < EJ; j++) a1[j] = key[j], a2[j] = 0u;
#pragma unroll
                for (int s = 1; s < EJ; s *= 2)
                    if (s < m)
#pragma unroll
                        for (int j = 0; j + s < EJ; j += 2 * s) top2_merge(a1[j], a2[j], a1[j + s], a2[j + s]);
                // every register's lane-wide top-2 (only group leaders j = g m are used): second largest =
                // the largest after the lowest lane holding the maximum swaps in its own second
#pragma unroll
                for (int j = 0; j < EJ; j++) {
                    const uint32_t m1 = __reduce_max_sync(0xffffffffu, a1[j]);
                    const uint32_t bal = __ballot_sync(0xffffffffu, a1[j] == m1);
                    const uint32_t m2 = __reduce_max_sync(0xffffffffu, (bal & (0u - bal)) == lane_bit ? a2[j] : a1[j]);
                    if (lane * m == j) gs = key_float(m1) + key_float(m2);
                }
            } else if (pow2) {
                // a group is a segment of gsz lanes of one register: top-2 merges across the segment
                const int segs = 32 / gsz, seg_shift = __ffs(segs) - 1;
#pragma unroll
                for (int j = 0; j < EJ; j++) {
                    uint32_t a1 = key[j], a2 = 0u;
                    for (int o = gsz / 2; o > 0; o >>= 1) {
                        const uint32_t b1 = __shfl_xor_sync(0xffffffffu, a1, o);
                        const uint32_t b2 = __shfl_xor_sync(0xffffffffu, a2, o);
                        top2_merge(a1, a2, b1, b2);
                    }
                    const float v = key_float(a1) + key_float(a2);
                    // group j * segs + s is held by lanes s * gsz ..; lane g takes its group's score
                    const float got = __shfl_sync(0xffffffffu, v, (lane & (segs - 1)) * gsz);
                    if ((lane >> seg_shift) == j) gs = got;
                }
            } else if (lane < p.n_groups) {
                // other group sizes: lane g scans its group
                int b1 = -1, b2 = -1;
                float v1 = 0.f, v2 = 0.f;
                for (int e = lane * gsz; e < (lane + 1) * gsz; e++) {
                    const float b = __ldcg(p.scores + (size_t)t * E + e) + __ldg(p.bias + e);
                    if (b1 < 0 || beats(b, e, v1, b1)) b2 = b1, v2 = v1, b1 = e, v1 = b;
                    else if (b2 < 0 || beats(b, e, v2, b2)) b2 = e, v2 = b;
                }
                gs = v1 + v2;
            }
            int rank = 0;
            for (int h = 0; h < p.n_groups; h++) {
                const float gh = __shfl_sync(0xffffffffu, gs, h);
                rank += beats(gh, h, gs, lane);
            }
            const uint32_t keepg = __ballot_sync(0xffffffffu, lane < p.n_groups && rank < p.topk_groups);
            // experts of the groups not kept become unselectable
            if (pow2) {
                const int gshift = __ffs(gsz) - 1;
#pragma unroll
                for (int j = 0; j < EJ; j++)
                    if (!((keepg >> (((lane + 32 * j) >> gshift) & 31)) & 1u)) key[j] = 0u;
            } else {
#pragma unroll
                for (int j = 0; j < EJ; j++)
                    if (!((keepg >> (((lane + 32 * j) / gsz) & 31)) & 1u)) key[j] = 0u;
            }
        }
        for (int i = 0; i < K; i++) {
            // lane argmax by a tree (ties to the lower register)
            uint32_t bk[EJ];
            int bj[EJ];
#pragma unroll
            for (int j = 0; j < EJ; j++) bk[j] = key[j], bj[j] = j;
#pragma unroll
            for (int s = 1; s < EJ; s *= 2)
#pragma unroll
                for (int j = 0; j + s < EJ; j += 2 * s)
                    if (bk[j + s] > bk[j]) bk[j] = bk[j + s], bj[j] = bj[j + s];
            const uint32_t mk = __reduce_max_sync(0xffffffffu, bk[0]);
            const int cand = (mk != 0u && bk[0] == mk) ? lane + 32 * bj[0] : INT_MAX;
            int win = __reduce_min_sync(0xffffffffu, cand);
            if (win == INT_MAX) {  // fewer candidates than topk: cannot happen for a validated layer
                if (lane == 0 && live) atomicOr(p.status, kErrBadTable);
                win = 0;
            }
            const int wj = lane == (win & 31) ? (win >> 5) : -1;
            float s_own = 0.f;
#pragma unroll
            for (int j = 0; j < EJ; j++)
                if (j == wj) key[j] = 0u, s_own = sv[j];
            const float s_win = __shfl_sync(0xffffffffu, s_own, win & 31);
            if (lane == i) mine = win, s_mine = s_win;
        }
    }
    // weights: unbiased scores normalised in top-k order (stbl/model.cu:450-451, 527-530)
    float sum = 0.f;
    for (int i = 0; i < K; i++) sum += __shfl_sync(0xffffffffu, s_mine, i);
    if (lane < K) {
        float wt = s_mine;
        wt /= sum + 1e-20f;
        wt *= p.route_scale;
        if (live) p.wts[t * K + lane] = wt;
        sel_row[lane] = mine;  // p.idx + t K in the live pass
        // dispatch counts and the expert's token bitmap (a token picks an expert at most once); bit
        // tb stands for the token
        atomicAdd(&cnt[mine], 1);
        atomicOr(&bm[mine * TW + (tb >> 5)], 1u << (tb & 31));
    }
}

// tokens selected by one CTA of the select kernel (one per warp)
constexpr int kSelTokensPerCta = kSelThreads / 32;

__host__ __device__ inline size_t router_select_smem(int E, int K, int T) {
    return (size_t)kSelTokensPerCta * K * 4 + 2 * (size_t)E * 4 + (size_t)E * ((T + 31) / 32) * 4;
}

// One CTA per 16 tokens (a warp per token).  Every CTA adds its tokens' choices to the global
// per-expert counts and token bitmaps (zeroed by the logits kernel); the last CTA to finish (by an
// atomic ticket) builds the bucketed dispatch for all T tokens.
__global__ void __launch_bounds__(kSelThreads) router_select_kernel(RouterParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int is_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int E = p.E, T = p.T, K = p.topk;
    int sh_r = __ffs(p.nt_routed) - 1, sh_s = __ffs(p.nt_shared) - 1;  // chunk sizes: powers of two
    __shared__ int s_wide;
    const int t0 = blockIdx.x * kSelTokensPerCta, n_own = min(kSelTokensPerCta, T - t0);
    int *s_idx = reinterpret_cast<int *>(smem);        // [16][K] (first pass)
    int *s_cnt = s_idx + kSelTokensPerCta * K;         // [E] (first pass)
    int *pk = s_cnt + E;                               // [E] exclusive scan of assignments | chunks << 16
    uint32_t *s_bm = reinterpret_cast<uint32_t *>(pk + E);  // [E][TW] (first pass: 16 tokens, one word)
    // registers per lane for E experts, rounded up to a power of two
    const int ej = E <= 32 ? 1 : E <= 64 ? 2 : E <= 128 ? 4 : E <= 256 ? 8 : 16;

    // Two passes over one copy of the code.  The first runs before the programmatic-launch wait,
    // while the logits kernel is still computing, on this CTA's tokens and shared memory only: it
    // reads whatever the scores buffer holds and stores nothing to global memory; it only brings this
    // kernel's instructions into the SM's instruction caches, so that the second, real pass does not
    // stall on instruction fetches.
#pragma unroll 1
    for (int pass = 0; pass < 2; pass++) {
        const bool live = pass == 1;
        // several CTAs (live pass): global counts and bitmaps of all T tokens; one CTA, or the first
        // pass: shared memory
        const bool global_state = live && gridDim.x > 1;
        int *cnt = global_state ? p.sel_cnt : s_cnt;
        uint32_t *bm = global_state ? p.sel_bm : s_bm;
        const int TW = live ? (T + 31) / 32 : 1;
        if (!global_state)
            for (int e = tid; e < E * TW; e += kSelThreads) s_bm[e] = 0;
        if (!global_state)
            for (int e = tid; e < E; e += kSelThreads) s_cnt[e] = 0;
        if (live) {
            pdl_wait();  // scores, quantized x and the zeroed global counts of the logits kernel
            pdl_launch_dependents();
        }
        __syncthreads();
        if (warp < n_own) {
            const int t = t0 + warp;
            int *sel_row = live ? p.idx + (size_t)t * K : s_idx + warp * K;
            const int tb = live ? t : warp;
            switch (ej) {
                case 1: select_token<1>(p, t, lane, sel_row, cnt, bm, TW, tb, live); break;
                case 2: select_token<2>(p, t, lane, sel_row, cnt, bm, TW, tb, live); break;
                case 4: select_token<4>(p, t, lane, sel_row, cnt, bm, TW, tb, live); break;
                case 8: select_token<8>(p, t, lane, sel_row, cnt, bm, TW, tb, live); break;
                default: select_token<16>(p, t, lane, sel_row, cnt, bm, TW, tb, live); break;
            }
        }
        if (global_state) {
            __threadfence();
            __syncthreads();
            if (tid == 0) is_last = atomicAdd(p.sel_ticket, 1u) == gridDim.x - 1;
            __syncthreads();
            if (!is_last) break;
            __threadfence();
            // every CTA's counts and bitmaps, into shared memory for the dispatch below
            for (int e = tid; e < E; e += kSelThreads) s_cnt[e] = __ldcg(p.sel_cnt + e);
            for (int i = tid; i < E * TW; i += kSelThreads) s_bm[i] = __ldcg(p.sel_bm + i);
            cnt = s_cnt;
            bm = s_bm;
        }
        __syncthreads();

        // bucketed dispatch over n tokens (live: all T; first pass: this CTA's), from shared memory.
        // Warp 0 scans (assignments | chunks << 16) over the experts, lane l owning experts
        // l * epl .. (l + 1) * epl - 1; every thread then places assignments by their stable rank among
        // the expert's tokens (the expert's token bitmap).
        const int n = live ? T : n_own;
        const int *sel = live ? p.idx : s_idx;
        if (live && p.adaptive_wide) {
            // 32-token chunks when they save more than a quarter of the 16-token ones (one item then
            // streams an expert's weights for up to 32 tokens; with few tokens per expert the 16-token
            // launch is faster)
            if (warp == 0) {
                int c16 = 0, c32 = 0;
                for (int e = lane; e < E; e += 32) c16 += (cnt[e] + 15) >> 4, c32 += (cnt[e] + 31) >> 5;
                if (p.has_shared) c16 += lane == 0 ? (T + 15) >> 4 : 0, c32 += lane == 0 ? (T + 31) >> 5 : 0;
                for (int o = 16; o > 0; o >>= 1) c16 += __shfl_xor_sync(0xffffffffu, c16, o), c32 += __shfl_xor_sync(0xffffffffu, c32, o);
                if (lane == 0) {
                    s_wide = 4 * c32 < 3 * c16;
                    *p.wide_sel = s_wide;
                }
            }
            __syncthreads();
            if (s_wide) sh_r = 5, sh_s = 5;
        }
        const int nt_r = 1 << sh_r, nt_s = 1 << sh_s;
        if (warp == 0) {
            const int epl = (E + 31) / 32, e0 = lane * epl;
            int run = 0;
            for (int i = 0; i < epl; i++) {
                const int e = e0 + i;
                if (e < E) {
                    const int c = cnt[e];
                    run += c | (((c + nt_r - 1) >> sh_r) << 16);
                }
            }
            int incl = run;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            int acc = incl - run;
            for (int i = 0; i < epl; i++) {
                const int e = e0 + i;
                if (e < E) {
                    pk[e] = acc;
                    const int c = cnt[e];
                    acc += c | (((c + nt_r - 1) >> sh_r) << 16);
                }
            }
        }
        __syncthreads();
        for (int a = tid; a < n * K; a += kSelThreads) {
            const int e = live ? __ldcg(sel + a) : sel[a], t = a / K;
            const uint32_t *row = bm + (size_t)e * TW;
            int rank = __popc(row[t >> 5] & ((1u << (t & 31)) - 1u));
            for (int w = 0; w < (t >> 5); w++) rank += __popc(row[w]);
            if (live) p.perm[(pk[e] & 0xffff) + rank] = a;
        }
        const int ns = p.has_shared ? (T + nt_s - 1) >> sh_s : 0;
        if (live) {
            for (int i = tid; i < ns; i += kSelThreads)
                p.chunks[i] = Chunk{E, T * K + (i << sh_s), min(nt_s, T - (i << sh_s)), 0};
            for (int e = tid; e < E; e += kSelThreads) {
                const int c_e = cnt[e], off = pk[e] & 0xffff, ch = pk[e] >> 16;
                p.counts[e] = c_e;
                p.offsets[e] = off;
                for (int c = 0; (c << sh_r) < c_e; c++)
                    p.chunks[ns + ch + c] = Chunk{e, off + (c << sh_r), min(nt_r, c_e - (c << sh_r)), 0};
                if (e == E - 1) {
                    p.offsets[E] = T * K;
                    p.n_chunks[0] = ns + ch + ((c_e + nt_r - 1) >> sh_r);
                    p.n_chunks[1] = ns;
                }
            }
        }
        __syncthreads();
    }
}

// ---- host side ---------------------------------------------------------------------------------------

cudaError_t router_setup() {
    return cudaFuncSetAttribute((const void *)router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)router_logits_smem(4 * kLgMaxSlice, kRouterMaxTokens));
}

cudaError_t launch_router(RouterParams r, cudaStream_t st, bool pdl_first) {
    if ((r.nt_routed & (r.nt_routed - 1)) || (r.nt_shared & (r.nt_shared - 1)) || r.nt_routed < 1 || r.nt_shared < 1)
        return cudaErrorInvalidValue;  // chunk sizes must be powers of two
    void *args[] = {&r};
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[2];
    cfg.gridDim = dim3(r.ksplit * ((r.E + kLgExperts - 1) / kLgExperts));
    cfg.blockDim = dim3(kLgThreads);
    cfg.dynamicSmemBytes = router_logits_smem(r.H, r.T);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = r.ksplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_first ? 2 : 1;
    cudaError_t e = cudaLaunchKernelExC(&cfg, (const void *)router_logits_kernel, args);
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3((r.T + kSelTokensPerCta - 1) / kSelTokensPerCta);
    cfg.blockDim = dim3(kSelThreads);
    cfg.dynamicSmemBytes = router_select_smem(r.E, r.topk, r.T);
    cfg.attrs = attr + 1;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, (const void *)router_select_kernel, args);
}

}  // namespace stbl
