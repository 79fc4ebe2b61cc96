// Grouped expert GEMVs of the MoE layer (small-batch decode path).
//
// One persistent CTA per SM walks a list of work items (chunk of <= kNT tokens of one expert, tile of
// RI output rows).  Warp 0 streams the item's weight rows (and MXFP4 scales) into a ring of shared
// memory stages with 1-D bulk copies (TMA engine, mbarrier completion).  Warps 1..14 hold the chunk's
// activations in registers as f16 pairs and take a fixed 32-value span of every weight row each:
// e4m3 / e2m1 pairs are widened to f16 with one cvt and multiplied into fp32 accumulators with the
// mixed-precision FMA; per-block weight and activation scales are applied once per span.  Lane
// partial sums are reduced by a reduce-scatter across the warp and a fixed-order sum across warps.
//
// up kernel (gate + up, SwiGLU with the routing weight, stbl/model.cu:536-537, kernels.cu:445-459):
//   h = bf16(silu(bf16(W1 x)) * bf16(W3 x) * w); when the last item of a 128-row group of a chunk
//   lands, that CTA re-quantizes the group (act_quant, ref/kernel.py:35-45) for the down kernel.
// down kernel (stbl/model.cu:538-539, 543-547, 589-592): eo = bf16(W2 hq); when the last of the
//   top-k routed experts and the shared expert of a token lands on a 128-row group, that CTA writes
//   y = bf16(sum of eo in top-k order + shared) for the group.
#include "layer.cuh"

namespace stbl {

constexpr int kRedSlots = 64 * 32;  // floats of cross-warp reduction space

struct ChunkInfo {
    int e, pos0, n, ok;
};

__device__ __forceinline__ ChunkInfo load_chunk(const ExpertParams &p, int c) {
    const Chunk ch = p.chunks[c];
    ChunkInfo ci{ch.e, ch.pos0, ch.n, 1};
    const int nrouted = p.T * p.topk;
    const bool shared = ch.e == p.E;
    const bool bad = ch.e < 0 || ch.e > p.E || (shared && !p.has_shared) || ch.n < 1 || ch.n > kNT ||
                     (shared ? (ch.pos0 < nrouted || ch.pos0 + ch.n > nrouted + p.T)
                             : (ch.pos0 < 0 || ch.pos0 + ch.n > nrouted));
    if (bad) ci = ChunkInfo{0, 0, 0, 0};
    return ci;
}

template <int FMT>
__device__ __forceinline__ int row_bytes(int K) {
    return FMT == kFmtFp8B128 ? K : K / 2;
}

// act_quant of 128 consecutive bf16 values (one warp, 4 per lane), read through L2 (written by other
// CTAs of this launch): codes and scales as ref/kernel.py:35-45.
__device__ void quant128_cg(const uint16_t *src, uint8_t *dst, float *sdst, int blk, int pow2, int lane) {
    const uint2 xv = __ldcg(reinterpret_cast<const uint2 *>(src + 4 * lane));
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
    *reinterpret_cast<uint32_t *>(dst + 4 * lane) = codes;
    if (((4 * lane) % blk) == 0) sdst[(4 * lane) / blk] = s;
}

template <int FMT, bool UP, int RPG>
__global__ void __launch_bounds__(kExpertThreads, 1)
    expert_kernel(ExpertParams p, int stage_bytes, int nst) {
    constexpr int NMAT = UP ? 2 : 1;
    constexpr int V = RPG * NMAT * kNT;
    constexpr int LOG2V = log2_const<V>();
    static_assert(V <= 32, "too many values per lane");

    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)nst * stage_bytes);
    uint64_t *empty = full + nst;
    float *red = reinterpret_cast<float *>(empty + nst);
    int *fin = reinterpret_cast<int *>(red + kRedSlots);  // [0] count, [1..] entries
    __shared__ int abort_flag;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = UP ? p.H : p.I;            // reduction length
    const int rows = UP ? p.I : p.H;         // output rows per matrix
    const int Lk = K / 32;                   // lanes per row
    const int n_rg = kConsumerThreads / Lk;  // rows in flight per CTA
    const int RI = n_rg * RPG;               // rows per item
    const int tiles = (rows + RI - 1) / RI;
    const int rb = row_bytes<FMT>(K);
    const int scale_off = NMAT * RI * rb;    // MXFP4 scales after the codes
    const int chunk_end = p.chunk_end >= 0 ? p.chunk_end : *(volatile const int *)p.n_chunks;
    const int n_items = max(0, chunk_end - p.chunk_begin) * tiles;

    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < nst; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == 0) {
        // ---- producer: one thread issues the bulk copies ----
        int issued = 0;
        if (lane == 0) {
            for (int it = 0;; it++) {
                const int item = blockIdx.x + it * gridDim.x;
                if (item >= n_items) break;
                const int c = p.chunk_begin + item / tiles, tile = item % tiles;
                const ChunkInfo ci = load_chunk(p, c);
                const ExpertPtrs ep = p.experts[ci.e];
                const int s = it % nst;
                if (!mbar_wait(&empty[s], ((it / nst) & 1) ^ 1, &abort_flag)) {
                    abort_flag = 1;
                    atomicOr(p.status, kErrWaitTimeout);
                    break;
                }
                const int r0 = tile * RI, nr = min(RI, rows - r0);
                bool ptr_ok = ci.ok;
#pragma unroll
                for (int m = 0; m < NMAT; m++) {
                    const int mat = UP ? m : 2;
                    ptr_ok = ptr_ok && ep.w[mat] != nullptr && (FMT != kFmtMxfp4 || ep.s[mat] != nullptr);
                }
                unsigned char *st = smem + (size_t)s * stage_bytes;
                if (!ptr_ok) {
                    mbar_arrive(&full[s]);  // consumers see an empty chunk (n = 0) or a flagged one
                } else {
                    const uint32_t bytes = NMAT * nr * rb + (FMT == kFmtMxfp4 ? NMAT * nr * (K / 32) : 0);
                    mbar_arrive_expect_tx(&full[s], bytes);
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        const int mat = UP ? m : 2;
                        bulk_g2s(st + (size_t)m * RI * rb, ep.w[mat] + (size_t)r0 * rb, nr * rb, &full[s]);
                        if (FMT == kFmtMxfp4)
                            bulk_g2s(st + scale_off + (size_t)m * RI * (K / 32),
                                     static_cast<const uint8_t *>(ep.s[mat]) + (size_t)r0 * (K / 32), nr * (K / 32),
                                     &full[s]);
                    }
                }
                issued = it + 1;
            }
            // leave only when every issued copy has landed (they write this CTA's shared memory)
            for (int it = max(0, issued - nst); it < issued; it++) {
                const int s = it % nst;
                uint64_t t0 = global_ns();
                while (!mbar_try_wait(&full[s], (it / nst) & 1)) {
                    if (global_ns() - t0 > kWaitLimitNs) {
                        atomicOr(p.status, kErrCopyTimeout);
                        break;
                    }
                }
            }
        }
        return;
    }

    // ---- consumers ----
    const int ct = tid - 32, wc = ct >> 5;
    const int rg = ct / Lk, pp = ct % Lk;
    const bool active = rg < n_rg;
    const int nG = (rows + 127) / 128;

    int cur = -1;
    ChunkInfo ci{0, 0, 0, 0};
    ExpertPtrs ep{};
    uint32_t xa[kNT][8], xb[kNT][8];  // FP8: spans p and p + Lk (16 values each); MXFP4: 32 values of span p
    float sxa[kNT], sxb[kNT];
    int tok[kNT], arow[kNT];
    float wt[kNT];

    for (int it = 0;; it++) {
        const int item = blockIdx.x + it * gridDim.x;
        if (item >= n_items) break;
        const int c = p.chunk_begin + item / tiles, tile = item % tiles;
        const int r0 = tile * RI, nr = min(RI, rows - r0);
        if (c != cur) {
            cur = c;
            ci = load_chunk(p, c);
            if (!ci.ok && ct == 0) atomicOr(p.status, kErrBadTable);
            ep = p.experts[ci.e];
            bool ptr_ok = true;
#pragma unroll
            for (int m = 0; m < NMAT; m++) ptr_ok = ptr_ok && ep.w[UP ? m : 2] != nullptr && ep.s[UP ? m : 2] != nullptr;
            if (!ptr_ok) {
                ci.n = 0;
                if (ct == 0) atomicOr(p.status, kErrBadTable);
            }
#pragma unroll
            for (int t = 0; t < kNT; t++) {
                tok[t] = 0, arow[t] = 0, wt[t] = 0.f, sxa[t] = 0.f, sxb[t] = 0.f;
#pragma unroll
                for (int j = 0; j < 8; j++) xa[t][j] = 0u, xb[t][j] = 0u;
                if (t < ci.n) {
                    const int pos = ci.pos0 + t;
                    if (ci.e < p.E) {
                        const int a = p.perm[pos];
                        arow[t] = a;
                        tok[t] = a / p.topk;
                        wt[t] = p.wts[a];
                    } else {
                        tok[t] = pos - p.T * p.topk;
                        wt[t] = 1.f;
                    }
                    const int xrow = UP ? tok[t] : pos;
                    const uint8_t *src = p.xq + (size_t)xrow * K;
                    const float *srow = p.xs + (size_t)xrow * p.xs_stride;
                    if (active) {
                        if (FMT == kFmtFp8B128) {
                            const uint4 qa = __ldg(reinterpret_cast<const uint4 *>(src + 16 * pp));
                            const uint4 qb = __ldg(reinterpret_cast<const uint4 *>(src + 16 * (pp + Lk)));
                            const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w}, wb[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
                            for (int j = 0; j < 4; j++) {
                                xa[t][2 * j] = e4m3x2_to_f16x2((uint16_t)(wa[j] & 0xffffu));
                                xa[t][2 * j + 1] = e4m3x2_to_f16x2((uint16_t)(wa[j] >> 16));
                                xb[t][2 * j] = e4m3x2_to_f16x2((uint16_t)(wb[j] & 0xffffu));
                                xb[t][2 * j + 1] = e4m3x2_to_f16x2((uint16_t)(wb[j] >> 16));
                            }
                            sxa[t] = __ldg(srow + (16 * pp) / p.act_blk);
                            sxb[t] = __ldg(srow + (16 * (pp + Lk)) / p.act_blk);
                        } else {
                            const uint4 qa = __ldg(reinterpret_cast<const uint4 *>(src + 32 * pp));
                            const uint4 qb = __ldg(reinterpret_cast<const uint4 *>(src + 32 * pp + 16));
                            const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w}, wb[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
                            for (int j = 0; j < 4; j++) {
                                xa[t][2 * j] = e4m3x2_to_f16x2((uint16_t)(wa[j] & 0xffffu));
                                xa[t][2 * j + 1] = e4m3x2_to_f16x2((uint16_t)(wa[j] >> 16));
                                xb[t][2 * j] = e4m3x2_to_f16x2((uint16_t)(wb[j] & 0xffffu));
                                xb[t][2 * j + 1] = e4m3x2_to_f16x2((uint16_t)(wb[j] >> 16));
                            }
                            sxa[t] = __ldg(srow + pp);
                        }
                    }
                }
            }
        }

        const int s = it % nst;
        const bool ok = mbar_wait(&full[s], (it / nst) & 1, &abort_flag);
        const unsigned char *st = smem + (size_t)s * stage_bytes;

        float v[V];
#pragma unroll
        for (int i = 0; i < V; i++) v[i] = 0.f;
        if (ok && active && ci.n > 0) {
#pragma unroll
            for (int i = 0; i < RPG; i++) {
                const int lr = rg + n_rg * i, r = r0 + lr;
                if (r < rows) {
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        const int mat = UP ? m : 2;
                        if (FMT == kFmtFp8B128) {
                            const unsigned char *rowp = st + (size_t)m * RI * rb + (size_t)lr * rb;
                            const uint4 qa = *reinterpret_cast<const uint4 *>(rowp + 16 * pp);
                            const uint4 qb = *reinterpret_cast<const uint4 *>(rowp + 16 * (pp + Lk));
                            const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w}, wb[4] = {qb.x, qb.y, qb.z, qb.w};
                            uint32_t fa[8], fb[8];
#pragma unroll
                            for (int j = 0; j < 4; j++) {
                                fa[2 * j] = e4m3x2_to_f16x2((uint16_t)(wa[j] & 0xffffu));
                                fa[2 * j + 1] = e4m3x2_to_f16x2((uint16_t)(wa[j] >> 16));
                                fb[2 * j] = e4m3x2_to_f16x2((uint16_t)(wb[j] & 0xffffu));
                                fb[2 * j + 1] = e4m3x2_to_f16x2((uint16_t)(wb[j] >> 16));
                            }
                            const float *wsr = static_cast<const float *>(ep.s[mat]) + (size_t)(r / 128) * ((K + 127) / 128);
                            const float swa = __ldg(wsr + (16 * pp) / 128), swb = __ldg(wsr + (16 * (pp + Lk)) / 128);
#pragma unroll
                            for (int t = 0; t < kNT; t++) {
                                if (t < ci.n) {
                                    float ra = 0.f, rb2 = 0.f;
#pragma unroll
                                    for (int j = 0; j < 8; j++) {
                                        ra = dot2_f16_f32(fa[j], xa[t][j], ra);
                                        rb2 = dot2_f16_f32(fb[j], xb[t][j], rb2);
                                    }
                                    v[(i * NMAT + m) * kNT + t] = fmaf(rb2, swb * sxb[t], ra * (swa * sxa[t]));
                                }
                            }
                        } else {
                            const unsigned char *rowp = st + (size_t)m * RI * rb + (size_t)lr * rb;
                            const uint4 q = *reinterpret_cast<const uint4 *>(rowp + 16 * pp);
                            const uint32_t sb = st[scale_off + (size_t)m * RI * (K / 32) + (size_t)lr * (K / 32) + pp];
                            const uint32_t wq[4] = {q.x, q.y, q.z, q.w};
                            uint32_t f[16];
#pragma unroll
                            for (int j = 0; j < 4; j++) {
#pragma unroll
                                for (int b = 0; b < 4; b++) f[4 * j + b] = e2m1x2_to_f16x2((wq[j] >> (8 * b)) & 0xffu);
                            }
                            const float sw = e8m0(sb);
#pragma unroll
                            for (int t = 0; t < kNT; t++) {
                                if (t < ci.n) {
                                    float ra = 0.f, rb2 = 0.f;
#pragma unroll
                                    for (int j = 0; j < 8; j++) {
                                        ra = dot2_f16_f32(f[j], xa[t][j], ra);
                                        rb2 = dot2_f16_f32(f[8 + j], xb[t][j], rb2);
                                    }
                                    v[(i * NMAT + m) * kNT + t] = (ra + rb2) * (sw * sxa[t]);
                                }
                            }
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);

        // reduce the lane partials: per row group, one value per (row, matrix, token)
        if (Lk >= 32) {
            const float r = warp_reduce_scatter<V>(v, lane);
            if ((lane & ((32 >> LOG2V) - 1)) == 0) red[wc * V + (lane >> (5 - LOG2V))] = r;
        } else {
#pragma unroll
            for (int i = 0; i < V; i++) {
                float x = v[i];
                for (int o = Lk / 2; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
                if (pp == 0 && active) red[rg * V + i] = x;
            }
        }
        if (bar_sync_or(1, kConsumerThreads, !ok)) {
            if (ct == 0) {
                abort_flag = 1;
                atomicOr(p.status, kErrWaitTimeout);
            }
            break;
        }
        const int wpr = Lk >= 32 ? Lk / 32 : 1;
        auto total = [&](int g, int vi) {
            float acc = 0.f;
            if (Lk >= 32) {
                for (int w = 0; w < wpr; w++) acc += red[(g * wpr + w) * V + vi];
            } else {
                acc = red[g * V + vi];
            }
            return acc;
        };
        // epilogue: one thread per (row group, row, token)
        for (int j = ct; j < n_rg * RPG * kNT; j += kConsumerThreads) {
            const int g = j / (RPG * kNT), i = (j / kNT) % RPG, t = j % kNT;
            const int r = r0 + g + n_rg * i;
            if (t >= ci.n || r >= rows) continue;
            if (UP) {
                float gv = bf16r(total(g, (i * 2 + 0) * kNT + t));
                float uv = bf16r(total(g, (i * 2 + 1) * kNT + t));
                if (p.swiglu_limit > 0.f) {
                    uv = fminf(fmaxf(uv, -p.swiglu_limit), p.swiglu_limit);
                    gv = fminf(gv, p.swiglu_limit);
                }
                const float hv = gv / (1.f + expf(-gv)) * uv * wt[t];
                p.h[(size_t)(ci.pos0 + t) * p.I + r] = f32_to_bf16_bits(hv);
            } else {
                const uint16_t o = f32_to_bf16_bits(total(g, i * kNT + t));
                if (ci.e < p.E) p.eo[(size_t)arow[t] * p.H + r] = o;
                else p.sh[(size_t)tok[t] * p.H + r] = o;
            }
        }
        bar_sync(1, kConsumerThreads);
        // completion counting per 128-row group (release: fence after the CTA's stores)
        if (ct == 0) {
            int nf = 0;
            if (ci.n > 0) {
                __threadfence();
                for (int gr = r0 / 128; gr <= (r0 + nr - 1) / 128; gr++) {
                    const int lo = max(r0, gr * 128), hi = min(r0 + nr, min(rows, gr * 128 + 128));
                    const int cnt = hi - lo, grp_rows = min(128, rows - gr * 128);
                    if (UP) {
                        if (atomicAdd(&p.hcnt[(size_t)c * nG + gr], cnt) + cnt == grp_rows) fin[1 + nf++] = gr;
                    } else {
                        const int need = (p.topk + p.has_shared) * grp_rows;
                        for (int t = 0; t < ci.n; t++)
                            if (atomicAdd(&p.ccnt[(size_t)tok[t] * nG + gr], cnt) + cnt == need) fin[1 + nf++] = gr * kNT + t;
                    }
                }
                if (nf) __threadfence();
            }
            fin[0] = nf;
        }
        bar_sync(1, kConsumerThreads);
        const int nf = fin[0];
        if (nf) {
            if (UP) {
                // re-quantize the finished 128-row groups of h for the down kernel
                for (int task = wc; task < nf * ci.n; task += kConsumerWarps) {
                    const int gr = fin[1 + task / ci.n], t = task % ci.n, pos = ci.pos0 + t;
                    if (gr * 128 + 4 * lane < p.I)
                        quant128_cg(p.h + (size_t)pos * p.I + gr * 128, p.hq + (size_t)pos * p.I + gr * 128,
                                    p.hs + (size_t)pos * p.hs_stride + gr * 128 / p.act_blk, p.act_blk,
                                    p.act_pow2, lane);
                }
            } else {
                // ordered combine of a finished (token, 128-row group): fp32 sum of the routed outputs in
                // top-k order, then the shared expert's, one bf16 rounding
                for (int task = ct; task < nf * 128; task += kConsumerThreads) {
                    const int f = fin[1 + task / 128];
                    const int gr = f / kNT, t = f % kNT, r = gr * 128 + task % 128;
                    if (r >= p.H) continue;
                    const int tk = tok[t];
                    float acc = 0.f;
                    for (int sl = 0; sl < p.topk; sl++)
                        acc = acc + bf16_bits_to_f32(__ldcg(p.eo + ((size_t)tk * p.topk + sl) * p.H + r));
                    if (p.has_shared) acc = acc + bf16_bits_to_f32(__ldcg(p.sh + (size_t)tk * p.H + r));
                    p.y[(size_t)tk * p.H + r] = f32_to_bf16_bits(acc);
                }
            }
        }
    }
}

// explicit instantiations (launched from moe.cu)
template __global__ void expert_kernel<kFmtFp8B128, true, 2>(ExpertParams, int, int);
template __global__ void expert_kernel<kFmtFp8B128, false, 2>(ExpertParams, int, int);
template __global__ void expert_kernel<kFmtMxfp4, true, 2>(ExpertParams, int, int);
template __global__ void expert_kernel<kFmtMxfp4, false, 2>(ExpertParams, int, int);

}  // namespace stbl

namespace stbl {
// host-side selection of the kernel instantiation for a weight format and direction
const void *expert_kernel_ptr(int fmt, bool up) {
    if (fmt == kFmtFp8B128)
        return up ? (const void *)expert_kernel<kFmtFp8B128, true, 2> : (const void *)expert_kernel<kFmtFp8B128, false, 2>;
    return up ? (const void *)expert_kernel<kFmtMxfp4, true, 2> : (const void *)expert_kernel<kFmtMxfp4, false, 2>;
}
}  // namespace stbl
