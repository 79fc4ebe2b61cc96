// Grouped expert GEMVs of the MoE layer (small-batch decode path) and the ordered combine.
//
// One persistent CTA per SM takes a contiguous range of work items (chunk of <= kNT tokens of one
// expert, tile of RI output rows).  Warp 0 streams the items' weight rows (and MXFP4 scales) into a
// ring of shared-memory stages with 1-D bulk copies (TMA engine, mbarrier completion).  Warps 1..14
// hold the chunk's activations in registers as f16 pairs and take a fixed 32-value span of every
// weight row: e4m3 / e2m1 pairs are widened to f16 with one cvt and multiplied into fp32
// accumulators by the mixed-precision FMA (products of two f16 holding e4m3 / e2m1 values are exact);
// block scales are applied once per span.  Lane partial sums are reduced by a reduce-scatter across
// the warp (about one shuffle per value, sized to the chunk's token count) and a fixed-order sum
// across the warps of a row.  One named barrier per item.
//
// up (gate + up, SwiGLU with the routing weight; stbl/model.cu:536-537, stbl/kernels.cu:445-459):
//   h = bf16(silu(bf16(W1 q(x))) * bf16(W3 q(x)) * w)
// down (stbl/model.cu:538-539, 543-547): eo = bf16(W2 q(h)), where q(h) is act_quant
//   (ref/kernel.py:35-45) computed in registers when the CTA reaches a new chunk.
// combine (stbl/model.cu:589-592): y = bf16(sum of eo in top-k order + shared output), fp32 sums.
#include "layer.cuh"

namespace stbl {

constexpr int kRedHalf = 1024;  // floats per reduction buffer; two buffers alternate by item

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

// 16 e4m3 codes (one uint4) -> 8 f16 pairs
__device__ __forceinline__ void codes16_to_f16(const uint4 q, uint32_t *f) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        f[2 * j] = e4m3x2_to_f16x2((uint16_t)(w[j] & 0xffffu));
        f[2 * j + 1] = e4m3x2_to_f16x2((uint16_t)(w[j] >> 16));
    }
}

// act_quant (ref/kernel.py:35-45) of 16 bf16 values held by this lane, whose block of `blk`
// values spans blk/16 consecutive lanes (a power of two <= 8); returns the scale, codes as f16 pairs.
__device__ __forceinline__ float quant16_lanes(const uint4 a, const uint4 b, int lanes, int pow2, uint32_t *f) {
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float v[16];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        v[2 * j] = __uint_as_float(w[j] << 16);
        v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 16; j++) amax = fmaxf(amax, fabsf(v[j]));
    for (int o = 1; o < lanes; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    amax = fmaxf(amax, 1e-4f);
    const float tq = amax * (1.0f / 448.0f);
    const float s = pow2 ? pow2_ceil(tq) : tq;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const uint32_t c0 = e4m3_code(fminf(fmaxf(v[2 * j] / s, -448.f), 448.f));
        const uint32_t c1 = e4m3_code(fminf(fmaxf(v[2 * j + 1] / s, -448.f), 448.f));
        f[j] = e4m3x2_to_f16x2((uint16_t)(c0 | (c1 << 8)));
    }
    return s;
}

template <int VN, int VT>
__device__ __forceinline__ float reduce_prefix(const float (&v)[VT], int lane) {
    float w[VN];
#pragma unroll
    for (int i = 0; i < VN; i++) w[i] = v[i];
    return warp_reduce_scatter<VN>(w, lane);
}

template <int FMT, bool UP, int RPG>
__global__ void __launch_bounds__(kExpertThreads, 1)
    expert_kernel(ExpertParams p, int stage_bytes, int nst) {
    constexpr int NMAT = UP ? 2 : 1;
    constexpr int RV = RPG * NMAT;           // values per token per lane
    constexpr int V = RV * kNT;
    static_assert(V <= 32, "too many values per lane");

    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)nst * stage_bytes);
    uint64_t *empty = full + nst;
    float *red = reinterpret_cast<float *>(empty + nst);  // [2][kRedHalf]
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

    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < nst; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();
    pdl_wait();  // routing tables, x codes and h come from the kernels before this one
    pdl_launch_dependents();

    const int chunk_end = p.chunk_end >= 0 ? p.chunk_end : *(volatile const int *)p.n_chunks;
    const long long n_items = (long long)max(0, chunk_end - p.chunk_begin) * tiles;
    const int lo = (int)(n_items * blockIdx.x / gridDim.x), hi = (int)(n_items * (blockIdx.x + 1) / gridDim.x);

    if (warp == 0) {
        // ---- producer: one thread issues the bulk copies ----
        if (lane == 0) {
            int issued = 0;
            for (int it = lo; it < hi; it++) {
                const int j = it - lo, s = j % nst;
                const int c = p.chunk_begin + it / tiles, tile = it % tiles;
                const ChunkInfo ci = load_chunk(p, c);
                const ExpertPtrs ep = p.experts[ci.e];
                if (!mbar_wait(&empty[s], ((j / nst) & 1) ^ 1, &abort_flag)) {
                    abort_flag = 1;
                    atomicOr(p.status, kErrWaitTimeout);
                    break;
                }
                const int r0 = tile * RI, nr = min(RI, rows - r0);
                bool ptr_ok = ci.ok;
#pragma unroll
                for (int m = 0; m < NMAT; m++) {
                    const int mat = UP ? m : 2;
                    ptr_ok = ptr_ok && ep.w[mat] != nullptr && ep.s[mat] != nullptr;
                }
                unsigned char *st = smem + (size_t)s * stage_bytes;
                if (!ptr_ok) {
                    mbar_arrive(&full[s]);  // consumers see an empty chunk
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
                issued = j + 1;
            }
            // leave only when every issued copy has landed (they write this CTA's shared memory)
            for (int j = max(0, issued - nst); j < issued; j++) {
                const int s = j % nst;
                const uint64_t t0 = global_ns();
                while (!mbar_try_wait(&full[s], (j / nst) & 1)) {
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
    const bool active = rg < n_rg;  // uniform per warp (Lk divides 32 or is a multiple of 32)

    int cur = -1, nt = 1;
    ChunkInfo ci{0, 0, 0, 0};
    ExpertPtrs ep{};
    uint32_t xa[kNT][8], xb[kNT][8];  // FP8: spans pp and pp + Lk (16 values each); MXFP4: 32 values of span pp
    float sxa[kNT], sxb[kNT];
    float wt[kNT];

    for (int it = lo; it < hi; it++) {
        const int j = it - lo;
        const int c = p.chunk_begin + it / tiles, tile = it % tiles;
        const int r0 = tile * RI;
        if (c != cur) {
            cur = c;
            ci = load_chunk(p, c);
            if (!ci.ok && ct == 0) atomicOr(p.status, kErrBadTable);
            ep = p.experts[ci.e];
            bool ptr_ok = true;
#pragma unroll
            for (int m = 0; m < NMAT; m++) ptr_ok = ptr_ok && ep.w[UP ? m : 2] != nullptr && ep.s[UP ? m : 2] != nullptr;
            if (!ptr_ok) ci.n = 0;
            nt = ci.n <= 1 ? 1 : (ci.n <= 2 ? 2 : 4);
#pragma unroll
            for (int t = 0; t < kNT; t++) {
                wt[t] = 0.f, sxa[t] = 0.f, sxb[t] = 0.f;
#pragma unroll
                for (int q = 0; q < 8; q++) xa[t][q] = 0u, xb[t][q] = 0u;
                if (t < ci.n) {
                    const int pos = ci.pos0 + t;
                    int tok;
                    if (ci.e < p.E) {
                        const int a = p.perm[pos];
                        tok = a / p.topk;
                        wt[t] = p.wts[a];
                    } else {
                        tok = pos - p.T * p.topk;
                        wt[t] = 1.f;
                    }
                    if (active) {
                        if (UP) {
                            const uint8_t *src = p.xq + (size_t)tok * K;
                            const float *srow = p.xs + (size_t)tok * p.xs_stride;
                            if (FMT == kFmtFp8B128) {
                                codes16_to_f16(__ldg(reinterpret_cast<const uint4 *>(src + 16 * pp)), xa[t]);
                                codes16_to_f16(__ldg(reinterpret_cast<const uint4 *>(src + 16 * (pp + Lk))), xb[t]);
                                sxa[t] = __ldg(srow + (16 * pp) / p.act_blk);
                                sxb[t] = __ldg(srow + (16 * (pp + Lk)) / p.act_blk);
                            } else {
                                codes16_to_f16(__ldg(reinterpret_cast<const uint4 *>(src + 32 * pp)), xa[t]);
                                codes16_to_f16(__ldg(reinterpret_cast<const uint4 *>(src + 32 * pp + 16)), xb[t]);
                                sxa[t] = __ldg(srow + pp);
                            }
                        } else {
                            // h of this position, re-quantized here (act_quant of the down projection input)
                            const uint16_t *hrow = p.h + (size_t)pos * K;
                            if (FMT == kFmtFp8B128) {
                                const uint4 *a4 = reinterpret_cast<const uint4 *>(hrow + 16 * pp);
                                const uint4 *b4 = reinterpret_cast<const uint4 *>(hrow + 16 * (pp + Lk));
                                sxa[t] = quant16_lanes(__ldg(a4), __ldg(a4 + 1), p.act_blk / 16, p.act_pow2, xa[t]);
                                sxb[t] = quant16_lanes(__ldg(b4), __ldg(b4 + 1), p.act_blk / 16, p.act_pow2, xb[t]);
                            } else {
                                const uint4 *a4 = reinterpret_cast<const uint4 *>(hrow + 32 * pp);
                                // one 32-block per lane: the two halves share the lane's scale
                                uint32_t fa[8], fb[8];
                                const uint4 q0 = __ldg(a4), q1 = __ldg(a4 + 1), q2 = __ldg(a4 + 2), q3 = __ldg(a4 + 3);
                                const uint32_t w[16] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w,
                                                        q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
                                float amax = 0.f;
#pragma unroll
                                for (int q = 0; q < 16; q++)
                                    amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(w[q] << 16)),
                                                             fabsf(__uint_as_float(w[q] & 0xffff0000u))));
                                amax = fmaxf(amax, 1e-4f);
                                const float s = pow2_ceil(amax * (1.0f / 448.0f));
#pragma unroll
                                for (int q = 0; q < 16; q++) {
                                    const uint32_t c0 = e4m3_code(fminf(fmaxf(__uint_as_float(w[q] << 16) / s, -448.f), 448.f));
                                    const uint32_t c1 = e4m3_code(fminf(fmaxf(__uint_as_float(w[q] & 0xffff0000u) / s, -448.f), 448.f));
                                    const uint32_t f = e4m3x2_to_f16x2((uint16_t)(c0 | (c1 << 8)));
                                    if (q < 8) fa[q] = f;
                                    else fb[q - 8] = f;
                                }
#pragma unroll
                                for (int q = 0; q < 8; q++) xa[t][q] = fa[q], xb[t][q] = fb[q];
                                sxa[t] = s;
                            }
                        }
                    }
                }
            }
        }

        const int s = j % nst;
        const bool ok = mbar_wait(&full[s], (j / nst) & 1, &abort_flag);
        const unsigned char *st = smem + (size_t)s * stage_bytes;

        // v[(t * RPG + i) * NMAT + m]: this lane's partial of row i, matrix m, token t
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
                        const unsigned char *rowp = st + (size_t)m * RI * rb + (size_t)lr * rb;
                        if (FMT == kFmtFp8B128) {
                            uint32_t fa[8], fb[8];
                            codes16_to_f16(*reinterpret_cast<const uint4 *>(rowp + 16 * pp), fa);
                            codes16_to_f16(*reinterpret_cast<const uint4 *>(rowp + 16 * (pp + Lk)), fb);
                            const float *wsr = static_cast<const float *>(ep.s[mat]) + (size_t)(r / 128) * ((K + 127) / 128);
                            const float swa = __ldg(wsr + (16 * pp) / 128), swb = __ldg(wsr + (16 * (pp + Lk)) / 128);
#pragma unroll
                            for (int t = 0; t < kNT; t++) {
                                if (t < ci.n) {
                                    float ra = 0.f, rb2 = 0.f;
#pragma unroll
                                    for (int q = 0; q < 8; q++) {
                                        ra = dot2_f16_f32(fa[q], xa[t][q], ra);
                                        rb2 = dot2_f16_f32(fb[q], xb[t][q], rb2);
                                    }
                                    v[(t * RPG + i) * NMAT + m] = fmaf(rb2, swb * sxb[t], ra * (swa * sxa[t]));
                                }
                            }
                        } else {
                            const uint4 q4 = *reinterpret_cast<const uint4 *>(rowp + 16 * pp);
                            const uint32_t sb = st[scale_off + (size_t)m * RI * (K / 32) + (size_t)lr * (K / 32) + pp];
                            const uint32_t wq[4] = {q4.x, q4.y, q4.z, q4.w};
                            uint32_t f[16];
#pragma unroll
                            for (int q = 0; q < 4; q++)
#pragma unroll
                                for (int b = 0; b < 4; b++) f[4 * q + b] = e2m1x2_to_f16x2((wq[q] >> (8 * b)) & 0xffu);
                            const float sw = e8m0(sb);
#pragma unroll
                            for (int t = 0; t < kNT; t++) {
                                if (t < ci.n) {
                                    float ra = 0.f, rb2 = 0.f;
#pragma unroll
                                    for (int q = 0; q < 8; q++) {
                                        ra = dot2_f16_f32(f[q], xa[t][q], ra);
                                        rb2 = dot2_f16_f32(f[8 + q], xb[t][q], rb2);
                                    }
                                    v[(t * RPG + i) * NMAT + m] = (ra + rb2) * (sw * sxa[t]);
                                }
                            }
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);

        // reduce the lane partials of the chunk's tokens: per row group, one value per
        // (token, row, matrix), written to this item's reduction buffer
        float *rbuf = red + (j & 1) * kRedHalf;
        const int VN = RV * nt;
        if (Lk >= 32) {
            float r;
            int sh;
            if (nt == 1) r = reduce_prefix<RV * 1>(v, lane), sh = 5 - log2_const<RV * 1>();
            else if (nt == 2) r = reduce_prefix<RV * 2>(v, lane), sh = 5 - log2_const<RV * 2>();
            else r = reduce_prefix<RV * 4>(v, lane), sh = 5 - log2_const<RV * 4>();
            if ((lane & ((1 << sh) - 1)) == 0) rbuf[wc * VN + (lane >> sh)] = r;
        } else {
#pragma unroll
            for (int i = 0; i < V; i++) {
                if (i < VN) {
                    float x = v[i];
                    for (int o = Lk / 2; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
                    if (pp == 0 && active) rbuf[rg * VN + i] = x;
                }
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
        // epilogue: one thread per (row group, row, token)
        for (int q = ct; q < n_rg * RPG * ci.n; q += kConsumerThreads) {
            const int g = q / (RPG * ci.n), i = (q / ci.n) % RPG, t = q % ci.n;
            const int r = r0 + g + n_rg * i;
            if (r >= rows) continue;
            float acc[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; m++) {
                const int vi = (t * RPG + i) * NMAT + m;
                float a = 0.f;
                if (Lk >= 32) {
                    for (int w = 0; w < wpr; w++) a += rbuf[(g * wpr + w) * VN + vi];
                } else {
                    a = rbuf[g * VN + vi];
                }
                acc[m] = a;
            }
            if (UP) {
                float gv = bf16r(acc[0]), uv = bf16r(acc[NMAT - 1]);
                if (p.swiglu_limit > 0.f) {
                    uv = fminf(fmaxf(uv, -p.swiglu_limit), p.swiglu_limit);
                    gv = fminf(gv, p.swiglu_limit);
                }
                const float hv = gv / (1.f + expf(-gv)) * uv * wt[t];
                p.h[(size_t)(ci.pos0 + t) * p.I + r] = f32_to_bf16_bits(hv);
            } else {
                const uint16_t o = f32_to_bf16_bits(acc[0]);
                const int pos = ci.pos0 + t;
                if (ci.e < p.E) p.eo[(size_t)p.perm[pos] * p.H + r] = o;
                else p.sh[(size_t)(pos - p.T * p.topk) * p.H + r] = o;
            }
        }
    }
}

// y[t] = bf16(fp32 sum of eo[t][0..topk-1] in slot order, + shared), eight columns per thread
__global__ void __launch_bounds__(256) combine_kernel(CombineParams p) {
    pdl_wait();
    pdl_launch_dependents();
    if (p.ep.n_ranks > 1) {
        // expert parallelism: this rank's down kernel (before this one) has finished writing into
        // every source rank's eo rows: say so everywhere, then wait until every rank has said so
        __shared__ int ok;
        if (threadIdx.x == 0) {
            if (blockIdx.x == 0) signal_all(p.ep, p.ep.L.done_flag);
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
    *reinterpret_cast<uint4 *>(p.y + (size_t)t * p.H + c) = make_uint4(o[0], o[1], o[2], o[3]);
}

template __global__ void expert_kernel<kFmtFp8B128, true, 2>(ExpertParams, int, int);
template __global__ void expert_kernel<kFmtFp8B128, false, 2>(ExpertParams, int, int);
template __global__ void expert_kernel<kFmtMxfp4, true, 2>(ExpertParams, int, int);
template __global__ void expert_kernel<kFmtMxfp4, false, 2>(ExpertParams, int, int);

// host-side selection of the kernel instantiation for a weight format and direction
const void *expert_kernel_ptr(int fmt, bool up) {
    if (fmt == kFmtFp8B128)
        return up ? (const void *)expert_kernel<kFmtFp8B128, true, 2> : (const void *)expert_kernel<kFmtFp8B128, false, 2>;
    return up ? (const void *)expert_kernel<kFmtMxfp4, true, 2> : (const void *)expert_kernel<kFmtMxfp4, false, 2>;
}

const void *combine_kernel_ptr() { return (const void *)combine_kernel; }

}  // namespace stbl
