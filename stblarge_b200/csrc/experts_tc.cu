// Grouped expert products on the 5th-generation tensor cores (FP8 128x128-block experts).
//
// Work item: (chunk of <= 16 tokens of one expert, output tile).  One persistent CTA per SM takes a
// contiguous range of items; six warps:
//   warp 0     TMA producer: per 128-K block one stage = a 128-row x 128-byte weight tile and a
//              16-row x 128-byte activation tile, both in the 128-byte swizzle layout;
//   warp 1     MMA issuer: tcgen05.mma kind::f8f6f4, M = 128 weight rows, N = 16 token columns,
//              K = 32 per instruction, four per 128-K block into one of eight TMEM accumulators;
//   warps 2-5  epilogue: read each block's partials from TMEM, apply the fp32 block scales (weight
//              block x activation block: the promotion of ref/kernel.py:85-91) and accumulate in
//              registers; then write the outputs.
// up: the tile is [64 gate rows; 64 up rows]; h = bf16(silu(bf16 g) * bf16 u * w) (stbl/kernels.cu:
//   445-459).  When both 64-row halves of a 128-row group of a chunk have landed, that CTA
//   re-quantizes the group (act_quant per 128, ref/kernel.py:35-45) for the down kernel.
// down: the tile is 128 rows of W2; eo = bf16(W2 q(h)); when the top-k routed experts and the shared
//   expert of a token have all landed on a tile, that CTA writes y = bf16(sum of eo in top-k order +
//   shared) for the tile (stbl/model.cu:589-592).
// Every wait is bounded; a CTA that gives up raises a status bit, drains its copies and MMAs, frees
// its TMEM and returns.
#include "layer.cuh"
#include "tc_params.cuh"
#include "umma.cuh"

namespace stbl {

constexpr int kTcThreads = 192;
constexpr int kTcN = 16;          // token columns per MMA (chunk size)
constexpr int kTcAcc = 8;         // TMEM accumulators (16 columns each)
constexpr int kTcTmemCols = 128;
constexpr int kATile = 128 * 128;
constexpr int kBTile = kTcN * 128;
constexpr int kStage = kATile + kBTile;  // 18 KB, a multiple of the 1 KB swizzle atom

struct TcChunk {
    int e, pos0, n, ok;
};

__device__ __forceinline__ TcChunk tc_chunk(const TcParams &p, int c) {
    const Chunk ch = p.chunks[c];
    TcChunk r{ch.e, ch.pos0, ch.n, 1};
    const int nrouted = p.T * p.topk;
    const bool shared = ch.e == p.E;
    const bool bad = ch.e < 0 || ch.e > p.E || (shared && !p.has_shared) || ch.n < 1 || ch.n > kTcN ||
                     (shared ? (ch.pos0 < nrouted || ch.pos0 + ch.n > nrouted + p.T)
                             : (ch.pos0 < 0 || ch.pos0 + ch.n > nrouted));
    if (bad) r = TcChunk{0, 0, 0, 0};
    return r;
}

__device__ __forceinline__ int tc_token(const TcParams &p, const TcChunk &c, int j) {
    const int pos = c.pos0 + j;
    return c.e < p.E ? p.perm[pos] / p.topk : pos - p.T * p.topk;
}

// first row of the chunk's B tiles: b_direct (x by token): routed chunks (T <= 16) read tokens 0..15
// and use column = token; shared chunks read their own 16 consecutive tokens, column = slot.
// Otherwise (rows by position) the chunk's first position, column = slot.
__device__ __forceinline__ int b_row(const TcParams &p, const TcChunk &ch) {
    if (!p.b_direct) return ch.pos0;
    return ch.e == p.E ? ch.pos0 - p.T * p.topk : 0;
}

template <bool UP>
__global__ void __launch_bounds__(kTcThreads, 1) expert_tc_kernel(const __grid_constant__ TcMaps maps, TcParams p,
                                                                  int nst) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int K = UP ? p.H : p.I;            // reduction length
    const int rows = UP ? p.I : p.H;         // output rows per matrix
    const int nkb = K / 128;
    const int tiles = UP ? rows / 64 : rows / 128;
    unsigned char *stages = smem;                                         // [nst][A tile | B tile]
    float *sx = reinterpret_cast<float *>(stages + (size_t)nst * kStage);  // [16][nkb] activation scales
    float *sw = sx + kTcN * nkb;                                          // [2][nkb] weight scales
    float *xacc = sw + 2 * nkb;                                           // [128][17] item sums
    uint64_t *full = reinterpret_cast<uint64_t *>(xacc + 128 * 17 + 2);
    uint64_t *empty = full + nst;
    uint64_t *acc_full = empty + nst;
    uint64_t *acc_empty = acc_full + kTcAcc;
    uint64_t *mma_done = acc_empty + kTcAcc;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    __shared__ int fin_flag[kTcN + 1];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < nst; s++) mbar_init(&full[s], 1), mbar_init(&empty[s], 1);
        for (int a = 0; a < kTcAcc; a++) mbar_init(&acc_full[a], 1), mbar_init(&acc_empty[a], 128);
        mbar_init(mma_done, 1);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(&tmem_base, kTcTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    pdl_wait();
    pdl_launch_dependents();
    const int chunk_end = p.chunk_end >= 0 ? p.chunk_end : *(volatile const int *)p.n_chunks;
    const long long n_items = (long long)max(0, chunk_end - p.chunk_begin) * tiles;
    const int lo = (int)(n_items * blockIdx.x / gridDim.x), hi = (int)(n_items * (blockIdx.x + 1) / gridDim.x);

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            for (int m = 0; m < 2; m++) tma_prefetch_map(&maps.w[m]), tma_prefetch_map(&maps.s[m]);
            tma_prefetch_map(&maps.b);
            int q = 0;  // running stage counter
            bool stop = false;
            for (int it = lo; it < hi && !stop; it++) {
                const int c = p.chunk_begin + it / tiles, tile = it % tiles;
                const TcChunk ch = tc_chunk(p, c);
                const bool shared = ch.e == p.E;
                const int z = shared ? 0 : ch.e;
                const int brow = b_row(p, ch);
                for (int kb = 0; kb < nkb; kb++, q++) {
                    const int s = q % nst;
                    if (!mbar_wait(&empty[s], ((q / nst) & 1) ^ 1, &abort_flag)) {
                        abort_flag = 1;
                        atomicOr(p.status, kErrWaitTimeout);
                        stop = true;
                        break;
                    }
                    unsigned char *a = stages + (size_t)s * kStage;
                    mbar_arrive_expect_tx(&full[s], kStage);
                    if (UP) {
                        tma_load_3d(a, shared ? &maps.s[0] : &maps.w[0], kb * 128, tile * 64, z, &full[s]);
                        tma_load_3d(a + kATile / 2, shared ? &maps.s[1] : &maps.w[1], kb * 128, tile * 64, z, &full[s]);
                    } else {
                        tma_load_3d(a, shared ? &maps.s[0] : &maps.w[0], kb * 128, tile * 128, z, &full[s]);
                    }
                    tma_load_2d(a + kATile, &maps.b, kb * 128, brow, &full[s]);
                }
            }
            // drain: every issued tile must land before the CTA may exit
            for (int j = max(0, q - nst); j < q; j++) {
                const uint64_t t0 = global_ns();
                while (!mbar_try_wait(&full[j % nst], (j / nst) & 1))
                    if (global_ns() - t0 > kWaitLimitNs) {
                        atomicOr(p.status, kErrCopyTimeout);
                        break;
                    }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f8_f32(128, kTcN);
            const int total = (hi - lo) * nkb;
            for (int q = 0; q < total; q++) {
                const int s = q % nst, b = q % kTcAcc;
                if (!mbar_wait(&full[s], (q / nst) & 1, &abort_flag) ||
                    !mbar_wait(&acc_empty[b], ((q / kTcAcc) & 1) ^ 1, &abort_flag)) {
                    abort_flag = 1;
                    atomicOr(p.status, kErrWaitTimeout);
                    break;
                }
                tc_fence_after();
                const unsigned char *a = stages + (size_t)s * kStage;
#pragma unroll
                for (int k = 0; k < 4; k++)
                    umma_f8(tmem + b * kTcN, sw128_desc(a + 32 * k), sw128_desc(a + kATile + 32 * k), idesc, k > 0);
                umma_commit(&empty[s]);
                umma_commit(&acc_full[b]);
            }
            // every issued MMA completes before TMEM is freed
            umma_commit(mma_done);
            const uint64_t t0 = global_ns();
            while (!mbar_try_wait(mma_done, 0))
                if (global_ns() - t0 > kWaitLimitNs) {
                    atomicOr(p.status, kErrCopyTimeout);
                    break;
                }
        }
    } else {
        // ---------------- epilogue warpgroup (warps 2..5) ----------------
        const int et = tid - 64;                   // 0..127
        const int row = 32 * (warp & 3) + lane;    // TMEM lane = tile row
        const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        int q = 0;
        for (int it = lo; it < hi; it++) {
            const int c = p.chunk_begin + it / tiles, tile = it % tiles;
            const TcChunk ch = tc_chunk(p, c);
            if (!ch.ok && et == 0) atomicOr(p.status, kErrBadTable);
            const bool shared = ch.e == p.E;
            // the item's scales: activation blocks of the 16 B rows, weight blocks of the tile
            bar_sync(2, 128);
            const int brow = b_row(p, ch);
            const int bvalid = p.b_direct && !shared ? p.T : ch.n;  // B rows holding real activations
            for (int u = et; u < kTcN * nkb; u += 128) {
                const int j = u / nkb, kb = u % nkb;
                sx[u] = j < bvalid ? __ldg(p.act_s + (size_t)(brow + j) * p.act_s_stride + kb) : 0.f;
            }
            {
                const int rblk = UP ? (tile * 64) / 128 : tile;
                for (int u = et; u < (UP ? 2 : 1) * nkb; u += 128) {
                    const int m = u / nkb, kb = u % nkb;
                    const float *base = shared ? p.s_scale[m] : p.w_scale[m] + (size_t)ch.e * p.w_scale_stride;
                    sw[u] = __ldg(base + (size_t)rblk * nkb + kb);
                }
            }
            bar_sync(2, 128);
            const int mrow = UP ? (row >> 6) : 0;  // up: rows 64..127 are the up matrix
            float acc[kTcN];
#pragma unroll
            for (int j = 0; j < kTcN; j++) acc[j] = 0.f;
            bool ok = true;
            for (int kb = 0; kb < nkb; kb++, q++) {
                const int b = q % kTcAcc;
                if (!mbar_wait(&acc_full[b], (q / kTcAcc) & 1, &abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                float d[16];
                tmem_ld16(tl + b * kTcN, d);
                tc_fence_before();
                mbar_arrive(&acc_empty[b]);
                const float wsc = sw[mrow * nkb + kb];
#pragma unroll
                for (int j = 0; j < kTcN; j++) acc[j] = fmaf(d[j], wsc * sx[j * nkb + kb], acc[j]);
            }
            if (bar_sync_or(2, 128, !ok)) {
                if (et == 0) {
                    abort_flag = 1;
                    atomicOr(p.status, kErrWaitTimeout);
                }
                break;
            }
            if (UP) {
                // every row's column sums to shared memory; a thread per (gate row, slot) applies SwiGLU
#pragma unroll
                for (int j = 0; j < kTcN; j++) xacc[row * 17 + j] = acc[j];
                bar_sync(2, 128);
                const int i = et & 63, r = tile * 64 + i;
                for (int j = et >> 6; j < ch.n; j += 2) {
                    const int pos = ch.pos0 + j;
                    const int col = p.b_direct && ch.e < p.E ? tc_token(p, ch, j) : j;
                    const float wt = ch.e < p.E ? p.wts[p.perm[pos]] : 1.f;
                    const float gv = bf16r(xacc[i * 17 + col]), uv = bf16r(xacc[(64 + i) * 17 + col]);
                    const float hv = gv / (1.f + expf(-gv)) * uv * wt;
                    p.h[(size_t)pos * p.I + r] = f32_to_bf16_bits(hv);
                }
                bar_sync(2, 128);
                // completion count of the 128-row group; the second half to land re-quantizes it
                if (et == 0) {
                    int f = 0;
                    if (ch.n > 0) {
                        __threadfence();
                        int *cnt = p.hcnt + (size_t)c * (p.I / 128) + tile / 2;
                        if (atomicAdd(cnt, 64) + 64 == 128) {
                            *cnt = 0;
                            __threadfence();
                            f = 1;
                        }
                    }
                    fin_flag[0] = f;
                }
                bar_sync(2, 128);
                if (fin_flag[0]) {
                    const int g = tile / 2;
                    for (int j = warp - 2; j < ch.n; j += 4) {
                        const int pos = ch.pos0 + j;
                        const uint16_t *src = p.h + (size_t)pos * p.I + g * 128;
                        const uint2 xv = __ldcg(reinterpret_cast<const uint2 *>(src + 4 * lane));
                        const float v[4] = {__uint_as_float(xv.x << 16), __uint_as_float(xv.x & 0xffff0000u),
                                            __uint_as_float(xv.y << 16), __uint_as_float(xv.y & 0xffff0000u)};
                        float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
                        amax = fmaxf(warp_max(amax), 1e-4f);
                        const float s = amax * (1.0f / 448.0f);
                        uint32_t codes = 0;
#pragma unroll
                        for (int u = 0; u < 4; u++) codes |= (uint32_t)e4m3_code(fminf(fmaxf(v[u] / s, -448.f), 448.f)) << (8 * u);
                        *reinterpret_cast<uint32_t *>(p.hq + (size_t)pos * p.I + g * 128 + 4 * lane) = codes;
                        if (lane == 0) p.hs[(size_t)pos * (p.I / 128) + g] = s;
                    }
                }
            } else {
                const int r = tile * 128 + row;
#pragma unroll
                for (int j = 0; j < kTcN; j++) {
                    if (j < ch.n) {
                        const int pos = ch.pos0 + j;
                        const uint16_t o = f32_to_bf16_bits(acc[j]);
                        if (ch.e < p.E) p.eo[(size_t)p.perm[pos] * p.H + r] = o;
                        else p.sh[(size_t)(pos - p.T * p.topk) * p.H + r] = o;
                    }
                }
                if (p.fuse_combine) {
                    bar_sync(2, 128);
                    // combine when the last of a token's top-k experts and the shared expert lands here
                    if (et < kTcN) {
                        int f = 0;
                        if (et < ch.n) {
                            __threadfence();
                            int *cnt = p.ccnt + (size_t)tc_token(p, ch, et) * (p.H / 128) + tile;
                            if (atomicAdd(cnt, 1) + 1 == p.topk + p.has_shared) {
                                *cnt = 0;
                                __threadfence();
                                f = 1;
                            }
                        }
                        fin_flag[et] = f;
                    }
                    bar_sync(2, 128);
                    for (int j = 0; j < ch.n; j++) {
                        if (!fin_flag[j]) continue;
                        const int tk = tc_token(p, ch, j);
                        float a = 0.f;
                        for (int sl = 0; sl < p.topk; sl++)
                            a = a + bf16_bits_to_f32(__ldcg(p.eo + ((size_t)tk * p.topk + sl) * p.H + r));
                        if (p.has_shared) a = a + bf16_bits_to_f32(__ldcg(p.sh + (size_t)tk * p.H + r));
                        p.y[(size_t)tk * p.H + r] = f32_to_bf16_bits(a);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTcTmemCols);
    }
}

// x codes and scales of every position (routed assignments in dispatch order, then the shared
// expert's tokens), for the up kernel's activation tiles when T > 16
__global__ void __launch_bounds__(256) gather_kernel(GatherParams p) {
    pdl_wait();
    pdl_launch_dependents();
    const int pos = blockIdx.x;
    const int nrouted = p.T * p.topk;
    const int tok = pos < nrouted ? p.perm[pos] / p.topk : pos - nrouted;
    const uint4 *src = reinterpret_cast<const uint4 *>(p.xq + (size_t)tok * p.H);
    uint4 *dst = reinterpret_cast<uint4 *>(p.xq_pos + (size_t)pos * p.H);
    for (int i = threadIdx.x; i < p.H / 16; i += blockDim.x) dst[i] = __ldg(src + i);
    for (int i = threadIdx.x; i < p.H / 128; i += blockDim.x)
        p.xs_pos[(size_t)pos * (p.H / 128) + i] = __ldg(p.xs + (size_t)tok * p.xs_stride + i);
}

template __global__ void expert_tc_kernel<true>(const __grid_constant__ TcMaps, TcParams, int);
template __global__ void expert_tc_kernel<false>(const __grid_constant__ TcMaps, TcParams, int);

const void *expert_tc_kernel_ptr(bool up) {
    return up ? (const void *)expert_tc_kernel<true> : (const void *)expert_tc_kernel<false>;
}

const void *gather_kernel_ptr() { return (const void *)gather_kernel; }

// dynamic shared-memory bytes of one launch (1 KB of it aligns the stages)
int expert_tc_smem_bytes(bool up, int H, int I, int nst) {
    const int K = up ? H : I, nkb = K / 128;
    return nst * kStage + 4 * (kTcN * nkb + 2 * nkb + 128 * 17 + 2) + 8 * (2 * nst + 2 * kTcAcc + 1) + 1024;
}

}  // namespace stbl
