// Grouped expert products for MXFP4 routed experts on the 5th-generation tensor cores.
//
// Weights: e2m1 codes (two per byte, even K index in the low nibble) with one e8m0 scale per 32 K
// values; activations: e4m3 codes with one power-of-two scale per 32 (the act_quant rule of the
// reference's MXFP4 path, stbl/kernels.cu:56-63), stored as e8m0.  This is exactly the operand format
// of tcgen05.mma.kind::mxf8f6f4.block_scale (A e2m1, B e4m3, ue8m0 scales per 32): the tensor cores
// apply both scales and accumulate a whole item in fp32 in TMEM, so the epilogue reads each
// accumulator once.  The numerics equal the reference's fp32 sum of dequantized products up to
// summation order (ref/kernel.py:94-102 fp4_gemm).
//
// Items are two 128-row weight tiles x one chunk of up to NTOK token columns (16, or 32 when a call
// has more than 16 tokens: an expert routed to by 17-32 of them then streams its weights once instead
// of twice), two accumulators: for the up product 128 gate rows AND the matching 128 up rows, so
// SwiGLU reads both from TMEM; for the down product 256 consecutive rows of W2.  Two independent accumulators per K step keep the tensor pipe
// busy: measured on one SM, a 128-K block of two matrices (3 scale copies + 8 MMAs) takes about as
// long as a block of one (2 copies + 4 MMAs).
// Stream-K over (item, 256-K unit) pairs, one persistent CTA per SM.  A pipeline stage is one
// 256-K unit: each weight matrix arrives as ONE 4-D TMA box of 128 rows x 2 K blocks (128 contiguous
// bytes of packed codes per row and op; single-K-block boxes read 64-byte row pieces, which streams
// about a third slower from HBM), the activations as one NTOK-row x 2-K-block box.  Six warps:
//   warp 0     producer: lane 0 issues every copy of a stage on the copy engine: the TMA boxes (the
//              packed codes land in the 128-byte swizzled layout the MMA reads, each 16 codes padded
//              to 16 bytes: tensor-map type 16U4_ALIGN16B) and bulk copies of the scales, which are
//              kept in HBM in the layout tcgen05.cp.32x128b.warpx4 spreads over TMEM (weights: per
//              128 rows x 128 K a 512-byte block, byte l * 16 + c * 4 + j = scale of row 32 c + l for
//              the K/32 sub-block j; activations: 16 bytes per row and 128-K block), so one barrier
//              with one transaction count covers the whole stage and no proxy fence is needed
//   warp 1     MMA issuer: per K block, tcgen05.cp of the scale blocks into a TMEM slot, then four
//              block-scaled MMAs per weight matrix (K = 32 each, scale byte j selected in the
//              instruction descriptor)
//   warps 2-5  epilogue: TMEM reads of the item's accumulators, stream-K partials, SwiGLU (up) /
//              outputs (down)
#include "tc8_body.cuh"

#include <algorithm>

namespace stbl {

constexpr int kT4Threads = 192;
constexpr int kT4Acc = 4;            // item accumulators in TMEM (2 x NTOK columns each)
constexpr int kT4Kb = kT4StageKb;    // K blocks per stage (one unit of stream-K)
constexpr int kT4ATile = 128 * 128;  // one K block of one weight matrix in shared memory (unpacked codes)
constexpr int kT4SfSlots = 4;        // scale-factor slots in TMEM, 16 columns each (A0, A1, B)
constexpr int kT4PartialCols = 64;   // floats per row in the stream-K partial buffer (2 x up to 32 columns)

template <bool UP, int NTOK>
struct T4 {
    static_assert(NTOK == 16 || NTOK == 32, "token columns per item: 16 or 32");
    static constexpr int nA = 2;                           // weight tiles per item (up: gate, up; down: 2 x 128 rows)
    static constexpr int BTile = NTOK * 128;               // one K block of activations
    static constexpr int A = nA * kT4Kb * kT4ATile;        // [m][kb][128 rows][128 B]
    static constexpr int B = kT4Kb * BTile;                // [kb][NTOK rows][128 B]
    // scales: [m | B][kb][512 B]; the activations' 512 bytes are the chunk's rows of 16 bytes (32 rows:
    // the tcgen05.cp 32x128b block, scale of token t at lane t, column 0)
    static constexpr int SF = (nA + 1) * kT4Kb * 512;
    static constexpr int stage = (A + B + SF + 1023) / 1024 * 1024;  // 71 KB (16 tokens), 75 KB (32)
    static constexpr int NV = nA * NTOK;                   // accumulator columns per item
    static constexpr int SfBase = kT4Acc * NV;             // first TMEM column of the scale slots
    static constexpr int TmemCols = SfBase + kT4SfSlots * 16 <= 256 ? 256 : 512;
    // chunk entries [chunk_begin, +Chunks) kept in shared memory (three 75 KB stages leave room for 16)
    static constexpr int Chunks = NTOK == 16 ? 192 : 16;
};
static_assert(T4<true, 16>::stage % 1024 == 0 && T4<false, 16>::stage % 1024 == 0 && T4<true, 32>::stage % 1024 == 0,
              "stages must keep 1 KB alignment");

__device__ __forceinline__ uint64_t plain_desc_32x16(const void *p) {
    // K-major, no swizzle: 8-row core matrices of 16-byte rows, 128 bytes apart (SBO), one along K
    const uint64_t a = smem_u32(p);
    return ((a & 0x3FFFFull) >> 4) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(128 >> 4) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::mxf8f6f4.block_scale: A e2m1 (7-9 = 5) or e4m3 (0), B e4m3 (10-12 =
// 0), K-major, N >> 3 at 17-22, scale type ue8m0 (bit 23), M >> 4 at 24-28; the scale byte of the K/32
// sub-block j for B at bits 4-5 and for A at bits 29-30.
template <int NTOK>
__device__ __forceinline__ uint32_t idesc_mx(int j, bool a8) {
    return ((uint32_t)j << 4) | ((a8 ? 0u : 5u) << 7) | ((uint32_t)(NTOK >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24) |
           ((uint32_t)j << 29);
}

__device__ __forceinline__ void umma_mx(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc, uint32_t sfa,
                                        uint32_t sfb) {
    asm volatile(
        "{.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
}

__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, const void *smem) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(plain_desc_32x16(smem)) : "memory");
}

// One CTA's share of the MXFP4 products: CTA `cta` of the `ncta` that run this body.
template <bool UP, int NTOK>
__device__ __forceinline__ void tc4_body(const TcMaps &maps, const TcParams &p, int nst, int cta, int ncta) {
    using S = T4<UP, NTOK>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int K = UP ? p.H : p.I;     // reduction length
    const int rows = UP ? p.I : p.H;  // output rows per matrix (down: H / 256 items of 2 tiles)
    const int nu = K / (128 * kT4Kb);     // units (stages) per item
    const int tiles = UP ? rows / 128 : rows / 256;
    // 128-row weight tile of matrix slot m of item tile t: up, gate (m 0) and up (m 1) rows of tile t;
    // down, the two halves of W2 rows [256 t, 256 t + 256)
    auto tile_row = [&](int t, int m) { return UP ? t : 2 * t + m; };
    unsigned char *stages = smem;                                                   // [nst][A | B | SF]
    int *col_dst = reinterpret_cast<int *>(stages + (size_t)nst * S::stage);        // [2][NTOK] by column
    float *col_w = reinterpret_cast<float *>(col_dst + 2 * NTOK);                  // [2][NTOK]
    Chunk *ctab = reinterpret_cast<Chunk *>(col_w + 2 * NTOK);                      // [S::Chunks] from chunk_begin
    uint64_t *full = reinterpret_cast<uint64_t *>(ctab + S::Chunks);
    uint64_t *empty = full + nst;
    uint64_t *acc_full = empty + nst;
    uint64_t *acc_empty = acc_full + kT4Acc;
    uint64_t *mma_done = acc_empty + kT4Acc;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag, s_chunk_end;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 32) {
        // the tensor maps are kernel parameters: fetch their descriptors while the previous kernel drains
        for (int m = 0; m < S::nA; m++) tma_prefetch_map(&maps.w[m]);
        tma_prefetch_map(&maps.b);
    }
    if (tid == 0) {
        abort_flag = 0;
        // full: the producer lane's arrival with the stage's transaction bytes
        for (int s = 0; s < nst; s++) mbar_init(&full[s], 1), mbar_init(&empty[s], 1);
        for (int a = 0; a < kT4Acc; a++) mbar_init(&acc_full[a], 1), mbar_init(&acc_empty[a], 128);
        mbar_init(mma_done, 1);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(&tmem_base, S::TmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    // The down product's chunk table, weights and weight scales do not depend on the kernel before it
    // (the up product, or the h quantizer): the router wrote the table, and it had finished before this
    // launch began.  So the table is read, and the weights of the first stages requested, before the
    // programmatic wait; the activation tiles and their scales wait for it.
    constexpr bool early = !UP;
    if (!early) {
        pdl_wait();
        pdl_launch_dependents();
    }
    // one round trip: the chunk count and the chunk table (each thread one entry, read concurrently)
    if (tid == 0) s_chunk_end = p.chunk_end >= 0 ? p.chunk_end : *(volatile const int *)p.n_chunks;
    if (tid < S::Chunks && p.chunk_begin + tid < p.chunk_cap) ctab[tid] = load_chunk(p.chunks + p.chunk_begin + tid);
    __syncthreads();
    const int chunk_end = s_chunk_end;
    const long long n_items = (long long)max(0, chunk_end - p.chunk_begin) * tiles;
    const long long n_units = n_items * nu;
    const long long u_lo = n_units * cta / ncta, u_hi = n_units * (cta + 1) / ncta;
    const int lo = (int)(u_lo / nu), hi = u_hi > u_lo ? (int)((u_hi - 1) / nu) + 1 : lo;
    auto u_range = [&](int it, int &ua, int &uz) {
        ua = (int)max(u_lo - (long long)it * nu, 0LL);
        uz = (int)min(u_hi - (long long)it * nu, (long long)nu);
    };
    auto chunk_of = [&](int c) -> TcChunk {
        const Chunk ch = (c - p.chunk_begin < S::Chunks) ? ctab[c - p.chunk_begin] : load_chunk(p.chunks + c);
        return tc_check(p, ch, NTOK);
    };
    const int nkb = K / 128;
    // a unit's copies: the weight boxes and their scale blocks (`early` part), then the activation box
    // and its scales, all on the stage's barrier, which expects their bytes
    auto copy_weights = [&](int s, int tile, int u, bool shared, int z, bool a8) {
        unsigned char *a = stages + (size_t)s * S::stage;
        unsigned char *sf = a + S::A + S::B;
        const uint32_t a_bytes = S::nA * kT4Kb * 128 * (a8 ? 128 : 64);
        mbar_arrive_expect_tx(&full[s], a_bytes + S::B + S::nA * kT4Kb * 512 + kT4Kb * NTOK * 16);
#pragma unroll
        for (int m = 0; m < S::nA; m++)
            tma_load_4d(a + m * kT4Kb * kT4ATile, shared ? &maps.s[m] : &maps.w[m], 0, tile_row(tile, m) * 128, kT4Kb * u, z,
                        &full[s]);
        // the unit's two 512-byte weight-scale blocks per matrix are adjacent
#pragma unroll
        for (int m = 0; m < S::nA; m++)
            bulk_g2s(sf + m * kT4Kb * 512,
                     (shared ? p.sf_s[m] : p.sf_a[m] + (size_t)z * p.sf_a_stride) + ((size_t)tile_row(tile, m) * nkb + kT4Kb * u) * 512,
                     kT4Kb * 512, &full[s]);
    };
    int n_early = 0;  // producer: stages whose weights were requested before the programmatic wait
    if (early) {
        if (tid == 0) {
            for (int it = lo; it < hi && n_early < nst; it++) {
                const TcChunk ch = chunk_of(p.chunk_begin + it / tiles);
                const bool shared = ch.e == p.E;
                int ua, uz;
                u_range(it, ua, uz);
                for (int u = ua; u < uz && n_early < nst; u++, n_early++)
                    copy_weights(n_early, it % tiles, u, shared, shared ? 0 : expert_slot(p, ch.e), shared ? p.s_a8 : p.w_a8);
            }
        }
        pdl_wait();
        pdl_launch_dependents();
    }

    if (warp == 0) {
        // ---------------- producer (lane 0: every copy of a stage, on the copy engine) ----------------
        if (lane == 0) {
            int q = 0;
            bool stop = false;
            for (int it = lo; it < hi && !stop; it++) {
                const int c = p.chunk_begin + it / tiles, tile = it % tiles;
                const TcChunk ch = chunk_of(c);
                const int brow = b_row(p, ch);
                // routed experts from their slots; the shared expert (its own maps and scale blocks) when the
                // layer's shared expert is in a block-scaled format too
                const bool shared = ch.e == p.E;
                const int z = shared ? 0 : expert_slot(p, ch.e);
                const bool a8 = shared ? p.s_a8 : p.w_a8;
                int ua, uz;
                u_range(it, ua, uz);
                for (int u = ua; u < uz; u++, q++) {
                    const int s = q % nst;
                    if (!mbar_wait(&empty[s], ((q / nst) & 1) ^ 1, &abort_flag)) {
                        abort_flag = 1;
                        atomicOr(p.status, kErrWaitTimeout);
                        stop = true;
                        break;
                    }
                    unsigned char *a = stages + (size_t)s * S::stage;
                    unsigned char *sf = a + S::A + S::B;
                    if (q >= n_early) copy_weights(s, tile, u, shared, z, a8);
                    tma_load_3d(a + S::A, &maps.b, 0, brow, kT4Kb * u, &full[s]);
                    // the activation scales: the chunk's NTOK rows of 16 bytes per K block
#pragma unroll
                    for (int g = 0; g < kT4Kb; g++)
                        bulk_g2s(sf + (S::nA * kT4Kb + g) * 512,
                                 p.act_e8 + ((size_t)(kT4Kb * u + g) * p.act_e8_rows + brow) * 16, NTOK * 16, &full[s]);
                }
            }
            // drain: every issued copy must land before the CTA may exit
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
            int q = 0, ia = 0;
            bool stop = false;
            for (int it = lo; it < hi && !stop; it++, ia++) {
                const int acc = ia % kT4Acc;
                if (!mbar_wait(&acc_empty[acc], ((ia / kT4Acc) & 1) ^ 1, &abort_flag)) {
                    stop = true;
                    break;
                }
                int ua, uz;
                u_range(it, ua, uz);
                const uint32_t d = tmem + (uint32_t)(acc * S::NV);
                const TcChunk ch = chunk_of(p.chunk_begin + it / tiles);
                const bool a8 = ch.e == p.E ? p.s_a8 : p.w_a8;
                for (int u = ua; u < uz; u++, q++) {
                    const int s = q % nst;
                    if (!mbar_wait(&full[s], (q / nst) & 1, &abort_flag)) {
                        stop = true;
                        break;
                    }
                    tc_fence_after();
                    const unsigned char *a = stages + (size_t)s * S::stage;
                    const unsigned char *sfs = a + S::A + S::B;
#pragma unroll
                    for (int g = 0; g < kT4Kb; g++) {
                        const uint32_t sf = tmem + (uint32_t)(S::SfBase + ((kT4Kb * q + g) % kT4SfSlots) * 16);
#pragma unroll
                        for (int m = 0; m < S::nA; m++) tmem_cp_sf(sf + 4 * m, sfs + (m * kT4Kb + g) * 512);
                        tmem_cp_sf(sf + 8, sfs + (S::nA * kT4Kb + g) * 512);
#pragma unroll
                        for (int m = 0; m < S::nA; m++)
#pragma unroll
                            for (int j = 0; j < 4; j++)
                                umma_mx(d + m * NTOK, sw128_desc(a + (m * kT4Kb + g) * kT4ATile + 32 * j),
                                        sw128_desc(a + S::A + g * S::BTile + 32 * j), idesc_mx<NTOK>(j, a8), (u > ua || g > 0 || j > 0),
                                        sf + 4 * m, sf + 8);
                    }
                    umma_commit(&empty[s]);
                }
                if (!stop) umma_commit(&acc_full[acc]);
            }
            if (stop) {
                abort_flag = 1;
                atomicOr(p.status, kErrWaitTimeout);
            }
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
        const int et = tid - 64;                 // 0..127
        const int row = 32 * (warp & 3) + lane;  // TMEM lane = tile row
        const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        // the next item's columns: assignment et's column, destination row (h position / eo row), weight
        int pcol = 0, pdst = 0;
        float pwt = 1.f;
        bool pval = false;
        auto prefetch = [&](int it) {
            const int c = p.chunk_begin + it / tiles;
            const TcChunk ch = chunk_of(c);
            pval = et < ch.n;
            if (pval) {
                const int pos = ch.pos0 + et;
                pcol = et, pdst = pos, pwt = 1.f;
                if (ch.e == p.E) {
                    if (!UP) pdst = pos - p.n_routed;  // shared expert: its output row is the token's
                } else {
                    const int a = __ldg(p.perm + pos);
                    if (UP) {
                        pwt = __ldg(p.wts + a);
                        if (p.b_direct) pcol = a / p.topk;  // x read by token: column = token
                    } else {
                        pdst = a;  // eo row
                    }
                }
            }
        };
        // scatter into the column table of buffer buf (all 128 threads; two barriers)
        auto park = [&](int buf) {
            if (et < NTOK) col_dst[buf * NTOK + et] = -1;
            bar_sync(2, 128);
            if (pval) col_dst[buf * NTOK + pcol] = pdst, col_w[buf * NTOK + pcol] = pwt;
            bar_sync(2, 128);
        };
        if (lo < hi) {
            prefetch(lo);
            park(0);
        }
        int ia = 0;
        for (int it = lo; it < hi; it++, ia++) {
            const int buf = (it - lo) & 1;
            const int c = p.chunk_begin + it / tiles, tile = it % tiles;
            const TcChunk ch = chunk_of(c);
            if (!ch.ok && et == 0) atomicOr(p.status, kErrBadTable);
            if (it + 1 < hi) prefetch(it + 1);
            const int acc_i = ia % kT4Acc;
            int ua, uz;
            u_range(it, ua, uz);
            bool ok = mbar_wait(&acc_full[acc_i], (ia / kT4Acc) & 1, &abort_flag);
            float va[NTOK], vb[NTOK];
            if (ok) {
                tc_fence_after();
#pragma unroll
                for (int h = 0; h < NTOK / 16; h++) {
                    float t[16];
                    tmem_ld16(tl + (uint32_t)(acc_i * S::NV + 16 * h), t);
#pragma unroll
                    for (int i = 0; i < 16; i++) va[16 * h + i] = t[i];
                    tmem_ld16(tl + (uint32_t)(acc_i * S::NV + NTOK + 16 * h), t);
#pragma unroll
                    for (int i = 0; i < 16; i++) vb[16 * h + i] = t[i];
                }
                tc_fence_before();
                mbar_arrive(&acc_empty[acc_i]);
            }
            if (bar_sync_or(2, 128, !ok)) {
                if (et == 0) {
                    abort_flag = 1;
                    atomicOr(p.status, kErrWaitTimeout);
                }
                break;
            }
            float *prow = p.partial + ((size_t)cta * 128 + row) * kT4PartialCols;
            if (ua > 0) {
                // the range starts inside this item: publish the partial sums for the CTA that finishes it
                float4 *dst = reinterpret_cast<float4 *>(prow);
#pragma unroll
                for (int j = 0; j < NTOK / 4; j++) dst[j] = make_float4(va[4 * j], va[4 * j + 1], va[4 * j + 2], va[4 * j + 3]);
#pragma unroll
                for (int j = 0; j < NTOK / 4; j++)
                    dst[NTOK / 4 + j] = make_float4(vb[4 * j], vb[4 * j + 1], vb[4 * j + 2], vb[4 * j + 3]);
                __threadfence();
                bar_sync(2, 128);
                if (et == 0) flag_release(p.flags + cta, p.seq);
                if (it + 1 < hi) park(buf ^ 1);
                continue;
            }
            bool got = true;
            for (int cb = cta + 1; cb < ncta; cb++) {
                const long long uc = n_units * cb / ncta;
                if (uc >= (long long)(it + 1) * nu) break;
                if (n_units * (cb + 1) / ncta == uc) continue;  // empty range
                if (et == 0) got = flag_wait(p.flags + cb, p.seq, &abort_flag) && got;
                bar_sync(2, 128);
                const float4 *src = reinterpret_cast<const float4 *>(p.partial + ((size_t)cb * 128 + row) * kT4PartialCols);
#pragma unroll
                for (int j = 0; j < NTOK / 4; j++) {
                    const float4 v = __ldcg(src + j);
                    va[4 * j] += v.x, va[4 * j + 1] += v.y, va[4 * j + 2] += v.z, va[4 * j + 3] += v.w;
                }
#pragma unroll
                for (int j = 0; j < NTOK / 4; j++) {
                    const float4 v = __ldcg(src + NTOK / 4 + j);
                    vb[4 * j] += v.x, vb[4 * j + 1] += v.y, vb[4 * j + 2] += v.z, vb[4 * j + 3] += v.w;
                }
            }
            if (!got) {
                abort_flag = 1;
                atomicOr(p.status, kErrWaitTimeout);
            }
            const int *cdst = col_dst + buf * NTOK;
            const float *cw = col_w + buf * NTOK;
            const int r = tile * 128 + row;
            if (UP) {
                // SwiGLU per column straight from the two accumulators (gate: va, up: vb); h is bf16
                // (stbl/kernels.cu:445-459) and goes to the down product as act_quant per 32 with a
                // power-of-two scale (stbl/kernels.cu:56-63): the 32 rows of this warp are one block,
                // so the block's amax is a warp reduction and h never leaves the SM unquantized
#pragma unroll
                for (int j = 0; j < NTOK; j++) {
                    const int dst = cdst[j];
                    if (dst < 0) continue;  // the same for every thread of the warpgroup
                    float gv = bf16r(va[j]), uv = bf16r(vb[j]);
                    if (p.swiglu_limit > 0.f) {
                        gv = fminf(gv, p.swiglu_limit);
                        uv = fminf(fmaxf(uv, -p.swiglu_limit), p.swiglu_limit);
                    }
                    const float hv = bf16r(gv / (1.f + expf(-gv)) * uv * cw[j]);
                    // the bf16 h itself too (0.2 % of the launch's bytes at T=16): the layer's
                    // activation readback checks the quantization below against the reference rule
                    p.h[(size_t)dst * p.I + r] = f32_to_bf16_bits(hv);
                    float amax = fabsf(hv);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                    amax = fmaxf(amax, 1e-4f);
                    const float s = pow2_ceil(amax * (1.0f / 448.0f));
                    p.hq[(size_t)dst * p.I + r] = e4m3_code(fminf(fmaxf(hv / s, -448.f), 448.f));
                    if (lane == 0) p.he8[((size_t)tile * p.he8_rows + dst) * 16 + (warp & 3)] = (uint8_t)(__float_as_uint(s) >> 23);
                }
            } else {
                // rows 256 tile + row (va) and 256 tile + 128 + row (vb) of W2's output
                const int r0 = tile * 256 + row;
#pragma unroll
                for (int j = 0; j < NTOK; j++)
                    if (j < ch.n) {
                        uint16_t *o = (ch.e == p.E ? p.sh : p.eo) + (size_t)cdst[j] * p.H;
                        o[r0] = f32_to_bf16_bits(va[j]);
                        o[r0 + 128] = f32_to_bf16_bits(vb[j]);
                    }
            }
            if (it + 1 < hi) park(buf ^ 1);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, S::TmemCols);
    }
}

// The MXFP4 launch: the routed experts' MXFP4 products and, on a share of the CTAs, the FP8 shared
// expert's (tc8_body), in one persistent grid, so the shared expert's 44 MB stream alongside the
// routed weights instead of in launches of their own.  The split follows the bytes each side streams
// (known only on the device: the routed chunk count comes from the router); p8 may hold no chunks.
template <bool UP, int NTOK>
__global__ void __launch_bounds__(kT4Threads, 1) expert_tc4_kernel(const __grid_constant__ TcMaps maps8, TcParams p8,
                                                                   int nst8, const __grid_constant__ TcMaps maps4,
                                                                   TcParams p4, int nst4) {
    // the down launch reads the router's chunk count before the programmatic wait: the router had
    // finished before this launch began (each body waits before it reads the kernel before's output)
    if (UP) pdl_wait();
    const int n4c = max(0, (p4.chunk_end >= 0 ? p4.chunk_end : *(volatile const int *)p4.n_chunks) - p4.chunk_begin);
    const int n8c = max(0, p8.chunk_end - p8.chunk_begin);
    // streamed bytes: MXFP4 up 128 x 2 rows x K/2, down 128 x K/2 per tile; FP8 128 x K per tile
    const double b4 = (double)n4c * (UP ? p4.I / 128 : p4.H / 128) * (UP ? 256.0 : 128.0) * (UP ? p4.H : p4.I) / 2;
    const double b8 = (double)n8c * (UP ? p8.I / 64 : p8.H / 128) * 128.0 * (UP ? p8.H : p8.I);
    // a CTA streams FP8 tiles about kRate8 times as fast as MXFP4 ones (measured on the full-size layer:
    // up 5.9 against 3.2-3.4 TB/s, down 5.5 against 3.0), so the split follows bytes / rate
    constexpr double kRate8 = 1.7;
    const int ncta = gridDim.x;
    int c8 = 0;
    if (n8c > 0) c8 = n4c > 0 ? min(ncta - 1, max(1, (int)(ncta * (b8 / kRate8) / (b8 / kRate8 + b4) + 0.5))) : ncta;
    // the FP8 shared expert keeps 16-token items here: the split above is calibrated for them (with 32-
    // token items this launch measured slower at T=64)
    if ((int)blockIdx.x < c8) tc8_body<UP, true, 16>(maps8, p8, nst8, blockIdx.x, c8);  // two-tile items
    else tc4_body<UP, NTOK>(maps4, p4, nst4, blockIdx.x - c8, ncta - c8);
}

template __global__ void expert_tc4_kernel<true, 16>(const __grid_constant__ TcMaps, TcParams, int,
                                                     const __grid_constant__ TcMaps, TcParams, int);
template __global__ void expert_tc4_kernel<false, 16>(const __grid_constant__ TcMaps, TcParams, int,
                                                      const __grid_constant__ TcMaps, TcParams, int);
template __global__ void expert_tc4_kernel<true, 32>(const __grid_constant__ TcMaps, TcParams, int,
                                                     const __grid_constant__ TcMaps, TcParams, int);
template __global__ void expert_tc4_kernel<false, 32>(const __grid_constant__ TcMaps, TcParams, int,
                                                      const __grid_constant__ TcMaps, TcParams, int);

// wide: items of up to 32 token columns (calls of more than 16 tokens), else 16
const void *expert_tc4_kernel_ptr(bool up, bool wide) {
    if (wide) return up ? (const void *)expert_tc4_kernel<true, 32> : (const void *)expert_tc4_kernel<false, 32>;
    return up ? (const void *)expert_tc4_kernel<true, 16> : (const void *)expert_tc4_kernel<false, 16>;
}

// dynamic shared-memory bytes of one launch (1 KB of it aligns the stages); up and down stages are
// equal (two 128-row tiles per item)
template <int NTOK>
int tc4_smem_bytes(int nst) {
    using S = T4<true, NTOK>;
    return nst * S::stage + 4 * (4 * NTOK) + (int)sizeof(Chunk) * S::Chunks + 8 * (2 * nst + 2 * kT4Acc + 1) + 1024;
}

int expert_tc4_smem_bytes(bool up, int nst, bool wide) {
    (void)up;
    return wide ? tc4_smem_bytes<32>(nst) : tc4_smem_bytes<16>(nst);
}

// e8m0 weight scales of slots [z0, z0 + nz) (slot z at src + z * src_stride) into the scale-block
// layout the expert kernel copies: per slot [rows/128][K/128][512 B], byte l*16 + c*4 + j = scale of
// row 32c + l, 32-block j (slot z at dst + z * dst_stride).  Source rows hold K/32 bytes and cover
// rps weight rows each: 1 for MXFP4 ([rows][K/32]), 32 for FP8 with 32x32 blocks ([rows/32][K/32]).
// One thread per 4-byte word.
__global__ void __launch_bounds__(256) sf_repack_kernel(const uint8_t *src, long long src_stride, uint8_t *dst,
                                                        long long dst_stride, int rows, int K, int z0, int nz, int rps) {
    const int nkb = K / 128;
    const long long per_slot = (long long)rows * nkb;  // words
    const long long total = per_slot * nz;
    for (long long w = (long long)blockIdx.x * blockDim.x + threadIdx.x; w < total; w += (long long)gridDim.x * blockDim.x) {
        const int z = z0 + (int)(w / per_slot);
        const long long r = w % per_slot;
        const int blk = (int)(r >> 7), i = (int)(r & 127);
        const int tile = blk / nkb, kb = blk % nkb, l = i >> 2, c = i & 3;
        const int row = tile * 128 + 32 * c + l;
        const uint32_t v = __ldg(reinterpret_cast<const uint32_t *>(src + (size_t)z * src_stride + (size_t)(row / rps) * (K / 32) + kb * 4));
        *reinterpret_cast<uint32_t *>(dst + (size_t)z * dst_stride + (size_t)r * 4) = v;
    }
}

cudaError_t launch_sf_repack(const uint8_t *src, long long src_stride, uint8_t *dst, long long dst_stride, int rows, int K,
                             int z0, int nz, int rps, cudaStream_t st) {
    const long long total = (long long)rows * (K / 128) * nz;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 4096);
    sf_repack_kernel<<<blocks, 256, 0, st>>>(src, src_stride, dst, dst_stride, rows, K, z0, nz, rps);
    return cudaGetLastError();
}

// floats per row of the stream-K partial buffer this kernel needs
int expert_tc4_partial_cols() { return kT4PartialCols; }

}  // namespace stbl
