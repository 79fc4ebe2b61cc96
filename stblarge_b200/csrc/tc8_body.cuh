// FP8 128x128-block expert products on the 5th-generation tensor cores: the per-CTA body shared by
// the FP8 expert kernel (experts_tc.cu) and the mixed MXFP4 + FP8 kernel (experts_tc4.cu).
//
// Work item: (chunk of <= NTOK tokens of one expert, output tile), nkb = K / 128 blocks of K each;
// NTOK = 16, or 32 in calls of more than 16 tokens (two-tile items only: an expert routed to by 17-32
// tokens then streams its weights once; its TMEM holds two accumulator groups instead of four, and
// its activation scales are parked in one buffer so that six stages still fit).
// One persistent CTA per SM takes an equal contiguous range of the (item, K block) units, so no SM
// idles while others finish a last item.  An item cut by a range boundary is finished by the CTA
// holding its first K block (which reaches it last, at the end of its range): the CTAs whose ranges
// start inside the item publish their partial sums first thing and raise a flag; the finishing CTA
// adds them in CTA order.  Publishers never wait, so the waits cannot form a cycle.  Six warps:
//   warp 0     TMA producer: per 128-K block one stage = the item's 128-row x 128-byte weight
//              tile(s) and an NTOK-row x 128-byte activation tile, all in the 128-byte swizzle layout
//              (down: the first stages' weight tiles are requested before the programmatic wait);
//   warp 1     MMA issuer: tcgen05.mma kind::f8f6f4, M = 128 weight rows, N = NTOK token columns
//              (16 for a chunk of at most 16 in a 32-token launch), K = 32 per instruction, four per
//              128-K block, each block into its own TMEM columns;
//              blocks are grouped by four (one completion signal per group), four groups in flight;
//   warps 2-5  epilogue: read a group's four blocks of partials from TMEM in one load, apply the
//              fp32 block scales (weight block x activation block: the promotion of
//              ref/kernel.py:85-91) and accumulate in registers; then write the outputs.
// up: the tile is [64 gate rows; 64 up rows]; h = bf16(silu(bf16 g) * bf16 u * w) (stbl/kernels.cu:
//   445-459).  hquant_kernel then re-quantizes h (act_quant per 128, ref/kernel.py:35-45).  With T2 an
//   up item is 128 gate rows and the matching 128 up rows (two boxes per stage, two accumulator sets),
//   so each epilogue thread holds a row's gate and up sums and applies SwiGLU directly.
// down: the tile is 128 rows of W2; eo = bf16(W2 q(h)); combine_kernel (combine.cu) adds them.  With
//   T2 an item takes two such tiles (256 rows, two boxes per stage, two accumulator sets in TMEM) and
//   the MMA issuer alternates between them: a 128-K block of two tiles costs the tensor pipe about as
//   long as one of one tile (measured on one SM), so the stages are released sooner.
// Every wait is bounded; a CTA that gives up raises a status bit, drains its copies and MMAs, frees
// its TMEM and returns.
#pragma once

#include "layer.cuh"
#include "tc_params.cuh"
#include "umma.cuh"
#include "tc_common.cuh"

namespace stbl {

constexpr int kTcThreads = 192;
constexpr int kTcG = 4;           // 128-K blocks per accumulator group (one TMEM read per group)
constexpr int kTcGroups = 4;      // accumulator groups in TMEM with 16-token items (4 x 4 x 16 columns per tile)
constexpr int kATile = 128 * 128; // one 128-row x 128-byte weight tile (a multiple of the 1 KB swizzle atom)
constexpr int kTcChunks = 192;    // chunk entries [chunk_begin, +192) kept in shared memory (one per thread)
constexpr int kTcBatch = 4;       // K blocks requested back to back (512 contiguous bytes of a weight row)

// Shapes and shared-memory layout of one body instance (T2: two weight tiles per item; NTOK: token
// columns per item).  The 16-token layout is the one the single-width body always had.
template <bool UP, bool T2, int NTOK>
struct Tc8 {
    static_assert(NTOK == 16 || (NTOK == 32 && T2), "32-token items exist in the two-tile forms only");
    static constexpr bool WIDE = NTOK > 16;
    static constexpr int NT = T2 ? 2 : 1;                    // weight tiles per item
    static constexpr int GROUPS = WIDE ? 2 : kTcGroups;      // accumulator groups in TMEM
    static constexpr int BTILE = NTOK * 128;                 // one K block of activations
    static constexpr int STAGE = NT * kATile + BTILE;        // 18 / 34 / 36 KB
    static constexpr int TMEM_COLS = NT * GROUPS * kTcG * NTOK;
    static constexpr int SXB = WIDE ? 1 : 2;                 // buffers of parked activation scales
    static constexpr int XACC = WIDE ? 0 : 128 * 17;         // item sums (single-tile up items)
    static constexpr int CHUNKS = WIDE ? 16 : kTcChunks;     // chunk entries kept in shared memory
    static constexpr int PRE = NTOK * 64 / 128;              // activation scales a thread prefetches (nkb <= 64)
    // dynamic shared-memory bytes (1 KB of it aligns the stages)
    __host__ __device__ static constexpr int smem_bytes(int nkb, int nst) {
        return nst * STAGE + 4 * (SXB * NTOK * nkb + 4 * nkb + XACC + 10 * NTOK) + (int)sizeof(Chunk) * CHUNKS +
               8 * (2 * nst + 2 * GROUPS + 1) + 1024;
    }
};
static_assert(Tc8<true, true, 16>::TMEM_COLS == 512 && Tc8<true, true, 32>::TMEM_COLS == 512 &&
              Tc8<true, false, 16>::TMEM_COLS == 256, "TMEM allocations");

// One CTA's share of an FP8 expert launch: CTA `cta` of the `ncta` that run this body (in a mixed
// launch these number themselves 0..ncta-1).
template <bool UP, bool T2 = false, int NTOK = 16>
__device__ __forceinline__ void tc8_body(const TcMaps &maps, const TcParams &p, int nst, int cta, int ncta) {
    using L = Tc8<UP, T2, NTOK>;
    constexpr int NT = L::NT;                            // weight tiles per item
    constexpr int STAGE = L::STAGE;
    constexpr int TMEM_COLS = L::TMEM_COLS;
    constexpr int GROUPS = L::GROUPS;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int K = UP ? p.H : p.I;            // reduction length
    const int rows = UP ? p.I : p.H;         // output rows per matrix
    const int nkb = K / 128;
    const int tiles = UP ? (T2 ? rows / 128 : rows / 64) : rows / (128 * NT);
    unsigned char *stages = smem;                                         // [nst][A tile(s) | B tile]
    float *sx = reinterpret_cast<float *>(stages + (size_t)nst * STAGE);  // [SXB][NTOK][nkb] activation scales
    float *sw = sx + L::SXB * NTOK * nkb;                                 // [2][2][nkb] weight scales
    float *xacc = sw + 4 * nkb;                                           // [128][17] item sums (XACC)
    float *slot_w = xacc + L::XACC;                                       // [2][NTOK] routing weights
    int *slot_col = reinterpret_cast<int *>(slot_w + 2 * NTOK);           // [2][NTOK] B column of a slot
    int *slot_dst = slot_col + 2 * NTOK;                                  // [2][NTOK] output row of a slot
    int *col_dst = slot_dst + 2 * NTOK;                                   // [2][NTOK] up T2: h row of a column (-1: none)
    float *col_w = reinterpret_cast<float *>(col_dst + 2 * NTOK);         // [2][NTOK] up T2: routing weight of a column
    Chunk *ctab = reinterpret_cast<Chunk *>(col_w + 2 * NTOK);            // [CHUNKS] from chunk_begin
    uint64_t *full = reinterpret_cast<uint64_t *>(ctab + L::CHUNKS);
    uint64_t *empty = full + nst;
    uint64_t *acc_full = empty + nst;
    uint64_t *acc_empty = acc_full + GROUPS;
    uint64_t *mma_done = acc_empty + GROUPS;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag, s_chunk_end;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (p.sel) {
        // one of two launches of different widths: the one the device did not choose for this call
        // returns before it allocates anything (the chosen one then sets up after the wait)
        pdl_wait();
        if (*(volatile const int *)p.sel != p.sel_val) return;
    }
    if (tid == 32) {
        // the tensor maps are kernel parameters: fetch their descriptors while the previous kernel drains
        for (int m = 0; m < 2; m++) tma_prefetch_map(&maps.w[m]), tma_prefetch_map(&maps.s[m]);
        tma_prefetch_map(&maps.b);
    }
    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < nst; s++) mbar_init(&full[s], 1), mbar_init(&empty[s], 1);
        for (int a = 0; a < GROUPS; a++) mbar_init(&acc_full[a], 1), mbar_init(&acc_empty[a], 128);
        mbar_init(mma_done, 1);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(&tmem_base, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    // The down product's chunk table and weights do not depend on the kernel before it (the h
    // quantizer): the router wrote the table, and it had finished before this launch began.  So on one
    // GPU the table is read, and the weight tiles of the first stages requested, before the
    // programmatic wait; only the activation tiles wait for it.
    const bool early = !UP && !p.sel && p.ep.n_ranks <= 1;
    if (!early) {
        pdl_wait();
        pdl_launch_dependents();
    }
    // expert parallelism: every rank's payload rows must have landed in this rank's receive rows
    // before they are read.  The payload kernel before this one has finished, so this rank's flag is
    // raised everywhere now; the producer waits for all of them after it has prefetched its first
    // weight tiles into L2 (weights do not depend on the payload), the epilogue before it reads the
    // rows' weights and origins.
    const bool ep_up = UP && p.ep.n_ranks > 1;
    const unsigned int *pay_flags = ep_up ? reinterpret_cast<const unsigned int *>(p.ep.region[p.ep.rank] + p.ep.L.pay_flag) : nullptr;
    if (ep_up && cta == 0 && tid == 0) signal_all(p.ep, p.ep.L.pay_flag);
    // one round trip: the chunk count and the chunk table (each thread one entry, read concurrently)
    if (tid == 0) s_chunk_end = p.chunk_end >= 0 ? p.chunk_end : *(volatile const int *)p.n_chunks;
    if (tid < L::CHUNKS && p.chunk_begin + tid < p.chunk_cap) ctab[tid] = load_chunk(p.chunks + p.chunk_begin + tid);
    __syncthreads();
    const int chunk_end = s_chunk_end;
    const long long n_items = (long long)max(0, chunk_end - p.chunk_begin) * tiles;
    const long long n_units = n_items * nkb;
    const long long u_lo = n_units * cta / ncta, u_hi = n_units * (cta + 1) / ncta;
    // items [lo, hi) touched by this CTA; item it covers K blocks [ka, kz) of it
    const int lo = (int)(u_lo / nkb), hi = u_hi > u_lo ? (int)((u_hi - 1) / nkb) + 1 : lo;
    auto k_range = [&](int it, int &ka, int &kz) {
        ka = (int)max(u_lo - (long long)it * nkb, 0LL);
        kz = (int)min(u_hi - (long long)it * nkb, (long long)nkb);
    };
    // chunks beyond the shared-memory table are read from global memory
    auto chunk_of = [&](int c) -> TcChunk {
        const Chunk ch = (c - p.chunk_begin < L::CHUNKS) ? ctab[c - p.chunk_begin] : load_chunk(p.chunks + c);
        return tc_check(p, ch, NTOK);
    };
    int n_early = 0;  // producer: stages whose weight tiles were requested before the programmatic wait
    if (early) {
        if (tid == 0) {
            // the first stages in the producer loop's order (each stage's barrier expects the weight
            // and activation bytes; the loop below adds only the activation tile for these)
            for (int it = lo; it < hi && n_early < nst; it++) {
                const int c = p.chunk_begin + it / tiles, tile = it % tiles;
                const TcChunk ch = chunk_of(c);
                const bool shared = ch.e == p.E;
                const int z = shared ? 0 : expert_slot(p, ch.e);
                int ka, kz;
                k_range(it, ka, kz);
                for (int kb = ka; kb < kz && n_early < nst; kb++, n_early++) {
                    unsigned char *a = stages + (size_t)n_early * STAGE;
                    mbar_arrive_expect_tx(&full[n_early], STAGE);
#pragma unroll
                    for (int m = 0; m < NT; m++)
                        tma_load_3d(a + m * kATile, shared ? &maps.s[0] : &maps.w[0], kb * 128, (NT * tile + m) * 128, z,
                                    &full[n_early]);
                }
            }
        }
        pdl_wait();
        pdl_launch_dependents();
    }

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int q = 0;  // running stage counter
            bool stop = false;
            if (ep_up) {
                // the weight tiles of the first stages into L2 while the other ranks' payload arrives
                int n_pf = 0;
                for (int it = lo; it < hi && n_pf < 2 * nst; it++) {
                    const int c = p.chunk_begin + it / tiles, tile = it % tiles;
                    const TcChunk ch = chunk_of(c);
                    const bool shared = ch.e == p.E;
                    const int z = shared ? 0 : expert_slot(p, ch.e);
                    int ka, kz;
                    k_range(it, ka, kz);
                    for (int kb = ka; kb < kz && n_pf < 2 * nst; kb++, n_pf++)
#pragma unroll
                        for (int m = 0; m < 2; m++)
                            tma_prefetch_l2_3d(shared ? &maps.s[m] : &maps.w[m], kb * 128, T2 ? tile * 128 : tile * 64, z);
                }
                if (!wait_flags_sys(pay_flags, p.ep.n_ranks, p.ep.epoch)) {
                    abort_flag = 1;
                    atomicOr(p.status, kErrWaitTimeout);
                    stop = true;
                }
                asm volatile("fence.proxy.async.global;" ::: "memory");  // the rows are read by TMA
            }
            for (int it = lo; it < hi && !stop; it++) {
                const int c = p.chunk_begin + it / tiles, tile = it % tiles;
                const TcChunk ch = chunk_of(c);
                const bool shared = ch.e == p.E;
                const int z = shared ? 0 : expert_slot(p, ch.e);
                const int brow = b_row(p, ch);
                int ka, kz;
                k_range(it, ka, kz);
                // K blocks are requested kTcBatch at a time, once as many stages are free, so that
                // DRAM sees consecutive 128-byte pieces of each weight row together
                for (int kb0 = ka; kb0 < kz && !stop; kb0 += kTcBatch) {
                  const int nb = min(kTcBatch, kz - kb0);
                  for (int u = 0; u < nb; u++) {
                    const int qq = q + u;
                    if (!mbar_wait(&empty[qq % nst], ((qq / nst) & 1) ^ 1, &abort_flag)) {
                        abort_flag = 1;
                        atomicOr(p.status, kErrWaitTimeout);
                        stop = true;
                        break;
                    }
                  }
                  for (int u = 0; u < nb && !stop; u++, q++) {
                    const int s = q % nst, kb = kb0 + u;
                    unsigned char *a = stages + (size_t)s * STAGE;
                    // (the first n_early stages have their weights requested already)
                    if (q >= n_early) mbar_arrive_expect_tx(&full[s], STAGE);
                    if (q < n_early) {
                    } else if (UP && !T2) {
                        tma_load_3d(a, shared ? &maps.s[0] : &maps.w[0], kb * 128, tile * 64, z, &full[s]);
                        tma_load_3d(a + kATile / 2, shared ? &maps.s[1] : &maps.w[1], kb * 128, tile * 64, z, &full[s]);
                    } else if (UP) {
                        // 128 gate rows, then the matching 128 up rows (maps of 128-row boxes)
#pragma unroll
                        for (int m = 0; m < 2; m++)
                            tma_load_3d(a + m * kATile, shared ? &maps.s[m] : &maps.w[m], kb * 128, tile * 128, z, &full[s]);
                    } else {
#pragma unroll
                        for (int m = 0; m < NT; m++)
                            tma_load_3d(a + m * kATile, shared ? &maps.s[0] : &maps.w[0], kb * 128, (NT * tile + m) * 128, z,
                                        &full[s]);
                    }
                    tma_load_2d(a + NT * kATile, &maps.b, kb * 128, brow, &full[s]);
                  }
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
            int q = 0, gq = 0;
            bool stop = false;
            for (int it = lo; it < hi && !stop; it++) {
                int ka, kz;
                k_range(it, ka, kz);
                // 32-token items: a chunk of at most 16 tokens takes N = 16 MMAs, its K blocks packed 16
                // columns apart (the 16-token layout), so the epilogue reads and scales 16 columns
                const bool half = L::WIDE && chunk_of(p.chunk_begin + it / tiles).n <= 16;
                const uint32_t idesc = idesc_f8_f32(128, half ? 16 : NTOK);
                const int bcols = half ? 16 : NTOK;  // TMEM columns between K blocks
                for (int kb0 = ka; kb0 < kz && !stop; kb0 += kTcG, gq++) {
                    const int g = gq % GROUPS;
                    if (!mbar_wait(&acc_empty[g], ((gq / GROUPS) & 1) ^ 1, &abort_flag)) {
                        stop = true;
                        break;
                    }
                    const int nb = min(kTcG, kz - kb0);
                    for (int u = 0; u < nb; u++, q++) {
                        const int s = q % nst;
                        if (!mbar_wait(&full[s], (q / nst) & 1, &abort_flag)) {
                            stop = true;
                            break;
                        }
                        tc_fence_after();
                        const unsigned char *a = stages + (size_t)s * STAGE;
                        // accumulator of (group g, K block u, tile m): columns (g NT + m) kTcG NTOK + u bcols
#pragma unroll
                        for (int m = 0; m < NT; m++) {
                            const uint32_t d = tmem + (uint32_t)((g * NT + m) * kTcG * NTOK + u * bcols);
#pragma unroll
                            for (int k = 0; k < 4; k++)
                                umma_f8(d, sw128_desc(a + m * kATile + 32 * k), sw128_desc(a + NT * kATile + 32 * k), idesc, k > 0);
                        }
                        umma_commit(&empty[s]);
                    }
                    if (!stop) umma_commit(&acc_full[g]);
                }
            }
            if (stop) {
                abort_flag = 1;
                atomicOr(p.status, kErrWaitTimeout);
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
        // Per item: scales and slot metadata of the NEXT item are loaded into registers before this
        // item's accumulators are drained (their latency hides behind the MMAs) and parked in the other
        // half of double-buffered shared arrays afterwards; nothing in the loop waits on global memory.
        const int et = tid - 64;                   // 0..127
        const int row = 32 * (warp & 3) + lane;    // TMEM lane = tile row
        const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        const int nsw = (UP ? 2 : NT) * nkb;
        float px[L::PRE];
        float pw = 0.f;
        int pcol = 0, pdst = 0;
        float pwt = 0.f;
        bool pval = false;
        // loads of item `it` into registers (thread et takes sx entries et, et + 128, ..., one weight scale
        // and, for et < 16, slot et's column, output row and routing weight)
        auto prefetch = [&](int it) {
            const int c = p.chunk_begin + it / tiles, tile = it % tiles;
            const TcChunk ch = chunk_of(c);
            const bool shared = ch.e == p.E;
            const int brow = b_row(p, ch);
            const int bvalid = p.b_direct && !shared ? p.T : ch.n;
#pragma unroll
            for (int k = 0; k < L::PRE; k++) {
                const int u = et + 128 * k;
                const int j = u / nkb, kb = u % nkb;
                px[k] = (u < NTOK * nkb && j < bvalid) ? __ldg(p.act_s + (size_t)(brow + j) * p.act_s_stride + kb) : 0.f;
            }
            if (et < nsw) {
                // up: the gate (m 0) and up (m 1) scales of the tile's 128-row block; down: tile m's block
                const int m = et / nkb, kb = et % nkb;
                const int rblk = UP ? (T2 ? tile : (tile * 64) / 128) : NT * tile + m;
                const int mat = UP ? m : 0;
                const float *base = shared ? p.s_scale[mat] : p.w_scale[mat] + (size_t)expert_slot(p, ch.e) * p.w_scale_stride;
                pw = __ldg(base + (size_t)rblk * nkb + kb);
            }
            if (et < NTOK) {
                const int pos = ch.pos0 + et;
                pcol = et, pdst = pos, pwt = 1.f;
                pval = et < ch.n;
                if (et < ch.n) {
                    if (!shared && p.pos_w) {
                        // expert parallelism: weight and origin of the receive row
                        if (UP) pwt = __ldcg(p.pos_w + pos);
                        else pdst = __ldcg(p.pos_meta + pos);  // source rank << 16 | assignment
                    } else if (!shared) {
                        const int a = __ldg(p.perm + pos);
                        if (UP) {
                            pwt = __ldg(p.wts + a);
                            if (p.b_direct) pcol = a / p.topk;
                        } else {
                            pdst = a;  // eo row
                        }
                    } else if (!UP) {
                        pdst = pos - p.n_routed;  // sh row
                    }
                }
            }
        };
        // (one buffer of activation scales with 32-token items: every thread has finished reading the
        // current item's when park runs, after the accumulation's closing barrier)
        auto park = [&](int buf) {
            const int bx = L::SXB > 1 ? buf : 0;
#pragma unroll
            for (int k = 0; k < L::PRE; k++) {
                const int u = et + 128 * k;
                if (u < NTOK * nkb) sx[bx * NTOK * nkb + u] = px[k];
            }
            if (et < nsw) sw[buf * 2 * nkb + et] = pw;
            if (et < NTOK) slot_col[buf * NTOK + et] = pcol, slot_dst[buf * NTOK + et] = pdst, slot_w[buf * NTOK + et] = pwt;
            if (UP && T2) {
                // the same by column (every column at most once: a token meets an expert at most once)
                if (et < NTOK) col_dst[buf * NTOK + et] = -1;
                bar_sync(2, 128);
                if (et < NTOK && pval) col_dst[buf * NTOK + pcol] = pdst, col_w[buf * NTOK + pcol] = pwt;
            }
        };
        int gq = 0;
        if (ep_up) {
            // pos_w / pos_meta of the receive rows come from the other ranks' payload kernels
            if (et == 0 && !wait_flags_sys(pay_flags, p.ep.n_ranks, p.ep.epoch)) {
                abort_flag = 1;
                atomicOr(p.status, kErrWaitTimeout);
            }
            bar_sync(2, 128);
        }
        if (lo < hi) {
            prefetch(lo);
            park(0);
        }
        bar_sync(2, 128);
        for (int it = lo; it < hi; it++) {
            const int buf = (it - lo) & 1;
            const int c = p.chunk_begin + it / tiles, tile = it % tiles;
            const TcChunk ch = chunk_of(c);
            if (!ch.ok && et == 0) atomicOr(p.status, kErrBadTable);
            const bool half = L::WIDE && ch.n <= 16;  // the MMA issuer's choice for this item
            if (it + 1 < hi) prefetch(it + 1);
            const float *sxb = sx + (L::SXB > 1 ? buf : 0) * NTOK * nkb, *swb = sw + buf * 2 * nkb;
            const int mrow = UP ? (row >> 6) : 0;  // up: rows 64..127 are the up matrix
            float acc2[NT][NTOK];                  // the item's sums, per weight tile
#pragma unroll
            for (int m = 0; m < NT; m++)
#pragma unroll
                for (int j = 0; j < NTOK; j++) acc2[m][j] = 0.f;
            float *acc = acc2[0];
            bool ok = true;
            int ka, kz;
            k_range(it, ka, kz);
            for (int kb0 = ka; kb0 < kz; kb0 += kTcG, gq++) {
                const int g = gq % GROUPS;
                if (!mbar_wait(&acc_full[g], (gq / GROUPS) & 1, &abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (L::WIDE && half) {
                    // a chunk of at most 16 tokens in a 32-token launch: four blocks of 16 columns per
                    // tile, two per 32-column read
#pragma unroll
                    for (int m = 0; m < NT; m++) {
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            float d[32];
                            tmem_ld32(tl + (uint32_t)((g * NT + m) * kTcG * NTOK + 32 * h), d);
                            if (m == NT - 1 && h == 1) {
                                tc_fence_before();
                                mbar_arrive(&acc_empty[g]);
                            }
#pragma unroll
                            for (int uu = 0; uu < 2; uu++) {
                                const int kb = kb0 + 2 * h + uu;
                                if (kb < kz) {
                                    const float wsc = swb[m * nkb + kb];
#pragma unroll
                                    for (int j = 0; j < 16; j++) acc2[m][j] = fmaf(d[uu * 16 + j], wsc * sxb[j * nkb + kb], acc2[m][j]);
                                }
                            }
                        }
                    }
                    continue;
                }
                // a group's kTcG blocks of NTOK columns per tile: four blocks in one 64-column read with
                // 16-token items, one block per 32-column read with 32-token items (registers)
                constexpr int W = NTOK == 16 ? 64 : 32;                // columns per read
                constexpr int LD = kTcG * NTOK / W, BPL = W / NTOK;    // reads per tile, blocks per read
#pragma unroll
                for (int m = 0; m < NT; m++) {
#pragma unroll
                    for (int h = 0; h < LD; h++) {
                        float d[W];
                        if constexpr (W == 64) tmem_ld64(tl + (uint32_t)((g * NT + m) * kTcG * NTOK + W * h), d);
                        else tmem_ld32(tl + (uint32_t)((g * NT + m) * kTcG * NTOK + W * h), d);
                        if (m == NT - 1 && h == LD - 1) {
                            tc_fence_before();
                            mbar_arrive(&acc_empty[g]);
                        }
#pragma unroll
                        for (int uu = 0; uu < BPL; uu++) {
                            const int kb = kb0 + h * BPL + uu;
                            if (kb < kz) {
                                const float wsc = swb[(UP && !T2 ? mrow : m) * nkb + kb];
#pragma unroll
                                for (int j = 0; j < NTOK; j++) acc2[m][j] = fmaf(d[uu * NTOK + j], wsc * sxb[j * nkb + kb], acc2[m][j]);
                            }
                        }
                    }
                }
            }
            if (bar_sync_or(2, 128, !ok)) {
                if (et == 0) {
                    abort_flag = 1;
                    atomicOr(p.status, kErrWaitTimeout);
                }
                break;
            }
            if (ka > 0) {
                // the range starts inside this item: publish the partial sums for the CTA that finishes it
                float4 *dst = reinterpret_cast<float4 *>(p.partial + ((size_t)cta * 128 + row) * (NT * NTOK));
#pragma unroll
                for (int m = 0; m < NT; m++)
#pragma unroll
                    for (int j = 0; j < NTOK / 4; j++)
                        dst[m * (NTOK / 4) + j] = make_float4(acc2[m][4 * j], acc2[m][4 * j + 1], acc2[m][4 * j + 2], acc2[m][4 * j + 3]);
                __threadfence();
                bar_sync(2, 128);
                if (et == 0) flag_release(p.flags + cta, p.seq);
                if (it + 1 < hi) park(buf ^ 1);
                bar_sync(2, 128);
                continue;
            }
            // this CTA holds the item's first K block: add the partials of the CTAs whose ranges start
            // inside the item, in CTA order
            bool got = true;
            for (int c = cta + 1; c < ncta; c++) {
                const long long uc = n_units * c / ncta;
                if (uc >= (long long)(it + 1) * nkb) break;
                if (n_units * (c + 1) / ncta == uc) continue;  // empty range
                if (et == 0) got = flag_wait(p.flags + c, p.seq, &abort_flag) && got;
                bar_sync(2, 128);
                const float4 *src = reinterpret_cast<const float4 *>(p.partial + ((size_t)c * 128 + row) * (NT * NTOK));
#pragma unroll
                for (int m = 0; m < NT; m++)
#pragma unroll
                    for (int j = 0; j < NTOK / 4; j++) {
                        const float4 v = __ldcg(src + m * (NTOK / 4) + j);
                        acc2[m][4 * j] += v.x, acc2[m][4 * j + 1] += v.y, acc2[m][4 * j + 2] += v.z, acc2[m][4 * j + 3] += v.w;
                    }
            }
            if (!got) {
                abort_flag = 1;
                atomicOr(p.status, kErrWaitTimeout);
            }
            const int *scol = slot_col + buf * NTOK, *sdst = slot_dst + buf * NTOK;
            const float *swt = slot_w + buf * NTOK;
            if (UP && T2) {
                // this thread holds row r's gate sums (tile 0) and up sums (tile 1) for every column
                const int *cd = col_dst + buf * NTOK;
                const float *cw = col_w + buf * NTOK;
                const int r = tile * 128 + row;
#pragma unroll
                for (int j = 0; j < NTOK; j++) {
                    const int dst = cd[j];
                    if (dst < 0) continue;
                    float gv = bf16r(acc2[0][j]), uv = bf16r(acc2[NT - 1][j]);
                    if (p.swiglu_limit > 0.f) {
                        gv = fminf(gv, p.swiglu_limit);
                        uv = fminf(fmaxf(uv, -p.swiglu_limit), p.swiglu_limit);
                    }
                    const float hv = gv / (1.f + expf(-gv)) * uv * cw[j];
                    p.h[(size_t)dst * p.I + r] = f32_to_bf16_bits(hv);
                }
            } else if (UP) {
                // every row's column sums to shared memory; a thread per (gate row, slot) applies SwiGLU
#pragma unroll
                for (int j = 0; j < NTOK; j++) xacc[row * 17 + j] = acc[j];
                bar_sync(2, 128);
                const int i = et & 63, r = tile * 64 + i;
                for (int j = et >> 6; j < ch.n; j += 2) {
                    const int col = scol[j];
                    float gv = bf16r(xacc[i * 17 + col]), uv = bf16r(xacc[(64 + i) * 17 + col]);
                    if (p.swiglu_limit > 0.f) {
                        gv = fminf(gv, p.swiglu_limit);
                        uv = fminf(fmaxf(uv, -p.swiglu_limit), p.swiglu_limit);
                    }
                    const float hv = gv / (1.f + expf(-gv)) * uv * swt[j];
                    p.h[(size_t)sdst[j] * p.I + r] = f32_to_bf16_bits(hv);
                }
            } else if constexpr (!L::WIDE) {
                // the item's bf16 outputs [tile m][column j][128 rows] through shared memory (xacc is
                // free in the down product), then 16-byte stores of 8 rows of one column: an eighth of
                // the store instructions, and whole 16-byte pieces over NVLink under expert parallelism
                uint16_t *ob = reinterpret_cast<uint16_t *>(xacc);
                static_assert(NT * 16 * 128 * 2 <= 128 * 17 * 4, "staging fits the item-sum buffer");
#pragma unroll
                for (int m = 0; m < NT; m++)
#pragma unroll
                    for (int j = 0; j < 16; j++) ob[(m * 16 + j) * 128 + row] = f32_to_bf16_bits(acc2[m][j]);
                bar_sync(2, 128);
                const bool remote = ch.e < p.E && p.pos_w;
                for (int c = et; c < NT * 16 * 16; c += 128) {
                    const int m = c >> 8, j = (c >> 4) & 15, q = c & 15;  // tile, column, 8-row piece
                    if (j >= ch.n) continue;
                    const uint4 v = *reinterpret_cast<const uint4 *>(ob + (m * 16 + j) * 128 + q * 8);
                    const int r = (NT * tile + m) * 128 + q * 8;
                    if (remote) {
                        // expert parallelism: straight into the source rank's eo row, over NVLink
                        const int meta = sdst[j], src = meta >> 16, a = meta & 0xffff;
                        if (src < 0 || src >= p.ep.n_ranks || a >= p.T_max_assign) {
                            atomicOr(p.status, kErrBadTable);
                            continue;
                        }
                        uint16_t *out = reinterpret_cast<uint16_t *>(p.ep.region[src] + p.ep.L.eo);
                        *reinterpret_cast<uint4 *>(out + (size_t)a * p.H + r) = v;
                    } else {
                        uint16_t *out = ch.e < p.E ? p.eo : p.sh;
                        *reinterpret_cast<uint4 *>(out + (size_t)sdst[j] * p.H + r) = v;
                    }
                }
            } else {
#pragma unroll
                for (int m = 0; m < NT; m++) {
                    const int r = (NT * tile + m) * 128 + row;
                    if (ch.e < p.E && p.pos_w) {
                        // expert parallelism: straight into the source rank's eo row, over NVLink
#pragma unroll
                        for (int j = 0; j < NTOK; j++)
                            if (j < ch.n) {
                                const int meta = sdst[j], src = meta >> 16, a = meta & 0xffff;
                                if (src < 0 || src >= p.ep.n_ranks || a >= p.T_max_assign) {
                                    if (row == 0) atomicOr(p.status, kErrBadTable);
                                    continue;
                                }
                                uint16_t *out = reinterpret_cast<uint16_t *>(p.ep.region[src] + p.ep.L.eo);
                                out[(size_t)a * p.H + r] = f32_to_bf16_bits(acc2[m][j]);
                            }
                    } else {
                        uint16_t *out = ch.e < p.E ? p.eo : p.sh;
#pragma unroll
                        for (int j = 0; j < NTOK; j++)
                            if (j < ch.n) out[(size_t)sdst[j] * p.H + r] = f32_to_bf16_bits(acc2[m][j]);
                    }
                }
            }
            if (it + 1 < hi) park(buf ^ 1);
            bar_sync(2, 128);
        }
        // expert parallelism: this CTA's output rows went into the source ranks' eo rows
        if (!UP && p.ep.n_ranks > 1) __threadfence_system();
    }
    tc_fence_before();
    __syncthreads();
    if (!UP && p.ep.n_ranks > 1 && tid == 0 && atomicAdd(p.ep_done_ctr, 1u) == (unsigned int)ncta - 1)
        signal_all(p.ep, p.ep.L.done_flag);  // every CTA's rows are visible: the combines may read them
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace stbl
