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
// Work split and roles as in experts_tc.cu (stream-K over (item, 128-K block) units, one persistent
// CTA per SM, six warps):
//   warp 0     producer: lane 0 issues TMA for the weight tile (the packed codes land in the 128-byte
//              swizzled layout the MMA reads, each 16 codes padded to 16 bytes: tensor-map type
//              16U4_ALIGN16B) and the activation tile; all 32 lanes copy the K block's scale words
//              (cp.async) into the stage, in the layout tcgen05.cp.32x128b.warpx4 spreads over TMEM:
//              byte (l * 16 + c * 4 + j) = scale of row 32 c + l for the K/32 sub-block j
//   warp 1     MMA issuer: per K block, tcgen05.cp of the two scale blocks into a TMEM slot, then four
//              block-scaled MMAs (K = 32 each, scale byte j selected in the instruction descriptor)
//   warps 2-5  epilogue: one TMEM read per item, stream-K partials, SwiGLU (up) / outputs (down)
#include "layer.cuh"
#include "tc_common.cuh"
#include "umma.cuh"

namespace stbl {

constexpr int kT4Threads = 192;
constexpr int kT4Acc = 4;            // item accumulators in TMEM (16 columns each)
constexpr int kT4SfSlots = 4;        // scale-factor slots in TMEM (4 columns A + 4 columns B each)
constexpr int kT4SfBase = 64;        // first TMEM column of the scale slots
constexpr int kT4TmemCols = 128;
constexpr int kT4A = 128 * 128;      // weight tile in shared memory (unpacked codes)
constexpr int kT4B = kTcN * 128;     // activation tile
constexpr int kT4Stage = kT4A + kT4B + 512 + 512;  // + scale blocks A and B: 19 KB
constexpr int kT4TxBytes = 128 * 64 + kT4B;          // TMA bytes per stage (packed codes + activations)
constexpr int kT4Batch = 4;          // K blocks requested back to back
constexpr int kT4Chunks = 32;

__device__ __forceinline__ uint64_t plain_desc_32x16(const void *p) {
    // K-major, no swizzle: 8-row core matrices of 16-byte rows, 128 bytes apart (SBO), one along K
    const uint64_t a = smem_u32(p);
    return ((a & 0x3FFFFull) >> 4) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(128 >> 4) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::mxf8f6f4.block_scale: A e2m1 (7-9 = 5), B e4m3 (10-12 = 0),
// K-major, N >> 3 at 17-22, scale type ue8m0 (bit 23), M >> 4 at 24-28; the scale byte of the K/32
// sub-block j for B at bits 4-5 and for A at bits 29-30.
__device__ __forceinline__ uint32_t idesc_mx(int j) {
    return ((uint32_t)j << 4) | (5u << 7) | ((uint32_t)(kTcN >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24) |
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

__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <bool UP>
__global__ void __launch_bounds__(kT4Threads, 1) expert_tc4_kernel(const __grid_constant__ TcMaps maps, TcParams p,
                                                                   int nst) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int K = UP ? p.H : p.I;     // reduction length
    const int rows = UP ? p.I : p.H;  // output rows per matrix
    const int nkb = K / 128, kw = K / 32;  // K blocks; scale bytes per row
    const int tiles = UP ? rows / 64 : rows / 128;
    unsigned char *stages = smem;                                               // [nst][A | B | SFA | SFB]
    float *xacc = reinterpret_cast<float *>(stages + (size_t)nst * kT4Stage);  // [128][17] item sums (up)
    float *slot_w = xacc + 128 * 17;                                            // [2][16]
    int *slot_col = reinterpret_cast<int *>(slot_w + 2 * kTcN);                 // [2][16]
    int *slot_dst = slot_col + 2 * kTcN;                                        // [2][16]
    Chunk *ctab = reinterpret_cast<Chunk *>(slot_dst + 2 * kTcN);               // [kT4Chunks]
    uint64_t *full = reinterpret_cast<uint64_t *>(ctab + kT4Chunks);
    uint64_t *empty = full + nst;
    uint64_t *acc_full = empty + nst;
    uint64_t *acc_empty = acc_full + kT4Acc;
    uint64_t *mma_done = acc_empty + kT4Acc;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        abort_flag = 0;
        // full: the producer lane's transaction arrival + one cp.async arrival per producer lane
        for (int s = 0; s < nst; s++) mbar_init(&full[s], 1 + 32), mbar_init(&empty[s], 1);
        for (int a = 0; a < kT4Acc; a++) mbar_init(&acc_full[a], 1), mbar_init(&acc_empty[a], 128);
        mbar_init(mma_done, 1);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(&tmem_base, kT4TmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    pdl_wait();
    pdl_launch_dependents();
    const int chunk_end = p.chunk_end >= 0 ? p.chunk_end : *(volatile const int *)p.n_chunks;
    const long long n_items = (long long)max(0, chunk_end - p.chunk_begin) * tiles;
    const long long n_units = n_items * nkb;
    const long long u_lo = n_units * blockIdx.x / gridDim.x, u_hi = n_units * (blockIdx.x + 1) / gridDim.x;
    const int lo = (int)(u_lo / nkb), hi = u_hi > u_lo ? (int)((u_hi - 1) / nkb) + 1 : lo;
    auto k_range = [&](int it, int &ka, int &kz) {
        ka = (int)max(u_lo - (long long)it * nkb, 0LL);
        kz = (int)min(u_hi - (long long)it * nkb, (long long)nkb);
    };
    const int c_lo = p.chunk_begin + lo / tiles;
    for (int i = tid; i < kT4Chunks; i += kT4Threads)
        if (lo < hi && c_lo + i <= p.chunk_begin + (hi - 1) / tiles) ctab[i] = p.chunks[c_lo + i];
    __syncthreads();
    auto chunk_of = [&](int c) -> TcChunk {
        const Chunk ch = (c - c_lo < kT4Chunks) ? ctab[c - c_lo] : p.chunks[c];
        return tc_check(p, ch);
    };

    if (warp == 0) {
        // ---------------- producer (lane 0: TMA; all lanes: scale words) ----------------
        if (lane == 0) {
            for (int m = 0; m < 2; m++) tma_prefetch_map(&maps.w[m]);
            tma_prefetch_map(&maps.b);
        }
        int q = 0;
        bool stop = false;
        for (int it = lo; it < hi && !stop; it++) {
            const int c = p.chunk_begin + it / tiles, tile = it % tiles;
            const TcChunk ch = chunk_of(c);
            const int brow = b_row(p, ch);
            const int z = expert_slot(p, ch.e);
            int ka, kz;
            k_range(it, ka, kz);
            // this lane's scale rows: A rows 32 cc + lane (cc = 0..3) of the tile, B row `lane` (< 16)
            const uint8_t *sa[4];
#pragma unroll
            for (int cc = 0; cc < 4; cc++) {
                const int m = 32 * cc + lane;
                const int mat = UP ? (m >> 6) : 0, r = UP ? tile * 64 + (m & 63) : tile * 128 + m;
                sa[cc] = p.w_e8[mat] + (size_t)z * p.w_e8_stride + (size_t)r * kw;
            }
            const uint8_t *sb = p.act_e8 + (size_t)(brow + (lane & 15)) * kw;
            for (int kb0 = ka; kb0 < kz && !stop; kb0 += kT4Batch) {
                const int nb = min(kT4Batch, kz - kb0);
                for (int u = 0; u < nb; u++) {
                    const int qq = q + u;
                    if (!mbar_wait(&empty[qq % nst], ((qq / nst) & 1) ^ 1, &abort_flag)) {
                        if (lane == 0) {
                            abort_flag = 1;
                            atomicOr(p.status, kErrWaitTimeout);
                        }
                        stop = true;
                        break;
                    }
                }
                if (__any_sync(0xffffffffu, stop)) {
                    stop = true;
                    break;
                }
                for (int u = 0; u < nb; u++, q++) {
                    const int s = q % nst, kb = kb0 + u;
                    unsigned char *a = stages + (size_t)s * kT4Stage;
                    if (lane == 0) {
                        mbar_arrive_expect_tx(&full[s], kT4TxBytes);
                        if (UP) {
                            tma_load_3d(a, &maps.w[0], kb * 128, tile * 64, z, &full[s]);
                            tma_load_3d(a + kT4A / 2, &maps.w[1], kb * 128, tile * 64, z, &full[s]);
                        } else {
                            tma_load_3d(a, &maps.w[0], kb * 128, tile * 128, z, &full[s]);
                        }
                        tma_load_2d(a + kT4A, &maps.b, kb * 128, brow, &full[s]);
                    }
                    uint32_t *sfa = reinterpret_cast<uint32_t *>(a + kT4A + kT4B);
                    uint32_t *sfb = sfa + 128;
#pragma unroll
                    for (int cc = 0; cc < 4; cc++) cp_async4(sfa + lane * 4 + cc, sa[cc] + kb * 4);
                    if (lane < 16) cp_async4(sfb + lane * 4, sb + kb * 4);
                    cp_async_arrive(&full[s]);
                }
            }
        }
        // drain: every issued copy must land before the CTA may exit
        if (lane == 0)
            for (int j = max(0, q - nst); j < q; j++) {
                const uint64_t t0 = global_ns();
                while (!mbar_try_wait(&full[j % nst], (j / nst) & 1))
                    if (global_ns() - t0 > kWaitLimitNs) {
                        atomicOr(p.status, kErrCopyTimeout);
                        break;
                    }
            }
        asm volatile("cp.async.wait_all;" ::: "memory");
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
                int ka, kz;
                k_range(it, ka, kz);
                const uint32_t d = tmem + (uint32_t)(acc * kTcN);
                for (int kb = ka; kb < kz; kb++, q++) {
                    const int s = q % nst;
                    if (!mbar_wait(&full[s], (q / nst) & 1, &abort_flag)) {
                        stop = true;
                        break;
                    }
                    fence_proxy_async_smem();  // scale words arrived through cp.async
                    tc_fence_after();
                    const unsigned char *a = stages + (size_t)s * kT4Stage;
                    const uint32_t sf = tmem + (uint32_t)(kT4SfBase + (q % kT4SfSlots) * 8);
                    tmem_cp_sf(sf, a + kT4A + kT4B);
                    tmem_cp_sf(sf + 4, a + kT4A + kT4B + 512);
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        umma_mx(d, sw128_desc(a + 32 * j), sw128_desc(a + kT4A + 32 * j), idesc_mx(j), (kb > ka || j > 0),
                                sf, sf + 4);
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
        int pcol = 0, pdst = 0;
        float pwt = 0.f;
        auto prefetch = [&](int it) {
            const int c = p.chunk_begin + it / tiles;
            const TcChunk ch = chunk_of(c);
            if (et < kTcN) {
                const int pos = ch.pos0 + et;
                pcol = et, pdst = pos, pwt = 1.f;
                if (et < ch.n) {
                    const int a = __ldg(p.perm + pos);
                    if (UP) {
                        pwt = __ldg(p.wts + a);
                        if (p.b_direct) pcol = a / p.topk;
                    } else {
                        pdst = a;  // eo row
                    }
                }
            }
        };
        auto park = [&](int buf) {
            if (et < kTcN) slot_col[buf * kTcN + et] = pcol, slot_dst[buf * kTcN + et] = pdst, slot_w[buf * kTcN + et] = pwt;
        };
        if (lo < hi) {
            prefetch(lo);
            park(0);
        }
        bar_sync(2, 128);
        int ia = 0;
        for (int it = lo; it < hi; it++, ia++) {
            const int buf = (it - lo) & 1;
            const int c = p.chunk_begin + it / tiles, tile = it % tiles;
            const TcChunk ch = chunk_of(c);
            if (!ch.ok && et == 0) atomicOr(p.status, kErrBadTable);
            if (it + 1 < hi) prefetch(it + 1);
            const int acc_i = ia % kT4Acc;
            int ka, kz;
            k_range(it, ka, kz);
            bool ok = mbar_wait(&acc_full[acc_i], (ia / kT4Acc) & 1, &abort_flag);
            float acc[kTcN];
            if (ok) {
                tc_fence_after();
                tmem_ld16(tl + (uint32_t)(acc_i * kTcN), acc);
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
            if (ka > 0) {
                // the range starts inside this item: publish the partial sums for the CTA that finishes it
                float4 *dst = reinterpret_cast<float4 *>(p.partial + ((size_t)blockIdx.x * 128 + row) * kTcN);
#pragma unroll
                for (int j = 0; j < kTcN / 4; j++) dst[j] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
                __threadfence();
                bar_sync(2, 128);
                if (et == 0) flag_release(p.flags + blockIdx.x, p.seq);
                if (it + 1 < hi) park(buf ^ 1);
                bar_sync(2, 128);
                continue;
            }
            bool got = true;
            for (int cb = blockIdx.x + 1; cb < (int)gridDim.x; cb++) {
                const long long uc = n_units * cb / gridDim.x;
                if (uc >= (long long)(it + 1) * nkb) break;
                if (n_units * (cb + 1) / gridDim.x == uc) continue;  // empty range
                if (et == 0) got = flag_wait(p.flags + cb, p.seq, &abort_flag) && got;
                bar_sync(2, 128);
                const float4 *src = reinterpret_cast<const float4 *>(p.partial + ((size_t)cb * 128 + row) * kTcN);
#pragma unroll
                for (int j = 0; j < kTcN / 4; j++) {
                    const float4 v = __ldcg(src + j);
                    acc[4 * j] += v.x, acc[4 * j + 1] += v.y, acc[4 * j + 2] += v.z, acc[4 * j + 3] += v.w;
                }
            }
            if (!got) {
                abort_flag = 1;
                atomicOr(p.status, kErrWaitTimeout);
            }
            const int *scol = slot_col + buf * kTcN, *sdst = slot_dst + buf * kTcN;
            const float *swt = slot_w + buf * kTcN;
            if (UP) {
                // every row's column sums to shared memory; a thread per (gate row, slot) applies SwiGLU
#pragma unroll
                for (int j = 0; j < kTcN; j++) xacc[row * 17 + j] = acc[j];
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
            } else {
                const int r = tile * 128 + row;
#pragma unroll
                for (int j = 0; j < kTcN; j++)
                    if (j < ch.n) p.eo[(size_t)sdst[j] * p.H + r] = f32_to_bf16_bits(acc[j]);
            }
            if (it + 1 < hi) park(buf ^ 1);
            bar_sync(2, 128);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kT4TmemCols);
    }
}

template __global__ void expert_tc4_kernel<true>(const __grid_constant__ TcMaps, TcParams, int);
template __global__ void expert_tc4_kernel<false>(const __grid_constant__ TcMaps, TcParams, int);

const void *expert_tc4_kernel_ptr(bool up) {
    return up ? (const void *)expert_tc4_kernel<true> : (const void *)expert_tc4_kernel<false>;
}

// dynamic shared-memory bytes of one launch (1 KB of it aligns the stages)
int expert_tc4_smem_bytes(int nst) {
    return nst * kT4Stage + 4 * (128 * 17 + 6 * kTcN) + (int)sizeof(Chunk) * kT4Chunks + 8 * (2 * nst + 2 * kT4Acc + 1) + 1024;
}

}  // namespace stbl
