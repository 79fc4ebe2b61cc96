// Expert parallelism: the count exchange and the payload dispatch of one layer call (the protocol
// is described with EpLayout in layer.cuh).  Replaces the all-to-all pair the reference's design
// notes ask for (dispatch and combine as NCCL all-to-all over NVLink) by stores into peer memory:
// each rank writes its assignments' rows directly into the owning rank's receive rows, in the
// owner's compute order, so the owner needs no receive-side permutation.
#include "ep.cuh"

namespace stbl {

// exclusive scan of one value per thread over a block of NT threads; returns the total
template <int NT>
__device__ int block_scan_excl(int v, int *warp_tot, int &total) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = lane < NT / 32 ? warp_tot[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < NT / 32) warp_tot[lane] = w;
    }
    __syncthreads();
    const int r = (warp ? warp_tot[warp - 1] : 0) + incl - v;
    total = warp_tot[NT / 32 - 1];
    __syncthreads();
    return r;
}

constexpr int kEpCountThreads = 512;  // one thread per expert (E <= kMaxExperts)

__global__ void __launch_bounds__(kEpCountThreads) ep_counts_kernel(EpCountsParams p) {
    __shared__ int warp_tot[kEpCountThreads / 32];
    __shared__ int dst_off[kMaxExperts];
    __shared__ int cnt[kEpMaxRanks * kMaxExperts];  // [source rank][expert] counts of this call
    __shared__ int timed_out;
    const int tid = threadIdx.x;
    const EpView &v = p.ep;
    pdl_wait();  // the router's counts, offsets and permutation
    pdl_launch_dependents();
    if (tid == 0) timed_out = 0, *p.done_ctr = 0;
    const unsigned int tag = v.epoch % 0xffffu + 1u;  // 1..65535, never the zeroed region's 0

    // 1. this rank's counts, tagged with the call, into every rank's inbox row [rank]
    for (int d = 0; d < v.n_ranks; d++) {
        unsigned int *inbox = reinterpret_cast<unsigned int *>(v.region[d] + v.L.inbox) + (size_t)v.rank * p.E;
        for (int e = tid; e < p.E; e += kEpCountThreads) inbox[e] = tag << 16 | (unsigned int)p.counts[e];
    }
    // 2. every rank's row of this rank's inbox, once it carries this call's tag (bounded wait).  A rank
    //    writes its row of call c + 1 only after its combine of call c, so the tag also says that every
    //    rank is done with the buffers of call c that this call's payload and outputs overwrite.
    const unsigned int *own = reinterpret_cast<const unsigned int *>(v.region[v.rank] + v.L.inbox);
    if (tid < p.E) {
        const uint64_t t0 = global_ns();
        for (int s = 0; s < v.n_ranks; s++) {
            unsigned int x;
            for (;;) {
                asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(x) : "l"(own + (size_t)s * p.E + tid) : "memory");
                if ((x >> 16) == tag) break;
                if (global_ns() - t0 > kWaitLimitNs) {
                    timed_out = 1;
                    break;
                }
            }
            cnt[s * kMaxExperts + tid] = (int)(x & 0xffffu);
        }
    }
    __syncthreads();
    if (tid == 0 && timed_out) atomicOr(p.status, kErrWaitTimeout);

    // every expert's total and this rank's place among its sources
    const int e = tid;
    int tot = 0, below = 0;
    if (e < p.E)
        for (int s = 0; s < v.n_ranks; s++) {
            const int c = cnt[s * kMaxExperts + e];
            tot += c;
            if (s < v.rank) below += c;
        }
    int total;
    const int excl = block_scan_excl<kEpCountThreads>(e < p.E ? tot : 0, warp_tot, total);
    // rows of an owner start at its first expert: subtract the scan value there
    __shared__ int seg_base[kEpMaxRanks];
    if (e < p.E && e % p.E_loc == 0) seg_base[e / p.E_loc] = excl;
    __syncthreads();
    if (e < p.E) dst_off[e] = excl - seg_base[e / p.E_loc] + below;
    __syncthreads();

    // 3. receive row of each of this rank's assignments at its owner
    for (int q = tid; q < p.T * p.topk; q += kEpCountThreads) {
        const int a = p.perm[q], ea = p.idx[a];
        p.a_dst[a] = dst_off[ea] + (q - p.offsets[ea]);
    }

    // 4. this rank's compute chunks: the shared expert's tokens, then each local expert's rows (rows
    //    of local expert el start at the sum of the earlier local experts' totals, the same place
    //    the senders computed in step 2)
    const int el = tid;
    int my_tot = 0;
    if (el < p.E_loc)
        for (int s = 0; s < v.n_ranks; s++) my_tot += cnt[s * kMaxExperts + v.rank * p.E_loc + el];
    int rows_total;
    const int base = block_scan_excl<kEpCountThreads>(el < p.E_loc ? my_tot : 0, warp_tot, rows_total);
    int nt_r = p.nt_routed, nt_s = p.nt_shared;
    if (p.adaptive_wide) {
        // 32-token chunks when they save more than a quarter of the 16-token ones (this rank's experts)
        int c16, c32;
        block_scan_excl<kEpCountThreads>(el < p.E_loc ? (my_tot + 15) / 16 : 0, warp_tot, c16);
        block_scan_excl<kEpCountThreads>(el < p.E_loc ? (my_tot + 31) / 32 : 0, warp_tot, c32);
        if (p.has_shared) c16 += (p.T + 15) / 16, c32 += (p.T + 31) / 32;
        const bool wide = 4 * c32 < 3 * c16;
        if (wide) nt_r = nt_s = 32;
        if (tid == 0) *p.wide_sel = wide;
    }
    const int nch = el < p.E_loc ? (my_tot + nt_r - 1) / nt_r : 0;
    int nch_total;
    const int ch0 = block_scan_excl<kEpCountThreads>(nch, warp_tot, nch_total);
    const int ns = p.has_shared ? (p.T + nt_s - 1) / nt_s : 0;
    const bool fits = rows_total <= p.routed_cap;  // always, unless a count exchange went wrong
    if (el < p.E_loc && fits)
        for (int c = 0; c < nch; c++)
            p.chunks[ns + ch0 + c] = Chunk{el, base + c * nt_r, min(nt_r, my_tot - c * nt_r), 0};
    for (int i = tid; i < ns; i += kEpCountThreads)
        p.chunks[i] = Chunk{p.E_loc, p.routed_cap + i * nt_s, min(nt_s, p.T - i * nt_s), 0};
    if (tid == 0) {
        p.n_chunks[0] = ns + (fits ? nch_total : 0);
        p.n_chunks[1] = ns;
        p.n_rows[0] = fits ? rows_total : 0;
        if (!fits) atomicOr(p.status, kErrBadTable);
    }
}

// One warp per row: an assignment's token codes and scales, routing weight and origin go to its
// owner's receive row; the shared expert's rows (this rank's own tokens) to this rank's shared rows.
__global__ void __launch_bounds__(256) ep_payload_kernel(EpPayloadParams p) {
    pdl_wait();  // the receive rows of every assignment (ep_counts_kernel)
    pdl_launch_dependents();
    const EpView &v = p.ep;
    const int lane = threadIdx.x & 31;
    const int nw = gridDim.x * (blockDim.x / 32);
    const int n_assign = p.T * p.topk, n_rows = n_assign + (p.has_shared ? p.T : 0);
    for (int u = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); u < n_rows; u += nw) {
        int t, d, row;
        if (u < n_assign) {
            t = u / p.topk;
            d = __ldg(p.idx + u) / p.E_loc;
            row = __ldg(p.a_dst + u);
            if (row < 0 || row >= p.routed_cap) continue;  // counted as a bad table by ep_counts_kernel
        } else {
            t = u - n_assign;
            d = v.rank;
            row = p.routed_cap + t;
        }
        char *dst = v.region[d];
        const uint4 *src = reinterpret_cast<const uint4 *>(p.xq + (size_t)t * p.H);
        uint4 *dq = reinterpret_cast<uint4 *>(dst + v.L.xq_pos + (size_t)row * p.H);
        for (int i = lane; i < p.H / 16; i += 32) dq[i] = __ldg(src + i);
        float *ds = reinterpret_cast<float *>(dst + v.L.xs_pos) + (size_t)row * (p.H / 128);
        for (int i = lane; i < p.H / 128; i += 32) ds[i] = __ldg(p.xs + (size_t)t * p.xs_stride + i);
        if (lane == 0 && u < n_assign) {
            reinterpret_cast<int *>(dst + v.L.pos_meta)[row] = (v.rank << 16) | u;
            reinterpret_cast<float *>(dst + v.L.pos_w)[row] = __ldg(p.wts + u);
        }
    }
}

cudaError_t launch_ep(const EpCountsParams &cp, const EpPayloadParams &pp, int sms, cudaStream_t st) {
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.stream = st;
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kEpCountThreads);
    EpCountsParams c = cp;
    void *a1[] = {&c};
    cudaError_t e = cudaLaunchKernelExC(&cfg, (const void *)ep_counts_kernel, a1);
    if (e != cudaSuccess) return e;
    EpPayloadParams q = pp;
    void *a2[] = {&q};
    const int rows = q.T * q.topk + (q.has_shared ? q.T : 0);
    cfg.gridDim = dim3(max(1, min(sms, (rows + 7) / 8)));
    cfg.blockDim = dim3(256);
    return cudaLaunchKernelExC(&cfg, (const void *)ep_payload_kernel, a2);
}

}  // namespace stbl
