// GPU expert cache over a host expert store: the reference's ExpertCache (stbl/model.cu:99-106,
// 347-422) with its demand reads (stbl/model.cu:269-296, 503-520), planned and copied on the GPU.
//
// The reference syncs the stream after routing, runs an LRU list on the host (cached experts of the
// call touched first, then the routed experts in top-k order: a hit moves to the front, a miss takes
// a never-used slot in order or else the least recently used one) and reads the missing experts
// with host threads.  Here the same decisions are made by one CTA right after the router, from the
// routed ids in device memory (no device->host copy): per slot a logical last-use clock stands for
// the list position, so the victims of a call's misses are the least recently used slots in order.
// The layer's expert kernels read the slot of each routed expert from the map row of their layer.
// Missing experts are then copied by a grid of CTAs reading the pinned host store directly
// (device-visible host memory, 16-byte loads, many in flight): the copy, like everything else in
// the call, is ordered on the layer's stream and needs no host thread.
//
// Prefetch (the reference's shadow next-layer guesses, stbl/model.cu:432-475, 555-586): the planner's
// second mode places guessed experts of a coming layer call without touching cached ones (its
// issue(), each new guess takes a never-used slot or the least recently used one and goes to the
// front), and the copy runs on a second stream, beside the current call's expert kernels (the copy
// kernel keeps no shared memory and few registers, so its CTAs fit next to theirs).  A prefetch never
// takes a slot the last demand call used (those experts may still be read), and the next demand call
// waits for the prefetch copy before planning: the guesses have always landed by then, which is the
// reference's case of reads that finished in time (it also cancels guesses not yet started).
#include "../../include/stbl_moe.h"
#include "cache.cuh"
#include "layer.cuh"

#include <algorithm>
#include <stdexcept>
#include <string>

#define CK(x)                                                                                        \
    do {                                                                                             \
        cudaError_t e_ = (x);                                                                        \
        if (e_ != cudaSuccess) throw std::runtime_error(std::string(#x) + ": " + cudaGetErrorString(e_)); \
    } while (0)

namespace stbl {

constexpr int kPlanThreads = 1024;
constexpr int kPlanMaxIds = 4096;     // routed ids per call (max_tokens 256 x topk 16): the planner's shared list
constexpr int kCopyThreads = 256;
constexpr int kCopyChunk = 32768;     // bytes per CTA work item
constexpr int kCopyUnroll = kCopyChunk / (kCopyThreads * 16);

struct CachePlanParams {
    const int *idx;
    int n, layer, E, S;
    int *map, *owner;
    unsigned long long *ts, *ctr;
    int2 *jobs;
    int *n_jobs;
    long long expert_bytes;
    uint32_t *status;
    // prefetch mode: consider the first `consider` distinct ids; pf_flag [S]: filled by a prefetch and
    // not yet routed to (counted as used at its first hit)
    int prefetch, consider;
    unsigned char *pf_flag;
};

struct CacheCopyParams {
    const int2 *jobs;
    const int *n_jobs;
    uint8_t *pool;
    long long slot_bytes;
    long long piece_bytes[6], piece_off[6], host_stride[6];
    long long host_rows;
    const uint8_t *host[6];
    int chunks[6];  // work items of each piece: kCopyChunk bytes, or (blocked scales) 8 row groups of a 128-row tile
    // MXFP4 caches: the scale pieces (3..5) are written in the expert kernel's scale-block layout
    // (per 128 rows x 128 K a 512-byte block, byte l*16 + c*4 + j = scale of row 32c + l, 32-block j)
    int blocked;
    int rows[3], K[3];
};

__device__ __forceinline__ unsigned long long min_u64_warp(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w < v ? w : v;
    }
    return v;
}

// One CTA.  Keys pack (last use, slot): the smallest key is the least recently used slot, ties (never
// used, clock 0) to the lower slot - the reference's sequential fill of fresh slots.
__global__ void __launch_bounds__(kPlanThreads) cache_plan_kernel(CachePlanParams p) {
    extern __shared__ int sm[];
    int *first = sm;                 // [E] first position of each expert in the call
    int *ulist = first + p.E;        // [n] distinct experts in order of first appearance
    __shared__ int wsum[kPlanThreads / 32];
    __shared__ unsigned long long wmin[kPlanThreads / 32];
    __shared__ int s_nu, s_bad;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_wait();
    pdl_launch_dependents();
    if (tid == 0) s_bad = 0;
    for (int e = tid; e < p.E; e += kPlanThreads) first[e] = INT_MAX;
    __syncthreads();
    for (int a = tid; a < p.n; a += kPlanThreads) {
        const int e = __ldcg(p.idx + a);
        if (e >= 0 && e < p.E) atomicMin(&first[e], a);
        else s_bad = 1;
    }
    __syncthreads();
    // ordered compaction: thread tid owns positions [tid c, tid c + c)
    const int c = (p.n + kPlanThreads - 1) / kPlanThreads;
    int mine = 0;
    for (int a = tid * c; a < min(p.n, tid * c + c); a++) {
        const int e = __ldcg(p.idx + a);
        mine += (e >= 0 && e < p.E && first[e] == a);
    }
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int v = wsum[lane];
        int w = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += u;
        }
        wsum[lane] = w - v;  // exclusive
        if (lane == 31) s_nu = w;
    }
    __syncthreads();
    int at = wsum[warp] + incl - mine;
    for (int a = tid * c; a < min(p.n, tid * c + c); a++) {
        const int e = __ldcg(p.idx + a);
        if (e >= 0 && e < p.E && first[e] == a) ulist[at++] = e;
    }
    __syncthreads();
    const int nu = s_nu;
    const unsigned long long base = p.ctr[0];
    int *row = p.map + (size_t)p.layer * p.E;
    // the call's cached experts are touched first (in order), so no miss of this call evicts one;
    // then each hit is touched again in order (the reference moves it to the front twice)
    // prefetch mode: cached guesses are not touched, and only the first `consider` guesses count
    const int nw = p.prefetch ? min(nu, p.consider) : nu;
    const unsigned long long guard = p.prefetch ? p.ctr[4] : base;  // slots with a later use are off limits
    int hits = 0, used = 0;
    for (int i = tid; i < nu && !p.prefetch; i += kPlanThreads) {
        const int s = row[ulist[i]];
        if (s >= 0) {
            p.ts[s] = base + 1 + nu + i, hits++;
            if (p.pf_flag[s]) p.pf_flag[s] = 0, used++;
        }
    }
    // misses, in order: each takes the least recently used slot (every slot this call touched is newer)
    for (int o = 16; o > 0; o >>= 1) hits += __shfl_xor_sync(0xffffffffu, hits, o), used += __shfl_xor_sync(0xffffffffu, used, o);
    if (lane == 0) wsum[warp] = hits | (used << 16);
    __syncthreads();
    int n_hits = 0, n_used = 0;
    for (int w = 0; w < kPlanThreads / 32; w++) n_hits += wsum[w] & 0xFFFF, n_used += wsum[w] >> 16;
    int j = 0;
    for (int i = 0; i < nw; i++) {
        const int e = ulist[i];
        if (row[e] >= 0) continue;  // uniform: row[] changes only below, after a barrier
        unsigned long long best = ~0ull;
        for (int s = tid; s < p.S; s += kPlanThreads) {
            const unsigned long long k = (p.ts[s] << 20) | (unsigned long long)s;
            best = k < best ? k : best;
        }
        best = min_u64_warp(best);
        if (lane == 0) wmin[warp] = best;
        __syncthreads();
        if (warp == 0) {
            unsigned long long v = wmin[lane];
            v = min_u64_warp(v);
            if (lane == 0) {
                const int s = (int)(v & 0xFFFFF);
                if ((v >> 20) > guard) {
                    // demand: every slot is in use by this call, too few slots (checked at attach);
                    // prefetch: the rest would evict experts of the last call: the prefetch stops
                    s_bad = p.prefetch ? 2 : 1;
                } else {
                    const int old = p.owner[s];
                    if (old >= 0) p.map[old] = -1;
                    p.owner[s] = p.layer * p.E + e;
                    row[e] = s;
                    p.ts[s] = p.prefetch ? base + 1 + i : base + 1 + nu + i;
                    p.pf_flag[s] = p.prefetch ? 1 : 0;
                    p.jobs[j] = make_int2(s, p.layer * p.E + e);
                }
            }
        }
        __syncthreads();
        if (s_bad) break;
        j++;
    }
    if (tid == 0) {
        if (p.prefetch) {
            p.ctr[0] = base + 1 + (unsigned long long)nw;
            p.ctr[5] += j;
            p.ctr[7] += (unsigned long long)j * p.expert_bytes;
        } else {
            p.ctr[0] = base + 1 + 2ull * nu;
            p.ctr[1] += n_hits;
            p.ctr[2] += j;
            p.ctr[3] += (unsigned long long)j * p.expert_bytes;
            p.ctr[4] = base;
            p.ctr[6] += n_used;
        }
        *p.n_jobs = j;
        if (s_bad == 1) atomicOr(p.status, kErrBadTable);
    }
}

__global__ void __launch_bounds__(kCopyThreads) cache_copy_kernel(CacheCopyParams p) {
    pdl_wait();
    pdl_launch_dependents();
    const int nj = *(volatile const int *)p.n_jobs;
    int per_job = 0;
#pragma unroll
    for (int q = 0; q < 6; q++) per_job += p.chunks[q];
    const long long items = (long long)nj * per_job;
    for (long long it = blockIdx.x; it < items; it += gridDim.x) {
        const int jb = (int)(it / per_job);
        int r = (int)(it % per_job), q = 0;
        while (q < 5 && r >= p.chunks[q]) r -= p.chunks[q++];
        const int2 job = p.jobs[jb];
        if (p.blocked && q >= 3) {
            // natural [rows][K/32] scales into their blocks, without shared memory: item r = (128-row
            // tile r / 4, group of 8 row groups l); warp w takes row group l = 8 (r % 4) + w, i.e. rows
            // 32 c + l of the tile (c < 4); lane j loads 16 bytes (the 4 words of blocks 4j..4j+3) of each
            // of the 4 rows and writes the 16-byte word (l, kb) of each of its blocks kb
            const int mt = q - 3, kw = p.K[mt] / 32, nkb = p.K[mt] / 128;
            const int tile = r >> 2, l = 8 * (r & 3) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
            const long long hrow = (long long)job.y % p.host_rows;
            const uint8_t *src = p.host[q] + (size_t)hrow * p.host_stride[q] + (size_t)tile * 128 * kw;
            uint8_t *dst = p.pool + (size_t)job.x * p.slot_bytes + p.piece_off[q] + (size_t)tile * nkb * 512;
            for (int jc = lane; jc < kw / 16; jc += 32) {
                uint4 v[4];
#pragma unroll
                for (int c = 0; c < 4; c++) v[c] = *reinterpret_cast<const uint4 *>(src + (size_t)(32 * c + l) * kw + 16 * jc);
                const uint32_t *w0 = &v[0].x, *w1 = &v[1].x, *w2 = &v[2].x, *w3 = &v[3].x;
#pragma unroll
                for (int b = 0; b < 4; b++)
                    *reinterpret_cast<uint4 *>(dst + (size_t)(4 * jc + b) * 512 + l * 16) = make_uint4(w0[b], w1[b], w2[b], w3[b]);
            }
            continue;
        }
        const long long off = (long long)r * kCopyChunk;
        const long long bytes = min((long long)kCopyChunk, p.piece_bytes[q] - off);
        const long long hrow = (long long)job.y % p.host_rows;
        const uint4 *src = reinterpret_cast<const uint4 *>(p.host[q] + (size_t)hrow * p.host_stride[q] + off);
        uint4 *dst = reinterpret_cast<uint4 *>(p.pool + (size_t)job.x * p.slot_bytes + p.piece_off[q] + off);
        const int words = (int)(bytes >> 4);
        uint4 v[kCopyUnroll];
#pragma unroll
        for (int u = 0; u < kCopyUnroll; u++) {
            const int w = threadIdx.x + u * kCopyThreads;
            if (w < words) v[u] = src[w];
        }
#pragma unroll
        for (int u = 0; u < kCopyUnroll; u++) {
            const int w = threadIdx.x + u * kCopyThreads;
            if (w < words) dst[w] = v[u];
        }
    }
}

void launch_pdl_k(const void *fn, dim3 grid, dim3 block, void **args, size_t smem, cudaStream_t st) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CK(cudaLaunchKernelExC(&cfg, fn, args));
}

// the copy of the jobs a planner wrote (jobs / n_jobs), on stream st
void launch_copy(stbl_cache *c, const int2 *jobs, const int *n_jobs, cudaStream_t st, bool pdl) {
    CacheCopyParams cp{};
    cp.jobs = jobs, cp.n_jobs = n_jobs, cp.pool = c->pool, cp.slot_bytes = c->slot_bytes;
    cp.host_rows = c->host_rows;
    cp.blocked = c->fmt == STBL_FMT_MXFP4;
    const int rows[3] = {c->I, c->I, c->H}, ks[3] = {c->H, c->H, c->I};
    for (int q = 0; q < 6; q++) {
        cp.piece_bytes[q] = c->piece_bytes[q], cp.piece_off[q] = c->piece_off[q], cp.host_stride[q] = c->host_stride[q];
        cp.host[q] = c->host[q];
        cp.chunks[q] = (int)((c->piece_bytes[q] + kCopyChunk - 1) / kCopyChunk);
        if (cp.blocked && q >= 3) {
            cp.rows[q - 3] = rows[q - 3], cp.K[q - 3] = ks[q - 3];
            cp.chunks[q] = rows[q - 3] / 128 * 4;
        }
    }
    void *a2[] = {&cp};
    if (pdl) {
        launch_pdl_k((const void *)cache_copy_kernel, dim3(c->copy_ctas), dim3(kCopyThreads), a2, 0, st);
    } else {
        CK(cudaLaunchKernel((const void *)cache_copy_kernel, dim3(c->copy_ctas), dim3(kCopyThreads), a2, 0, st));
    }
}

void launch_cache(stbl_cache *c, int layer, const int *idx, int n, uint32_t *status, cudaStream_t st) {
    if (n < 1 || n > kPlanMaxIds) throw std::runtime_error("routed ids per call out of range for the cache planner");
    // a prefetch copy still running may be filling slots this call reads or evicts
    if (c->pf_pending) CK(cudaStreamWaitEvent(st, c->pf_done, 0));
    CachePlanParams pp{idx, n, layer, c->E, c->S, c->map, c->owner, c->ts, c->ctr, c->jobs, c->n_jobs, c->expert_bytes, status,
                       0, 0, c->pf_flag};
    void *a1[] = {&pp};
    launch_pdl_k((const void *)cache_plan_kernel, dim3(1), dim3(kPlanThreads), a1, sizeof(int) * (c->E + n), st);
    launch_copy(c, c->jobs, c->n_jobs, st, true);
}

void launch_prefetch(stbl_cache *c, int layer, const int *ids, int n, int consider, uint32_t *status, cudaStream_t st,
                     cudaStream_t copy_st) {
    if (n < 1 || n > kPlanMaxIds) throw std::runtime_error("prefetch ids out of range for the cache planner");
    // the previous prefetch's jobs list and slots are reused: its copy must be done
    if (c->pf_pending) CK(cudaStreamWaitEvent(st, c->pf_done, 0));
    CachePlanParams pp{ids, n, layer, c->E, c->S, c->map, c->owner, c->ts, c->ctr, c->pf_jobs, c->pf_n_jobs, c->expert_bytes,
                       status, 1, consider, c->pf_flag};
    void *a1[] = {&pp};
    launch_pdl_k((const void *)cache_plan_kernel, dim3(1), dim3(kPlanThreads), a1, sizeof(int) * (c->E + n), st);
    CK(cudaEventRecord(c->pf_planned, st));
    CK(cudaStreamWaitEvent(copy_st, c->pf_planned, 0));
    launch_copy(c, c->pf_jobs, c->pf_n_jobs, copy_st, false);
    CK(cudaEventRecord(c->pf_done, copy_st));
    c->pf_pending = true;
}

}  // namespace stbl

using namespace stbl;

namespace {

long long piece_size(int fmt, int rows, int k, bool scales) {
    if (fmt == STBL_FMT_FP8_B128)
        return scales ? 4LL * ((rows + 127) / 128) * ((k + 127) / 128) : (long long)rows * k;
    return scales ? (long long)rows * (k / 32) : (long long)rows * (k / 2);
}

int fail(char *err, int errlen, const std::string &m) {
    if (err && errlen > 0) {
        const size_t n = std::min((size_t)errlen - 1, m.size());
        m.copy(err, n);
        err[n] = 0;
    }
    return -1;
}

}  // namespace

extern "C" {

int stbl_cache_create(const stbl_cache_desc *d, stbl_cache **out, char *err, int errlen) {
    stbl_cache *c = nullptr;
    try {
        if (!d || !out) throw std::runtime_error("null argument");
        if (d->n_layers < 1 || d->n_experts < 1 || d->n_experts > 512) throw std::runtime_error("n_layers >= 1, n_experts in 1..512");
        if (d->slots < 0 || d->slots > (1 << 20) - 1) throw std::runtime_error("slots must be in 0..2^20-1");
        if (d->fmt != STBL_FMT_FP8_B128 && d->fmt != STBL_FMT_MXFP4) throw std::runtime_error("bad fmt");
        if (d->hidden <= 0 || d->inter <= 0 || d->hidden % 512 || d->inter % 512)
            throw std::runtime_error("hidden and inter must be multiples of 512");
        if ((long long)d->n_layers * d->n_experts >= (1LL << 31)) throw std::runtime_error("store too large");
        c = new stbl_cache();
        c->L = d->n_layers, c->E = d->n_experts, c->S = d->slots, c->fmt = d->fmt, c->H = d->hidden, c->I = d->inter;
        if (d->host_rows < 0 || d->host_rows > (long long)c->L * c->E) throw std::runtime_error("host_rows must be in 0..n_layers*n_experts");
        c->host_rows = d->host_rows ? d->host_rows : (long long)c->L * c->E;
        CK(cudaGetDevice(&c->dev));
        const int rows[3] = {c->I, c->I, c->H}, ks[3] = {c->H, c->H, c->I};
        long long off = 0;
        for (int q = 0; q < 6; q++) {
            const int mt = q % 3;
            c->piece_bytes[q] = piece_size(c->fmt, rows[mt], ks[mt], q >= 3);
            c->piece_off[q] = off;
            off += (c->piece_bytes[q] + 1023) & ~1023LL;
            c->expert_bytes += c->piece_bytes[q];
            const void *h = q < 3 ? d->host_w[q] : d->host_s[q - 3];
            const long long hs = q < 3 ? d->host_w_stride[q] : d->host_s_stride[q - 3];
            c->host_stride[q] = hs ? hs : c->piece_bytes[q];
            if (!h) throw std::runtime_error("host store pointer missing");
            if (((uintptr_t)h & 15) || (c->host_stride[q] & 15))
                throw std::runtime_error("host store pieces must be 16-byte aligned (base and stride)");
            if (c->host_stride[q] < c->piece_bytes[q]) throw std::runtime_error("host store stride smaller than a piece");
            cudaPointerAttributes pa{};
            CK(cudaPointerGetAttributes(&pa, h));
            if (pa.type != cudaMemoryTypeHost || !pa.devicePointer)
                throw std::runtime_error("host store must be page-locked host memory (cudaHostAlloc / cudaHostRegister)");
            c->host[q] = static_cast<const uint8_t *>(pa.devicePointer);
        }
        c->slot_bytes = off;
        if (c->S == 0) {
            // sized from the device's free memory (the reference sizes its cache from the host's available
            // memory, stbl/model.cu:960-977): all of it but a headroom of max(4 GiB, 5 %), at most one slot
            // per expert of the store
            size_t free_b = 0, total_b = 0;
            CK(cudaMemGetInfo(&free_b, &total_b));
            const long long headroom = std::max<long long>(4LL << 30, (long long)(total_b / 20));
            const long long room = (long long)free_b - headroom;
            c->S = (int)std::min<long long>({room > 0 ? room / c->slot_bytes : 0, (long long)c->L * c->E, (1 << 20) - 1});
            if (c->S < 1) throw std::runtime_error("not enough device memory for an expert cache slot");
        }
        int sms = 0;
        CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c->dev));
        c->copy_ctas = 2 * sms;
        CK(cudaMalloc(&c->pool, (size_t)c->S * c->slot_bytes));
        CK(cudaMalloc(&c->map, sizeof(int) * (size_t)c->L * c->E));
        CK(cudaMemset(c->map, 0xFF, sizeof(int) * (size_t)c->L * c->E));
        CK(cudaMalloc(&c->owner, sizeof(int) * c->S));
        CK(cudaMemset(c->owner, 0xFF, sizeof(int) * c->S));
        CK(cudaMalloc(&c->ts, sizeof(unsigned long long) * c->S));
        CK(cudaMemset(c->ts, 0, sizeof(unsigned long long) * c->S));
        CK(cudaMalloc(&c->ctr, sizeof(unsigned long long) * 8));
        CK(cudaMemset(c->ctr, 0, sizeof(unsigned long long) * 8));
        CK(cudaMalloc(&c->jobs, sizeof(int2) * c->S));
        CK(cudaMalloc(&c->n_jobs, sizeof(int)));
        CK(cudaMemset(c->n_jobs, 0, sizeof(int)));
        CK(cudaMalloc(&c->pf_jobs, sizeof(int2) * c->S));
        CK(cudaMalloc(&c->pf_n_jobs, sizeof(int)));
        CK(cudaMemset(c->pf_n_jobs, 0, sizeof(int)));
        CK(cudaMalloc(&c->pf_flag, c->S));
        CK(cudaMemset(c->pf_flag, 0, c->S));
        CK(cudaEventCreateWithFlags(&c->pf_done, cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&c->pf_planned, cudaEventDisableTiming));
        CK(cudaMalloc(&c->status, sizeof(uint32_t)));
        CK(cudaMemset(c->status, 0, sizeof(uint32_t)));
        CK(cudaDeviceSynchronize());
        *out = c;
        return 0;
    } catch (const std::exception &e) {
        if (c) stbl_cache_destroy(c);
        return fail(err, errlen, e.what());
    }
}

int stbl_cache_layer_desc(const stbl_cache *c, stbl_moe_desc *d) {
    if (!c || !d) return -1;
    d->routed_fmt = c->fmt;
    d->n_slots = c->S;
    d->routed_s_blocked = c->fmt == STBL_FMT_MXFP4;  // the copy writes MXFP4 scales in the block layout
    for (int q = 0; q < 3; q++) {
        d->routed_w[q] = c->pool + c->piece_off[q];
        d->routed_s[q] = c->pool + c->piece_off[q + 3];
        d->routed_w_stride[q] = c->slot_bytes;
        d->routed_s_stride[q] = c->slot_bytes;
    }
    return 0;
}

int stbl_cache_info(const stbl_cache *c, int *slots, uint64_t *slot_bytes) {
    if (!c) return -1;
    if (slots) *slots = c->S;
    if (slot_bytes) *slot_bytes = (uint64_t)c->slot_bytes;
    return 0;
}

int stbl_cache_stats(const stbl_cache *c, uint64_t *hits, uint64_t *misses, uint64_t *bytes) {
    if (!c) return -1;
    unsigned long long v[4];
    if (cudaMemcpy(v, c->ctr, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (hits) *hits = v[1];
    if (misses) *misses = v[2];
    if (bytes) *bytes = v[3];
    return 0;
}

int stbl_cache_prefetch_stats(const stbl_cache *c, uint64_t *prefetched, uint64_t *used, uint64_t *bytes) {
    if (!c) return -1;
    unsigned long long v[8];
    if (cudaMemcpy(v, c->ctr, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (prefetched) *prefetched = v[5];
    if (used) *used = v[6];
    if (bytes) *bytes = v[7];
    return 0;
}

int stbl_cache_prefetch(stbl_cache *c, int layer, const int *ids, int n, int consider, cudaStream_t stream,
                        cudaStream_t copy_stream) {
    try {
        if (!c || !ids) throw std::runtime_error("null argument");
        if (layer < 0 || layer >= c->L) throw std::runtime_error("layer out of the cache's range");
        if (consider < 1) throw std::runtime_error("consider must be >= 1");
        launch_prefetch(c, layer, ids, n, consider, c->status, stream, copy_stream);
        return 0;
    } catch (const std::exception &e) {
        c->err = e.what();
        return -1;
    }
}

int stbl_cache_state(const stbl_cache *c, int *map, int *owner) {
    if (!c) return -1;
    if (map && cudaMemcpy(map, c->map, sizeof(int) * (size_t)c->L * c->E, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (owner && cudaMemcpy(owner, c->owner, sizeof(int) * c->S, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    return 0;
}

void stbl_cache_destroy(stbl_cache *c) {
    if (!c) return;
    cudaDeviceSynchronize();
    cudaFree(c->pool);
    cudaFree(c->map);
    cudaFree(c->owner);
    cudaFree(c->ts);
    cudaFree(c->ctr);
    cudaFree(c->jobs);
    cudaFree(c->n_jobs);
    cudaFree(c->pf_jobs);
    cudaFree(c->pf_n_jobs);
    cudaFree(c->pf_flag);
    cudaFree(c->status);
    if (c->pf_done) cudaEventDestroy(c->pf_done);
    if (c->pf_planned) cudaEventDestroy(c->pf_planned);
    delete c;
}

}  // extern "C"
