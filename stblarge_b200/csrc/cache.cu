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
// issue(), each new guess takes a freed slot, a never-used one or the least recently used one and goes
// to the front), and the copy runs on a second stream, beside the current call's expert kernels (one
// CTA per SM of at most 64 registers and no dynamic shared memory fits next to theirs).  A prefetch
// never takes a slot the last demand call used (those experts may still be read).
// Cancellation (the reference's PfJob states, stbl/model.cu:92-97, 319-345, 397-414, 478-494): each
// prefetched slot carries a claim word in device memory, queued -> copying -> landed.  The copy kernel
// claims a job (queued -> copying) before it writes any of its bytes and marks it landed after the last
// one; the next demand planner runs without waiting for that copy and, for the guesses of its own layer
// still queued, cancels the ones it did not route to (the slot is freed and taken first by later
// misses) and takes over the ones it did (queued -> its own copy job, counted as a miss).  Guesses it
// routes to that are being copied or have landed are hits; the call's expert kernels wait for the
// prefetch copy.  Victims skip slots still queued or being copied.  Claims are atomic, so a job is
// either copied whole by the prefetch or not touched by it.
//
// File-backed store (stbl_cache_create_file; the reference's expert tensors kept as file offsets and
// read on a miss, stbl/model.cu:269-308, 940-949, 978-987): the planner writes its jobs into mapped
// page-locked memory, a host step (cudaLaunchHostFunc, on a reader stream joined to the copying stream
// by events) reads the listed experts' GGUF MXFP4 blocks with the reader threads into page-locked
// staging, and the copy kernel converts the staged 17-byte blocks into the slot layout (codes and
// block-layout scales) while it copies them into device memory.  The staging has two buffers, so the
// reads of one round overlap the copy of the one before.  The stream waits for the reads in order, so a call still needs no
// host synchronisation; a prefetch's reads run on its own stream beside the current call's kernels.
// A failed read raises status bit 8 (that call's output is not valid) and marks its slots; the next
// planner drops them from the cache, so a later call that routes to those experts reads them again.
#include "../../include/stbl_moe.h"
#include "cache.cuh"
#include "layer.cuh"
#include "reader.cuh"

#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

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
    // prefetch mode: consider the first `consider` distinct ids; pf_flag [S]: 1 = filled by a prefetch
    // and not yet routed to (counted at its first hit), 2 = freed by a cancelled prefetch
    int prefetch, consider;
    unsigned char *pf_flag;
    // claim words [S] (kPfLanded / kPfQueued / kPfCopying) and landed work items [S] of the prefetch
    // jobs; null for file-backed stores, whose demand calls wait for the prefetch before planning
    unsigned int *pf_state, *pf_items;
    // file-backed store: slots whose read failed (mapped host memory written by the read step) and a
    // flag that any are marked; null otherwise
    unsigned char *bad;
    int *n_bad;
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
    // prefetch copies: the jobs' claim words and landed-item counters (cache_plan_kernel); null for
    // demand copies, which own their slots
    unsigned int *state, *items;
};

// prefetch job claim words (the reference's PfJob::state 0 queued, 1 reading, 2 landed; cancelled and
// taken-on-demand jobs go straight back to kPfLanded, the word of a slot with no job in flight)
constexpr unsigned int kPfLanded = 0, kPfQueued = 1, kPfCopying = 2;

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
__global__ void __launch_bounds__(kPlanThreads, 1) cache_plan_kernel(CachePlanParams p) {
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
    if (p.n_bad) {
        // slots a failed read left behind become free (never used) before anything is planned
        __shared__ int s_any;
        if (tid == 0) s_any = *(volatile int *)p.n_bad;
        __syncthreads();
        if (s_any) {
            volatile unsigned char *bad = p.bad;
            for (int s = tid; s < p.S; s += kPlanThreads)
                if (bad[s]) {
                    const int old = p.owner[s];
                    if (old >= 0) p.map[old] = -1;
                    p.owner[s] = -1, p.ts[s] = 0, p.pf_flag[s] = 0;
                    bad[s] = 0;
                }
            __syncthreads();
            if (tid == 0) *(volatile int *)p.n_bad = 0;
        }
    }
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
    __shared__ int s_taken;
    if (tid == 0) s_taken = 0;
    // demand mode, before anything is touched (stbl/model.cu:478-494): guesses of this layer still
    // queued and not routed to are cancelled (their slots freed); landed guesses of earlier layers are
    // forgotten (a later hit on them is a plain hit)
    int cancelled = 0;
    if (!p.prefetch) {
        for (int s = tid; s < p.S; s += kPlanThreads) {
            if (p.pf_flag[s] != 1) continue;
            const int key = p.owner[s], l = key / p.E, e = key - l * p.E;
            if (l == p.layer && first[e] == INT_MAX) {
                if (p.pf_state && atomicCAS(p.pf_state + s, kPfQueued, kPfLanded) == kPfQueued) {
                    row[e] = -1;
                    p.owner[s] = -1, p.ts[s] = 0, p.pf_flag[s] = 2;
                    cancelled++;
                }
            } else if (l < p.layer && (!p.pf_state || atomicAdd(p.pf_state + s, 0) == kPfLanded)) {
                p.pf_flag[s] = 0;
            }
        }
    }
    __syncthreads();
    // the call's cached experts are touched first (in order), so no miss of this call evicts one;
    // then each hit is touched again in order (the reference moves it to the front twice).  A guess
    // still queued is taken over (stbl/model.cu:404-408): its slot gets this call's copy, a miss.
    // prefetch mode: cached guesses are not touched, and only the first `consider` guesses count
    const int nw = p.prefetch ? min(nu, p.consider) : nu;
    const unsigned long long guard = p.prefetch ? p.ctr[4] : base;  // slots with a later use are off limits
    int hits = 0, landed = 0, reading = 0;
    for (int i = tid; i < nu && !p.prefetch; i += kPlanThreads) {
        const int e = ulist[i], s = row[e];
        if (s < 0) continue;
        p.ts[s] = base + 1 + nu + i;
        if (p.pf_flag[s] != 1) {
            hits++;
            continue;
        }
        p.pf_flag[s] = 0;
        const unsigned int st = p.pf_state ? atomicCAS(p.pf_state + s, kPfQueued, kPfLanded) : kPfLanded;
        if (st == kPfQueued) {
            p.jobs[atomicAdd(&s_taken, 1)] = make_int2(s, p.layer * p.E + e);
        } else {
            hits++;
            if (st == kPfCopying) reading++;
            else landed++;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        hits += __shfl_xor_sync(0xffffffffu, hits, o), landed += __shfl_xor_sync(0xffffffffu, landed, o);
        reading += __shfl_xor_sync(0xffffffffu, reading, o), cancelled += __shfl_xor_sync(0xffffffffu, cancelled, o);
    }
    if (lane == 0) wsum[warp] = hits | (landed << 16), wmin[warp] = (unsigned long long)reading | ((unsigned long long)cancelled << 32);
    __syncthreads();
    int n_hits = 0, n_landed = 0, n_reading = 0, n_cancelled = 0;
    for (int w = 0; w < kPlanThreads / 32; w++) {
        n_hits += wsum[w] & 0xFFFF, n_landed += wsum[w] >> 16;
        n_reading += (int)(wmin[w] & 0xFFFFFFFFu), n_cancelled += (int)(wmin[w] >> 32);
    }
    const int n_taken = s_taken;
    __syncthreads();  // wsum / wmin are reused below
    // misses, in order: each takes a freed slot, else a never-used one (in slot order), else the least
    // recently used one (every slot this call touched is newer); slots a prefetch is still filling are
    // skipped (stbl/model.cu:347-372).  Key = (class, slot): freed 0, never used 1, else last use + 1.
    int j = n_taken;
    for (int i = 0; i < nw; i++) {
        const int e = ulist[i];
        if (row[e] >= 0) continue;  // uniform: row[] changes only below, after a barrier
        unsigned long long best = ~0ull;
        for (int s = tid; s < p.S; s += kPlanThreads) {
            const unsigned char fl = p.pf_flag[s];
            unsigned long long k;
            if (fl == 1 && p.pf_state && atomicAdd(p.pf_state + s, 0) != kPfLanded) k = ~0ull;
            else if (fl == 2) k = (unsigned long long)s;
            else k = ((p.ts[s] + 1) << 20) | (unsigned long long)s;
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
                if ((v >> 20) > guard + 1) {
                    // demand: every slot is in use by this call or being filled (too few slots);
                    // prefetch: the rest would evict experts of the last call: the prefetch stops
                    s_bad = p.prefetch ? 2 : 1;
                } else {
                    const int old = p.owner[s];
                    if (old >= 0) p.map[old] = -1;
                    p.owner[s] = p.layer * p.E + e;
                    row[e] = s;
                    p.ts[s] = p.prefetch ? base + 1 + i : base + 1 + nu + i;
                    p.pf_flag[s] = p.prefetch ? 1 : 0;
                    if (p.prefetch && p.pf_state) p.pf_state[s] = kPfQueued, p.pf_items[s] = 0;
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
            p.ctr[6] += n_landed;
            // jobs the prefetch copy will not write: bytes prefetched counts what it copied
            p.ctr[7] -= (unsigned long long)(n_cancelled + n_taken) * p.expert_bytes;
            p.ctr[8] += n_reading;
            p.ctr[9] += n_cancelled;
            p.ctr[10] += n_taken;
        }
        *p.n_jobs = j;
        if (s_bad == 1) atomicOr(p.status, kErrBadTable);
    }
}

// A prefetch job's item claims it first (queued -> copying; a job already copying goes on, a cancelled
// or taken-over one is skipped); the item that completes the job marks it landed.
__global__ void __launch_bounds__(kCopyThreads, 4) cache_copy_kernel(const __grid_constant__ CacheCopyParams p) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ unsigned int s_go;
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
        if (p.state) {
            __syncthreads();  // s_go of the previous item has been read
            if (threadIdx.x == 0) {
                const unsigned int st = atomicCAS(p.state + job.x, kPfQueued, kPfCopying);
                s_go = st == kPfQueued || st == kPfCopying;
            }
            __syncthreads();
            if (!s_go) continue;
        }
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
        } else {
            const long long off = (long long)r * kCopyChunk;
            const long long bytes = min((long long)kCopyChunk, p.piece_bytes[q] - off);
            const long long hrow = (long long)job.y % p.host_rows;
            const uint4 *src = reinterpret_cast<const uint4 *>(p.host[q] + (size_t)hrow * p.host_stride[q] + off);
            uint4 *dst = reinterpret_cast<uint4 *>(p.pool + (size_t)job.x * p.slot_bytes + p.piece_off[q] + off);
            const int words = (int)(bytes >> 4);
            // two halves of 16 KB per CTA in flight: the kernel stays within 64 registers, so a CTA of it
            // fits beside an expert kernel's CTA on the same SM
#pragma unroll 1
            for (int h = 0; h < 2; h++) {
                uint4 v[kCopyUnroll / 2];
#pragma unroll
                for (int u = 0; u < kCopyUnroll / 2; u++) {
                    const int w = threadIdx.x + (h * kCopyUnroll / 2 + u) * kCopyThreads;
                    if (w < words) v[u] = src[w];
                }
#pragma unroll
                for (int u = 0; u < kCopyUnroll / 2; u++) {
                    const int w = threadIdx.x + (h * kCopyUnroll / 2 + u) * kCopyThreads;
                    if (w < words) dst[w] = v[u];
                }
            }
        }
        if (p.state) {
            __threadfence();  // this item's bytes before the count that may mark the job landed
            __syncthreads();
            if (threadIdx.x == 0 && atomicAdd(p.items + job.x, 1u) == (unsigned int)per_job - 1) {
                __threadfence();
                atomicExch(p.state + job.x, kPfLanded);
            }
        }
    }
}

// ---- file-backed store ---------------------------------------------------------------------------

struct FileStore;

struct FileRound {  // the argument of one read step: round `round` of the demand (0) or prefetch (1) jobs
    stbl_cache *c;
    int round, which;
};

struct FileStore {
    ExpertReader *reader = nullptr;
    std::vector<uint64_t> offset;       // [L][3] file offset of expert 0's gate / up / down blocks
    uint64_t gbytes[3] = {};            // bytes of one expert's matrix in the file (17 per 32 values)
    long long region_off[3] = {}, row_bytes = 0;  // one staged expert: three aligned read regions
    int cap = 0;                        // experts staged per round
    // two staging buffers: round r reads into buffer r % 2 while the copy of round r - 1 converts the other
    uint8_t *stage_alloc = nullptr;     // page-locked allocation holding the staging (small ones need not
                                        // start on a page)
    uint8_t *stage = nullptr, *stage_d = nullptr;       // [2][cap][row_bytes], 4096-aligned (host, device view)
    // per staging buffer, the round's table for the conversion kernel (RoundTab layout: job count, read
    // status, jobs, device address of each staged matrix): written by the read step in page-locked
    // memory, copied to device memory in stream order before the conversion, so the kernel's CTAs
    // never read host memory for it
    char *tab = nullptr, *tab_d = nullptr;
    size_t tab_bytes = 0;
    cudaStream_t rstream = nullptr;     // the read steps run here, ahead of the copies on the caller's stream
    cudaEvent_t ev_plan = nullptr;      // the planner has written the jobs list
    std::vector<cudaEvent_t> ev_read, ev_copy;  // per round: its reads / its copy are done
    unsigned char *bad = nullptr, *bad_d = nullptr;     // [S] slots whose read failed
    int *n_bad = nullptr, *n_bad_d = nullptr;
    int2 *jobs_h[2] = {};               // host views of the demand / prefetch jobs lists
    int *n_jobs_h[2] = {};
    std::vector<FileRound> rounds[2];
    std::atomic<uint64_t> failed_rounds{0};
    std::mutex mu;
    std::string err;
};

// a round's table: n jobs (slot, key) and the device address of each staged matrix [n][3]
struct RoundTab {
    int n;
    uint32_t bad;                  // 1: the round's reads failed
    int pad[2];
    // followed by int2 jobs[cap], then const uint8_t *src[cap][3]
};
__host__ __device__ inline int2 *tab_jobs(char *t) { return reinterpret_cast<int2 *>(t + sizeof(RoundTab)); }
__host__ __device__ inline const uint8_t **tab_src(char *t, int cap) {
    return reinterpret_cast<const uint8_t **>(t + sizeof(RoundTab) + sizeof(int2) * cap);
}
inline size_t tab_size(int cap) { return (sizeof(RoundTab) + (sizeof(int2) + 3 * sizeof(void *)) * cap + 255) & ~(size_t)255; }

struct FileCopyParams {
    char *tab;                     // this round's table (device memory)
    int cap;
    uint32_t *status;
    uint8_t *pool;
    long long slot_bytes, piece_off[6];
    int K[3], tiles[3];            // gate, up: K = hidden, I / 128 tiles; down: K = inter, H / 128 tiles
};

// 16 GGUF MXFP4 blocks (272 bytes: per block the e8m0 scale, then values i and 16 + i in the low and
// high nibble of byte i, as 17 uint4 words) -> 256 bytes of codes (values 2j, 2j + 1 in byte j, low
// nibble first) in codes[16] and the 16 scales as four words of the scale-block layout in sw[4]
__device__ __forceinline__ void convert_group(const uint4 *src, uint4 (&codes)[16], uint32_t (&sw)[4]) {
    uint32_t w[69];
#pragma unroll
    for (int i = 0; i < 17; i++) {
        const uint4 v = src[i];
        w[4 * i] = v.x, w[4 * i + 1] = v.y, w[4 * i + 2] = v.z, w[4 * i + 3] = v.w;
    }
    w[68] = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) sw[i] = 0u;
#pragma unroll
    for (int b = 0; b < 16; b++) {
        const int o = 17 * b;
        sw[b >> 2] |= ((w[o >> 2] >> (8 * (o & 3))) & 0xFFu) << (8 * (b & 3));
        uint32_t q[4];
#pragma unroll
        for (int m = 0; m < 4; m++) {
            const int ob = o + 1 + 4 * m;
            q[m] = (ob & 3) ? __funnelshift_r(w[ob >> 2], w[(ob >> 2) + 1], 8 * (ob & 3)) : w[ob >> 2];
        }
        // a | a >> 4 puts the nibble pairs (2j, 2j + 1) into bytes 0 and 2; the permute keeps those
        auto pack = [](uint32_t a, uint32_t c) { return __byte_perm(a | (a >> 4), c | (c >> 4), 0x6420); };
        const uint32_t l0 = q[0] & 0x0F0F0F0Fu, l1 = q[1] & 0x0F0F0F0Fu, l2 = q[2] & 0x0F0F0F0Fu, l3 = q[3] & 0x0F0F0F0Fu;
        const uint32_t h0 = (q[0] >> 4) & 0x0F0F0F0Fu, h1 = (q[1] >> 4) & 0x0F0F0F0Fu, h2 = (q[2] >> 4) & 0x0F0F0F0Fu,
                       h3 = (q[3] >> 4) & 0x0F0F0F0Fu;
        codes[b] = make_uint4(pack(l0, l1), pack(l2, l3), pack(h0, h1), pack(h2, h3));
    }
}

constexpr int kFileWarps = 2;                        // warps per CTA of the conversion
constexpr int kFileGroupBytes = 272;                 // 16 GGUF blocks: 512 values of one row
constexpr int kFileRunBytes = 32 * kFileGroupBytes;  // the 32 consecutive groups a warp converts at a time

// The staged GGUF rows of one matrix are one contiguous array of 272-byte groups (group u = row
// u / G, groups g = u % G of K / 512 per row), and the slot's codes of that matrix one contiguous
// array of 256-byte groups in the same order.  A warp takes 32 consecutive groups (8,704 bytes): it
// reads them from page-locked host memory with coalesced 512-byte loads (lane l the 16 bytes at
// 16 l of each), parks them in its shared-memory buffer, converts group `lane` from there, parks the
// 8 KB of codes back (rotated by lane so the 16-byte stores hit distinct banks) and writes them to the
// slot with coalesced 512-byte stores; the four scale words of each group go to the scale-block
// layout directly.  Host memory sees only whole 512-byte requests.  The round's table (job count,
// read status, jobs, where each staged matrix starts) is read from device memory: read from mapped host
// memory by every CTA, the same few host lines halved the conversion rate (measured with 592 CTAs:
// 24.8 GB/s, against 50.9 GB/s from device memory; the link's ceiling is 51.4 GB/s).
__global__ void __launch_bounds__(kFileWarps * 32) cache_file_copy_kernel(FileCopyParams p) {
    extern __shared__ uint4 fsm[];
    const RoundTab *tab = reinterpret_cast<const RoundTab *>(p.tab);
    if (tab->bad) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(p.status, kErrRead);
        return;
    }
    const int n = min(tab->n, p.cap);
    if (n <= 0) return;
    const int2 *s_jobs = tab_jobs(p.tab);
    const uint8_t *const *s_src = tab_src(p.tab, p.cap);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint4 *buf = fsm + (size_t)warp * (kFileRunBytes / 16);
    int runs[3];
#pragma unroll
    for (int q = 0; q < 3; q++) runs[q] = p.tiles[q] * 128 * (p.K[q] / 512) / 32;
    const int per_job = runs[0] + runs[1] + runs[2];
    const long long total = (long long)n * per_job;
    for (long long wj = (long long)blockIdx.x * kFileWarps + warp; wj < total; wj += (long long)gridDim.x * kFileWarps) {
        const int j = (int)(wj / per_job);
        int run = (int)(wj % per_job), q = 0;
        while (q < 2 && run >= runs[q]) run -= runs[q++];
        const int2 job = s_jobs[j];
        const int K = p.K[q], G = K / 512;
        const uint4 *src = reinterpret_cast<const uint4 *>(s_src[j * 3 + q] + (size_t)run * kFileRunBytes);
#pragma unroll
        for (int k = 0; k < 17; k++) buf[k * 32 + lane] = __ldg(src + k * 32 + lane);
        __syncwarp();
        uint4 codes[16];
        uint32_t sw[4];
        convert_group(buf + lane * 17, codes, sw);
        __syncwarp();
        // codes of group `lane` into the buffer, 16-byte unit b at lane * 16 + ((b + lane) & 15)
#pragma unroll
        for (int b = 0; b < 16; b++) buf[lane * 16 + ((b + lane) & 15)] = codes[b];
        __syncwarp();
        uint8_t *slot = p.pool + (size_t)job.x * p.slot_bytes;
        uint4 *dst = reinterpret_cast<uint4 *>(slot + p.piece_off[q] + (size_t)run * (32 * 256));
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const int U = k * 32 + lane, gl = U >> 4, b = U & 15;  // unit b of the run's group gl
            dst[U] = buf[gl * 16 + ((b + gl) & 15)];
        }
        // the group's 16 scales: four words of the scale-block layout of its row's 128-row tile
        const int u = run * 32 + lane, r = u / G, g = u % G;
        uint8_t *sdst = slot + p.piece_off[3 + q] + (size_t)(r >> 7) * (K / 128) * 512 + (size_t)(4 * g) * 512 +
                        (r & 31) * 16 + ((r & 127) >> 5) * 4;
#pragma unroll
        for (int kk = 0; kk < 4; kk++) *reinterpret_cast<uint32_t *>(sdst + kk * 512) = sw[kk];
        __syncwarp();  // the buffer is reused by the next run
    }
}

// marks round fr's jobs as failed: status for its copy, slots for the next planner, the message
void file_round_failed(const FileRound *fr, int begin, int n, const std::string &why) {
    FileStore *f = fr->c->file;
    const volatile int2 *jobs = f->jobs_h[fr->which];
    volatile unsigned char *bad = f->bad;
    for (int j = 0; j < n; j++) bad[jobs[begin + j].x] = 1;
    *(volatile int *)f->n_bad = 1;
    reinterpret_cast<volatile RoundTab *>(f->tab + (fr->round & 1) * f->tab_bytes)->bad = 1;
    f->failed_rounds++;
    std::lock_guard<std::mutex> lk(f->mu);
    f->err = "expert read failed: " + why;
    std::atomic_thread_fence(std::memory_order_seq_cst);
}

void file_round_read(const FileRound *fr);

// The read step of one round, run by the CUDA runtime in stream order (no CUDA calls here).  Nothing
// may escape a runtime callback: an exception counts as a failed read.
void CUDART_CB file_round_host(void *arg) {
    const FileRound *fr = static_cast<const FileRound *>(arg);
    try {
        file_round_read(fr);
    } catch (const std::exception &e) {
        FileStore *f = fr->c->file;
        const int nj = *(volatile const int *)f->n_jobs_h[fr->which];
        const int begin = fr->round * f->cap, n = std::max(0, std::min(nj, begin + f->cap) - begin);
        file_round_failed(fr, begin, n, e.what());
    }
}

// reads the round's experts into the staging rows and publishes where each matrix's data starts
void file_round_read(const FileRound *fr) {
    stbl_cache *c = fr->c;
    FileStore *f = c->file;
    const int buf = fr->round & 1;
    char *tab = f->tab + buf * f->tab_bytes;
    volatile RoundTab *rt = reinterpret_cast<volatile RoundTab *>(tab);
    const int nj = *(volatile const int *)f->n_jobs_h[fr->which];
    const int begin = fr->round * f->cap, n = std::min(nj, begin + f->cap) - begin;
    rt->n = std::max(0, n), rt->bad = 0;
    if (n <= 0) return;
    std::vector<uint64_t> off(3 * n), bytes(3 * n), at(3 * n);
    std::vector<uint8_t *> region(3 * n);
    const volatile int2 *jobs = f->jobs_h[fr->which];
    for (int j = 0; j < n; j++) {
        const int key = jobs[begin + j].y, l = key / c->E, e = key % c->E;
        for (int q = 0; q < 3; q++) {
            off[3 * j + q] = f->offset[3 * l + q] + (uint64_t)e * f->gbytes[q];
            bytes[3 * j + q] = f->gbytes[q];
            region[3 * j + q] = f->stage + ((size_t)buf * f->cap + j) * f->row_bytes + f->region_off[q];
        }
    }
    if (!f->reader->read(3 * n, off.data(), bytes.data(), region.data(), at.data())) {
        file_round_failed(fr, begin, n, f->reader->error());
        return;
    }
    int2 *tj = tab_jobs(tab);
    for (int j = 0; j < n; j++) tj[j] = make_int2(jobs[begin + j].x, jobs[begin + j].y);
    const uint8_t **ts = tab_src(tab, f->cap);
    for (int i = 0; i < 3 * n; i++) ts[i] = f->stage_d + (region[i] - f->stage) + at[i];
    std::atomic_thread_fence(std::memory_order_seq_cst);
}

void launch_file_copy(stbl_cache *c, int which, int round, uint32_t *status, cudaStream_t st) {
    FileStore *f = c->file;
    FileCopyParams fp{};
    // the round's table, as the read step left it, into device memory (stream order: after the read)
    const size_t toff = (size_t)(round & 1) * f->tab_bytes;
    CK(cudaMemcpyAsync(f->tab_d + toff, f->tab + toff, f->tab_bytes, cudaMemcpyHostToDevice, st));
    fp.tab = f->tab_d + toff, fp.cap = f->cap, fp.status = status;
    fp.pool = c->pool, fp.slot_bytes = c->slot_bytes;
    for (int q = 0; q < 6; q++) fp.piece_off[q] = c->piece_off[q];
    const int rows[3] = {c->I, c->I, c->H}, ks[3] = {c->H, c->H, c->I};
    for (int q = 0; q < 3; q++) fp.K[q] = ks[q], fp.tiles[q] = rows[q] / 128;
    cache_file_copy_kernel<<<2 * c->copy_ctas, kFileWarps * 32, kFileWarps * kFileRunBytes, st>>>(fp);
    CK(cudaGetLastError());
}

// `jobs` experts at most in the jobs list: rounds of read step (on the reader stream) + copy (on st); a
// failed read raises kErrRead in `status` (the calling layer's status word).  Round r + 1's reads run
// while round r's copy converts; round r + 2 reuses round r's buffer after its copy.  Every event is
// recorded before anything here waits for it, so no wait can see a recording of an earlier call.
void launch_file_rounds(stbl_cache *c, int which, int jobs, uint32_t *status, cudaStream_t st) {
    FileStore *f = c->file;
    const int rounds = (jobs + f->cap - 1) / f->cap;
    if (rounds > (int)f->rounds[which].size()) throw std::runtime_error("too many experts per call for the staging rounds");
    CK(cudaEventRecord(f->ev_plan, st));
    CK(cudaStreamWaitEvent(f->rstream, f->ev_plan, 0));
    for (int r = 0; r < rounds; r++) {
        if (r >= 2) CK(cudaStreamWaitEvent(f->rstream, f->ev_copy[r - 2], 0));
        CK(cudaLaunchHostFunc(f->rstream, file_round_host, &f->rounds[which][r]));
        CK(cudaEventRecord(f->ev_read[r], f->rstream));
        CK(cudaStreamWaitEvent(st, f->ev_read[r], 0));
        launch_file_copy(c, which, r, status, st);
        CK(cudaEventRecord(f->ev_copy[r], st));
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
void launch_copy(stbl_cache *c, const int2 *jobs, const int *n_jobs, cudaStream_t st, bool pdl, bool prefetch) {
    CacheCopyParams cp{};
    cp.jobs = jobs, cp.n_jobs = n_jobs, cp.pool = c->pool, cp.slot_bytes = c->slot_bytes;
    if (prefetch) cp.state = c->pf_state, cp.items = c->pf_items;
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
    // a demand copy has the GPU to itself (the call's expert kernels wait for it): two CTAs per SM; a
    // prefetch copy runs beside the expert kernels, whose persistent CTAs leave room on each SM for
    // one CTA of it (64 registers x 256 threads, no dynamic shared memory): one per SM
    const int grid = prefetch ? std::max(1, c->copy_ctas / 2) : c->copy_ctas;
    if (pdl) {
        launch_pdl_k((const void *)cache_copy_kernel, dim3(grid), dim3(kCopyThreads), a2, 0, st);
    } else {
        CK(cudaLaunchKernel((const void *)cache_copy_kernel, dim3(grid), dim3(kCopyThreads), a2, 0, st));
    }
}

void launch_cache(stbl_cache *c, int layer, const int *idx, int n, uint32_t *status, cudaStream_t st) {
    if (n < 1 || n > kPlanMaxIds) throw std::runtime_error("routed ids per call out of range for the cache planner");
    // host store: the planner runs beside a prefetch copy still in flight (claim words decide which of
    // its jobs it cancels or takes over) and the call's expert kernels, enqueued after this, wait for
    // that copy; file-backed store (no claims): the planner waits for the prefetch's reads and copy
    if (c->pf_pending && c->file) CK(cudaStreamWaitEvent(st, c->pf_done, 0));
    CachePlanParams pp{idx, n, layer, c->E, c->S, c->map, c->owner, c->ts, c->ctr, c->jobs, c->n_jobs, c->expert_bytes, status,
                       0, 0, c->pf_flag, c->pf_state, c->pf_items, c->file ? c->file->bad_d : nullptr,
                       c->file ? c->file->n_bad_d : nullptr};
    void *a1[] = {&pp};
    launch_pdl_k((const void *)cache_plan_kernel, dim3(1), dim3(kPlanThreads), a1, sizeof(int) * (c->E + n), st);
    if (c->file) {
        launch_file_rounds(c, 0, std::min(n, c->S), status, st);
    } else {
        launch_copy(c, c->jobs, c->n_jobs, st, true, false);
        if (c->pf_pending) CK(cudaStreamWaitEvent(st, c->pf_done, 0));
    }
}

void launch_prefetch(stbl_cache *c, int layer, const int *ids, int n, int consider, uint32_t *status, cudaStream_t st,
                     cudaStream_t copy_st) {
    if (n < 1 || n > kPlanMaxIds) throw std::runtime_error("prefetch ids out of range for the cache planner");
    // the previous prefetch's jobs list and slots are reused: its copy must be done
    if (c->pf_pending) CK(cudaStreamWaitEvent(st, c->pf_done, 0));
    CachePlanParams pp{ids, n, layer, c->E, c->S, c->map, c->owner, c->ts, c->ctr, c->pf_jobs, c->pf_n_jobs, c->expert_bytes,
                       status, 1, consider, c->pf_flag, c->pf_state, c->pf_items, c->file ? c->file->bad_d : nullptr,
                       c->file ? c->file->n_bad_d : nullptr};
    void *a1[] = {&pp};
    launch_pdl_k((const void *)cache_plan_kernel, dim3(1), dim3(kPlanThreads), a1, sizeof(int) * (c->E + n), st);
    CK(cudaEventRecord(c->pf_planned, st));
    CK(cudaStreamWaitEvent(copy_st, c->pf_planned, 0));
    if (c->file) launch_file_rounds(c, 1, std::min({n, consider, c->S}), status, copy_st);
    else launch_copy(c, c->pf_jobs, c->pf_n_jobs, copy_st, false, true);
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

// page-locked host memory, mapped: (host view, device view)
template <class T>
void host_mapped(T **h, T **d, size_t bytes) {
    CK(cudaHostAlloc((void **)h, bytes, cudaHostAllocMapped));
    memset((void *)*h, 0, bytes);
    CK(cudaHostGetDevicePointer((void **)d, (void *)*h, 0));
}

void file_desc_check(const stbl_cache_desc *d, const stbl_cache_file_desc *fd) {
    if (!fd->path || !fd->offset) throw std::runtime_error("file desc: path and offset are required");
    if (fd->readers < 0 || fd->stage_experts < 0) throw std::runtime_error("file desc: readers and stage_experts must be >= 0");
    for (long long i = 0; i < 3LL * d->n_layers; i++)
        if (fd->offset[i] % 16) throw std::runtime_error("expert tensor offsets must be multiples of 16 (GGUF alignment >= 16)");
}

void file_store_new(stbl_cache *c, const stbl_cache_file_desc *fd) {
    FileStore *f = new FileStore();
    c->file = f;
    const int rows[3] = {c->I, c->I, c->H}, ks[3] = {c->H, c->H, c->I};
    for (int q = 0; q < 3; q++) f->gbytes[q] = (uint64_t)rows[q] * (ks[q] / 32) * 17;
    f->offset.assign(fd->offset, fd->offset + 3 * (size_t)c->L);
    long long off = 0;
    for (int q = 0; q < 3; q++) f->region_off[q] = off, off += (long long)read_region_bytes(f->gbytes[q]);
    f->row_bytes = off;
    f->cap = std::min(fd->stage_experts ? fd->stage_experts : 2, c->S);  // small rounds overlap best
    f->reader = new ExpertReader(fd->path, fd->readers, fd->direct != 0);
    uint8_t *alloc_d = nullptr;
    host_mapped(&f->stage_alloc, &alloc_d, 2 * (size_t)f->cap * f->row_bytes + kReadAlign);
    const size_t pad = (kReadAlign - (uintptr_t)f->stage_alloc % kReadAlign) % kReadAlign;  // O_DIRECT buffers
    f->stage = f->stage_alloc + pad, f->stage_d = alloc_d + pad;
    f->tab_bytes = tab_size(f->cap);
    CK(cudaHostAlloc((void **)&f->tab, 2 * f->tab_bytes, cudaHostAllocDefault));
    memset(f->tab, 0, 2 * f->tab_bytes);
    CK(cudaMalloc((void **)&f->tab_d, 2 * f->tab_bytes));
    CK(cudaStreamCreateWithFlags(&f->rstream, cudaStreamNonBlocking));
    CK(cudaEventCreateWithFlags(&f->ev_plan, cudaEventDisableTiming));
    host_mapped(&f->bad, &f->bad_d, (size_t)c->S);
    host_mapped(&f->n_bad, &f->n_bad_d, sizeof(int));
    for (int w = 0; w < 2; w++) {
        host_mapped(&f->jobs_h[w], w ? &c->pf_jobs : &c->jobs, sizeof(int2) * c->S);
        host_mapped(&f->n_jobs_h[w], w ? &c->pf_n_jobs : &c->n_jobs, sizeof(int));
        const int most = std::min(c->S, kPlanMaxIds);
        for (int r = 0; r < (most + f->cap - 1) / f->cap; r++) f->rounds[w].push_back(FileRound{c, r, w});
    }
    for (size_t r = 0; r < f->rounds[0].size(); r++) {
        f->ev_read.push_back(nullptr), f->ev_copy.push_back(nullptr);
        CK(cudaEventCreateWithFlags(&f->ev_read.back(), cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&f->ev_copy.back(), cudaEventDisableTiming));
    }
}

void file_store_free(stbl_cache *c) {
    FileStore *f = c->file;
    if (!f) return;
    delete f->reader;
    for (cudaEvent_t e : f->ev_read)
        if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : f->ev_copy)
        if (e) cudaEventDestroy(e);
    if (f->ev_plan) cudaEventDestroy(f->ev_plan);
    if (f->rstream) cudaStreamDestroy(f->rstream);
    cudaFreeHost(f->stage_alloc);
    cudaFreeHost(f->tab);
    cudaFree(f->tab_d);
    cudaFreeHost(f->bad);
    cudaFreeHost(f->n_bad);
    for (int w = 0; w < 2; w++) cudaFreeHost(f->jobs_h[w]), cudaFreeHost(f->n_jobs_h[w]);
    c->jobs = c->pf_jobs = nullptr;
    c->n_jobs = c->pf_n_jobs = nullptr;
    delete f;
    c->file = nullptr;
}

}  // namespace

extern "C" {

// the cache of desc d over the pinned host store d->host_* (f null) or over the checkpoint file f
static stbl_cache *cache_new(const stbl_cache_desc *d, const stbl_cache_file_desc *f) {
    stbl_cache *c = nullptr;
    try {
        if (!d) throw std::runtime_error("null argument");
        if (d->n_layers < 1 || d->n_experts < 1 || d->n_experts > 512) throw std::runtime_error("n_layers >= 1, n_experts in 1..512");
        if (d->slots < 0 || d->slots > (1 << 20) - 1) throw std::runtime_error("slots must be in 0..2^20-1");
        if (d->fmt != STBL_FMT_FP8_B128 && d->fmt != STBL_FMT_MXFP4) throw std::runtime_error("bad fmt");
        if (f && d->fmt != STBL_FMT_MXFP4) throw std::runtime_error("a file-backed cache holds MXFP4 experts (GGUF type 39)");
        if (f) file_desc_check(d, f);  // before any device call
        if (d->hidden <= 0 || d->inter <= 0 || d->hidden % 512 || d->inter % 512)
            throw std::runtime_error("hidden and inter must be multiples of 512");
        if ((long long)d->n_layers * d->n_experts >= (1LL << 31)) throw std::runtime_error("store too large");
        c = new stbl_cache();
        c->L = d->n_layers, c->E = d->n_experts, c->S = d->slots, c->fmt = d->fmt, c->H = d->hidden, c->I = d->inter;
        if (!f && (d->host_rows < 0 || d->host_rows > (long long)c->L * c->E))
            throw std::runtime_error("host_rows must be in 0..n_layers*n_experts");
        c->host_rows = !f && d->host_rows ? d->host_rows : (long long)c->L * c->E;
        CK(cudaGetDevice(&c->dev));
        const int rows[3] = {c->I, c->I, c->H}, ks[3] = {c->H, c->H, c->I};
        long long off = 0;
        for (int q = 0; q < 6; q++) {
            const int mt = q % 3;
            c->piece_bytes[q] = piece_size(c->fmt, rows[mt], ks[mt], q >= 3);
            c->piece_off[q] = off;
            off += (c->piece_bytes[q] + 1023) & ~1023LL;
            c->expert_bytes += c->piece_bytes[q];
            if (f) continue;  // no host store
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
        CK(cudaMalloc(&c->ctr, sizeof(unsigned long long) * kCtrWords));
        CK(cudaMemset(c->ctr, 0, sizeof(unsigned long long) * kCtrWords));
        if (f) {
            file_store_new(c, f);
        } else {
            CK(cudaMalloc(&c->jobs, sizeof(int2) * c->S));
            CK(cudaMalloc(&c->n_jobs, sizeof(int)));
            CK(cudaMemset(c->n_jobs, 0, sizeof(int)));
            CK(cudaMalloc(&c->pf_jobs, sizeof(int2) * c->S));
            CK(cudaMalloc(&c->pf_n_jobs, sizeof(int)));
            CK(cudaMemset(c->pf_n_jobs, 0, sizeof(int)));
            CK(cudaMalloc(&c->pf_state, sizeof(unsigned int) * c->S));
            CK(cudaMemset(c->pf_state, 0, sizeof(unsigned int) * c->S));
            CK(cudaMalloc(&c->pf_items, sizeof(unsigned int) * c->S));
            CK(cudaMemset(c->pf_items, 0, sizeof(unsigned int) * c->S));
        }
        CK(cudaMalloc(&c->pf_flag, c->S));
        CK(cudaMemset(c->pf_flag, 0, c->S));
        CK(cudaEventCreateWithFlags(&c->pf_done, cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&c->pf_planned, cudaEventDisableTiming));
        CK(cudaMalloc(&c->status, sizeof(uint32_t)));
        CK(cudaMemset(c->status, 0, sizeof(uint32_t)));
        CK(cudaDeviceSynchronize());
        return c;
    } catch (...) {
        if (c) stbl_cache_destroy(c);
        throw;
    }
}

int stbl_cache_create(const stbl_cache_desc *d, stbl_cache **out, char *err, int errlen) {
    try {
        if (!out) throw std::runtime_error("null argument");
        *out = cache_new(d, nullptr);
        return 0;
    } catch (const std::exception &e) {
        return fail(err, errlen, e.what());
    }
}

int stbl_cache_create_file(const stbl_cache_desc *d, const stbl_cache_file_desc *f, stbl_cache **out, char *err, int errlen) {
    try {
        if (!out || !f) throw std::runtime_error("null argument");
        *out = cache_new(d, f);
        return 0;
    } catch (const std::exception &e) {
        return fail(err, errlen, e.what());
    }
}

int stbl_cache_file_stats(const stbl_cache *c, uint64_t *pieces, uint64_t *bytes, double *seconds, int *direct,
                          uint64_t *failed_rounds) {
    if (!c || !c->file) return -1;
    c->file->reader->stats(pieces, bytes, seconds, direct);
    if (failed_rounds) *failed_rounds = c->file->failed_rounds.load();
    return 0;
}

int stbl_cache_inject_read_error(stbl_cache *c, int64_t after, int err_no) {
    if (!c || !c->file || after < 0 || err_no < 0) return -1;
    c->file->reader->inject_error(after, err_no);
    return 0;
}

const char *stbl_cache_error(const stbl_cache *c) {
    if (!c) return "null cache";
    if (c->file) {
        std::lock_guard<std::mutex> lk(c->file->mu);
        if (!c->file->err.empty()) {
            thread_local std::string msg;
            msg = c->file->err;
            return msg.c_str();
        }
    }
    return c->err.c_str();
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
    unsigned long long v[kCtrWords];
    if (cudaMemcpy(v, c->ctr, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (prefetched) *prefetched = v[5];
    if (used) *used = v[6] + v[8];
    if (bytes) *bytes = v[7];
    return 0;
}

int stbl_cache_prefetch_counters(const stbl_cache *c, uint64_t *out) {
    if (!c || !out) return -1;
    unsigned long long v[kCtrWords];
    if (cudaMemcpy(v, c->ctr, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    out[0] = v[5], out[1] = v[6], out[2] = v[8], out[3] = v[9];
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
    file_store_free(c);  // mapped jobs lists
    cudaFree(c->jobs);
    cudaFree(c->n_jobs);
    cudaFree(c->pf_jobs);
    cudaFree(c->pf_n_jobs);
    cudaFree(c->pf_flag);
    cudaFree(c->pf_state);
    cudaFree(c->pf_items);
    cudaFree(c->status);
    if (c->pf_done) cudaEventDestroy(c->pf_done);
    if (c->pf_planned) cudaEventDestroy(c->pf_planned);
    delete c;
}

}  // extern "C"
