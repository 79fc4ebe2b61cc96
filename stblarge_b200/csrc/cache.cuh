// GPU expert cache (include/stbl_moe.h: stbl_cache_*): declarations shared by cache.cu and moe.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace stbl {
struct FileStore;
constexpr int kCtrWords = 16;  // stbl_cache::ctr
}

struct stbl_cache {
    int L = 0, E = 0, S = 0, fmt = 0, H = 0, I = 0, dev = 0;
    // one expert = six pieces: codes of gate, up, down, then their scales; slot s holds piece p at
    // pool + s * slot_bytes + piece_off[p]
    long long piece_bytes[6] = {}, piece_off[6] = {}, slot_bytes = 0, expert_bytes = 0;
    const uint8_t *host[6] = {};      // device-visible addresses of the host store (pinned memory)
    long long host_stride[6] = {};    // bytes between store rows of a piece
    long long host_rows = 0;          // store rows; expert (l, e) is row (l * E + e) mod host_rows
    uint8_t *pool = nullptr;          // [S][slot_bytes]
    int *map = nullptr;               // [L][E] slot of (layer, expert), -1 when not resident
    int *owner = nullptr;             // [S] l * E + e held by the slot, -1 when free
    unsigned long long *ts = nullptr; // [S] last use (a logical clock), 0 never used
    // [0] clock, [1] hits, [2] misses, [3] bytes copied, [4] clock before the last demand call,
    // [5] experts prefetched (issued), [6] prefetched experts routed to after they landed, [7] bytes the
    // prefetch copies wrote, [8] prefetched experts routed to while being copied, [9] prefetches
    // cancelled, [10] prefetches taken over by a demand call (copied by it, counted as misses)
    unsigned long long *ctr = nullptr;
    int2 *jobs = nullptr;             // [S] (slot, l * E + e) to fill in the current call
    int *n_jobs = nullptr;
    int copy_ctas = 0;
    // prefetch (stbl_cache_prefetch): its own jobs list, per-slot "prefetched, not yet routed to"
    // flags, the event after its copy (the next call's expert kernels wait for it) and status bits
    int2 *pf_jobs = nullptr;
    int *pf_n_jobs = nullptr;
    unsigned char *pf_flag = nullptr;
    unsigned int *pf_state = nullptr, *pf_items = nullptr;  // host store: claim words, landed items [S]
    cudaEvent_t pf_done = nullptr, pf_planned = nullptr;
    bool pf_pending = false;
    uint32_t *status = nullptr;
    std::string err;
    // file-backed store (stbl_cache_create_file): the jobs lists above live in mapped page-locked memory
    // and the missing experts are read from the checkpoint by a host step on the copying stream
    stbl::FileStore *file = nullptr;
};

namespace stbl {
// Enqueues the cache step of one layer call: the planner (hits, LRU victims, the layer's slot table
// = map row `layer`) and the copy of the missing experts from the host store into their slots.
// idx: device [n] routed expert ids of the call (token-major, top-k order).
void launch_cache(stbl_cache *c, int layer, const int *idx, int n, uint32_t *status, cudaStream_t st);
// Enqueues a prefetch for layer `layer`: the planner (prefetch mode) on st, the copy on copy_st.
// ids: device [n] guessed expert ids in priority order; the first `consider` distinct ones count.
void launch_prefetch(stbl_cache *c, int layer, const int *ids, int n, int consider, uint32_t *status, cudaStream_t st,
                     cudaStream_t copy_st);
}  // namespace stbl
