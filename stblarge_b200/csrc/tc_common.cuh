// Device helpers shared by the tensor-core expert kernels (experts_tc.cu: FP8, experts_tc4.cu: MXFP4).
#pragma once

#include "tc_params.cuh"

namespace stbl {

constexpr int kTcN = 16;  // token columns per MMA (chunk size)

struct TcChunk {
    int e, pos0, n, ok;
};

// a chunk entry checked against the launch (max_n: token columns per item)
__device__ __forceinline__ TcChunk tc_check(const TcParams &p, const Chunk ch, int max_n = kTcN) {
    TcChunk r{ch.e, ch.pos0, ch.n, 1};
    const int nrouted = p.n_routed;
    const bool shared = ch.e == p.E;
    const bool bad = ch.e < 0 || ch.e > p.E || (shared && !p.has_shared) || ch.n < 1 || ch.n > max_n ||
                     (shared ? (ch.pos0 < nrouted || ch.pos0 + ch.n > nrouted + p.T)
                             : (ch.pos0 < 0 || ch.pos0 + ch.n > nrouted));
    if (bad) r = TcChunk{0, 0, 0, 0};
    return r;
}

// first row of the chunk's B tiles: b_direct (x by token): routed chunks (T <= 16) read tokens 0..15
// and use column = token; shared chunks read their own 16 or 32 consecutive tokens, column = slot.
// Otherwise (rows by position) the chunk's first position, column = slot.
__device__ __forceinline__ int b_row(const TcParams &p, const TcChunk &ch) {
    if (!p.b_direct) return ch.pos0;
    return ch.e == p.E ? ch.pos0 - p.n_routed : 0;
}

// storage slot of a routed expert in the strided weight arrays (the expert cache re-points experts).
// Read at L2 (the cache planner rewrites the table between calls; the down kernels read it before
// their programmatic wait).
__device__ __forceinline__ int expert_slot(const TcParams &p, int e) { return p.slot ? __ldcg(p.slot + e) : e; }

// a chunk-table entry, read at L2 (written by the router of this call; the down kernels read the
// table before their programmatic wait)
__device__ __forceinline__ Chunk load_chunk(const Chunk *c) {
    const int4 v = __ldcg(reinterpret_cast<const int4 *>(c));
    return Chunk{v.x, v.y, v.z, v.w};
}

__device__ __forceinline__ void flag_release(unsigned int *f, unsigned int v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}

// wait until *f == v; gives up when *abort is raised or after kWaitLimitNs
__device__ __forceinline__ bool flag_wait(const unsigned int *f, unsigned int v, volatile int *abort) {
    const uint64_t t0 = global_ns();
    for (;;) {
        unsigned int x;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(x) : "l"(f) : "memory");
        if (x == v) return true;
        if (*abort || global_ns() - t0 > kWaitLimitNs) return false;
    }
}

}  // namespace stbl
