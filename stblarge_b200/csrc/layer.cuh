// Device-side structures of the MoE layer: the expert pointer table, the dispatch chunks and the
// parameter blocks of the three kernels that make up one layer call (router, expert up, expert down).
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace stbl {

enum : int { kFmtNone = 0, kFmtFp8B128 = 1, kFmtMxfp4 = 2 };
enum : int { kScoreSigmoid = 0, kScoreSqrtSoftplus = 1 };

constexpr int kMaxExperts = 512;    // router: a lane holds experts l, l+32, ... (16 per lane)
constexpr int kMaxTopk = 16;
constexpr int kRouterMaxTokens = 256;
constexpr int kLgThreads = 256;     // router logits kernel: 8 warps
constexpr int kLgExperts = 8;       // experts per logits CTA (two quads of 4)
constexpr int kLgRound = 32;        // tokens staged in shared memory at a time
constexpr int kLgMaxSlice = 2048;   // longest hidden slice (H / ksplit) the logits kernel stages
constexpr int kSelThreads = 512;    // router selection kernel: one CTA, a warp per token
constexpr int kExpertWarps = 15;    // warp 0 streams weights, warps 1..14 compute
constexpr int kConsumerWarps = kExpertWarps - 1;
constexpr int kConsumerThreads = 32 * kConsumerWarps;  // 448
constexpr int kExpertThreads = 32 * kExpertWarps;      // 480
constexpr int kNT = 4;              // tokens of one expert handled per pass over its weights

// Device addresses of one expert's three matrices (0 gate [I][H], 1 up [I][H], 2 down [H][I]) and
// their scales.  Entry E of the table is the shared expert.  The expert cache re-points entries.
struct ExpertPtrs {
    const uint8_t *w[3];
    const void *s[3];
};

// Up to kNT tokens of one expert.  Rows pos0 .. pos0+n-1 of the position-ordered buffers (h, hq)
// belong to it.  Routed positions are the bucketed dispatch order; position p < T*topk is assignment
// perm[p] = token * topk + slot.  Shared-expert positions are T*topk + token.
struct Chunk {
    int e;
    int pos0;
    int n;
    int pad;
};

// Router split of the hidden dimension: the logits are summed over kRouterSplit(H) slices
// (the CPU oracle restates this order).
__host__ __device__ inline int router_ksplit(int H) { return (H % 512 == 0) ? 4 : 1; }

struct RouterParams {
    const float *W;          // [E][H]
    const float *bias;       // [E]
    const uint16_t *x;       // [T][H] bf16
    int T, E, H, topk, n_groups, topk_groups, score_fn;
    float route_scale;
    int ksplit;
    int has_shared;
    int nt_routed, nt_shared;  // tokens per chunk of a routed / the shared expert
    float *scores;           // [T][E]
    int *idx;                // [T][topk]
    float *wts;              // [T][topk]
    int *counts;             // [E]
    int *offsets;            // [E + 1]
    int *perm;               // [T * topk]
    Chunk *chunks;           // [T * topk + T]
    int *n_chunks;           // [0] total, [1] shared chunks
    // activation quantization of x for the routed (a) and shared (b) experts' formats; scale rows
    // hold H / 32 floats whatever the block
    uint8_t *xq_a;
    float *xs_a;
    int blk_a, pow2_a;
    uint8_t *xq_b;
    float *xs_b;
    int blk_b, pow2_b;
    uint32_t *status;
};

// Sets the logits kernel's shared-memory limit on the current device (once per device, before any
// stream capture).
cudaError_t router_setup();
// Enqueues the router's two kernels (logits + scores, then selection + dispatch).  pdl_first lets
// the logits kernel start while the previous kernel on the stream drains.  H / router_ksplit(H)
// must be at most kLgMaxSlice and T at most kRouterMaxTokens.
cudaError_t launch_router(RouterParams r, cudaStream_t st, bool pdl_first);

// One launch of the expert kernels covers chunks [chunk_begin, chunk_end); chunk_end < 0 means
// "up to n_chunks[0]" (known only on the device).  Each CTA takes one contiguous range of the
// launch's work items (chunk-major, tile-minor), so a CTA streams long contiguous runs of one
// expert's rows and reloads its activations only when the chunk changes.
struct ExpertParams {
    const ExpertPtrs *experts;
    const Chunk *chunks;
    const int *n_chunks;
    int chunk_begin, chunk_end;
    int T, topk, E, H, I;
    const int *perm;
    const float *wts;
    // up: x codes [T][H] + scales [T][xs_stride] from the router kernel
    const uint8_t *xq;
    const float *xs;
    int xs_stride;           // scale floats per x row (H / 32: room for per-32 scales)
    int act_blk, act_pow2;   // act_quant rule of this launch's weight format
    float swiglu_limit;
    uint16_t *h;             // [pos][I] bf16: written by up, read (and re-quantized in registers) by down
    uint16_t *eo;            // [T * topk][H] bf16, routed outputs in (token, slot) order
    uint16_t *sh;            // [T][H] bf16, shared-expert outputs
    int has_shared;
    uint32_t *status;
};

struct CombineParams {
    const uint16_t *eo;
    const uint16_t *sh;
    uint16_t *y;
    int T, topk, H, has_shared;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace stbl
