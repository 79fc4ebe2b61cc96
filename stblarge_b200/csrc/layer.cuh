// Device-side structures of the MoE layer: the expert pointer table, the dispatch chunks and the
// parameter blocks of the router and combine kernels.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace stbl {

enum : int { kFmtNone = 0, kFmtFp8B128 = 1, kFmtMxfp4 = 2 };
enum : int { kScoreSigmoid = 0, kScoreSqrtSoftplus = 1 };
// activation quantization rules (RouterParams::pow2_a / pow2_b): 0 fp32 scale amax/448, 1 power-of-two
// scale, kActQ8 int8 codes with an fp32 scale amax/127 per 32 (ref/emulate_ds4.py:23-30)
constexpr int kActQ8 = 2;
// rows after the position-ordered activation buffers (x by position, h): a chunk's TMA box and the
// bulk copy of its scales read whole 16- or 32-row blocks from its first position
constexpr int kPosPad = 32;
constexpr int kQ8ChunkTokens = 8;   // tokens per routed chunk of an act_q8 layer (experts_q8.cu)

constexpr int kMaxExperts = 512;    // router: a lane holds experts l, l+32, ... (16 per lane)
constexpr int kMaxTopk = 16;
constexpr int kRouterMaxTokens = 256;
constexpr int kLgThreads = 256;     // router logits kernel: 8 warps
constexpr int kLgExperts = 8;       // experts per logits CTA (two quads of 4)
constexpr int kLgRound = 32;        // tokens staged in shared memory at a time
constexpr int kLgMaxSlice = 2048;   // longest hidden slice (H / ksplit) the logits kernel stages
constexpr int kSelThreads = 512;    // router selection kernel: one CTA, a warp per token

// Up to 16 tokens of one expert.  Rows pos0 .. pos0+n-1 of the position-ordered buffers (h, hq)
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
    // adaptive chunking (FP8 layers, calls of more than 16 tokens): chunks of 32 tokens instead of
    // nt_routed / nt_shared (16) when that saves more than a quarter of the chunks; the choice goes to
    // *wide_sel (1: 32-token chunks), which the expert launches of both widths read
    int adaptive_wide;
    int *wide_sel;
    float *scores;           // [T][E]
    int *idx;                // [T][topk]
    float *wts;              // [T][topk]
    int *counts;             // [E]
    int *offsets;            // [E + 1]
    int *perm;               // [T * topk]
    Chunk *chunks;           // [T * topk + T]
    int *n_chunks;           // [0] total, [1] shared chunks
    // activation quantization of x for the routed (a) and shared (b) experts' formats; scale rows
    // hold H / 32 floats whatever the block (xq_a null: no quantization, routing only)
    uint8_t *xq_a;
    float *xs_a;
    int blk_a, pow2_a;
    uint8_t *xe8_a;          // optional: scales of a as e8m0 bytes (per-32 power-of-two rule) in the
                             // tensor cores' activation-scale layout [H/128][xe8_rows][16 B]: row t's
                             // bytes 0..3 = the scales of its four 32-blocks of one 128-K block
    int xe8_rows;
    uint8_t *xq_b;
    float *xs_b;
    int blk_b, pow2_b;
    // selection state shared by the select kernel's CTAs: [E] counts, [E][ceil(T/32)] token bitmaps,
    // a ticket; zeroed by the logits kernel
    int *sel_cnt;
    uint32_t *sel_bm;
    unsigned int *sel_ticket;
    uint32_t *status;
    const int *forced_idx;   // optional: [T][topk] experts given instead of selected (forced routes)
    // optional fused RMSNorm (x_pre non-null; x is then not read): the layer input is
    // bf16(norm_w * (x_pre * rsqrt(mean(x_pre^2) + norm_eps))), computed per token as the reference's
    // k_rms_norm does (stbl/kernels.cu:217-236): 256 strided partial sums, two xor-butterfly warp sums
    const float *x_pre;      // [T][H] fp32
    const float *norm_w;     // [H]
    float norm_eps;
};

// Sets the logits kernel's shared-memory limit on the current device (once per device, before any
// stream capture).
cudaError_t router_setup();
// Enqueues the router's two kernels (logits + scores, then selection + dispatch).  pdl_first lets
// the logits kernel start while the previous kernel on the stream drains.  H / router_ksplit(H)
// must be at most kLgMaxSlice and T at most kRouterMaxTokens.
cudaError_t launch_router(RouterParams r, cudaStream_t st, bool pdl_first);

// ---- expert parallelism ------------------------------------------------------------------------
//
// Rank r of n holds routed experts [r E/n, (r+1) E/n).  Every rank owns one exchange region, mapped
// into every other rank's address space (CUDA IPC over NVLink); the regions have the same layout on
// every rank.  Per layer call (epoch = the call's number, the same on every rank):
//   counts  each rank writes its per-expert assignment counts into every rank's inbox[r], each word
//           tagged with the call (tag << 16 | count, the tag cycling over 1..65535); every rank waits
//           until all n rows of its inbox carry this call's tag (a word is written whole, so no fence
//           or flag is needed), then knows where each of its assignments lands in its owner's receive
//           rows (expert-major, then source rank, then the source's token order)
//   payload each rank writes the FP8 codes + scales of each assignment's token, its routing weight
//           and (source rank, assignment) into the owner's receive rows; the owner's up kernel, once
//           the payload kernel before it has finished, raises pay_flag[r] on every rank and waits for
//           all n pay_flags
//   outputs the owner's down kernel stores each assignment's bf16 output row straight into the source
//           rank's eo rows; each of its CTAs fences its stores and the last one to finish raises
//           done_flag[r] on every rank; the combine kernel waits for all n
// Every wait is bounded.  A rank never waits for a later step of another rank, so the waits cannot
// form a cycle; the count exchange of call c+1 cannot start on any rank before every rank has
// finished call c's combine, which protects every buffer that peers write.
constexpr int kEpMaxRanks = 8;

struct EpLayout {            // byte offsets inside an exchange region
    long long inbox;         // u32 [n][E]: call tag << 16 | assignment count per expert, by source rank
    long long cnt_flag;      // u32 [n] (unused: the inbox words carry the call)
    long long pay_flag;      // u32 [n]
    long long done_flag;     // u32 [n]
    long long xq_pos;        // u8 [rows][H]: receive rows (routed, capacity n Tmax topk), then the shared rows
    long long xs_pos;        // f32 [rows][H / 128]
    long long pos_meta;      // int [routed capacity]: source rank << 16 | assignment (token * topk + slot)
    long long pos_w;         // f32 [routed capacity]: routing weight of the row
    long long eo;            // bf16 [Tmax topk][H]: this rank's routed outputs, written by the owners
    long long bytes;
};

struct EpView {
    char *region[kEpMaxRanks];  // every rank's exchange region (this rank's own at [rank])
    EpLayout L;
    int rank, n_ranks;
    unsigned int epoch;
};

__device__ __forceinline__ void st_release_sys(unsigned int *f, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}

// wait until flags[s] == v for every s < n (flags written by other GPUs); false after kWaitLimitNs
__device__ __forceinline__ bool wait_flags_sys(const unsigned int *flags, int n, unsigned int v) {
    const uint64_t t0 = global_ns();
    for (int s = 0; s < n; s++) {
        for (;;) {
            unsigned int x;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(x) : "l"(flags + s) : "memory");
            if (x == v) break;
            if (global_ns() - t0 > kWaitLimitNs) return false;
        }
    }
    return true;
}

// raise flag `which` (a byte offset of the layout) at index rank on every rank's region
__device__ __forceinline__ void signal_all(const EpView &v, long long which) {
    __threadfence_system();
    for (int d = 0; d < v.n_ranks; d++)
        st_release_sys(reinterpret_cast<unsigned int *>(v.region[d] + which) + v.rank, v.epoch);
}

struct CombineParams {
    const uint16_t *eo;
    const uint16_t *sh;
    uint16_t *y;             // [T][H] bf16 (null: not written)
    int T, topk, H, has_shared;
    // expert parallelism (ep.n_ranks > 1): raise done_flag on every rank, wait for all of them
    EpView ep;
    uint32_t *status;
    // optional fused hyper-connection post (hout non-null; the reference's k_hc_post,
    // stbl/kernels.cu:328-338, per token): hout[t][j][d] = bf16(post[t][j] * y[t][d] +
    // sum_a comb[t][a][j] * res[t][a][d]), products and sums rounded step by step in a's order
    const float *res;        // [T][hc][H]
    const float *post;       // [T][hc]
    const float *comb;       // [T][hc][hc]
    float *hout;             // [T][hc][H], bf16 values
    int hc;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace stbl
