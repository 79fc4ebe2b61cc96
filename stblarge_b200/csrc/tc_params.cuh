// Host/device parameter blocks of the tensor-core expert kernels (experts_tc.cu).
#pragma once

#include <cuda.h>

#include "layer.cuh"

namespace stbl {

// K blocks of 128 per pipeline stage of the block-scaled (MXFP4 / FP8-e8m0) expert kernels; the
// weight and activation tensor maps' boxes span this many K blocks
constexpr int kT4StageKb = 2;

struct TcMaps {
    CUtensorMap w[2];  // up: routed gate, routed up; down: routed down (twice)
    CUtensorMap s[2];  // up: shared gate, shared up; down: shared down (twice)
    CUtensorMap b;     // activation operand: 16-row x 128-byte tiles of e4m3 codes
};

struct TcParams {
    const int *slot;           // [E] storage slot of each routed expert in the weight arrays (null: e)
    const Chunk *chunks;
    const int *n_chunks;
    int chunk_begin, chunk_end;
    int chunk_cap;             // entries of the chunks array (reads beyond the live count stay inside it)
    int T, topk, E, H, I;
    const int *perm;
    const float *wts;
    // B tiles: 16 rows of the activation map.  b_direct: the map holds x by token; a routed chunk
    // (T <= 16) reads tokens 0..15 and finds token t in column t, a shared-expert chunk reads its 16
    // consecutive tokens.  Otherwise the map holds rows by position and a chunk reads its own.
    int b_direct;
    const float *act_s;        // per-128 activation scales of the map's rows, row stride act_s_stride
    int act_s_stride;
    const float *w_scale[2];   // routed block scales of the two matrices (up) / one (down), [E][rb][kb]
    long long w_scale_stride;  // floats per expert
    // MXFP4 routed experts (experts_tc4.cu): e8m0 weight scales [E][rows][K / 32] of the two
    // matrices (up) / one (down), bytes per expert; e8m0 activation scales [rows][K / 32] of the B rows
    // MXFP4: weight scales in the tensor cores' scale-block layout (per matrix [rows/128][K/128][512 B]:
    // byte l*16 + c*4 + j = scale of row 32c + l, 32-block j), slot z at sf_a[m] + z * sf_a_stride; the
    // activation scales [K/128][act_e8_rows][16 B]
    const uint8_t *sf_a[2];
    long long sf_a_stride;
    // weights of the block-scaled kernel in e4m3 (FP8 with e8m0 32x32 block scales) instead of e2m1:
    // routed (w_a8) and shared expert (s_a8); the shared expert's scale blocks (one copy per matrix)
    int w_a8, s_a8;
    const uint8_t *sf_s[2];
    const uint8_t *act_e8;
    int act_e8_rows;
    const float *s_scale[2];   // shared expert block scales
    float swiglu_limit;        // > 0: SwiGLU clamps (stbl/kernels.cu:445-459)
    uint16_t *h;               // up out: [pos][I] bf16
    uint8_t *hq, *he8;         // MXFP4 up out: h quantized for the down product: e4m3 [pos][I], e8m0
    int he8_rows;              // scales in the activation-scale layout [I/128][he8_rows][16 B]
    uint16_t *eo, *sh;         // down outputs: routed [T * topk][H] in (token, slot) order, shared [T][H]
    int has_shared;
    // rows [0, n_routed) are routed assignments, the shared expert's rows follow (row n_routed + token)
    int n_routed;
    // expert parallelism (ep.n_ranks > 1): the rows are this rank's receive rows; pos_w / pos_meta give
    // each routed row's routing weight and origin (source rank << 16 | assignment); the up kernel
    // raises pay_flag on every rank and waits for all of them first; the down kernel stores routed
    // outputs into the source rank's eo rows
    const float *pos_w;
    const int *pos_meta;
    int T_max_assign;          // rows of a source rank's eo (max_tokens x topk)
    EpView ep;
    // split items: CTA b publishes the partial sums of the item its range starts inside in
    // partial[b] ([128 rows][16 columns] fp32) and then sets flags[b] = seq
    float *partial;
    unsigned int *flags;
    unsigned int seq;          // this launch's number, never 0
    unsigned int *ep_done_ctr; // expert parallelism, down: CTA ticket; the last CTA raises done_flag
    // adaptive chunk width: the launch runs only when *sel == sel_val (the router's or count exchange's
    // choice, read after the programmatic-launch wait); otherwise it returns at once.  sel null: always
    const int *sel;
    int sel_val;
    uint32_t *status;
};

// act_quant of h (positions x I) into e4m3 codes and per-128 scales for the down kernel
struct HquantParams {
    const uint16_t *h;
    uint8_t *hq;
    float *hs;                 // scales [pos][I / 128] (per-128 rule); unused for the per-32 rule
    int n_pos, I;
    // expert parallelism: rows [0, *n_routed_dev) (known on the device) and [n_pos, n_pos + n_tail)
    const int *n_routed_dev;
    int n_tail;
    // per-32 power-of-two rule (MXFP4 experts) instead of per-128: scales as e8m0 bytes [pos][I / 32]
    uint8_t *he8;
};

// gathers x codes and scales into position order for the up kernel when T > 16
struct GatherParams {
    const int *perm;
    int T, topk, H;
    int has_shared;
    const uint8_t *xq;
    const float *xs;
    int xs_stride;
    uint8_t *xq_pos;
    float *xs_pos;             // [pos][H / 128]
    // MXFP4 routed experts: e8m0 scales in the activation-scale layout [H/128][rows][16 B], token rows
    // (xe8_rows) -> position rows (xe8_pos_rows); then only routed positions
    const uint8_t *xe8;
    uint8_t *xe8_pos;
    int xe8_rows, xe8_pos_rows;
};

// the Q8 routed expert products (experts_q8.cu): routed MXFP4 experts x int8 activations per 32
struct Q8Params {
    const int *slot;          // [E] storage slot of each routed expert (null: e)
    const Chunk *chunks;
    const int *n_chunks;      // [0] total chunks, [1] the shared expert's (first); routed chunks follow
    int T, topk, E, H, I;
    const int *perm;
    const float *wts;
    const uint8_t *w[2];      // up: gate, up codes; down: down codes ([rows][K / 2] per slot)
    long long w_stride[2];    // bytes between slots
    const uint8_t *s[2];      // e8m0 scales [rows][K / 32] per slot
    long long s_stride[2];
    const int8_t *xq;         // activation codes: up, x by token [.][H]; down, h by position [.][I]
    const float *xd;          // their per-32 scales, xd_stride floats per row
    int xd_stride;
    int8_t *hq;               // up out: Q8 codes of h by position [pos][I]
    float *hd;                // up out: their scales [pos][I / 32]
    uint16_t *h;              // up out: h (bf16) by position [pos][I]
    float swiglu_limit;
    uint16_t *eo;             // down out: [T * topk][H] by assignment
    uint32_t *status;
};

}  // namespace stbl
