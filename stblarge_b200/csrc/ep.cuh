// Parameter blocks of the expert-parallel exchange kernels (ep.cu).
#pragma once

#include "layer.cuh"

namespace stbl {

struct EpCountsParams {
    EpView ep;
    const int *counts;   // [E] this rank's assignments per (global) expert, from the router
    const int *offsets;  // [E + 1] bucketed dispatch offsets
    const int *perm;     // [T topk] assignments in bucketed order
    const int *idx;      // [T][topk] expert of each assignment
    int T, topk, E, E_loc, nt_routed, nt_shared, has_shared, routed_cap;
    int *a_dst;          // [T topk] out: receive row of each assignment at its owner
    Chunk *chunks;       // out: this rank's compute chunks (shared expert first; e = local expert)
    int *n_chunks;       // out: [0] all, [1] shared
    int *n_rows;         // out: [0] routed rows received
    unsigned int *done_ctr;  // the down kernel's CTA ticket (zeroed here, before that kernel runs)
    int adaptive_wide;   // chunks of 32 tokens when that saves more than a quarter of the chunks
    int *wide_sel;       // out (adaptive_wide): 1 when the chunks are of 32 tokens
    uint32_t *status;
};

struct EpPayloadParams {
    EpView ep;
    const int *idx;
    const float *wts;
    const int *a_dst;
    const uint8_t *xq;   // [T][H] e4m3 codes of this rank's tokens (per-128 act_quant)
    const float *xs;     // [T][xs_stride] their scales
    int xs_stride;
    int T, topk, H, E_loc, routed_cap, has_shared;
};

// Enqueues the count exchange (one CTA) and the payload dispatch (up to `sms` CTAs).
cudaError_t launch_ep(const EpCountsParams &cp, const EpPayloadParams &pp, int sms, cudaStream_t st);

}  // namespace stbl
