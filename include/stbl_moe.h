/* B200-native MoE decode layer: layer-level C ABI (libstbl_moe.so).
 *
 * Drop-in for the reference's MoE layer, stbl/model.cu:426-594 (moe(), the body of
 * stbl_block_test stage 4, stbl/stbl.h:25-31), in the reference's C-ABI style: plain pointers and
 * sizes, int status (0 ok, -1 error, message from stbl_moe_error), caller-owned device buffers,
 * work ordered on the caller's cudaStream_t.  Routing, dispatch, the expert products and the
 * combine all stay on the GPU: there is no device->host copy inside a layer call.
 *
 * Numerics (checked against the CPU oracle, oracle/moe_oracle.c):
 *   logits = W_g x (fp32), score = sigmoid (DeepSeek-V3) or sqrt(softplus) (the reference engine),
 *   selection over score + bias (group-limited when n_groups > 1 and topk_groups < n_groups; ties go
 *   to the lower expert id), weights = score / (sum + 1e-20) * route_scale (stbl/model.cu:444-451,
 *   527-530); per expert g, u = bf16(W1 q(x)), bf16(W3 q(x)), h = bf16(silu(g) u w) (clamped when
 *   swiglu_limit > 0, stbl/kernels.cu:445-459), out = bf16(W2 q(h)); y = bf16(sum of outputs in top-k
 *   order + shared expert) (stbl/model.cu:589-592).  q() is act_quant (ref/kernel.py:35-45): per-128
 *   fp32 scales for STBL_FMT_FP8_B128 weights, per-32 power-of-two scales for STBL_FMT_MXFP4.
 */
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* weight formats */
enum {
    STBL_FMT_NONE = 0,
    STBL_FMT_FP8_B128 = 1, /* e4m3 codes [rows][k]; fp32 scales [ceil(rows/128)][ceil(k/128)] */
    STBL_FMT_MXFP4 = 2,    /* e2m1 codes [rows][k/2], even k in the low nibble; e8m0 scales [rows][k/32] */
    STBL_FMT_FP8_E8M0 = 3  /* e4m3 codes [rows][k]; e8m0 scales [ceil(rows/32)][k/32], one per 32x32 block: the
                              reference engine's FP8 format (stbl/kernels.cu:98-132, tools/convert_official.py:74-81).
                              Routed (with an FP8-e8m0 or no shared expert, or with MXFP4 routed experts) and
                              shared (with MXFP4 or FP8-e8m0 routed experts); activations are quantized per 32
                              with power-of-two scales (stbl/kernels.cu:56-63) */
};

/* router score functions */
enum { STBL_SCORE_SIGMOID = 0, STBL_SCORE_SQRT_SOFTPLUS = 1 };

typedef struct stbl_moe stbl_moe;

typedef struct stbl_moe_desc {
    int hidden;        /* H: multiple of 512, at most 8192 */
    int inter;         /* I: moe_intermediate, multiple of 512 */
    int n_experts;     /* E routed experts, <= 512, multiple of n_groups */
    int topk;          /* <= 16 */
    int n_groups;      /* expert groups for group-limited routing (1: none), <= 32 */
    int topk_groups;   /* groups kept */
    int score_fn;      /* STBL_SCORE_* */
    float route_scale; /* routed scaling factor */
    float swiglu_limit;/* 0: no SwiGLU clamps */
    int routed_fmt;    /* STBL_FMT_FP8_B128 or STBL_FMT_MXFP4 */
    int shared_fmt;    /* STBL_FMT_FP8_B128 or STBL_FMT_NONE */
    int max_tokens;    /* largest T passed to stbl_moe_forward, <= 256 */
    const float *router_w;    /* device fp32 [E][H], 16-byte aligned */
    const float *router_bias; /* device fp32 [E] (score-correction bias) */
    /* routed experts, device: expert e of matrix m (0 gate [I][H], 1 up [I][H], 2 down [H][I]) starts
       at routed_w[m] + e * routed_w_stride[m] bytes (stride 0: the packed size of one matrix) */
    const void *routed_w[3];
    const void *routed_s[3];
    long long routed_w_stride[3];
    long long routed_s_stride[3];
    /* shared expert, device */
    const void *shared_w[3];
    const void *shared_s[3];
    /* slots in the routed arrays (0: n_experts); an expert cache's pool may hold fewer or more
       slots than a layer has experts (stbl_cache_layer_desc fills this and the routed pointers; a
       layer with fewer slots than experts runs only once its cache is attached) */
    int n_slots;
    /* MXFP4 only: 1 when routed_s already holds the scales in the tensor cores' scale-block layout
       (per slot and matrix [rows/128][k/128][512 B], byte l*16 + c*4 + j = scale of row 32c + l,
       32-block j of the 128-k block; an expert cache's pool holds them so).  0: the natural
       [rows][k/32] layout; the layer then keeps its own copy in the block layout, made at create for
       every slot and again for a slot when stbl_moe_set_expert points an expert at it. */
    int routed_s_blocked;
    /* 1: the routed MXFP4 experts take Q8 activations instead of FP8: x and h quantized per 32 values
       to int8 with an fp32 scale amax / 127, round-half-even (ref/emulate_ds4.py:23-30, 69-77; the
       reference's ds4 numerics), products on the CUDA cores with exact integer block sums.  Needs
       routed_fmt STBL_FMT_MXFP4 with natural scales (routed_s_blocked 0), a shared expert in
       STBL_FMT_FP8_B128 (it keeps its FP8 rule) or none, hidden <= 8192, inter <= 4096, one GPU, no
       expert cache.  0: the FP8 rule of the weight format. */
    int act_q8;
} stbl_moe_desc;

/* Validate the description, allocate the layer's workspace on the current device and build its
 * expert table.  Weight pointers must be 16-byte aligned.  Returns 0, or -1 with err filled. */
int stbl_moe_create(const stbl_moe_desc *desc, stbl_moe **out, char *err, int errlen);

/* y = MoE(x) for T decode tokens: x and y are device bf16 [T][H], x 16-byte aligned.  Enqueued on
 * `stream`; returns without waiting.  Returns -1 (see stbl_moe_error) for a bad argument. */
int stbl_moe_forward(stbl_moe *m, const void *x_bf16, int T, void *y_bf16, cudaStream_t stream);

/* The same with host buffers (pinned or pageable): copies x in, runs the layer, copies y out and
 * waits for the stream.  The reference's stbl_block_test(stage 4) contract (stbl/model.cu:1065-1071). */
int stbl_moe_forward_host(stbl_moe *m, const void *x_bf16_host, int T, void *y_bf16_host, cudaStream_t stream);

/* Routing of the last call, copied to host (waits for the stream): idx [T][topk] in selection order
 * (stbl_last_route, stbl/stbl.h:35-36), weights [T][topk], counts [E], offsets [E+1] and the
 * bucketed dispatch permutation perm [T*topk] (perm[p] = token * topk + slot, expert-major, token
 * order inside an expert).  Any pointer may be NULL.  Returns T of that call, or -1. */
int stbl_moe_last_route(stbl_moe *m, int *idx, float *weights, int *counts, int *offsets, int *perm);

/* Router scores of the last call (fp32 [T][E]), for parity checks.  Returns T, or -1. */
int stbl_moe_last_scores(stbl_moe *m, float *scores);

/* The quantized activations of the last call as the expert kernels read them, copied to host (waits
 * for the device), for bit-exact checks of the layer's own act_quant steps against the reference's
 * rule (ref/kernel.py:35-45; stbl/kernels.cu:56-63; the reference tests them at tolerance 0,
 * stbl/test_kernels.py:63-69).  `which`:
 *   STBL_ACTS_X_ROUTED  x as the routed experts read it: rows T, width hidden
 *   STBL_ACTS_X_SHARED  x as the shared expert reads it: rows T, width hidden
 *   STBL_ACTS_H_ROUTED  h of the routed assignments by dispatch position (perm): rows T*topk, width inter
 *   STBL_ACTS_H_SHARED  h of the shared expert by token: rows T, width inter
 * h_bf16 (h rows only; may be NULL): the bf16 values that were quantized, [rows][width]; codes: e4m3
 * [rows][width]; scales: fp32 [rows][width / blk], blk 128 (fp32 scale amax/448) for FP8 128x128
 * weights, 32 (power-of-two scale, stored as e8m0) for MXFP4 and FP8-e8m0 weights; for the routed
 * rows of an act_q8 layer, int8 codes and fp32 scales amax/127 per 32.  Any output
 * pointer may be NULL.  Single-GPU layers.  Returns the row count, or -1. */
#define STBL_ACTS_X_ROUTED 0
#define STBL_ACTS_X_SHARED 1
#define STBL_ACTS_H_ROUTED 2
#define STBL_ACTS_H_SHARED 3
int stbl_moe_last_acts(stbl_moe *m, int which, void *h_bf16, void *codes, float *scales);

/* Point routed expert e at another slot of the layer's expert arrays (an expert cache: the arrays
 * passed in the description are the slot pool, slot j at routed_w[m] + j * routed_w_stride[m]).  w and
 * s must be the same slot j for all three matrices and their scales.  Takes effect for calls enqueued
 * on `stream` after this one. */
int stbl_moe_set_expert(stbl_moe *m, int e, const void *const w[3], const void *const s[3], cudaStream_t stream);

/* y = MoE(x) with the routed experts given instead of selected: idx is device int [T][topk], the
 * expert ids of each token in the order their outputs are added (distinct within a token, in
 * 0..n_experts-1; a token that breaks this is routed to experts 0..topk-1 and status bit 2 is
 * raised).  Weights are the router's, for the given experts: score / (sum + 1e-20) * route_scale in
 * the given order.  The reference's forced-route replay of a recorded route trace. */
int stbl_moe_forward_routed(stbl_moe *m, const void *x_bf16, int T, const int *idx, void *y_bf16, cudaStream_t stream);

/* GPU expert cache over a host expert store: the reference's expert cache and demand reads
 * (stbl/model.cu:99-106, 269-296, 347-422; stbl_stats, stbl/stbl.h:20), with the planning and the
 * copies done on the GPU.  The store holds every expert of n_layers layers in page-locked host memory
 * (cudaHostAlloc / cudaMallocHost / cudaHostRegister): piece q of expert e of layer l at
 * host_w[q] (codes, q = 0 gate [I][H], 1 up, 2 down [H][I]) or host_s[q] (scales) + (l * n_experts +
 * e) * stride (stride 0: the packed size), 16-byte aligned.  The cache is `slots` expert slots in
 * device memory shared by all attached layers.  A layer created from stbl_cache_layer_desc and
 * attached with stbl_moe_attach_cache brings the experts each call selects into the cache before its
 * expert kernels run: right after the router one CTA replays the reference's LRU order (the call's
 * cached experts touched first, then its experts in token-major top-k order: a hit is touched again,
 * a miss takes a never-used slot in order or else the least recently used slot) and one grid copies
 * the missing experts from the store (the GPU reads the page-locked memory directly).  No host
 * synchronisation; the copies are ordered on the layer call's stream.  Calls of attached layers on
 * different streams must not overlap (they share the cache state). */
typedef struct stbl_cache stbl_cache;
typedef struct stbl_cache_desc {
    int n_layers, n_experts;
    int slots;               /* device slots; 0: as many as the free device memory holds after a headroom of
                                max(4 GiB, 5 %), at most n_layers * n_experts (stbl_cache_info reports it) */
    int fmt;                 /* STBL_FMT_FP8_B128 or STBL_FMT_MXFP4 */
    int hidden, inter;       /* multiples of 512 */
    const void *host_w[3];
    const void *host_s[3];
    long long host_w_stride[3];
    long long host_s_stride[3];
    /* experts held by the store (0: n_layers * n_experts); expert (l, e) reads store row
       (l * n_experts + e) mod host_rows, so a store smaller than the model repeats its experts
       (synthetic benchmarks: every miss still moves a whole expert) */
    long long host_rows;
} stbl_cache_desc;
int stbl_cache_create(const stbl_cache_desc *desc, stbl_cache **out, char *err, int errlen);
/* Points desc's routed weights at the cache's slot pool (routed_w/routed_s, strides, n_slots,
 * routed_fmt); the caller fills the rest and creates the layer with stbl_moe_create. */
int stbl_cache_layer_desc(const stbl_cache *c, stbl_moe_desc *desc);
/* Layer m (made from stbl_cache_layer_desc, single GPU) becomes layer `layer` of the cache.  Needs
 * slots >= max_tokens * topk (a call's experts must fit at once). */
int stbl_moe_attach_cache(stbl_moe *m, stbl_cache *c, int layer);
/* Slots of the cache and bytes per slot (one expert: codes and scales of its three matrices). */
int stbl_cache_info(const stbl_cache *c, int *slots, uint64_t *slot_bytes);
/* Counters since creation (waits for the device): routed experts found in the cache, experts copied
 * in, bytes copied.  The reference's stbl_stats(hits, misses). */
int stbl_cache_stats(const stbl_cache *c, uint64_t *hits, uint64_t *misses, uint64_t *bytes);
/* Residency (waits for the device): map [n_layers][n_experts] slot or -1; owner [slots] l * E + e or -1. */
int stbl_cache_state(const stbl_cache *c, int *map, int *owner);
void stbl_cache_destroy(stbl_cache *c);

/* File-backed cache: the reference's expert streaming from the checkpoint (stbl/model.cu:269-308 reads,
 * 940-949 experts kept as file offsets, 978-987 readers and O_DIRECT).  Instead of a host store the
 * routed experts stay in the GGUF file as MXFP4 blocks (type 39, ffn_{gate,up,down}_exps.weight, dims
 * (k, rows, n_experts), 17 bytes per 32 values); desc->host_* and host_rows are ignored and desc->fmt
 * must be STBL_FMT_MXFP4.  Each call's missing experts are read by `readers` host threads (pread in
 * 2 MiB pieces, O_DIRECT where the file system takes it; include/stbl_io.h) into page-locked staging of
 * `stage_experts` experts, from host steps (cudaLaunchHostFunc) on a reader stream that the call's
 * stream waits for through events, then converted into the slot layout by the copy kernel; the missing
 * experts are read in rounds of stage_experts, double-buffered.  The stream waits for the reads; the caller does not (a
 * prefetch reads on its copy stream, beside the current call's kernels).  A failed read raises status
 * bit 8 in the layer (stbl_moe_status; that call's output is not valid), is counted, and its message
 * is kept (stbl_cache_error); the experts it was reading leave the cache at the next call, so a later
 * call routed to them reads them again. */
typedef struct stbl_cache_file_desc {
    const char *path;         /* the GGUF checkpoint */
    const uint64_t *offset;   /* [n_layers][3] absolute file offset of cache layer l's gate / up / down
                                 expert tensor (multiples of 16); expert e's matrix q starts at
                                 offset[3 l + q] + e * rows_q * (k_q / 32) * 17 */
    int readers;              /* reader threads, 0: 4 (the reference's default), at most 64 */
    int direct;               /* 1: O_DIRECT where the file system takes it, 0: buffered reads */
    int stage_experts;        /* experts per staging round, 0: 2 (two buffers of it, page-locked; round r + 1 is
                                 read while round r is converted, so small rounds hide the conversion) */
} stbl_cache_file_desc;
int stbl_cache_create_file(const stbl_cache_desc *desc, const stbl_cache_file_desc *file, stbl_cache **out, char *err,
                           int errlen);
/* File-backed caches: pieces read, bytes read, seconds the read steps took, *direct = 1 while reads go
 * through O_DIRECT, and read rounds that failed.  -1 for a cache over a host store. */
int stbl_cache_file_stats(const stbl_cache *c, uint64_t *pieces, uint64_t *bytes, double *seconds, int *direct,
                          uint64_t *failed_rounds);
/* Host-side fault injection for tests (file-backed caches): counting from this call, read number `after`
 * and every later one fail with errno err_no (0 switches it off); see stbl_reader_inject_error. */
int stbl_cache_inject_read_error(stbl_cache *c, int64_t after, int err_no);
/* The message of the cache's last error ("" when none). */
const char *stbl_cache_error(const stbl_cache *c);

/* Prefetch into the cache, the reference's shadow next-layer guesses (stbl/model.cu:432-475 predict,
 * 555-586 issue, 347-373 take_slot): of the first `consider` distinct ids (device [n], guessed experts of
 * layer `layer` in priority order) the ones not cached take a freed slot, a never-used one or the least
 * recently used one and become the most recent; cached ones are not touched.  Planned on `stream` (after
 * what is queued there), copied on `copy_stream`.  A slot the last call used is never taken: the prefetch
 * stops there.  The cache's next call plans beside that copy (the reference's PfJob states,
 * stbl/model.cu:92-97, 397-414, 478-494): a guess of its layer not yet claimed by the copy is cancelled
 * when the call does not route to it (its slot is freed) and taken over when it does (the call copies
 * it; a miss); guesses being copied or landed are hits, and the call's expert kernels wait for the copy.
 * Landed guesses of earlier layers are forgotten (no longer counted as prefetched).  File-backed caches
 * read whole prefetches: their next call waits for the prefetch before planning, so nothing is
 * cancelled.  Counters: experts prefetched, prefetched experts a later call routed to (landed or being
 * copied), bytes the prefetch copies wrote. */
int stbl_cache_prefetch(stbl_cache *c, int layer, const int *ids, int n, int consider, cudaStream_t stream,
                        cudaStream_t copy_stream);
int stbl_cache_prefetch_stats(const stbl_cache *c, uint64_t *prefetched, uint64_t *used, uint64_t *bytes);
/* The same counters in the layout of the reference's stbl_prefetch (stbl/stbl.h:23-24, printed by
 * stbl/run.py:100): out[0] guesses issued, out[1] guesses routed to after they landed, out[2] guesses
 * routed to while still being copied, out[3] guesses cancelled (guesses a call took over count as its
 * misses, as in the reference).  Waits for the device. */
int stbl_cache_prefetch_counters(const stbl_cache *c, uint64_t *out);
/* Each call of layer m (attached to a cache) then also runs `next`'s router on m's input and prefetches
 * its top n_predict experts per token (first `consider` distinct ones, stbl_cache_prefetch) for `next`,
 * copied on copy_stream beside m's expert kernels.  next: a layer attached to the same cache, or NULL
 * to stop.  Single-GPU; n_predict <= 16. */
int stbl_moe_attach_prefetch(stbl_moe *m, const stbl_moe *next, int n_predict, int consider, cudaStream_t copy_stream);

/* The reference engine's MXFP4 storage, GGUF blocks of 17 bytes per 32 values (the e8m0 scale, then 16
 * bytes holding values 0..15 in the low nibbles and 16..31 in the high nibbles; stbl/kernels.cu:134-141,
 * tools/convert_official.py:187-201), into the layer's STBL_FMT_MXFP4 layout: codes [rows][k/2] (even
 * index in the low nibble) and scales [rows][k/32].  Device buffers, enqueued on `stream`; k a multiple of
 * 32.  Lossless: the reference's weights load into a layer this way, once. */
int stbl_mxfp4_from_gguf(const void *blocks, int rows, int k, void *codes, void *scales, cudaStream_t stream);

/* The layer inside its transformer block, the reference's FFN sub-block (stbl/model.cu:803-805), in the
 * layer's own launches:
 *   x = bf16(norm_w * (x_pre * rsqrt(mean(x_pre^2) + eps)))   stbl_rms_norm (stbl/kernels.cu:217-236, 594-596),
 *       fused into the router kernel, same operations and reduction order (bit-identical)
 *   y = the layer's output for x                             moe() / stbl_moe_forward
 *   h_out[t][j][d] = bf16(post[t][j] * y[t][d] + sum_a comb[t][a][j] * res[t][a][d]) for j < hc
 *                                                            stbl_hc_post (stbl/kernels.cu:328-338, 609-612),
 *       fused into the combine kernel, same rounding steps (bit-identical)
 * x_pre fp32 [T][hidden] (the hc_pre output), norm_w fp32 [hidden], res fp32 [T][hc][hidden], post fp32
 * [T][hc], comb fp32 [T][hc][hc], h_out fp32 [T][hc][hidden] (bf16 values); device pointers, x_pre,
 * norm_w, res and h_out 16-byte aligned; hc <= 16; single-GPU layers. */
int stbl_moe_forward_block(stbl_moe *m, const float *x_pre, const float *norm_w, float eps, const float *res,
                           const float *post, const float *comb, int hc, int T, float *h_out, cudaStream_t stream);

/* Device status bits raised by kernels since the last call of this function (waits for the
 * device): 1 a wait timed out, 2 a dispatch entry was out of range, 4 copies were still in flight
 * when a CTA gave up, 8 an expert read from the checkpoint failed (file-backed cache).  0 when every
 * call so far ran cleanly. */
int stbl_moe_status(stbl_moe *m, uint32_t *status);

/* Per-kernel device timing, the counterpart of the reference's STBL_TIMING / stbl_timing
 * (stbl/model.cu:13-15, 250-258; stbl/stbl.h:32-34), without its stream synchronisations: while
 * enabled, every call records CUDA events on its stream around the router, expert-up and
 * expert-down launches.  stbl_moe_timing waits for the recorded events, adds their durations to
 * per-section totals in seconds (order: router, expert up, expert down; sec[3] = number of calls
 * timed) and returns the number of entries written (4). */
int stbl_moe_set_timing(stbl_moe *m, int enable);
int stbl_moe_timing(stbl_moe *m, double *sec, int n);

/* Kernel launches per forward call and layer counters. */
void stbl_moe_stats(const stbl_moe *m, uint64_t *calls, uint64_t *tokens, int *launches_per_call);

const char *stbl_moe_error(const stbl_moe *m);
void stbl_moe_destroy(stbl_moe *m);

/* Expert parallelism over the GPUs of one node (NVLink / NVSwitch).  Rank `rank` of `n_ranks` (<= 8,
 * dividing n_experts) holds routed experts [rank E/n, (rank+1) E/n): desc->routed_w/routed_s point at
 * the first of them (desc->n_experts stays the global count; the router and its weights are global,
 * the shared expert is replicated).  Each rank routes its own tokens; dispatch and combine are done by
 * the layer's kernels with stores into peer GPUs' memory through one exchange region per rank (no
 * host synchronisation, no collective library in the data path).  Needs FP8 routed experts.
 * Bring-up: every rank creates its layer, exports its region with stbl_moe_ep_handle, the host
 * side gathers the n_ranks handles in rank order (any transport: the Python mirror uses
 * torch.distributed all_gather_object) and passes them to stbl_moe_ep_connect.  After that every
 * rank must call stbl_moe_forward the same number of times, in the same order across layers (each
 * call exchanges with every rank); device waits on other ranks time out after 1 s and raise status
 * bit 1.  This replaces the reference design's NCCL all-to-all pair (dispatch, combine). */
#define STBL_EP_HANDLE_BYTES 64
int stbl_moe_create_ep(const stbl_moe_desc *desc, int rank, int n_ranks, stbl_moe **out, char *err, int errlen);
int stbl_moe_ep_handle(stbl_moe *m, void *handle /* STBL_EP_HANDLE_BYTES */);
int stbl_moe_ep_connect(stbl_moe *m, const void *handles /* n_ranks x STBL_EP_HANDLE_BYTES, rank order */);

/* Routing without allocating.  This entry point has no counterpart in the reference; it exists for
 * callers that cannot allocate device memory: engines that own a fixed memory pool and allow no
 * allocation outside it, embedded runtimes without an allocator.  It runs the layer's router (logits, scores, group-limited top-k, routing weights,
 * bucketed dispatch; the same kernels and results as stbl_moe_forward's routing) for T tokens with
 * all of its working memory in one fixed array inside the library (86,784 bytes, held by every GPU
 * that loads the library until the process exits; x is not quantized for expert kernels here).  Limits: T <= 64, n_experts <= 256, hidden a
 * multiple of 128 up to 8192 (up to 2048 when it is not a multiple of 512), topk <= 16; larger sizes
 * are rejected with a message in err.  router_w and x must be 16-byte aligned.  Inputs and outputs
 * are device buffers owned by the caller: idx, weights [T][topk], counts [E], offsets [E+1],
 * perm [T*topk] (as stbl_moe_last_route).  Every call shares the array, so calls that overlap on the
 * GPU race: serialise them.  The first call on each device looks the array up
 * (cudaGetSymbolAddress); make it before any stream capture.  Returns 0, or -1 with err filled. */
int stbl_route_noalloc(const float *router_w, const float *router_bias, const void *x_bf16, int T, int n_experts,
                       int hidden, int topk, int n_groups, int topk_groups, int score_fn, float route_scale, int *idx,
                       float *weights, int *counts, int *offsets, int *perm, cudaStream_t stream, char *err,
                       int errlen);

/* The Q8 linear of the act_q8 layers alone: y[t][r] = sum over K of dequantized w[r] times
 * dequantized q[t], for MXFP4 weights (codes [rows][k/2], value 2j in the low nibble of byte j; e8m0
 * scales [rows][k/32]) and Q8 activations (int8 codes q [n_tok][k], fp32 scales d [n_tok][k/32], the
 * rule of ref/emulate_ds4.py:23-30).  The FP4 branch of the reference's emulated linear
 * (ref/emulate_ds4.py:69-77), which the reference's kernels.h has no launcher for: per 32-value
 * block an exact integer dot product (twice every e2m1 value is an integer), scaled in fp32.  Device
 * buffers, w and q 16-byte aligned, k a multiple of 32; fp32 out [n_tok][rows], not rounded.
 * Enqueued on `stream`.  Returns 0, or -1 for a bad argument or launch. */
int stbl_gemv_mxfp4_q8(float *y, const void *w, const void *scales, const int8_t *q, const float *d, int rows, int k,
                       int n_tok, cudaStream_t stream);

/* Status bits the router kernels raised during the stbl_route_noalloc calls on the current device
 * since the last read (waits for the device, then clears them; bits as stbl_moe_status: 1 a bounded
 * wait ran out, 2 a table entry was out of range).  Each stbl_route_noalloc call clears the word on
 * its stream before its kernels run, so a read right after a call covers that call.  Non-zero: the
 * outputs of those calls are not valid.  Returns 0, or -1 if the device could not be read. */
int stbl_route_noalloc_status(uint32_t *status);

#ifdef __cplusplus
}
#endif
