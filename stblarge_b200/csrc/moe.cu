// Layer object and C ABI of the MoE decode path (include/stbl_moe.h).
//
// One layer call is six kernel launches on the caller's stream for FP8 experts (seven above 16
// tokens, eight when the routed experts are MXFP4): router logits, router selection + dispatch,
// expert up (+ SwiGLU), act_quant of h, expert down, combine.  They are chained with programmatic
// dependent launch, so each kernel's CTAs start while the previous kernel drains.  No host
// synchronisation inside a call.
#include <stdio.h>
#include <string.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/stbl_moe.h"
#include "layer.cuh"
#include "tc_params.cuh"
#include "ep.cuh"
#include "cache.cuh"

namespace stbl {
const void *combine_kernel_ptr();                 // combine.cu
const void *expert_tc_kernel_ptr(bool up, bool two, bool wide);  // experts_tc.cu
const void *expert_tc4_kernel_ptr(bool up, bool wide);  // experts_tc4.cu
int expert_tc4_smem_bytes(bool up, int nst, bool wide);
int expert_tc4_partial_cols();
cudaError_t launch_sf_repack(const uint8_t *src, long long src_stride, uint8_t *dst, long long dst_stride, int rows, int K,
                             int z0, int nz, int rps, cudaStream_t st);
const void *gather_kernel_ptr();                  // experts_tc.cu
const void *hquant_kernel_ptr();                  // experts_tc.cu
int expert_tc_smem_bytes(bool up, int H, int I, int nst, bool two, bool wide);
cudaError_t launch_q8(bool up, const Q8Params &p, int sms, cudaStream_t st);  // experts_q8.cu
}  // namespace stbl

using namespace stbl;

#define CK(x)                                                                                        \
    do {                                                                                             \
        cudaError_t e_ = (x);                                                                        \
        if (e_ != cudaSuccess) throw std::runtime_error(std::string(#x) + ": " + cudaGetErrorString(e_)); \
    } while (0)

namespace {

// events of one timed call: before the router, after it, after the up launches, after the downs
struct TimedCall {
    cudaEvent_t ev[4];
};

int act_blk_of(int fmt) { return fmt == STBL_FMT_FP8_B128 ? 128 : 32; }
int act_pow2_of(int fmt) { return fmt == STBL_FMT_FP8_B128 ? 0 : 1; }

long long mat_bytes(int fmt, int rows, int k, bool scales) {
    if (fmt == STBL_FMT_FP8_B128)
        return scales ? 4LL * ((rows + 127) / 128) * ((k + 127) / 128) : (long long)rows * k;
    if (fmt == STBL_FMT_FP8_E8M0) return scales ? (long long)((rows + 31) / 32) * (k / 32) : (long long)rows * k;
    return scales ? (long long)rows * (k / 32) : (long long)rows * (k / 2);
}

// weight rows that share one row of e8m0 scales: 32 for FP8 with 32x32 blocks, 1 for MXFP4
int scale_rows_of(int fmt) { return fmt == STBL_FMT_FP8_E8M0 ? 32 : 1; }



}  // namespace

struct stbl_moe {
    stbl_moe_desc d{};
    int E = 0, H = 0, I = 0, K = 0, Tmax = 0, ksplit = 1, sms = 0, has_shared = 0;
    // expert parallelism: this rank holds routed experts [ep_rank E_loc, (ep_rank + 1) E_loc)
    int ep_rank = 0, ep_n = 1, E_loc = 0;
    int routed_cap = 0;               // routed rows of the position-ordered buffers
    char *ep_region = nullptr;        // exchange region (expert parallelism), exported by CUDA IPC
    EpLayout ep_L{};
    char *ep_peer[kEpMaxRanks] = {};
    bool ep_connected = false;
    unsigned int ep_epoch = 0;
    int *a_dst = nullptr, *n_rows = nullptr;
    unsigned int *ep_done_ctr = nullptr;
    int *wide_sel = nullptr;  // the call's chunk width choice (1: 32 tokens), written by the router / count exchange  // expert parallelism: the down kernel's CTA ticket (ep.cu zeroes it per call)
    int *sel_cnt = nullptr;
    uint32_t *sel_bm = nullptr;
    unsigned int *sel_ticket = nullptr;
    void *ws = nullptr;
    size_t ws_bytes = 0;
    float *scores = nullptr, *wts = nullptr, *xs_a = nullptr, *xs_b = nullptr;
    int *idx = nullptr, *counts = nullptr, *offsets = nullptr, *perm = nullptr, *n_chunks = nullptr;
    Chunk *chunks = nullptr;
    uint8_t *xq_a = nullptr, *xq_b = nullptr;
    uint16_t *h = nullptr, *eo = nullptr, *sh = nullptr, *xin = nullptr, *yout = nullptr;
    uint32_t *status = nullptr;
    float *tc_partial = nullptr;      // split-item partial sums: FP8 body [sms][128][<= 64], then MXFP4 [sms][128][64]
    unsigned int *tc_flags = nullptr; // [2][sms] launch number whose partial a CTA slot holds (FP8, MXFP4 bodies)
    unsigned int tc_seq = 0;
    // expert slots: routed expert e reads slot slot[e] of the strided weight arrays (an expert cache
    // re-points experts at other slots, stbl_moe_set_expert)
    int *slot = nullptr;
    std::vector<int> host_slot;
    int n_slots = 0;                  // slots in the routed arrays
    bool slots_moved = false;         // some expert reads a slot other than its own id
    stbl_cache *cache = nullptr;      // attached expert cache (stbl_moe_attach_cache), layer cache_layer
    int cache_layer = 0;
    // shadow next-layer prefetch (stbl_moe_attach_prefetch): the next layer's router on this layer's
    // input, its top pf_predict experts per token prefetched into the cache (pf_consider counted)
    const stbl_moe *pf_next = nullptr;
    int pf_predict = 0, pf_consider = 0;
    cudaStream_t pf_stream = nullptr;
    void *pf_ws = nullptr;
    RouterParams pf_r{};              // the shadow router's buffers (inputs and routing set per call)
    long long w_stride[3] = {0, 0, 0}, s_stride[3] = {0, 0, 0};  // bytes between slots
    // tensor-core kernels (FP8 experts): tensor maps, launch shape
    TcMaps tc_up{}, tc_down{};
    int tc_nst_up = 0, tc_nst_down = 0, tc_smem_up = 0, tc_smem_down = 0;
    int tc_nst_down2 = 0, tc_smem_down2 = 0;  // the down kernel with two-tile items (T >= 4)
    int tc_nst_up2 = 0, tc_smem_up2 = 0;      // the up kernel with two-tile items (128 gate + 128 up rows)
    int tc_nst_upw = 0, tc_smem_upw = 0, tc_nst_downw = 0, tc_smem_downw = 0;  // two-tile items of up to 32 tokens
    TcMaps tc_up2{};                          // its maps: 128-row boxes of the gate and up matrices
    bool routed_tc = false;           // routed experts on the FP8 tensor-core kernels
    bool routed_bs = false;           // routed experts MXFP4 or FP8-e8m0: the block-scaled tensor-core kernels
    bool shared_bs = false;           // shared expert FP8-e8m0: handled by the block-scaled kernels too
    uint8_t *sf_shared = nullptr;     // the shared expert's scales in the scale-block layout (3 matrices)
    long long sf_shared_off[3] = {0, 0, 0};
    TcMaps tc4_up{}, tc4_down{};      // MXFP4 weight maps (16 codes padded to 16 bytes in shared memory)
    int tc4_nst[2][2] = {}, tc4_nst8[2][2] = {}, tc4_smem[2][2] = {};  // [up][wide]: stages of both bodies, bytes
    uint8_t *xe8_a = nullptr, *xe8_pos = nullptr, *he8 = nullptr;  // e8m0 activation scales (per 32), [K/128][rows][16 B]
    int Tpad = 0, pos_rows = 0;       // rows of the token-ordered and position-ordered activation buffers
    // MXFP4 weight scales in the scale-block layout: the layer's own copy (natural scales given), slot z
    // of matrix m at sf_own + z * sf_own_stride + sf_own_off[m]
    uint8_t *sf_own = nullptr;
    long long sf_own_stride = 0, sf_own_off[3] = {0, 0, 0};
    uint8_t *hq = nullptr, *xq_pos = nullptr;
    float *hs = nullptr, *xs_pos = nullptr;
    bool act_q8 = false;              // routed MXFP4 experts with Q8 activations (CUDA-core kernels)
    float *hd8 = nullptr;             // Q8 scales of h by position [pos][I / 32]
    CUtensorMap bmap_xa{}, bmap_xb{}, bmap_xpos{}, bmap_hq{};  // activation tiles for the tensor-core kernels
    CUtensorMap bmap_xa32{}, bmap_xb32{}, bmap_xpos32{}, bmap_hq32{};  // the same in 32-row tiles (32-token items)
    CUtensorMap bmap4_xa{}, bmap4_xpos{}, bmap4_hq{};         // the same, two K blocks per box (MXFP4 kernels)
    CUtensorMap bmap4w_xpos{}, bmap4w_hq{};                   // 32-row boxes (MXFP4 items of up to 32 tokens)

    int last_T = 0;
    uint64_t calls = 0, tokens = 0;
    int launches = 0;
    std::string err;
    // timing (stbl_moe_set_timing)
    int timing = 0;
    std::vector<TimedCall> pending, event_pool;
    double tsum[3] = {0, 0, 0};
    uint64_t tcalls = 0;
};

namespace {

template <typename T>
T *carve(char *&p, size_t n) {
    T *r = reinterpret_cast<T *>(p);
    p += (n * sizeof(T) + 255) & ~(size_t)255;
    return r;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !ptr) throw std::runtime_error("cuTensorMapEncodeTiled unavailable");
        fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// 3-D tensor map over `experts` matrices of [rows][K] e4m3 codes (expert stride in bytes), read in
// tiles of 128 bytes x box_rows rows with the 128-byte swizzle the MMA descriptors expect
CUtensorMap weight_map(const void *base, int K, int rows, int experts, long long estride, int box_rows) {
    CUtensorMap m;
    const cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)experts};
    const cuuint64_t strides[2] = {(cuuint64_t)K, (cuuint64_t)estride};
    const cuuint32_t box[3] = {128, (cuuint32_t)box_rows, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, es,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed for an expert weight tensor");
    return m;
}

// The same over MXFP4 codes (two per byte), as a 4-D view {128 codes, rows, K blocks, experts} whose
// K-block dimension (64 bytes apart) comes after the rows: one box is 128 rows x 2 K blocks, 128
// contiguous bytes of each row, landing as two [128 rows][128 B] tiles.  The map's data type unpacks
// each 16 codes to 16 bytes in shared memory, the layout kind::mxf8f6f4 reads e2m1 operands in; the
// transaction count of a box is its packed size.  Needs 32-byte aligned base and strides.
// The same view of e4m3 codes (FP8 with e8m0 32x32 block scales): one box is 128 rows x 2 K blocks of
// 128 bytes, landing as two [128 rows][128 B] tiles, the operand layout of the block-scaled MMA.
CUtensorMap weight_map8x2(const void *base, int K, int rows, int experts, long long estride) {
    CUtensorMap m;
    if (((uintptr_t)base & 15) || (estride & 15) || (K & 15))
        throw std::runtime_error("FP8 expert weights must be 16-byte aligned (base, row and expert strides)");
    const cuuint64_t dims[4] = {128, (cuuint64_t)rows, (cuuint64_t)(K / 128), (cuuint64_t)experts};
    const cuuint64_t strides[3] = {(cuuint64_t)K, 128, (cuuint64_t)(estride ? estride : (long long)rows * K)};
    const cuuint32_t box[4] = {128, 128, (cuuint32_t)kT4StageKb, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void *>(base), dims, strides, box, es,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed for an FP8-e8m0 expert weight tensor");
    return m;
}

CUtensorMap weight_map4(const void *base, int K, int rows, int experts, long long estride) {
    CUtensorMap m;
    if (((uintptr_t)base & 31) || (estride & 31) || ((K / 2) & 31))
        throw std::runtime_error("MXFP4 expert weights must be 32-byte aligned (base, row and expert strides)");
    const cuuint64_t dims[4] = {128, (cuuint64_t)rows, (cuuint64_t)(K / 128), (cuuint64_t)experts};
    const cuuint64_t strides[3] = {(cuuint64_t)(K / 2), 64, (cuuint64_t)estride};
    const cuuint32_t box[4] = {128, 128, (cuuint32_t)kT4StageKb, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 4, const_cast<void *>(base), dims, strides, box,
                                   es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed for an MXFP4 expert weight tensor");
    return m;
}

void launch_pdl(const void *fn, dim3 grid, dim3 block, void **args, size_t smem, cudaStream_t st);

// 3-D view {128 codes, rows, K blocks} of [rows][K] e4m3 activation codes: one box is box_rows (16 or
// 32) rows x 2 K blocks, landing as two [box_rows][128 B] tiles (128B swizzle); the MXFP4 kernels' B
// operand
CUtensorMap act_map2(const void *base, int K, int rows, int box_rows = 16) {
    CUtensorMap m;
    const cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)(K / 128)};
    const cuuint64_t strides[2] = {(cuuint64_t)K, 128};
    const cuuint32_t box[3] = {128, (cuuint32_t)box_rows, (cuuint32_t)kT4StageKb};
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, es,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed for an activation tensor");
    return m;
}

// 2-D tensor map over [rows][K] e4m3 activation codes, read in 16-row x 128-byte tiles (128B swizzle)
CUtensorMap act_map(const void *base, int K, int rows, int box_rows = 16) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, es,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed for an activation tensor");
    return m;
}

// exchange-region layout (expert parallelism); the same on every rank
EpLayout ep_layout(int E, int n, int routed_cap, int Tmax, int K, int H) {
    EpLayout L{};
    long long o = 0;
    auto take = [&](long long bytes) {
        const long long r = o;
        o += (bytes + 255) & ~255LL;
        return r;
    };
    L.inbox = take(4LL * n * E);
    L.cnt_flag = take(4LL * kEpMaxRanks);
    L.pay_flag = take(4LL * kEpMaxRanks);
    L.done_flag = take(4LL * kEpMaxRanks);
    L.xq_pos = take((long long)(routed_cap + Tmax + kPosPad) * H);
    L.xs_pos = take(4LL * (routed_cap + Tmax + kPosPad) * (H / 128));
    L.pos_meta = take(4LL * routed_cap);
    L.pos_w = take(4LL * routed_cap);
    L.eo = take(2LL * Tmax * K * H);
    L.bytes = o;
    return L;
}

void create(stbl_moe *m, const stbl_moe_desc *d, int ep_rank = 0, int ep_n = 1) {
    if (!d) throw std::runtime_error("null description");
    m->d = *d;
    const int H = d->hidden, I = d->inter, Eg = d->n_experts, K = d->topk;
    if (ep_n < 1 || ep_n > kEpMaxRanks || ep_rank < 0 || ep_rank >= ep_n) throw std::runtime_error("bad rank / n_ranks (n_ranks <= 8)");
    if (Eg % ep_n) throw std::runtime_error("n_experts must be a multiple of n_ranks");
    if (ep_n > 1 && d->routed_fmt != STBL_FMT_FP8_B128) throw std::runtime_error("expert parallelism needs FP8 routed experts");
    m->ep_rank = ep_rank, m->ep_n = ep_n;
    // the router sees every expert; the expert kernels see this rank's E / n_ranks
    const int E = Eg / ep_n;
    if (H <= 0 || I <= 0 || H % 512 || I % 512) throw std::runtime_error("hidden and inter must be multiples of 512");
    if (Eg < 1 || Eg > kMaxExperts) throw std::runtime_error("n_experts must be in 1..512");
    if (K < 1 || K > kMaxTopk || K > Eg) throw std::runtime_error("topk must be in 1..16 and <= n_experts");
    if (d->n_groups < 1 || d->n_groups > 32 || Eg % d->n_groups) throw std::runtime_error("n_groups must divide n_experts and be <= 32");
    if (d->topk_groups < 1 || d->topk_groups > d->n_groups) throw std::runtime_error("topk_groups must be in 1..n_groups");
    const int gsz = Eg / d->n_groups;
    const bool grouped = d->n_groups > 1 && d->topk_groups < d->n_groups;
    if (grouped && (gsz < 2 || d->topk_groups * gsz < K)) throw std::runtime_error("kept groups hold fewer than topk experts");
    if (d->score_fn != STBL_SCORE_SIGMOID && d->score_fn != STBL_SCORE_SQRT_SOFTPLUS) throw std::runtime_error("bad score_fn");
    if (d->routed_fmt != STBL_FMT_FP8_B128 && d->routed_fmt != STBL_FMT_MXFP4 && d->routed_fmt != STBL_FMT_FP8_E8M0)
        throw std::runtime_error("bad routed_fmt");
    if (d->shared_fmt != STBL_FMT_FP8_B128 && d->shared_fmt != STBL_FMT_FP8_E8M0 && d->shared_fmt != STBL_FMT_NONE)
        throw std::runtime_error("bad shared_fmt");
    if (d->routed_fmt == STBL_FMT_FP8_B128 && d->shared_fmt == STBL_FMT_FP8_E8M0)
        throw std::runtime_error("an FP8-e8m0 shared expert needs block-scaled routed experts (MXFP4 or FP8-e8m0)");
    if (d->max_tokens < 1 || d->max_tokens > kRouterMaxTokens) throw std::runtime_error("max_tokens must be in 1..256");
    if (d->act_q8 != 0 && d->act_q8 != 1) throw std::runtime_error("act_q8 must be 0 or 1");
    if (d->act_q8) {
        if (d->routed_fmt != STBL_FMT_MXFP4) throw std::runtime_error("act_q8 needs MXFP4 routed experts");
        if (d->shared_fmt != STBL_FMT_FP8_B128 && d->shared_fmt != STBL_FMT_NONE)
            throw std::runtime_error("act_q8 needs an FP8 128x128 shared expert or none");
        if (d->routed_s_blocked) throw std::runtime_error("act_q8 reads the natural MXFP4 scale layout (routed_s_blocked 0)");
        if (ep_n > 1) throw std::runtime_error("act_q8 layers are single-GPU");
        if (d->inter > 4096) throw std::runtime_error("act_q8 needs inter <= 4096");
    }
    if (H / router_ksplit(H) > kLgMaxSlice) throw std::runtime_error("hidden must be at most 8192");
    if (!d->router_w || !d->router_bias) throw std::runtime_error("router weights missing");
    if ((uintptr_t)d->router_w & 15) throw std::runtime_error("router weights must be 16-byte aligned");
    m->E = Eg, m->E_loc = E, m->H = H, m->I = I, m->K = K, m->Tmax = d->max_tokens;
    m->ksplit = router_ksplit(H);
    m->has_shared = d->shared_fmt != STBL_FMT_NONE;

    // routed experts: slots of strided arrays (slot e = expert e until an expert cache re-points it)
    if (d->n_slots < 0 || d->n_slots > (1 << 20)) throw std::runtime_error("n_slots must be in 0..2^20");
    if (ep_n > 1 && d->n_slots > 0 && d->n_slots != E) throw std::runtime_error("expert parallelism takes no extra slots");
    m->n_slots = d->n_slots > 0 ? d->n_slots : E;
    m->host_slot.resize(E);
    for (int e = 0; e < E; e++) m->host_slot[e] = e < m->n_slots ? e : 0;  // fewer slots: an expert cache places them
    const int rows[3] = {I, I, H}, ks[3] = {H, H, I};
    for (int mt = 0; mt < 3; mt++) {
        if (!d->routed_w[mt] || !d->routed_s[mt]) throw std::runtime_error("routed expert weights missing");
        m->w_stride[mt] = d->routed_w_stride[mt] ? d->routed_w_stride[mt] : mat_bytes(d->routed_fmt, rows[mt], ks[mt], false);
        m->s_stride[mt] = d->routed_s_stride[mt] ? d->routed_s_stride[mt] : mat_bytes(d->routed_fmt, rows[mt], ks[mt], true);
        if (((uintptr_t)d->routed_w[mt] & 15) || ((uintptr_t)d->routed_s[mt] & 15) || (m->w_stride[mt] & 15) || (m->s_stride[mt] & 3))
            throw std::runtime_error("expert weights must be 16-byte aligned");
        if (m->has_shared) {
            if (!d->shared_w[mt] || !d->shared_s[mt]) throw std::runtime_error("shared expert weights missing");
            if (((uintptr_t)d->shared_w[mt] & 15) || ((uintptr_t)d->shared_s[mt] & 15))
                throw std::runtime_error("shared expert weights must be 16-byte aligned");
        }
    }

    int dev = 0, max_smem = 0;
    CK(cudaGetDevice(&dev));
    CK(cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, dev));
    CK(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));

    // workspace (+ the exchange region under expert parallelism)
    const int T = m->Tmax, Tpad = (T + 15) / 16 * 16;
    m->routed_cap = ep_n * T * K;
    const int npos = m->routed_cap + T;
    if (ep_n > 1) {
        m->ep_L = ep_layout(Eg, ep_n, m->routed_cap, T, K, H);
        CK(cudaMalloc(&m->ep_region, m->ep_L.bytes));
        CK(cudaMemset(m->ep_region, 0, m->ep_L.bytes));
        m->ep_peer[ep_rank] = m->ep_region;
    }
    auto layout = [&](char *base) {
        char *p = base;
        m->slot = carve<int>(p, E);
        m->scores = carve<float>(p, (size_t)T * Eg);
        m->idx = carve<int>(p, (size_t)T * K);
        m->wts = carve<float>(p, (size_t)T * K);
        m->counts = carve<int>(p, Eg);
        m->offsets = carve<int>(p, Eg + 1);
        m->perm = carve<int>(p, (size_t)T * K);
        m->chunks = carve<Chunk>(p, npos);
        m->n_chunks = carve<int>(p, 4);
        m->xq_a = carve<uint8_t>(p, (size_t)Tpad * H);
        m->xs_a = carve<float>(p, (size_t)Tpad * (H / 32));
        m->xq_b = carve<uint8_t>(p, (size_t)Tpad * H);
        m->xs_b = carve<float>(p, (size_t)Tpad * (H / 32));
        m->xe8_a = carve<uint8_t>(p, (size_t)(H / 128) * Tpad * 16);
        m->xe8_pos = carve<uint8_t>(p, (size_t)(H / 128) * (npos + kPosPad) * 16);
        m->he8 = carve<uint8_t>(p, (size_t)(I / 128) * (npos + kPosPad) * 16);
        m->xq_pos = ep_n > 1 ? nullptr : carve<uint8_t>(p, (size_t)(npos + kPosPad) * H);
        m->xs_pos = ep_n > 1 ? nullptr : carve<float>(p, (size_t)(npos + kPosPad) * (H / 128));
        m->h = carve<uint16_t>(p, (size_t)npos * I);
        m->hq = carve<uint8_t>(p, (size_t)(npos + kPosPad) * I);
        m->hs = carve<float>(p, (size_t)(npos + kPosPad) * (I / 128));
        m->hd8 = d->act_q8 ? carve<float>(p, (size_t)(npos + kPosPad) * (I / 32)) : nullptr;
        m->eo = ep_n > 1 ? nullptr : carve<uint16_t>(p, (size_t)T * K * H);
        m->sh = carve<uint16_t>(p, (size_t)T * H);
        m->xin = carve<uint16_t>(p, (size_t)T * H);
        m->yout = carve<uint16_t>(p, (size_t)T * H);
        m->status = carve<uint32_t>(p, 4);
        m->tc_partial = carve<float>(p, (size_t)m->sms * 128 * (64 + 64));
        m->tc_flags = carve<unsigned int>(p, 2 * m->sms);
        m->a_dst = carve<int>(p, (size_t)T * K);
        m->n_rows = carve<int>(p, 4);
        m->ep_done_ctr = carve<unsigned int>(p, 1);
        m->wide_sel = carve<int>(p, 1);
        m->sel_cnt = carve<int>(p, Eg);
        m->sel_bm = carve<uint32_t>(p, (size_t)Eg * ((T + 31) / 32));
        m->sel_ticket = carve<unsigned int>(p, 4);
        return (size_t)(p - base);
    };
    m->ws_bytes = layout(nullptr);
    CK(cudaMalloc(&m->ws, m->ws_bytes));
    CK(cudaMemset(m->ws, 0, m->ws_bytes));
    layout(static_cast<char *>(m->ws));
    if (ep_n > 1) {
        m->xq_pos = reinterpret_cast<uint8_t *>(m->ep_region + m->ep_L.xq_pos);
        m->xs_pos = reinterpret_cast<float *>(m->ep_region + m->ep_L.xs_pos);
        m->eo = reinterpret_cast<uint16_t *>(m->ep_region + m->ep_L.eo);
    }
    CK(cudaMemcpy(m->slot, m->host_slot.data(), sizeof(int) * E, cudaMemcpyHostToDevice));
    m->Tpad = Tpad, m->pos_rows = npos + kPosPad;

    CK(router_setup());
    m->routed_tc = d->routed_fmt == STBL_FMT_FP8_B128;
    m->act_q8 = d->act_q8 != 0;
    m->routed_bs = !m->routed_tc;
    m->shared_bs = d->shared_fmt == STBL_FMT_FP8_E8M0;
    if (H % 128 || I % 128 || H > 8192 || I > 8192)
        throw std::runtime_error("experts need hidden and inter multiples of 128, at most 8192");
    if (m->routed_bs && !m->act_q8) {
        const bool e8 = d->routed_fmt == STBL_FMT_FP8_E8M0;
        const long long wst4[3] = {m->w_stride[0], m->w_stride[1], m->w_stride[2]};
        const int ns = m->n_slots, rps = scale_rows_of(d->routed_fmt);
        if (!d->routed_s_blocked) {
            // the layer's own copy of every slot's scales in the scale-block layout
            long long off = 0;
            for (int mt = 0; mt < 3; mt++) {
                m->sf_own_off[mt] = off;
                off += ((long long)rows[mt] * (ks[mt] / 32) + 1023) & ~1023LL;
            }
            m->sf_own_stride = off;
            CK(cudaMalloc(&m->sf_own, (size_t)ns * off));
            for (int mt = 0; mt < 3; mt++)
                CK(launch_sf_repack(static_cast<const uint8_t *>(d->routed_s[mt]), m->s_stride[mt], m->sf_own + m->sf_own_off[mt],
                                    m->sf_own_stride, rows[mt], ks[mt], 0, ns, rps, 0));
            CK(cudaDeviceSynchronize());
        } else {
            for (int mt = 0; mt < 3; mt++)
                if (m->s_stride[mt] & 511) throw std::runtime_error("block-layout MXFP4 scales need a slot stride multiple of 512");
        }
        auto wmap = [&](const void *base, int K, int R, int n, long long st) {
            return e8 ? weight_map8x2(base, K, R, n, st) : weight_map4(base, K, R, n, st);
        };
        m->tc4_up.w[0] = wmap(d->routed_w[0], H, I, ns, wst4[0]);
        m->tc4_up.w[1] = wmap(d->routed_w[1], H, I, ns, wst4[1]);
        m->tc4_down.w[0] = m->tc4_down.w[1] = wmap(d->routed_w[2], I, H, ns, wst4[2]);
        m->tc4_up.s[0] = m->tc4_up.s[1] = m->tc4_up.w[0];
        m->tc4_down.s[0] = m->tc4_down.s[1] = m->tc4_down.w[0];
        if (m->shared_bs) {
            // FP8-e8m0 shared expert on the same kernels: its own maps and scale blocks
            m->tc4_up.s[0] = weight_map8x2(d->shared_w[0], H, I, 1, (long long)I * H);
            m->tc4_up.s[1] = weight_map8x2(d->shared_w[1], H, I, 1, (long long)I * H);
            m->tc4_down.s[0] = m->tc4_down.s[1] = weight_map8x2(d->shared_w[2], I, H, 1, (long long)H * I);
            long long off = 0;
            for (int mt = 0; mt < 3; mt++) {
                m->sf_shared_off[mt] = off;
                off += ((long long)rows[mt] * (ks[mt] / 32) + 1023) & ~1023LL;
            }
            CK(cudaMalloc(&m->sf_shared, (size_t)off));
            for (int mt = 0; mt < 3; mt++)
                CK(launch_sf_repack(static_cast<const uint8_t *>(d->shared_s[mt]), 0, m->sf_shared + m->sf_shared_off[mt], 0,
                                    rows[mt], ks[mt], 0, 1, 32, 0));
            CK(cudaDeviceSynchronize());
        }
        for (int mt = 0; mt < 3; mt++)
            if (((uintptr_t)d->routed_s[mt] & 15) || (m->s_stride[mt] & 15))
                throw std::runtime_error("block-scaled expert scales must be 16-byte aligned (base and expert stride)");
    }
    {
        // tensor maps: up boxes of 64 rows (T < 4: 64 gate + 64 up rows per item) and of 128 rows (128
        // gate + 128 up rows), down boxes of 128 rows (one or two per item)
        const long long wst[3] = {
            d->routed_w_stride[0] ? d->routed_w_stride[0] : (long long)I * H,
            d->routed_w_stride[1] ? d->routed_w_stride[1] : (long long)I * H,
            d->routed_w_stride[2] ? d->routed_w_stride[2] : (long long)H * I};
        if (m->routed_tc) {
            m->tc_up.w[0] = weight_map(d->routed_w[0], H, I, m->n_slots, wst[0], 64);
            m->tc_up.w[1] = weight_map(d->routed_w[1], H, I, m->n_slots, wst[1], 64);
            m->tc_up2.w[0] = weight_map(d->routed_w[0], H, I, m->n_slots, wst[0], 128);
            m->tc_up2.w[1] = weight_map(d->routed_w[1], H, I, m->n_slots, wst[1], 128);
            m->tc_down.w[0] = weight_map(d->routed_w[2], I, H, m->n_slots, wst[2], 128);
            m->tc_down.w[1] = m->tc_down.w[0];
        }
        if (m->has_shared && !m->shared_bs) {
            m->tc_up.s[0] = weight_map(d->shared_w[0], H, I, 1, (long long)I * H, 64);
            m->tc_up.s[1] = weight_map(d->shared_w[1], H, I, 1, (long long)I * H, 64);
            m->tc_up2.s[0] = weight_map(d->shared_w[0], H, I, 1, (long long)I * H, 128);
            m->tc_up2.s[1] = weight_map(d->shared_w[1], H, I, 1, (long long)I * H, 128);
            m->tc_down.s[0] = weight_map(d->shared_w[2], I, H, 1, (long long)H * I, 128);
            m->tc_down.s[1] = m->tc_down.s[0];
        }
        if (!m->routed_tc && m->has_shared && !m->shared_bs) {
            m->tc_up.w[0] = m->tc_up.w[1] = m->tc_up.s[0], m->tc_down.w[0] = m->tc_down.w[1] = m->tc_down.s[0];
            m->tc_up2.w[0] = m->tc_up2.w[1] = m->tc_up2.s[0];
        }
        if (!m->has_shared && m->routed_tc) {
            m->tc_up.s[0] = m->tc_up.s[1] = m->tc_up.w[0], m->tc_down.s[0] = m->tc_down.s[1] = m->tc_down.w[0];
            m->tc_up2.s[0] = m->tc_up2.s[1] = m->tc_up2.w[0];
        }
        if (!m->routed_tc && (!m->has_shared || m->shared_bs)) m->tc_up = m->tc_up2 = m->tc4_up, m->tc_down = m->tc4_down;  // unused, valid
        m->bmap_xa = act_map(m->xq_a, H, Tpad);
        m->bmap_xb = act_map(m->xq_b, H, Tpad);
        m->bmap_xpos = act_map(m->xq_pos, H, npos + kPosPad);
        m->bmap_hq = act_map(m->hq, I, npos + kPosPad);
        m->bmap_xa32 = act_map(m->xq_a, H, Tpad, 32);
        m->bmap_xb32 = act_map(m->xq_b, H, Tpad, 32);
        m->bmap_xpos32 = act_map(m->xq_pos, H, npos + kPosPad, 32);
        m->bmap_hq32 = act_map(m->hq, I, npos + kPosPad, 32);
        m->bmap4_xa = act_map2(m->xq_a, H, Tpad);
        m->bmap4_xpos = act_map2(m->xq_pos, H, npos + kPosPad);
        m->bmap4_hq = act_map2(m->hq, I, npos + kPosPad);
        m->bmap4w_xpos = act_map2(m->xq_pos, H, npos + kPosPad, 32);
        m->bmap4w_hq = act_map2(m->hq, I, npos + kPosPad, 32);
        // stages: at least kTcBatch (4: the producer requests K blocks four at a time and first waits
        // for four free stages), at most 8 of one tile (more outstanding requests only lengthen the
        // DRAM queues, measured) or 6 of two
        auto pick = [&](bool up, bool two, bool wide, int &nst, int &smem) {
            cudaFuncAttributes fa{};
            CK(cudaFuncGetAttributes(&fa, expert_tc_kernel_ptr(up, two, wide)));
            const int nmax = two ? 6 : 8, nmin = 4;
            for (nst = nmax; nst >= nmin; nst--)
                if (expert_tc_smem_bytes(up, H, I, nst, two, wide) + (int)fa.sharedSizeBytes <= max_smem) break;
            if (nst < nmin) throw std::runtime_error("tensor-core expert kernel does not fit in shared memory");
            smem = expert_tc_smem_bytes(up, H, I, nst, two, wide);
            CK(cudaFuncSetAttribute(expert_tc_kernel_ptr(up, two, wide), cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        };
        pick(true, false, false, m->tc_nst_up, m->tc_smem_up);
        pick(true, true, false, m->tc_nst_up2, m->tc_smem_up2);
        pick(false, false, false, m->tc_nst_down, m->tc_smem_down);
        pick(false, true, false, m->tc_nst_down2, m->tc_smem_down2);
        pick(true, true, true, m->tc_nst_upw, m->tc_smem_upw);
        pick(false, true, true, m->tc_nst_downw, m->tc_smem_downw);
        if (m->routed_bs) {
            // the MXFP4 launch runs both bodies (MXFP4 routed, FP8 shared): as many stages of each as
            // fit; a MXFP4 stage is one 256-K unit of two 128-row tiles (71 KB with 16-token items, 75
            // KB with 32-token ones)
            for (int up = 1; up >= 0; up--)
                for (int wide = 0; wide < 2; wide++) {
                    cudaFuncAttributes fa{};
                    CK(cudaFuncGetAttributes(&fa, expert_tc4_kernel_ptr(up, wide)));
                    const int room = max_smem - (int)fa.sharedSizeBytes;
                    // the FP8 body takes two-tile items here (34 KB stages, 4 to 6)
                    int n4 = 6, n8 = 6;
                    const int n8min = 4;
                    while (n4 >= 2 && expert_tc4_smem_bytes(up, n4, wide) > room) n4--;
                    while (n8 >= n8min && expert_tc_smem_bytes(up, H, I, n8, true, false) > room) n8--;
                    if (n4 < 2 || n8 < n8min) throw std::runtime_error("MXFP4 tensor-core expert kernel does not fit in shared memory");
                    const int smem = std::max(expert_tc4_smem_bytes(up, n4, wide), expert_tc_smem_bytes(up, H, I, n8, true, false));
                    CK(cudaFuncSetAttribute(expert_tc4_kernel_ptr(up, wide), cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
                    m->tc4_nst[up][wide] = n4, m->tc4_nst8[up][wide] = n8, m->tc4_smem[up][wide] = smem;
                }
        }
    }
}

EpView ep_view(const stbl_moe *m) {
    EpView v{};
    v.n_ranks = m->ep_n;
    v.rank = m->ep_rank;
    v.epoch = m->ep_epoch;
    v.L = m->ep_L;
    for (int d = 0; d < m->ep_n; d++) v.region[d] = m->ep_peer[d];
    return v;
}

TcParams tc_params(stbl_moe *m, int T, bool up, bool direct = true) {
    TcParams p{};
    // slot table: the cache's map row, the layer's own table once an expert was re-pointed, else none
    // (slot = expert: the kernels skip the lookup)
    p.slot = m->cache ? m->cache->map + (size_t)m->cache_layer * m->E : (m->slots_moved ? m->slot : nullptr);
    p.chunk_cap = m->routed_cap + m->Tmax;
    p.chunks = m->chunks;
    p.n_chunks = m->n_chunks;
    p.T = T, p.topk = m->K, p.E = m->E_loc, p.H = m->H, p.I = m->I;
    p.ep = ep_view(m);
    if (m->ep_n > 1) {
        p.n_routed = m->routed_cap;
        p.pos_w = reinterpret_cast<const float *>(m->ep_region + m->ep_L.pos_w);
        p.pos_meta = reinterpret_cast<const int *>(m->ep_region + m->ep_L.pos_meta);
        p.T_max_assign = m->Tmax * m->K;
        p.ep_done_ctr = m->ep_done_ctr;
    } else {
        p.n_routed = T * m->K;
    }
    p.perm = m->perm;
    p.wts = m->wts;
    const stbl_moe_desc &d = m->d;
    if (up) {
        // direct: x codes by token for the FP8 (per-128) rule (the routed buffer when the routed experts
        // are FP8, else the shared expert's); gathered: codes by position (gather_kernel)
        p.b_direct = direct;
        if (direct) {
            p.act_s = m->routed_tc ? m->xs_a : m->xs_b;
            p.act_s_stride = m->H / 32;
        } else {
            p.act_s = m->xs_pos;
            p.act_s_stride = m->H / 128;
        }
    } else {
        p.b_direct = 0;
        p.act_s = m->hs;
        p.act_s_stride = m->I / 128;
    }
    const int I = m->I, H = m->H;
    const int mats[2] = {up ? 0 : 2, up ? 1 : 2};
    for (int i = 0; i < 2; i++) {
        const int mt = mats[i];
        p.w_scale[i] = m->routed_tc ? static_cast<const float *>(d.routed_s[mt]) : nullptr;
        p.s_scale[i] = m->has_shared ? static_cast<const float *>(d.shared_s[mt]) : nullptr;
    }
    const int rows = up ? I : H, K = up ? H : I;
    const long long sst = d.routed_s_stride[mats[0]] ? d.routed_s_stride[mats[0]]
                                                       : 4LL * ((rows + 127) / 128) * ((K + 127) / 128);
    p.w_scale_stride = sst / 4;
    if (m->routed_bs) {
        for (int i = 0; i < 2; i++)
            p.sf_a[i] = m->sf_own ? m->sf_own + m->sf_own_off[mats[i]] : static_cast<const uint8_t *>(d.routed_s[mats[i]]);
        p.sf_a_stride = m->sf_own ? m->sf_own_stride : m->s_stride[mats[0]];
        p.act_e8 = up ? (direct ? m->xe8_a : m->xe8_pos) : m->he8;
        p.act_e8_rows = up && direct ? m->Tpad : m->pos_rows;
        p.he8_rows = m->pos_rows;
        p.w_a8 = d.routed_fmt == STBL_FMT_FP8_E8M0;
        p.s_a8 = m->shared_bs;
        for (int i = 0; i < 2; i++) p.sf_s[i] = m->sf_shared ? m->sf_shared + m->sf_shared_off[mats[i]] : nullptr;
    }
    p.h = m->h;
    p.hq = m->hq, p.he8 = m->he8;
    p.swiglu_limit = m->d.swiglu_limit;
    p.eo = m->eo, p.sh = m->sh;
    p.has_shared = m->has_shared;
    p.partial = m->tc_partial;
    p.flags = m->tc_flags;
    if (++m->tc_seq == 0) m->tc_seq = 1;
    p.seq = m->tc_seq;
    p.status = m->status;
    return p;
}

// the Q8 routed products' parameters (act_q8 layers): up reads x codes by token, down h codes by
// position; weights and natural e8m0 scales of the routed slots
Q8Params q8_params(stbl_moe *m, int T, bool up) {
    Q8Params q{};
    q.slot = m->slots_moved ? m->slot : nullptr;
    q.chunks = m->chunks, q.n_chunks = m->n_chunks;
    q.T = T, q.topk = m->K, q.E = m->E_loc, q.H = m->H, q.I = m->I;
    q.perm = m->perm, q.wts = m->wts;
    const int mats[2] = {up ? 0 : 2, up ? 1 : 2};
    for (int i = 0; i < 2; i++) {
        q.w[i] = static_cast<const uint8_t *>(m->d.routed_w[mats[i]]);
        q.w_stride[i] = m->w_stride[mats[i]];
        q.s[i] = static_cast<const uint8_t *>(m->d.routed_s[mats[i]]);
        q.s_stride[i] = m->s_stride[mats[i]];
    }
    q.xq = reinterpret_cast<const int8_t *>(up ? m->xq_a : m->hq);
    q.xd = up ? m->xs_a : m->hd8;
    q.xd_stride = up ? m->H / 32 : m->I / 32;
    q.hq = reinterpret_cast<int8_t *>(m->hq), q.hd = m->hd8, q.h = m->h;
    q.swiglu_limit = m->d.swiglu_limit;
    q.eo = m->eo;
    q.status = m->status;
    return q;
}

// act_quant of h for the positions of [pos_begin, pos_end) (the down kernel's B operand)
void launch_hquant(stbl_moe *m, int pos_begin, int pos_end, cudaStream_t st) {
    if (pos_end <= pos_begin) return;
    HquantParams hp{m->h + (size_t)pos_begin * m->I, m->hq + (size_t)pos_begin * m->I, m->hs + (size_t)pos_begin * (m->I / 128),
                    pos_end - pos_begin, m->I};
    void *args[] = {&hp};
    const int warps = hp.n_pos * (m->I / 128);
    launch_pdl(hquant_kernel_ptr(), dim3((warps + 7) / 8), dim3(256), args, 0, st);
}

// Chunk widths of calls of more than 16 tokens (their chunks are read by position then).
//  * Block-scaled (MXFP4 / FP8-e8m0) routed experts, and a block-scaled shared expert, always take
//    items of up to 32 tokens: an expert routed to by 17-32 of the call's tokens streams its weights
//    once, not twice.
//  * FP8 layers choose on the device, per call (the router, or under expert parallelism the count
//    exchange): 32-token chunks when they save more than a quarter of the 16-token ones (experts with
//    many tokens, e.g. skewed routing), else 16 (the 16-token launch is faster when experts have few
//    tokens: its TMEM holds twice as many K blocks ahead of the epilogue).  Both launches of each
//    product are enqueued; the one not chosen takes no items.
//  * An FP8 shared expert inside the MXFP4 launch, and the shared expert of a Q8 layer, keep 16.
//  * Q8 routed experts keep their own 8-token chunks.
bool wide_call(int T) { return T > 16; }
bool tc4_wide(const stbl_moe *m, int T) { return m->routed_bs && !m->act_q8 && wide_call(T); }
bool fp8_adaptive(const stbl_moe *m, int T) { return m->routed_tc && wide_call(T); }
int routed_chunk_tokens(const stbl_moe *m, int T) { return m->act_q8 ? kQ8ChunkTokens : tc4_wide(m, T) ? 32 : 16; }
int shared_chunk_tokens(const stbl_moe *m, int T) { return tc4_wide(m, T) && m->shared_bs ? 32 : 16; }

// up items of 128 gate + 128 up rows from this many tokens on (the up kernel's two-tile form).
// Measured on one GPU: cfg2 T=16 up 407 -> 351 us, cfg4 T=256 layer 2.29 -> 2.07 ms; at T=1 the
// single-tile form stays (73 against 76 us).  Under expert parallelism (2 GPUs, cfg4): 1.282 ->
// 1.198 ms per step.
constexpr int kUpTwoMinT = 4;

// adaptive (fp8_adaptive): enqueue the 16-token launch and the 32-token one; each runs only if the
// device chose its width for this call (TcParams::sel).  Returns the launches enqueued.
int launch_tc(stbl_moe *m, bool up, TcParams p, cudaStream_t st, bool adaptive = false) {
    const bool up2 = up && p.T >= kUpTwoMinT;
    TcMaps maps = up ? (up2 ? m->tc_up2 : m->tc_up) : m->tc_down;
    if (adaptive) {
        // the 32-token form (two-tile items; T > 16 implies them), after the 16-token one below
        TcMaps mw = maps;
        if (up) mw.b = p.b_direct ? (m->routed_tc ? m->bmap_xa32 : m->bmap_xb32) : m->bmap_xpos32;
        else mw.b = m->bmap_hq32;
        TcParams pw = p;
        p.sel = pw.sel = m->wide_sel;
        p.sel_val = 0, pw.sel_val = 1;
        launch_tc(m, up, p, st);
        void *args[] = {&mw, &pw, up ? &m->tc_nst_upw : &m->tc_nst_downw};
        launch_pdl(expert_tc_kernel_ptr(up, true, true), dim3(m->sms), dim3(192), args, up ? m->tc_smem_upw : m->tc_smem_downw, st);
        return 2;
    }
    if (up) maps.b = p.b_direct ? (m->routed_tc ? m->bmap_xa : m->bmap_xb) : m->bmap_xpos;
    else maps.b = m->bmap_hq;
    // down items of two 128-row tiles from T = 4 on (measured at 256 experts, down kernel: T=16 218 ->
    // 185 us; at T=1 a single-tile item's shorter ramp wins, 46 against 50 us, and still with the first
    // stages' weights requested before the programmatic wait: layer call 141.3 against 144.4 us); under expert parallelism
    // too (the epilogue stores each tile's rows into the source ranks' eo rows)
    const bool two = up ? up2 : p.T >= 4;
    void *args[] = {&maps, &p, up ? (two ? &m->tc_nst_up2 : &m->tc_nst_up) : (two ? &m->tc_nst_down2 : &m->tc_nst_down)};
    launch_pdl(expert_tc_kernel_ptr(up, two, false), dim3(m->sms), dim3(192), args,
               up ? (two ? m->tc_smem_up2 : m->tc_smem_up) : (two ? m->tc_smem_down2 : m->tc_smem_down), st);
    return 1;
}

// the MXFP4 launch: p4 the routed MXFP4 chunks, p8 the FP8 shared expert's chunks (none: an empty range).
// wide: the call's block-scaled chunks hold up to 32 tokens (tc4_wide), read by position
void launch_tc4(stbl_moe *m, bool up, TcParams p8, TcParams p4, bool wide, cudaStream_t st) {
    TcMaps maps8 = up ? m->tc_up2 : m->tc_down;  // the FP8 body's two-tile items (128-row boxes)
    maps8.b = up ? m->bmap_xb : m->bmap_hq;
    TcMaps maps4 = up ? m->tc4_up : m->tc4_down;
    if (wide) maps4.b = up ? m->bmap4w_xpos : m->bmap4w_hq;
    else maps4.b = up ? (p4.b_direct ? m->bmap4_xa : m->bmap4_xpos) : m->bmap4_hq;
    p4.flags = m->tc_flags + m->sms;
    p4.partial = m->tc_partial + (size_t)m->sms * 128 * 64;
    int *n8 = &m->tc4_nst8[up][wide], *n4 = &m->tc4_nst[up][wide];
    void *args[] = {&maps8, &p8, n8, &maps4, &p4, n4};
    launch_pdl(expert_tc4_kernel_ptr(up, wide), dim3(m->sms), dim3(192), args, m->tc4_smem[up][wide], st);
}

void launch_gather(stbl_moe *m, int T, cudaStream_t st) {
    GatherParams g{m->perm, T, m->K, m->H, m->has_shared, m->xq_a, m->xs_a, m->H / 32, m->xq_pos, m->xs_pos, nullptr, nullptr};
    if (m->routed_bs) g.xe8 = m->xe8_a, g.xe8_pos = m->xe8_pos, g.xe8_rows = m->Tpad, g.xe8_pos_rows = m->pos_rows;
    void *args[] = {&g};
    // the shared expert's rows too when it reads by position (not when the FP8 body reads x by token)
    const int rows = T * m->K + (m->has_shared && (!m->routed_bs || m->shared_bs) ? T : 0);
    launch_pdl(gather_kernel_ptr(), dim3(rows), dim3(256), args, 0, st);
}


// Launch with programmatic dependent launch: the kernel may start while the previous one in the
// stream drains (its CTAs block in griddepcontrol.wait until that grid has completed).
void launch_pdl(const void *fn, dim3 grid, dim3 block, void **args, size_t smem, cudaStream_t st) {
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

TimedCall take_events(stbl_moe *m);
void collect_timing(stbl_moe *m, size_t keep);

// the block around the layer (stbl_moe_forward_block): RMSNorm before it, hyper-connection post after
struct BlockIO {
    const float *x_pre, *norm_w;
    float eps;
    const float *res, *post, *comb;
    int hc;
    float *hout;
};

void forward(stbl_moe *m, const void *x, int T, void *y, cudaStream_t st, const int *forced = nullptr,
             const BlockIO *io = nullptr) {
    if (T < 1 || T > m->Tmax) throw std::runtime_error("T must be in 1..max_tokens");
    if (io) x = io->x_pre, y = io->hout;
    if (!x || !y) throw std::runtime_error("null x or y");
    if (m->ep_n > 1 && !m->ep_connected) throw std::runtime_error("expert-parallel layer not connected (stbl_moe_ep_connect)");
    if (m->ep_n > 1 && ++m->ep_epoch == 0) m->ep_epoch = 1;
    if ((uintptr_t)x & 15) throw std::runtime_error("x must be 16-byte aligned");
    if (m->n_slots < m->E_loc && !m->cache) throw std::runtime_error("the layer has fewer slots than experts: attach its expert cache first");
    TimedCall tc{};
    if (m->timing) {
        if (m->pending.size() >= 256) collect_timing(m, 0);
        tc = take_events(m);
        CK(cudaEventRecord(tc.ev[0], st));
    }
    RouterParams r{};
    r.W = m->d.router_w, r.bias = m->d.router_bias, r.x = io ? nullptr : static_cast<const uint16_t *>(x);
    if (io) r.x_pre = io->x_pre, r.norm_w = io->norm_w, r.norm_eps = io->eps;
    r.T = T, r.E = m->E, r.H = m->H, r.topk = m->K, r.n_groups = m->d.n_groups, r.topk_groups = m->d.topk_groups;
    r.score_fn = m->d.score_fn, r.route_scale = m->d.route_scale, r.ksplit = m->ksplit, r.has_shared = m->has_shared;
    r.scores = m->scores, r.idx = m->idx, r.wts = m->wts;
    r.counts = m->counts, r.offsets = m->offsets, r.perm = m->perm, r.chunks = m->chunks, r.n_chunks = m->n_chunks;
    const int fr = m->d.routed_fmt, fs = m->has_shared ? m->d.shared_fmt : fr;
    // the routed experts' rule: the weight format's FP8 rule, or Q8 (int8 per 32) for an act_q8 layer
    const int rule_a = m->act_q8 ? kActQ8 : act_pow2_of(fr);
    r.xq_a = m->xq_a, r.xs_a = m->xs_a, r.blk_a = act_blk_of(fr), r.pow2_a = rule_a;
    if (act_blk_of(fs) == act_blk_of(fr) && act_pow2_of(fs) == rule_a)  // one quantization serves both
        r.xq_b = m->xq_a, r.xs_b = m->xs_a, r.blk_b = r.blk_a, r.pow2_b = r.pow2_a;
    else r.xq_b = m->xq_b, r.xs_b = m->xs_b, r.blk_b = act_blk_of(fs), r.pow2_b = act_pow2_of(fs);
    r.xe8_a = m->routed_bs && !m->act_q8 ? m->xe8_a : nullptr;
    r.xe8_rows = m->Tpad;
    r.nt_routed = routed_chunk_tokens(m, T);
    r.nt_shared = shared_chunk_tokens(m, T);
    r.adaptive_wide = fp8_adaptive(m, T);
    r.wide_sel = m->wide_sel;
    r.sel_cnt = m->sel_cnt, r.sel_bm = m->sel_bm, r.sel_ticket = m->sel_ticket;
    r.status = m->status;
    r.forced_idx = forced;
    CK(launch_router(r, st, true));
    int launches = 2;
    if (m->cache) {
        // bring the call's routed experts into the cache: plan (hits, LRU victims), copy the misses
        launch_cache(m->cache, m->cache_layer, m->idx, T * m->K, m->status, st);
        launches += 2;
        if (m->pf_next) {
            // the next layer's router on this layer's input (stbl/model.cu:432-436), then its guesses
            // into the cache: planned here, copied on the prefetch stream beside this call's experts
            const stbl_moe *nx = m->pf_next;
            RouterParams sr = m->pf_r;
            sr.x = r.x, sr.x_pre = r.x_pre, sr.norm_w = r.norm_w, sr.norm_eps = r.norm_eps;
            sr.W = nx->d.router_w, sr.bias = nx->d.router_bias;
            sr.T = T, sr.E = nx->E, sr.H = nx->H, sr.topk = m->pf_predict, sr.n_groups = nx->d.n_groups;
            sr.topk_groups = nx->d.topk_groups, sr.score_fn = nx->d.score_fn, sr.route_scale = nx->d.route_scale;
            sr.ksplit = nx->ksplit;
            CK(launch_router(sr, st, true));
            launch_prefetch(m->cache, nx->cache_layer, sr.idx, T * m->pf_predict, m->pf_consider, m->status, st, m->pf_stream);
            launches += 4;
        }
    }
    if (m->timing) CK(cudaEventRecord(tc.ev[1], st));

    const int npos = T * m->K + (m->has_shared ? T : 0);
    if (m->ep_n > 1) {
        // expert parallelism: counts exchange -> payload into the owners' receive rows -> up (waits
        // for every rank's payload) -> hquant -> down (outputs into the source ranks' eo rows)
        EpCountsParams cpp{};
        cpp.ep = ep_view(m);
        cpp.counts = m->counts, cpp.offsets = m->offsets, cpp.perm = m->perm, cpp.idx = m->idx;
        cpp.T = T, cpp.topk = m->K, cpp.E = m->E, cpp.E_loc = m->E_loc;
        cpp.nt_routed = routed_chunk_tokens(m, T), cpp.nt_shared = shared_chunk_tokens(m, T);
        cpp.adaptive_wide = fp8_adaptive(m, T), cpp.wide_sel = m->wide_sel;
        cpp.has_shared = m->has_shared, cpp.routed_cap = m->routed_cap;
        cpp.a_dst = m->a_dst, cpp.chunks = m->chunks, cpp.n_chunks = m->n_chunks, cpp.n_rows = m->n_rows;
        cpp.done_ctr = m->ep_done_ctr;
        cpp.status = m->status;
        EpPayloadParams ppp{};
        ppp.ep = cpp.ep;
        ppp.idx = m->idx, ppp.wts = m->wts, ppp.a_dst = m->a_dst;
        ppp.xq = m->xq_a, ppp.xs = m->xs_a, ppp.xs_stride = m->H / 32;
        ppp.T = T, ppp.topk = m->K, ppp.H = m->H, ppp.E_loc = m->E_loc, ppp.routed_cap = m->routed_cap;
        ppp.has_shared = m->has_shared;
        CK(launch_ep(cpp, ppp, m->sms, st));
        TcParams pu = tc_params(m, T, true, false), pd = tc_params(m, T, false);
        pu.chunk_begin = pd.chunk_begin = 0;
        pu.chunk_end = pd.chunk_end = -1;
        launches += launch_tc(m, true, pu, st, fp8_adaptive(m, T));
        if (m->timing) CK(cudaEventRecord(tc.ev[2], st));
        HquantParams hp{m->h, m->hq, m->hs, m->routed_cap, m->I, m->n_rows, m->has_shared ? T : 0};
        void *hargs[] = {&hp};
        // two CTAs per SM: they fit beside the down kernel's CTAs, which start early (programmatic launch)
        launch_pdl(hquant_kernel_ptr(), dim3(2 * m->sms), dim3(256), hargs, 0, st);
        launches += launch_tc(m, false, pd, st, fp8_adaptive(m, T));
        launches += 3;
    } else if (m->act_q8) {
        // routed MXFP4 experts x Q8 activations on the CUDA cores (chunks of <= 8 tokens); the FP8
        // shared expert on the tensor cores (its chunks, first in the table, read x by token):
        // [shared up] -> routed up (+ SwiGLU, Q8 of h) -> [hquant of the shared rows] -> [shared down]
        // -> routed down -> combine
        const int ns = m->has_shared ? (T + shared_chunk_tokens(m, T) - 1) / shared_chunk_tokens(m, T) : 0;
        if (ns) {
            TcParams su = tc_params(m, T, true, true);
            su.chunk_begin = 0, su.chunk_end = ns;
            launch_tc(m, true, su, st);
            launches++;
        }
        CK(launch_q8(true, q8_params(m, T, true), m->sms, st));
        if (m->timing) CK(cudaEventRecord(tc.ev[2], st));
        launches++;
        if (ns) {
            launch_hquant(m, T * m->K, npos, st);
            TcParams sd = tc_params(m, T, false);
            sd.chunk_begin = 0, sd.chunk_end = ns;
            launch_tc(m, false, sd, st);
            launches += 2;
        }
        CK(launch_q8(false, q8_params(m, T, false), m->sms, st));
        launches++;
    } else if (m->routed_tc) {
        // every expert on the tensor cores: [gather] -> up (16- and 32-token launches when the
        // width is chosen on the device) -> hquant -> down (likewise) -> combine
        const bool direct = T <= 16;
        if (!direct) {
            launch_gather(m, T, st);
            launches++;
        }
        TcParams pu = tc_params(m, T, true, direct), pd = tc_params(m, T, false);
        pu.chunk_begin = pd.chunk_begin = 0;
        pu.chunk_end = pd.chunk_end = -1;
        launches += launch_tc(m, true, pu, st, fp8_adaptive(m, T));
        if (m->timing) CK(cudaEventRecord(tc.ev[2], st));
        launch_hquant(m, 0, npos, st);
        launches += launch_tc(m, false, pd, st, fp8_adaptive(m, T));
        launches += 1;
    } else {
        // routed experts MXFP4 or FP8-e8m0 on the block-scaled tensor cores.  An FP8 128x128 shared
        // expert (its chunks read x by token, as 16 or 32 consecutive tokens, at any T) runs on a share of the
        // same launches' CTAs; an FP8-e8m0 shared expert is one more set of chunks of the block-scaled
        // body.  [gather] -> up (h quantized per 32 in its epilogue for every block-scaled row) ->
        // [hquant per 128 of the FP8 128x128 shared rows] -> down -> combine
        const bool direct = T <= 16;
        const int ns = m->has_shared ? (T + shared_chunk_tokens(m, T) - 1) / shared_chunk_tokens(m, T) : 0;
        const int n8 = m->shared_bs ? 0 : ns;  // chunks of the FP8 128x128 body (the shared expert's, first)
        if (!direct) {
            launch_gather(m, T, st);
            launches++;
        }
        TcParams su = tc_params(m, T, true, true), pu = tc_params(m, T, true, direct);
        su.chunk_begin = 0, su.chunk_end = n8;
        pu.chunk_begin = n8, pu.chunk_end = -1;
        launch_tc4(m, true, su, pu, tc4_wide(m, T), st);
        if (m->timing) CK(cudaEventRecord(tc.ev[2], st));
        launches += 1;
        if (n8) {
            launch_hquant(m, T * m->K, npos, st);
            launches++;
        }
        TcParams sd = tc_params(m, T, false), pd = tc_params(m, T, false);
        sd.chunk_begin = 0, sd.chunk_end = n8;
        pd.chunk_begin = n8, pd.chunk_end = -1;
        launch_tc4(m, false, sd, pd, tc4_wide(m, T), st);
        launches += 1;
    }
    CombineParams cp{m->eo, m->sh, io ? nullptr : static_cast<uint16_t *>(y), T, m->K, m->H, m->has_shared, ep_view(m), m->status};
    if (io) cp.res = io->res, cp.post = io->post, cp.comb = io->comb, cp.hout = io->hout, cp.hc = io->hc;
    void *cargs[] = {&cp};
    const int cthreads = T * (m->H / 8);
    launch_pdl(combine_kernel_ptr(), dim3((cthreads + 255) / 256), dim3(256), cargs, 0, st);
    launches += 1;
    if (m->timing) {
        CK(cudaEventRecord(tc.ev[3], st));
        m->pending.push_back(tc);
    }
    m->launches = launches;
    m->last_T = T;
    m->calls++;
    m->tokens += T;
}

TimedCall take_events(stbl_moe *m) {
    if (!m->event_pool.empty()) {
        TimedCall t = m->event_pool.back();
        m->event_pool.pop_back();
        return t;
    }
    TimedCall t{};
    for (auto &e : t.ev) CK(cudaEventCreate(&e));
    return t;
}

// wait for the pending timed calls (all but the newest `keep`) and add their durations
void collect_timing(stbl_moe *m, size_t keep) {
    while (m->pending.size() > keep) {
        TimedCall t = m->pending.front();
        m->pending.erase(m->pending.begin());
        CK(cudaEventSynchronize(t.ev[3]));
        for (int i = 0; i < 3; i++) {
            float ms = 0.f;
            CK(cudaEventElapsedTime(&ms, t.ev[i], t.ev[i + 1]));
            m->tsum[i] += ms * 1e-3;
        }
        m->tcalls++;
        m->event_pool.push_back(t);
    }
}

}  // namespace

extern "C" {

int stbl_moe_create(const stbl_moe_desc *desc, stbl_moe **out, char *err, int errlen) {
    return stbl_moe_create_ep(desc, 0, 1, out, err, errlen);
}

int stbl_moe_create_ep(const stbl_moe_desc *desc, int rank, int n_ranks, stbl_moe **out, char *err, int errlen) {
    stbl_moe *m = new stbl_moe();
    try {
        create(m, desc, rank, n_ranks);
        *out = m;
        return 0;
    } catch (const std::exception &e) {
        if (err && errlen > 0) snprintf(err, errlen, "%s", e.what());
        if (m->ws) cudaFree(m->ws);
        if (m->ep_region) cudaFree(m->ep_region);
        delete m;
        *out = nullptr;
        return -1;
    }
}

int stbl_moe_ep_handle(stbl_moe *m, void *handle) {
    try {
        if (m->ep_n < 2) throw std::runtime_error("not an expert-parallel layer");
        static_assert(sizeof(cudaIpcMemHandle_t) == STBL_EP_HANDLE_BYTES, "IPC handle size");
        cudaIpcMemHandle_t h;
        CK(cudaIpcGetMemHandle(&h, m->ep_region));
        memcpy(handle, &h, sizeof h);
        return 0;
    } catch (const std::exception &e) {
        m->err = e.what();
        return -1;
    }
}

int stbl_moe_ep_connect(stbl_moe *m, const void *handles) {
    try {
        if (m->ep_n < 2) throw std::runtime_error("not an expert-parallel layer");
        if (m->ep_connected) throw std::runtime_error("already connected");
        for (int d = 0; d < m->ep_n; d++) {
            if (d == m->ep_rank) continue;
            cudaIpcMemHandle_t h;
            memcpy(&h, static_cast<const char *>(handles) + (size_t)d * STBL_EP_HANDLE_BYTES, sizeof h);
            void *ptr = nullptr;
            CK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
            m->ep_peer[d] = static_cast<char *>(ptr);
        }
        m->ep_connected = true;
        return 0;
    } catch (const std::exception &e) {
        for (int d = 0; d < m->ep_n; d++)
            if (d != m->ep_rank && m->ep_peer[d]) cudaIpcCloseMemHandle(m->ep_peer[d]), m->ep_peer[d] = nullptr;
        m->err = e.what();
        return -1;
    }
}

int stbl_moe_forward(stbl_moe *m, const void *x_bf16, int T, void *y_bf16, cudaStream_t stream) {
    try {
        forward(m, x_bf16, T, y_bf16, stream);
        return 0;
    } catch (const std::exception &e) {
        m->err = e.what();
        return -1;
    }
}

int stbl_moe_forward_block(stbl_moe *m, const float *x_pre, const float *norm_w, float eps, const float *res,
                           const float *post, const float *comb, int hc, int T, float *h_out, cudaStream_t stream) {
    try {
        if (!x_pre || !norm_w || !res || !post || !comb || !h_out) throw std::runtime_error("null argument");
        if (hc < 1 || hc > 16) throw std::runtime_error("hc must be in 1..16");
        if (m->ep_n > 1) throw std::runtime_error("the fused block is single-GPU");
        for (const void *ptr : {(const void *)x_pre, (const void *)norm_w, (const void *)res, (const void *)h_out})
            if ((uintptr_t)ptr & 15) throw std::runtime_error("x_pre, norm_w, res and h_out must be 16-byte aligned");
        const BlockIO io{x_pre, norm_w, eps, res, post, comb, hc, h_out};
        forward(m, nullptr, T, nullptr, stream, nullptr, &io);
        return 0;
    } catch (const std::exception &e) {
        m->err = e.what();
        return -1;
    }
}

int stbl_moe_forward_routed(stbl_moe *m, const void *x_bf16, int T, const int *idx, void *y_bf16, cudaStream_t stream) {
    try {
        if (!idx) throw std::runtime_error("null idx");
        if (m->ep_n > 1) throw std::runtime_error("forced routes are single-GPU");
        forward(m, x_bf16, T, y_bf16, stream, idx);
        return 0;
    } catch (const std::exception &e) {
        m->err = e.what();
        return -1;
    }
}

int stbl_moe_attach_prefetch(stbl_moe *m, const stbl_moe *next, int n_predict, int consider, cudaStream_t copy_stream) {
    try {
        if (m->pf_ws) {
            CK(cudaDeviceSynchronize());
            CK(cudaFree(m->pf_ws));
            m->pf_ws = nullptr;
        }
        m->pf_next = nullptr;
        if (!next) return 0;
        if (!m->cache || next->cache != m->cache) throw std::runtime_error("both layers must be attached to the same expert cache");
        if (next->E != m->E || next->H != m->H) throw std::runtime_error("the next layer's shape differs");
        if (n_predict < 1 || n_predict > 16 || n_predict > next->E) throw std::runtime_error("n_predict must be in 1..16 and <= n_experts");
        if (consider < 1) throw std::runtime_error("consider must be >= 1");
        if (next->d.n_groups > 1 && next->d.topk_groups < next->d.n_groups &&
            next->d.topk_groups * (next->E / next->d.n_groups) < n_predict)
            throw std::runtime_error("the next layer's kept groups hold fewer than n_predict experts");
        const int T = m->Tmax, E = m->E, H = m->H, K = n_predict;
        const size_t bytes = ((size_t)T * E * 4 + 255) + 2 * ((size_t)T * K * 4 + 255) + 2 * ((size_t)(E + 1) * 4 + 255) +
                             ((size_t)T * K * 4 + 255) + ((size_t)T * (K + 1) * sizeof(Chunk) + 255) + 2 * 256 +
                             ((size_t)T * H + 255) + ((size_t)T * (H / 32) * 4 + 255) + ((size_t)E * 4 + 255) +
                             ((size_t)E * ((T + 31) / 32) * 4 + 255) + 4096;
        CK(cudaMalloc(&m->pf_ws, bytes));
        char *p = static_cast<char *>(m->pf_ws);
        RouterParams &r = m->pf_r;
        r = RouterParams{};
        r.scores = carve<float>(p, (size_t)T * E);
        r.idx = carve<int>(p, (size_t)T * K);
        r.wts = carve<float>(p, (size_t)T * K);
        r.counts = carve<int>(p, E + 1);
        r.offsets = carve<int>(p, E + 1);
        r.perm = carve<int>(p, (size_t)T * K);
        r.chunks = carve<Chunk>(p, (size_t)T * (K + 1));
        r.n_chunks = carve<int>(p, 4);
        r.status = m->status;
        r.xq_a = r.xq_b = carve<uint8_t>(p, (size_t)T * H);
        r.xs_a = r.xs_b = carve<float>(p, (size_t)T * (H / 32));
        r.blk_a = r.blk_b = 128, r.pow2_a = r.pow2_b = 0;
        r.sel_cnt = carve<int>(p, E);
        r.sel_bm = carve<uint32_t>(p, (size_t)E * ((T + 31) / 32));
        r.sel_ticket = carve<unsigned int>(p, 4);
        r.has_shared = 0, r.nt_routed = 16, r.nt_shared = 16;
        m->pf_next = next, m->pf_predict = n_predict, m->pf_consider = consider, m->pf_stream = copy_stream;
        return 0;
    } catch (const std::exception &e) {
        m->err = e.what();
        return -1;
    }
}

int stbl_moe_attach_cache(stbl_moe *m, stbl_cache *c, int layer) {
    try {
        if (!c) throw std::runtime_error("null cache");
        if (m->ep_n > 1) throw std::runtime_error("the expert cache is single-GPU");
        if (m->act_q8) throw std::runtime_error("act_q8 layers read the natural MXFP4 scales; the expert cache holds the block layout");
        if (layer < 0 || layer >= c->L) throw std::runtime_error("layer out of the cache's range");
        int dev = 0;
        CK(cudaGetDevice(&dev));
        if (dev != c->dev) throw std::runtime_error("the cache lives on another device");
        if (c->E != m->E || c->H != m->H || c->I != m->I || c->fmt != m->d.routed_fmt)
            throw std::runtime_error("cache and layer shapes or formats differ");
        if (m->n_slots != c->S) throw std::runtime_error("layer not made from stbl_cache_layer_desc (n_slots)");
        for (int q = 0; q < 3; q++)
            if (m->d.routed_w[q] != c->pool + c->piece_off[q] || m->d.routed_s[q] != c->pool + c->piece_off[q + 3] ||
                m->w_stride[q] != c->slot_bytes || m->s_stride[q] != c->slot_bytes)
                throw std::runtime_error("layer not made from stbl_cache_layer_desc (routed pointers)");
        if ((long long)c->S < std::min((long long)m->Tmax * m->K, (long long)m->E))
            throw std::runtime_error("the cache needs at least min(max_tokens * topk, n_experts) slots");
        m->cache = c;
        m->cache_layer = layer;
        return 0;
    } catch (const std::exception &e) {
        m->err = e.what();
        return -1;
    }
}

int stbl_moe_forward_host(stbl_moe *m, const void *x_bf16_host, int T, void *y_bf16_host, cudaStream_t stream) {
    try {
        if (T < 1 || T > m->Tmax) throw std::runtime_error("T must be in 1..max_tokens");
        const size_t bytes = (size_t)T * m->H * 2;
        CK(cudaMemcpyAsync(m->xin, x_bf16_host, bytes, cudaMemcpyHostToDevice, stream));
        forward(m, m->xin, T, m->yout, stream);
        CK(cudaMemcpyAsync(y_bf16_host, m->yout, bytes, cudaMemcpyDeviceToHost, stream));
        CK(cudaStreamSynchronize(stream));
        return 0;
    } catch (const std::exception &e) {
        m->err = e.what();
        return -1;
    }
}

int stbl_moe_last_route(stbl_moe *m, int *idx, float *weights, int *counts, int *offsets, int *perm) {
    try {
        const int T = m->last_T;
        CK(cudaDeviceSynchronize());
        if (idx) CK(cudaMemcpy(idx, m->idx, sizeof(int) * T * m->K, cudaMemcpyDeviceToHost));
        if (weights) CK(cudaMemcpy(weights, m->wts, sizeof(float) * T * m->K, cudaMemcpyDeviceToHost));
        if (counts) CK(cudaMemcpy(counts, m->counts, sizeof(int) * m->E, cudaMemcpyDeviceToHost));
        if (offsets) CK(cudaMemcpy(offsets, m->offsets, sizeof(int) * (m->E + 1), cudaMemcpyDeviceToHost));
        if (perm) CK(cudaMemcpy(perm, m->perm, sizeof(int) * T * m->K, cudaMemcpyDeviceToHost));
        return T;
    } catch (const std::exception &e) {
        m->err = e.what();
        return -1;
    }
}

int stbl_moe_last_scores(stbl_moe *m, float *scores) {
    try {
        CK(cudaDeviceSynchronize());
        CK(cudaMemcpy(scores, m->scores, sizeof(float) * m->last_T * m->E, cudaMemcpyDeviceToHost));
        return m->last_T;
    } catch (const std::exception &e) {
        m->err = e.what();
        return -1;
    }
}

int stbl_moe_last_acts(stbl_moe *m, int which, void *h_bf16, void *codes, float *scales) {
    try {
        if (m->ep_n > 1) throw std::runtime_error("activation readback is for single-GPU layers");
        if (which < STBL_ACTS_X_ROUTED || which > STBL_ACTS_H_SHARED) throw std::runtime_error("bad `which`");
        const int T = m->last_T;
        if (T < 1) throw std::runtime_error("no call yet");
        const bool x = which == STBL_ACTS_X_ROUTED || which == STBL_ACTS_X_SHARED;
        const bool shared = which == STBL_ACTS_X_SHARED || which == STBL_ACTS_H_SHARED;
        if (shared && !m->has_shared) throw std::runtime_error("the layer has no shared expert");
        const int fr = m->d.routed_fmt, fmt = shared ? m->d.shared_fmt : fr;
        const int blk = act_blk_of(fmt);
        const int width = x ? m->H : m->I;
        const int rows = x ? T : (shared ? T : T * m->K);
        const int pos0 = x ? 0 : (shared ? T * m->K : 0);  // first position of the h rows
        CK(cudaDeviceSynchronize());
        // x: the routed format's buffer, or the shared expert's own when its rule differs (forward())
        const bool own_b = x && shared && !(act_blk_of(fmt) == act_blk_of(fr) && act_pow2_of(fmt) == act_pow2_of(fr));
        const uint8_t *src_codes = x ? (own_b ? m->xq_b : m->xq_a) : m->hq + (size_t)pos0 * width;
        if (codes) CK(cudaMemcpy(codes, src_codes, (size_t)rows * width, cudaMemcpyDeviceToHost));
        if (h_bf16 && !x) CK(cudaMemcpy(h_bf16, m->h + (size_t)pos0 * width, (size_t)rows * width * 2, cudaMemcpyDeviceToHost));
        if (scales) {
            const int ns = width / blk;
            std::vector<float> out((size_t)rows * ns);
            if (m->act_q8 && !shared) {
                // Q8: fp32 scales per 32, x rows H / 32 floats, h rows I / 32
                const float *src = x ? m->xs_a : m->hd8 + (size_t)pos0 * (width / 32);
                CK(cudaMemcpy(out.data(), src, out.size() * 4, cudaMemcpyDeviceToHost));
            } else if (blk == 128) {
                // fp32 scales: x rows hold H / 32 floats (the first H / 128 used), h rows I / 128
                const float *src = x ? (own_b ? m->xs_b : m->xs_a) : m->hs + (size_t)pos0 * (width / 128);
                const int stride = x ? m->H / 32 : width / 128;
                std::vector<float> buf((size_t)rows * stride);
                CK(cudaMemcpy(buf.data(), src, buf.size() * 4, cudaMemcpyDeviceToHost));
                for (int r = 0; r < rows; r++)
                    for (int j = 0; j < ns; j++) out[(size_t)r * ns + j] = buf[(size_t)r * stride + j];
            } else {
                // e8m0 bytes in the tensor cores' activation-scale layout [width/128][rows_of_layout][16 B]
                const uint8_t *src = x ? m->xe8_a : m->he8;
                const int lrows = x ? m->Tpad : m->pos_rows;
                std::vector<uint8_t> buf((size_t)(width / 128) * lrows * 16);
                CK(cudaMemcpy(buf.data(), src, buf.size(), cudaMemcpyDeviceToHost));
                for (int r = 0; r < rows; r++)
                    for (int j = 0; j < ns; j++) {
                        const uint8_t b = buf[((size_t)(j / 4) * lrows + pos0 + r) * 16 + (j % 4)];
                        uint32_t bits = (uint32_t)b << 23;
                        float f;
                        memcpy(&f, &bits, 4);
                        out[(size_t)r * ns + j] = f;
                    }
            }
            memcpy(scales, out.data(), out.size() * 4);
        }
        return rows;
    } catch (const std::exception &e) {
        m->err = e.what();
        return -1;
    }
}

int stbl_moe_set_expert(stbl_moe *m, int e, const void *const w[3], const void *const s[3], cudaStream_t stream) {
    try {
        if (e < 0 || e >= m->E_loc) throw std::runtime_error("expert id out of range (local experts of this rank)");
        if (m->cache) throw std::runtime_error("the layer's experts are placed by its expert cache");
        // the new memory must be one slot of the layer's strided expert arrays, the same slot for all
        // three matrices and their scales
        const long long off = (long long)(static_cast<const char *>(w[0]) - static_cast<const char *>(m->d.routed_w[0]));
        if (!w[0] || off < 0 || off % m->w_stride[0]) throw std::runtime_error("expert memory must be a slot of the layer's expert arrays");
        const long long sl = off / m->w_stride[0];
        if (sl >= m->n_slots) throw std::runtime_error("expert slot out of range");
        for (int i = 0; i < 3; i++)
            if (w[i] != static_cast<const char *>(m->d.routed_w[i]) + sl * m->w_stride[i] ||
                s[i] != static_cast<const char *>(m->d.routed_s[i]) + sl * m->s_stride[i])
                throw std::runtime_error("the three matrices and scales of an expert must share one slot");
        m->host_slot[e] = (int)sl;
        if (sl != e) m->slots_moved = true;
        if (m->sf_own) {
            // the slot's MXFP4 scales as they are now, into the layer's scale-block copy
            const int rows[3] = {m->I, m->I, m->H}, ks[3] = {m->H, m->H, m->I};
            for (int mt = 0; mt < 3; mt++)
                CK(launch_sf_repack(static_cast<const uint8_t *>(m->d.routed_s[mt]), m->s_stride[mt], m->sf_own + m->sf_own_off[mt],
                                    m->sf_own_stride, rows[mt], ks[mt], (int)sl, 1, scale_rows_of(m->d.routed_fmt), stream));
        }
        CK(cudaMemcpyAsync(m->slot + e, &m->host_slot[e], sizeof(int), cudaMemcpyHostToDevice, stream));
        return 0;
    } catch (const std::exception &e2) {
        m->err = e2.what();
        return -1;
    }
}

int stbl_moe_status(stbl_moe *m, uint32_t *status) {
    try {
        CK(cudaDeviceSynchronize());
        uint32_t s = 0;
        CK(cudaMemcpy(&s, m->status, 4, cudaMemcpyDeviceToHost));
        CK(cudaMemset(m->status, 0, 4));
        *status = s;
        return 0;
    } catch (const std::exception &e) {
        m->err = e.what();
        return -1;
    }
}

int stbl_moe_set_timing(stbl_moe *m, int enable) {
    try {
        if (!enable) collect_timing(m, 0);
        m->timing = enable != 0;
        return 0;
    } catch (const std::exception &e) {
        m->err = e.what();
        return -1;
    }
}

int stbl_moe_timing(stbl_moe *m, double *sec, int n) {
    try {
        collect_timing(m, 0);
        for (int i = 0; i < n && i < 3; i++) sec[i] = m->tsum[i];
        if (n > 3) sec[3] = (double)m->tcalls;
        return 4;
    } catch (const std::exception &e) {
        m->err = e.what();
        return -1;
    }
}

void stbl_moe_stats(const stbl_moe *m, uint64_t *calls, uint64_t *tokens, int *launches_per_call) {
    if (calls) *calls = m->calls;
    if (tokens) *tokens = m->tokens;
    if (launches_per_call) *launches_per_call = m->launches;
}

const char *stbl_moe_error(const stbl_moe *m) { return m ? m->err.c_str() : "null layer"; }

void stbl_moe_destroy(stbl_moe *m) {
    if (!m) return;
    for (auto &t : m->pending) cudaEventSynchronize(t.ev[3]), m->event_pool.push_back(t);
    for (auto &t : m->event_pool)
        for (auto e : t.ev) cudaEventDestroy(e);
    if (m->ws) cudaFree(m->ws);
    if (m->pf_ws) cudaFree(m->pf_ws);
    if (m->sf_own) cudaFree(m->sf_own);
    if (m->sf_shared) cudaFree(m->sf_shared);
    for (int d = 0; d < m->ep_n; d++)
        if (d != m->ep_rank && m->ep_peer[d]) cudaIpcCloseMemHandle(m->ep_peer[d]);
    if (m->ep_region) cudaFree(m->ep_region);
    delete m;
}

}  // extern "C"
