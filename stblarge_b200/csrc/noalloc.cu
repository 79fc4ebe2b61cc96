// Allocation-free routing entry point (stbl_route_noalloc, include/stbl_moe.h).
//
// Some callers cannot allocate device memory: engines that own a fixed memory pool and forbid
// allocations outside it, and embedded runtimes that never link an allocator.  For them this entry point runs the router
// kernels (router.cu, the same launches as the layer's) with all of their working memory in one
// fixed-size array that the library declares at file scope; the caller passes only its inputs and
// output buffers.
//
// Limits: T <= kNaMaxTokens tokens, E <= kNaMaxExperts experts, H <= kNaMaxHidden (and at most
// 2048 when H is not a multiple of 512: the router's hidden slice), topk <= 16.
// The array (kNaBytes = 86,784 bytes) is part of the library image: every GPU that loads the library
// holds it until the process exits.  All calls share it, so calls that overlap on the GPU (two
// streams, two threads) race; serialise them.  The first call on each device looks up the array's
// device address (cudaGetSymbolAddress); make that first call before any stream capture.
// The router kernels raise status bits in the array (a bounded wait that ran out, a bad table
// entry); each call clears the word on its stream before the kernels run (a memset: no allocation),
// and stbl_route_noalloc_status reads and clears it.  A non-zero status means the outputs of the
// calls since the last read are not valid.
#include <mutex>
#include <stdio.h>

#include "../../include/stbl_moe.h"
#include "layer.cuh"

using namespace stbl;

namespace {

constexpr int kNaMaxTokens = 64;
constexpr int kNaMaxExperts = 256;
constexpr int kNaMaxHidden = 8192;
constexpr int kNaMaxTopk = 16;

// byte layout of the scratch array (routing only: x is not quantized for expert kernels here)
constexpr size_t kNaScores = 0;                                                        // f32 [T][E]
constexpr size_t kNaChunks = kNaScores + sizeof(float) * kNaMaxTokens * kNaMaxExperts;  // Chunk [T * (topk + 1)]
constexpr size_t kNaNChunks = kNaChunks + sizeof(Chunk) * kNaMaxTokens * (kNaMaxTopk + 1);  // int [4]
constexpr size_t kNaStatus = kNaNChunks + 256;                                         // u32 status
constexpr size_t kNaSelCnt = kNaStatus + 256;                                          // int [E]
constexpr size_t kNaSelBm = kNaSelCnt + sizeof(int) * kNaMaxExperts;                  // u32 [E][T / 32]
constexpr size_t kNaSelTicket = kNaSelBm + sizeof(uint32_t) * kNaMaxExperts * (kNaMaxTokens / 32);  // u32
constexpr size_t kNaBytes = kNaSelTicket + 256;
static_assert(kNaBytes == 86784, "the array size stated in stbl_moe.h and this file's header");

static __device__ __align__(256) unsigned char g_route_scratch[kNaBytes];

constexpr int kNaMaxDevices = 64;
std::mutex g_na_mu;
unsigned char *g_na_addr[kNaMaxDevices] = {};

int fail(char *err, int errlen, const char *msg) {
    if (err && errlen > 0) snprintf(err, errlen, "%s", msg);
    return -1;
}

}  // namespace

extern "C" int stbl_route_noalloc(const float *router_w, const float *router_bias, const void *x_bf16, int T, int E,
                                  int H, int topk, int n_groups, int topk_groups, int score_fn, float route_scale,
                                  int *idx, float *weights, int *counts, int *offsets, int *perm, cudaStream_t stream,
                                  char *err, int errlen) {
    if (T < 1 || T > kNaMaxTokens) return fail(err, errlen, "stbl_route_noalloc: T must be in 1..64");
    if (E < 1 || E > kNaMaxExperts) return fail(err, errlen, "stbl_route_noalloc: n_experts must be in 1..256");
    if (H < 128 || H > kNaMaxHidden || H % 128) return fail(err, errlen, "stbl_route_noalloc: hidden must be a multiple of 128, at most 8192");
    if (H / router_ksplit(H) > kLgMaxSlice)
        return fail(err, errlen, "stbl_route_noalloc: hidden must be at most 2048 when it is not a multiple of 512");
    if ((uintptr_t)router_w & 15 || (uintptr_t)x_bf16 & 15)
        return fail(err, errlen, "stbl_route_noalloc: router_w and x must be 16-byte aligned");
    if (topk < 1 || topk > kNaMaxTopk || topk > E) return fail(err, errlen, "stbl_route_noalloc: topk must be in 1..16 and <= n_experts");
    if (n_groups < 1 || n_groups > 32 || E % n_groups || topk_groups < 1 || topk_groups > n_groups)
        return fail(err, errlen, "stbl_route_noalloc: bad expert groups");
    const int gsz = E / n_groups;
    if (n_groups > 1 && topk_groups < n_groups && (gsz < 2 || topk_groups * gsz < topk))
        return fail(err, errlen, "stbl_route_noalloc: kept groups hold fewer than topk experts");
    if (score_fn != STBL_SCORE_SIGMOID && score_fn != STBL_SCORE_SQRT_SOFTPLUS) return fail(err, errlen, "stbl_route_noalloc: bad score_fn");
    if (!router_w || !router_bias || !x_bf16 || !idx || !weights || !counts || !offsets || !perm)
        return fail(err, errlen, "stbl_route_noalloc: null pointer");

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNaMaxDevices)
        return fail(err, errlen, "stbl_route_noalloc: no current CUDA device");
    unsigned char *base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_na_mu);
        if (!g_na_addr[dev]) {
            void *ptr = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&ptr, g_route_scratch);
            if (e != cudaSuccess || !ptr) {
                if (err && errlen > 0) snprintf(err, errlen, "stbl_route_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
                return -1;
            }
            const cudaError_t e2 = router_setup();
            if (e2 != cudaSuccess) {
                if (err && errlen > 0) snprintf(err, errlen, "stbl_route_noalloc: %s", cudaGetErrorString(e2));
                return -1;
            }
            g_na_addr[dev] = static_cast<unsigned char *>(ptr);
        }
        base = g_na_addr[dev];
    }

    RouterParams r{};
    r.W = router_w, r.bias = router_bias, r.x = static_cast<const uint16_t *>(x_bf16);
    r.T = T, r.E = E, r.H = H, r.topk = topk, r.n_groups = n_groups, r.topk_groups = topk_groups;
    r.score_fn = score_fn, r.route_scale = route_scale, r.ksplit = router_ksplit(H), r.has_shared = 0;
    r.nt_routed = kNaMaxTopk, r.nt_shared = kNaMaxTopk;
    r.scores = reinterpret_cast<float *>(base + kNaScores);
    r.idx = idx, r.wts = weights, r.counts = counts, r.offsets = offsets, r.perm = perm;
    r.chunks = reinterpret_cast<Chunk *>(base + kNaChunks);
    r.n_chunks = reinterpret_cast<int *>(base + kNaNChunks);
    r.xq_a = r.xq_b = nullptr;  // no expert kernels follow: skip the activation quantization
    r.xs_a = r.xs_b = nullptr;
    r.blk_a = r.blk_b = 128, r.pow2_a = r.pow2_b = 0;
    r.status = reinterpret_cast<uint32_t *>(base + kNaStatus);
    r.sel_cnt = reinterpret_cast<int *>(base + kNaSelCnt);
    r.sel_bm = reinterpret_cast<uint32_t *>(base + kNaSelBm);
    r.sel_ticket = reinterpret_cast<unsigned int *>(base + kNaSelTicket);
    // this call's status starts clear (stream-ordered, so a later read covers this call only)
    cudaError_t e = cudaMemsetAsync(base + kNaStatus, 0, sizeof(uint32_t), stream);
    if (e == cudaSuccess) e = launch_router(r, stream, false);
    if (e != cudaSuccess) {
        if (err && errlen > 0) snprintf(err, errlen, "stbl_route_noalloc: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

extern "C" int stbl_route_noalloc_status(uint32_t *status) {
    if (!status) return -1;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNaMaxDevices) return -1;
    unsigned char *base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_na_mu);
        base = g_na_addr[dev];
    }
    if (!base) {  // no call on this device yet: nothing can have been raised
        *status = 0;
        return 0;
    }
    uint32_t s = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return -1;
    if (cudaMemcpy(&s, base + kNaStatus, sizeof s, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (cudaMemset(base + kNaStatus, 0, sizeof s) != cudaSuccess) return -1;
    *status = s;
    return 0;
}
