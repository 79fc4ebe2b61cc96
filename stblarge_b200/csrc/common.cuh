// Device helpers shared by the sm_100a kernels: number formats, warp reductions, and the
// mbarrier / bulk-copy (TMA, non-tensor) primitives used to stream weight tiles into shared memory.
// Every wait is bounded: it gives up after a time limit, raises a flag in the caller's status word
// and lets the kernel leave cleanly, so a logic error can never hang the GPU.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace stbl {

// status bits written by kernels into the layer's device status word
enum : uint32_t {
    kErrWaitTimeout = 1u,   // an mbarrier wait ran out of time
    kErrBadTable = 2u,      // a dispatch table entry was out of range
    kErrCopyTimeout = 4u,   // copies still in flight when a CTA gave up
    kErrRead = 8u,          // an expert read from the checkpoint file failed (file-backed expert cache)
};

// one second: far above any legal wait (a whole layer takes well under a millisecond)
constexpr uint64_t kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// 2^ceil(log2 t) for positive normal t by exponent and mantissa bits (ref/kernel.py:22-26).
__device__ __forceinline__ float pow2_ceil(float t) {
    const uint32_t b = __float_as_uint(t);
    const int e = (int)((b >> 23) & 0xff) - 127 + ((b & 0x7fffffu) != 0);
    return __uint_as_float((uint32_t)(e + 127) << 23);
}

// E8M0 byte -> 2^(b - 127); code 0 (2^-127) maps to 0, as in the reference (stbl/kernels.cu:32); the
// quantizers never produce it.
__device__ __forceinline__ float e8m0(uint32_t b) { return __uint_as_float(b << 23); }

__device__ __forceinline__ float e4m3_value(uint8_t c) {
    __nv_fp8_e4m3 v;
    v.__x = c;
    return (float)v;
}

// round to nearest even on the e4m3 grid, saturating to +-448
__device__ __forceinline__ uint8_t e4m3_code(float x) {
    return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}

// two e4m3 codes (low byte first) -> f16x2, exact (every e4m3 value is an f16 value)
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t two) {
    uint32_t r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(two));
    return r;
}

// two e2m1 codes in one byte (low nibble first) -> f16x2, exact
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
    uint32_t r;
    asm("{.reg .b8 t; cvt.u8.u32 t, %1; cvt.rn.f16x2.e2m1x2 %0, t;}" : "=r"(r) : "r"(byte));
    return r;
}

// acc += w.lo * x.lo + w.hi * x.hi with f16 operands and an fp32 accumulator; each product of two
// f16 values holding e4m3 / e2m1 numbers is exact in fp32.
__device__ __forceinline__ float dot2_f16_f32(uint32_t w, uint32_t x, float acc) {
    asm("{.reg .f16 wl, wh, xl, xh;\n\t"
        "mov.b32 {wl, wh}, %1;\n\t"
        "mov.b32 {xl, xh}, %2;\n\t"
        "fma.rn.f32.f16 %0, wl, xl, %0;\n\t"
        "fma.rn.f32.f16 %0, wh, xh, %0;}"
        : "+f"(acc)
        : "r"(w), "r"(x));
    return acc;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum V values (V a power of two, at most 32) over the 32 lanes of a warp and scatter them: on
// return lane l holds in v[0] the warp total of value l >> (5 - log2 V).  About one shuffle per value.
template <int V>
__device__ __forceinline__ float warp_reduce_scatter(float (&v)[V], int lane) {
    int off = 16;
#pragma unroll
    for (int half = V / 2; half >= 1; half /= 2, off >>= 1) {
        const bool upper = lane & off;
#pragma unroll
        for (int i = 0; i < half; i++) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    float r = v[0];
    for (; off >= 1; off >>= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
    return r;
}

template <int V>
__device__ __forceinline__ constexpr int log2_const() {
    return V <= 1 ? 0 : 1 + log2_const<V / 2>();
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- mbarrier + bulk copy ------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{.reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0];}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{.reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;}" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete.  Gives up when *abort becomes non-zero
// (another warp of the CTA gave up) or after kWaitLimitNs; returns false then.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (global_ns() - t0 > kWaitLimitNs) return false;
    }
}

// 1-D bulk copy global -> shared (TMA engine), completing on the mbarrier's transaction count.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// named barrier over `threads` threads (id 1..15), with an OR over a predicate
__device__ __forceinline__ bool bar_sync_or(int id, int threads, bool pred) {
    uint32_t r;
    asm volatile(
        "{.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;}"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(threads)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint4 lds128(const void *p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p)));
    return v;
}

// float key that orders like the float (for redux.sync max); -0 and +0 map apart but the router
// never compares them (scores are positive)
__device__ __forceinline__ uint32_t float_key(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

}  // namespace stbl
