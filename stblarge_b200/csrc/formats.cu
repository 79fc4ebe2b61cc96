// Weight-format conversion for loading the reference engine's weights into a layer.
//
// GGUF MXFP4 (stbl/kernels.cu:134-141, tools/convert_official.py:187-201): per 32 values 17 bytes, the
// e8m0 scale then 16 bytes with value i (i < 16) in the low nibble of byte i and value 16 + i in its
// high nibble.  The layer's layout (ref/kernel.py:94-102) packs values 2i, 2i + 1 into byte i, low
// nibble first, and keeps the scales apart.  One thread per 32-value block.
#include "../../include/stbl_moe.h"

#include <stdint.h>

namespace {

__global__ void __launch_bounds__(256) mxfp4_from_gguf_kernel(const uint8_t *blocks, long long n_blocks, uint8_t *codes,
                                                              uint8_t *scales) {
    for (long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x; b < n_blocks; b += (long long)gridDim.x * blockDim.x) {
        const uint8_t *src = blocks + b * 17;
        uint8_t v[32];
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const uint8_t x = src[1 + i];
            v[i] = x & 15, v[16 + i] = x >> 4;
        }
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            w[q] = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int byte = 4 * q + i;
                w[q] |= (uint32_t)(v[2 * byte] | (v[2 * byte + 1] << 4)) << (8 * i);
            }
        }
        *reinterpret_cast<uint4 *>(codes + b * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        scales[b] = src[0];
    }
}

}  // namespace

extern "C" int stbl_mxfp4_from_gguf(const void *blocks, int rows, int k, void *codes, void *scales, cudaStream_t stream) {
    if (!blocks || !codes || !scales || rows < 1 || k < 32 || k % 32) return -1;
    if ((uintptr_t)codes & 15) return -1;  // 16-byte stores of each block's codes
    const long long n = (long long)rows * (k / 32);
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    mxfp4_from_gguf_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint8_t *>(blocks), n, static_cast<uint8_t *>(codes),
                                                   static_cast<uint8_t *>(scales));
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
