// CHW f32 frames -> interleaved RGB24 bytes, the reference's output
// conversion (tools/tp-cli.cpp:43-53, the frame handed to the video encoder):
// per pixel and channel, v clamped to [-1, 1] with the same comparisons
// (v < -1 ? -1 : (v > 1 ? 1 : v)), then (unsigned char) ((v + 1) / 2 * 255)
// in f32 with truncation toward zero; the operations are spelled as
// round-to-nearest intrinsics so no contraction changes a byte.
//
// HBM-bound: 12 bytes read and 3 written per pixel. Each thread converts
// four consecutive pixels: three 16-byte plane loads, three 4-byte stores
// (12 contiguous output bytes), so a warp reads and writes contiguous lines.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <string>

#include "../../include/tpmd.h"
#include "tpmd_internal.h"

namespace tpmd {
namespace {

__device__ __forceinline__ uint32_t to_u8(float v) {
    v = v < -1.0f ? -1.0f : (v > 1.0f ? 1.0f : v);
    const float s = __fmul_rn(__fmul_rn(__fadd_rn(v, 1.0f), 0.5f), 255.0f);
    return (uint32_t) (unsigned char) __float2uint_rz(s);
}

// one thread per 4 pixels of one frame: hw4 = H*W/4 quads per frame
__global__ void __launch_bounds__(256) chw_to_rgb24_kernel(const float4 *__restrict__ chw,
                                                           uint32_t *__restrict__ rgb, int64_t hw4,
                                                           int64_t total) {
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t) gridDim.x * blockDim.x) {
        const int64_t f = i / hw4, q = i - f * hw4;
        const float4 *src = chw + f * 3 * hw4 + q;
        const float4 r = __ldg(src), g = __ldg(src + hw4), b = __ldg(src + 2 * hw4);
        const uint32_t p0 = to_u8(r.x) | to_u8(g.x) << 8 | to_u8(b.x) << 16 | to_u8(r.y) << 24;
        const uint32_t p1 = to_u8(g.y) | to_u8(b.y) << 8 | to_u8(r.z) << 16 | to_u8(g.z) << 24;
        const uint32_t p2 = to_u8(b.z) | to_u8(r.w) << 8 | to_u8(g.w) << 16 | to_u8(b.w) << 24;
        uint32_t *dst = rgb + (f * hw4 + q) * 3;
        dst[0] = p0;
        dst[1] = p1;
        dst[2] = p2;
    }
}

}  // namespace

cudaError_t launch_chw_to_rgb24(const float *chw, int64_t n, int64_t hw, uint8_t *rgb, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (hw % 4 || (uintptr_t) chw % 16 || (uintptr_t) rgb % 4) return cudaErrorInvalidValue;
    const int64_t total = n * (hw / 4);
    const int blocks = (int) std::min<int64_t>((total + 255) / 256, (int64_t) 148 * 8);
    chw_to_rgb24_kernel<<<blocks, 256, 0, st>>>((const float4 *) chw, (uint32_t *) rgb, hw / 4, total);
    return cudaGetLastError();
}

}  // namespace tpmd

extern "C" int tpk_chw_to_rgb24(const float *chw, int64_t n, int H, int W, uint8_t *rgb, void *stream) {
    if (n < 0 || H <= 0 || W <= 0) return tpmd::tpk_fail("tpk_chw_to_rgb24: bad shape");
    if (n == 0) return 0;
    if (!chw || !rgb) return tpmd::tpk_fail("tpk_chw_to_rgb24: null pointer");
    if (((int64_t) H * W) % 4 || (uintptr_t) chw % 16 || (uintptr_t) rgb % 4)
        return tpmd::tpk_fail("tpk_chw_to_rgb24: H*W must be a multiple of 4, chw 16-byte and rgb 4-byte aligned");
    const cudaError_t e = tpmd::launch_chw_to_rgb24(chw, n, (int64_t) H * W, rgb, (cudaStream_t) stream);
    if (e != cudaSuccess) return tpmd::tpk_fail(std::string("tpk_chw_to_rgb24: ") + cudaGetErrorString(e));
    return 0;
}
