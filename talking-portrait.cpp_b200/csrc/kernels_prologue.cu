// Per-batch prologue of the decoder: every conv's per-frame style and
// demodulation denominator, computed once for the whole batch, and the styled
// constant input of conv1.
//
//  style:  s[b][row] = Wmod_all[row] . latent[b] + bmod_all[row] over the 22
//          modulation linears stacked row-wise (src/motion_dec.cpp:267-272);
//  den:    inv_den[b][o] = 1/sqrt(S_aug[o] . [s^2; 1]) per demodulated conv
//          (src/motion_dec.cpp:275-280; S_aug is pre-halved so this also
//          folds the FusedLeakyReLU sqrt(2));
//  conv1:  x0[b][p][c] = input[p][c] * s_conv1[b][c] (src/motion_dec.cpp:375-384).
//
// Both reductions are one warp per output row: the row (512 or IC+1 floats)
// sits in registers, read once, and is reused for every frame of the batch,
// so the weight stream is read once per batch, coalesced.
#include "tpmd_internal.h"

namespace tpmd {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void __launch_bounds__(256)
style_kernel(const float *__restrict__ wmod, const float *__restrict__ bmod, int rows,
             const float *__restrict__ lat, int B, float *__restrict__ s_all) {
    const int lane = threadIdx.x & 31;
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;
    float w[STYLE_DIM / 32];
#pragma unroll
    for (int i = 0; i < STYLE_DIM / 32; i++) w[i] = __ldg(wmod + (int64_t) row * STYLE_DIM + lane + 32 * i);
    const float bias = __ldg(bmod + row);
    // four frames per pass: independent loads and reductions overlap
    for (int b0 = 0; b0 < B; b0 += 4) {
        float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int f = 0; f < 4; f++) {
            if (b0 + f >= B) continue;
            const float *l = lat + (int64_t) (b0 + f) * STYLE_DIM;
#pragma unroll
            for (int i = 0; i < STYLE_DIM / 32; i++) a[f] = fmaf(w[i], __ldg(l + lane + 32 * i), a[f]);
        }
#pragma unroll
        for (int f = 0; f < 4; f++) a[f] = warp_sum(a[f]);
        if (lane < 4 && b0 + lane < B) {
            const float v = lane == 0 ? a[0] : lane == 1 ? a[1] : lane == 2 ? a[2] : a[3];
            s_all[(int64_t) (b0 + lane) * rows + row] = v + bias;
        }
    }
}

__global__ void __launch_bounds__(256)
den_kernel(const float *__restrict__ saug, den_table t, const float *__restrict__ s_all,
           int s_stride, int B, float *__restrict__ inv_den, int d_stride) {
    const int lane = threadIdx.x & 31;
    const int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (g >= t.row0[t.n]) return;
    int c = 0;
    while (g >= t.row0[c + 1]) c++;
    const int o = g - t.row0[c];
    const int IC = t.ic[c];
    const float *r = saug + t.saug_off[c] + (int64_t) o * (IC + 1);
    constexpr int MAXPER = 512 / 32;
    float w[MAXPER];
    const int per = IC / 32;  // IC is a multiple of 32 (32..512)
#pragma unroll
    for (int i = 0; i < MAXPER; i++) w[i] = i < per ? __ldg(r + lane + 32 * i) : 0.0f;
    const float eps = __ldg(r + IC);
    for (int b0 = 0; b0 < B; b0 += 4) {  // four frames per pass
        float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int f = 0; f < 4; f++) {
            if (b0 + f >= B) continue;
            const float *s = s_all + (int64_t) (b0 + f) * s_stride + t.s_off[c];
#pragma unroll
            for (int i = 0; i < MAXPER; i++) {
                if (i < per) {
                    const float v = __ldg(s + lane + 32 * i);
                    a[f] = fmaf(w[i], v * v, a[f]);
                }
            }
        }
#pragma unroll
        for (int f = 0; f < 4; f++) a[f] = warp_sum(a[f]) + eps;
        if (lane < 4 && b0 + lane < B) {
            const float v = lane == 0 ? a[0] : lane == 1 ? a[1] : lane == 2 ? a[2] : a[3];
            inv_den[(int64_t) (b0 + lane) * d_stride + t.d_off[c] + o] = 1.0f / sqrtf(v);
        }
    }
}

template <typename T>
__device__ __forceinline__ T to_t(float v);
template <>
__device__ __forceinline__ float to_t<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half to_t<__half>(float v) { return __float2half_rn(v); }

template <typename T>
__global__ void conv1_input_kernel(const float *__restrict__ input, const float *__restrict__ s,
                                   int s_stride, int B, T *__restrict__ x0) {
    const int64_t n = (int64_t) B * 16 * 512;
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t) gridDim.x * blockDim.x) {
        const int c = (int) (i % 512);
        const int p = (int) ((i / 512) % 16);
        const int64_t b = i / (16 * 512);
        x0[i] = to_t<T>(__ldg(input + p * 512 + c) * __ldg(s + b * s_stride + c));
    }
}

}  // namespace

cudaError_t launch_style(const float *wmod, const float *bmod, int rows, const float *lat, int B,
                         float *s_all, cudaStream_t st) {
    const int blocks = (rows * 32 + 255) / 256;
    style_kernel<<<blocks, 256, 0, st>>>(wmod, bmod, rows, lat, B, s_all);
    return cudaGetLastError();
}

cudaError_t launch_den(const float *saug, const den_table &t, const float *s_all, int s_stride,
                       int B, float *inv_den, int d_stride, cudaStream_t st) {
    const int rows = t.row0[t.n];
    const int blocks = (rows * 32 + 255) / 256;
    den_kernel<<<blocks, 256, 0, st>>>(saug, t, s_all, s_stride, B, inv_den, d_stride);
    return cudaGetLastError();
}

cudaError_t launch_conv1_input(bool f16, const float *input, const float *s, int s_stride, int B,
                               void *x0, cudaStream_t st) {
    const int blocks = (B * 16 * 512 + 255) / 256;
    if (f16)
        conv1_input_kernel<__half><<<blocks, 256, 0, st>>>(input, s, s_stride, B, (__half *) x0);
    else
        conv1_input_kernel<float><<<blocks, 256, 0, st>>>(input, s, s_stride, B, (float *) x0);
    return cudaGetLastError();
}

}  // namespace tpmd
