// Kernels of the motion encoder (motion_enc::run, src/motion_enc.cpp:46-184),
// run once per portrait in float32 (the reference keeps the encoder f32,
// src/tp.cpp:22-25). Activations are channel-last [H][W][C], batch 1.
//
//  stem:   x[p][o] = lrelu(sum_c W[o][c] img[c][p] + b[o])       (1x1, CHW in)
//  conv:   y[p][o] = act(sum_k W[o][k] x[..] (+ b[o])) (+ res[p][o]); k =
//          (kh*KW + kw)*IC + ic, stride s, zero padding p on every side —
//          EqualConv2d with its scale folded (src/ops_common.h:12-26)
//  blur:   upfirdn2d(up 1, pad (p0, p1)) with a 4x4 FIR, depthwise
//          correlation (src/ops_common.h:39-43)
//  head:   five plain EqualLinears (a warp per output) and motion = Q lambda
//
// The conv is im2col (rows of K*K*IC floats, zeros outside the map) and the
// library's tcgen05 GEMM with f32 operands by the three-pass TF32 split
// (kernels_gemm_tc.cu), bias, leaky ReLU and the residual in its epilogue.
#include "tpmd_internal.h"

#include <algorithm>

namespace tpmd {
namespace {

__global__ void __launch_bounds__(256) enc_stem_kernel(const float *__restrict__ img, int P,
                                                       const float *__restrict__ w,
                                                       const float *__restrict__ b,
                                                       float *__restrict__ y) {
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= P) return;
    const float c0 = __ldg(img + p), c1 = __ldg(img + P + p), c2 = __ldg(img + 2 * P + p);
    float4 *out = reinterpret_cast<float4 *>(y + (int64_t) p * 32);
#pragma unroll
    for (int o4 = 0; o4 < 8; o4++) {
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int o = 4 * o4 + i;
            float a = __ldg(w + 3 * o) * c0;
            a = fmaf(__ldg(w + 3 * o + 1), c1, a);
            a = fmaf(__ldg(w + 3 * o + 2), c2, a);
            a += __ldg(b + o);
            v[i] = fmaxf(a, 0.2f * a);
        }
        out[o4] = make_float4(v[0], v[1], v[2], v[3]);
    }
}

// col[m][k] = x[oy*s - p + kh][ox*s - p + kw][ic] (zero outside), m = oy*OW +
// ox, k = (kh*K + kw)*IC + ic; a block per output pixel (grid-stride), four
// channels per thread (IC % 4 == 0)
__global__ void __launch_bounds__(128) enc_im2col_kernel(const float *__restrict__ x, int IH, int IW, int IC, int K,
                                                         int stride, int pad, int OH, int OW,
                                                         float *__restrict__ col) {
    const int IC4 = IC >> 2, row4 = K * K * IC4;
    const int64_t M = (int64_t) OH * OW;
    for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
        const int oy = (int) (m / OW), ox = (int) (m - (int64_t) oy * OW);
        float4 *dst = reinterpret_cast<float4 *>(col) + m * row4;
        for (int r = threadIdx.x; r < row4; r += blockDim.x) {
            const int t = r / IC4, c4 = r - t * IC4;
            const int iy = oy * stride - pad + t / K, ix = ox * stride - pad + t % K;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (iy >= 0 && iy < IH && ix >= 0 && ix < IW)
                v = __ldg(reinterpret_cast<const float4 *>(x + ((int64_t) iy * IW + ix) * IC) + c4);
            dst[r] = v;
        }
    }
}

__global__ void __launch_bounds__(256) enc_blur_kernel(const float *__restrict__ x, int IH, int IW, int C,
                                                       const float *__restrict__ k4, int p0, int OH, int OW,
                                                       float *__restrict__ y) {
    const int C4 = C / 4;
    const int64_t n = (int64_t) OH * OW * C4;
    float k[16];
#pragma unroll
    for (int i = 0; i < 16; i++) k[i] = __ldg(k4 + i);
    for (int64_t e = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t) gridDim.x * blockDim.x) {
        const int c4 = (int) (e % C4);
        const int64_t q = e / C4;
        const int X = (int) (q % OW), Y = (int) (q / OW);
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int a = 0; a < 4; a++) {
            const int sy = Y + a - p0;
            if (sy < 0 || sy >= IH) continue;
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int sx = X + b - p0;
                if (sx < 0 || sx >= IW) continue;
                const float4 v = __ldg(reinterpret_cast<const float4 *>(x + ((int64_t) sy * IW + sx) * C) + c4);
                const float kv = k[a * 4 + b];
                acc.x = fmaf(kv, v.x, acc.x);
                acc.y = fmaf(kv, v.y, acc.y);
                acc.z = fmaf(kv, v.z, acc.z);
                acc.w = fmaf(kv, v.w, acc.w);
            }
        }
        reinterpret_cast<float4 *>(y + q * C)[c4] = acc;
    }
}

// appearance [512] -> five EqualLinears (512 -> 512 x4 -> 20) -> lambda [20];
// motion = Q lambda with Q [512][20]. One block of 512 threads, a warp per
// output row with coalesced weight reads, layers separated by barriers.
// one EqualLinear of the head: out[o] = W[o] . in + b[o] over 512 inputs,
// one warp per output (16-byte weight loads, four per lane)
__global__ void __launch_bounds__(256) enc_fc_kernel(const float *__restrict__ in, const float *__restrict__ W,
                                                     const float *__restrict__ b, int N, float *__restrict__ out) {
    const int lane = threadIdx.x & 31, o = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (o >= N) return;
    const float4 *w4 = reinterpret_cast<const float4 *>(W + (int64_t) o * 512);
    const float4 *x4 = reinterpret_cast<const float4 *>(in);
    float a = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float4 w = __ldg(w4 + lane + 32 * k), x = __ldg(x4 + lane + 32 * k);
        a = fmaf(w.x, x.x, a);
        a = fmaf(w.y, x.y, a);
        a = fmaf(w.z, x.z, a);
        a = fmaf(w.w, x.w, a);
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) a += __shfl_xor_sync(0xffffffffu, a, s);
    if (lane == 0) out[o] = a + __ldg(b + o);
}

// motion = Q lambda (Q [512][20])
__global__ void __launch_bounds__(512) enc_motion_kernel(const float *__restrict__ lam, const float *__restrict__ Q,
                                                         float *__restrict__ motion) {
    const int t = threadIdx.x;
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < 20; k++) m = fmaf(__ldg(Q + t * 20 + k), __ldg(lam + k), m);
    motion[t] = m;
}

__global__ void convert_feats_kernel(const float *__restrict__ src, int64_t n, __half *__restrict__ dst) {
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x)
        dst[i] = __float2half_rn(src[i]);
}

}  // namespace

cudaError_t launch_convert_feats(const float *src, int64_t n, bool f16, void *dst, cudaStream_t st) {
    if (!f16) return cudaMemcpyAsync(dst, src, (size_t) n * 4, cudaMemcpyDeviceToDevice, st);
    const int blocks = (int) std::min<int64_t>((n + 255) / 256, 148 * 16);
    convert_feats_kernel<<<blocks, 256, 0, st>>>(src, n, (__half *) dst);
    return cudaGetLastError();
}

cudaError_t launch_enc_stem(const float *img, const float *w, const float *b, float *y, cudaStream_t st) {
    const int P = 512 * 512;
    enc_stem_kernel<<<(P + 255) / 256, 256, 0, st>>>(img, P, w, b, y);
    return cudaGetLastError();
}

cudaError_t launch_enc_conv(const enc_conv_params &p, cudaStream_t st) {
    if (p.IC % 4 || p.OC % 4 || p.OH <= 0 || p.OW <= 0 || !p.err) return cudaErrorInvalidValue;
    const int64_t M = (int64_t) p.OH * p.OW, Kall = (int64_t) p.K * p.K * p.IC;
    if (M * Kall > p.col_floats || M >= (1ll << 31) || Kall >= (1ll << 31)) return cudaErrorInvalidValue;
    enc_im2col_kernel<<<(unsigned) std::min<int64_t>(M, 148 * 32), 128, 0, st>>>(p.x, p.IH, p.IW, p.IC, p.K, p.stride,
                                                                               p.pad, p.OH, p.OW, p.col);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    gemm_desc d;
    d.f32 = true;
    d.X = p.col;
    d.ldx = Kall;
    d.W = p.w;
    d.ldw = Kall;
    d.Y = p.y;
    d.ldy = p.OC;
    d.M = (int) M;
    d.N = p.OC;
    d.K = (int) Kall;
    d.bias = p.bias;
    d.act = p.lrelu ? 3 : 0;
    d.res = p.res;
    d.err = p.err;
    return gemm_tc(d, st);
}

cudaError_t launch_enc_blur(const float *x, int IH, int IW, int C, const float *k4, int p0, int p1, float *y,
                            cudaStream_t st) {
    if (C % 4) return cudaErrorInvalidValue;
    const int OH = IH + p0 + p1 - 3, OW = IW + p0 + p1 - 3;
    const int64_t n = (int64_t) OH * OW * (C / 4);
    const int blocks = (int) std::min<int64_t>((n + 255) / 256, 148 * 16);
    enc_blur_kernel<<<blocks, 256, 0, st>>>(x, IH, IW, C, k4, p0, OH, OW, y);
    return cudaGetLastError();
}

cudaError_t launch_enc_head(const float *app, const enc_head_params &h, float *lam, float *motion, float *scratch,
                            cudaStream_t st) {
    // fc 0..3 (512 -> 512) alternate between the two scratch rows, fc 4 (512 -> 20) into lam
    float *t0 = scratch, *t1 = scratch + 512;
    const float *in = app;
    for (int l = 0; l < 4; l++) {
        float *o = (l & 1) ? t1 : t0;
        enc_fc_kernel<<<512 * 32 / 256, 256, 0, st>>>(in, h.W[l], h.b[l], 512, o);
        in = o;
    }
    enc_fc_kernel<<<(20 * 32 + 255) / 256, 256, 0, st>>>(in, h.W[4], h.b[4], 20, lam);
    enc_motion_kernel<<<1, 512, 0, st>>>(lam, h.Q, motion);
    return cudaGetLastError();
}

}  // namespace tpmd
