// Modulated 3x3 conv as an FFMA implicit GEMM (fp32 parity mode).
//
// GEMM view: M = output-grid pixels of the batch (B*H*W), N = OC (dense) or
// 4*OC (sub-pixel up-conv, parity classes stacked on N), K = 9*IC in the cf
// order k = tap*IC + ic. The A operand is never materialised: each block
// loads, per (tap, 16-channel slice), the shifted channel-last input rows of
// its 128 pixels straight from HBM/L2 (zero outside the map = the conv's
// padding), which removes the reference's 9x im2col write (src/motion_dec.cpp
// :340-354, patch:827-904) from the path.
//
// The epilogue applies the demodulation (x inv_den[b][o], S_aug halved so the
// FusedLeakyReLU gain is included), + activate bias, leaky ReLU 0.2, and x the
// next conv's per-frame style (style applied to activations, so weights stay
// shared across frames), then stores channel-last; the up-conv scatters the
// four parity classes to (2y+by, 2x+bx) (the subpix_lrelu_cl interleave,
// patch:488-530).
//
// Tiles: 128 pixels x 64 columns x 16 k, 256 threads, 8x4 outputs per thread.
#include "tpmd_internal.h"

namespace tpmd {
namespace {

constexpr int BM = 128, BN = 64, BK = 16;

__device__ __forceinline__ void ld8(const float *p, float *v) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void ld8(const __half *p, float *v) {
    const uint4 q = __ldg(reinterpret_cast<const uint4 *>(p));
    const __half2 *h = reinterpret_cast<const __half2 *>(&q);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 f = __half22float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void ld4(const float *p, float *v) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
__device__ __forceinline__ void ld4(const __half *p, float *v) {
    const uint2 q = __ldg(reinterpret_cast<const uint2 *>(p));
    const __half2 *h = reinterpret_cast<const __half2 *>(&q);
    const float2 a = __half22float2(h[0]), b = __half22float2(h[1]);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void st1(float *p, float v) { *p = v; }
__device__ __forceinline__ void st1(__half *p, float v) { *p = __float2half_rn(v); }

template <typename T, bool UP>
__global__ void __launch_bounds__(256) conv_simt_kernel(conv_params p) {
    __shared__ __align__(16) float As[BK][BM + 4];
    __shared__ __align__(16) float Bs[BK][BN + 4];
    const int H = p.H, W = p.W, IC = p.IC, OC = p.OC;
    const int N = UP ? 4 * OC : OC;
    const int K = 9 * IC;
    const int64_t M = (int64_t) p.B * H * W;
    const int64_t m0 = (int64_t) blockIdx.x * BM;
    const int n0 = blockIdx.y * BN;
    const int tid = threadIdx.x;

    // A loads: pixel row tid%128, channels (tid/128)*8 .. +8 of the slice
    const int a_row = tid & (BM - 1), a_c = (tid >> 7) * 8;
    const int64_t am = m0 + a_row;
    const bool a_valid = am < M;
    int ax = 0, ay = 0;
    int64_t ab = 0;
    if (a_valid) {
        ax = (int) (am % W);
        const int64_t t = am / W;
        ay = (int) (t % H);
        ab = t / H;
    }
    const T *xb = (const T *) p.x + ab * H * W * (int64_t) IC;
    // B loads: column tid/4, k (tid%4)*4 .. +4 of the slice
    const int b_n = tid >> 2, b_k = (tid & 3) * 4;
    const bool b_valid = n0 + b_n < N;
    const T *wrow = (const T *) p.w + (int64_t) (b_valid ? n0 + b_n : 0) * K;
    // compute: rows tm*8 .. +8, columns tn*4 .. +4
    const int tn = tid & 15, tm = tid >> 4;

    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;

    for (int tap = 0; tap < 9; tap++) {
        const int iy = ay + tap / 3 - 1, ix = ax + tap % 3 - 1;
        const bool in_b = a_valid && iy >= 0 && iy < H && ix >= 0 && ix < W;
        const T *xp = xb + ((int64_t) iy * W + ix) * IC + a_c;
        const T *wp = wrow + (int64_t) tap * IC + b_k;
        for (int c0 = 0; c0 < IC; c0 += BK) {
            float av[8], bv[4];
            if (in_b) {
                ld8(xp + c0, av);
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) av[i] = 0.0f;
            }
            if (b_valid) {
                ld4(wp + c0, bv);
            } else {
#pragma unroll
                for (int i = 0; i < 4; i++) bv[i] = 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 8; i++) As[a_c + i][a_row] = av[i];
#pragma unroll
            for (int i = 0; i < 4; i++) Bs[b_k + i][b_n] = bv[i];
            __syncthreads();
#pragma unroll
            for (int kk = 0; kk < BK; kk++) {
                const float4 a0 = *reinterpret_cast<const float4 *>(&As[kk][tm * 8]);
                const float4 a1 = *reinterpret_cast<const float4 *>(&As[kk][tm * 8 + 4]);
                const float4 bq = *reinterpret_cast<const float4 *>(&Bs[kk][tn * 4]);
                const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float b[4] = {bq.x, bq.y, bq.z, bq.w};
#pragma unroll
                for (int i = 0; i < 8; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
            }
            __syncthreads();
        }
    }

    // epilogue
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int64_t m = m0 + tm * 8 + i;
        if (m >= M) continue;
        const int x = (int) (m % W);
        const int64_t t = m / W;
        const int y = (int) (t % H);
        const int64_t b = t / H;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int n = n0 + tn * 4 + j;
            if (n >= N) continue;
            const int o = UP ? n % OC : n;
            float v = fmaf(acc[i][j], __ldg(p.inv_den + b * p.den_stride + o), __ldg(p.bias + o));
            v = v > 0.0f ? v : 0.2f * v;
            if (p.snext) v *= __ldg(p.snext + b * p.snext_stride + o);
            int64_t dst;
            if (UP) {
                const int k = n / OC;
                const int Y = 2 * y + (k >> 1), X = 2 * x + (k & 1);
                dst = ((b * 2 * H + Y) * 2 * W + X) * (int64_t) OC + o;
            } else {
                dst = ((b * H + y) * W + x) * (int64_t) OC + o;
            }
            st1((T *) p.y + dst, v);
        }
    }
}

}  // namespace

cudaError_t launch_conv_simt(bool f16, bool up, const conv_params &p, cudaStream_t st) {
    if (p.IC % BK != 0) return cudaErrorInvalidValue;
    const int64_t M = (int64_t) p.B * p.H * p.W;
    const int N = up ? 4 * p.OC : p.OC;
    const dim3 grid((unsigned) ((M + BM - 1) / BM), (unsigned) ((N + BN - 1) / BN));
    if (f16) {
        if (up)
            conv_simt_kernel<__half, true><<<grid, 256, 0, st>>>(p);
        else
            conv_simt_kernel<__half, false><<<grid, 256, 0, st>>>(p);
    } else {
        if (up)
            conv_simt_kernel<float, true><<<grid, 256, 0, st>>>(p);
        else
            conv_simt_kernel<float, false><<<grid, 256, 0, st>>>(p);
    }
    return cudaGetLastError();
}

}  // namespace tpmd
