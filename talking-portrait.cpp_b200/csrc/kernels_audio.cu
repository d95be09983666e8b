// Kernels of the audio encoder (audio_model::encode, src/audio_enc.cpp:55-236),
// float32, around the library's tcgen05 GEMMs (tpae_api.cu). Activations are time-major
// [T][C] (the conv stack) and token-major [S][H] (the transformer).
#include "tpmd_internal.h"

#include <algorithm>

namespace tpmd {
namespace {

__device__ __forceinline__ float gelu_erf(float v) { return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f)); }
__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }
constexpr int AUD_STAT_BLOCKS = 256;
inline int grid_for(int64_t n) { return (int) std::min<int64_t>((n + 255) / 256, 148 * 16); }

// out[g][t][c*K + k] = x[t*s + k - p][c_off + g*C + c] (zero outside), the
// column order of a torch conv1d weight row [C][K]; rows of ldo floats
// (the GEMM's 16-byte row stride; the padding is not written)
__global__ void im2col1d_kernel(const float *__restrict__ x, int64_t T, int ld, int C, int K, int s, int p,
                                int64_t OT, float *__restrict__ out, int ldo) {
    const int g = blockIdx.y;
    const int CK = C * K;
    const int64_t n = OT * CK;
    float *o = out + (int64_t) g * OT * ldo;
    for (int64_t e = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t) gridDim.x * blockDim.x) {
        const int ck = (int) (e % CK);
        const int k = ck % K;
        const int c = ck / K;
        const int64_t t = e / CK;
        const int64_t ti = t * s + k - p;
        o[t * ldo + ck] = (ti >= 0 && ti < T) ? x[ti * ld + (int64_t) g * C + c] : 0.0f;
    }
}

// dst[c][j] = src[j][c] for c < C, j < S (src rows of lds floats, dst rows of
// ldd): 32 x 32 tiles through shared memory
__global__ void transpose_kernel(const float *__restrict__ src, int64_t S, int lds, int C, float *__restrict__ dst,
                                 int ldd) {
    __shared__ float t[32][33];
    const int c0 = blockIdx.x * 32;
    const int64_t j0 = (int64_t) blockIdx.y * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int64_t j = j0 + r;
        const int c = c0 + threadIdx.x;
        t[r][threadIdx.x] = (j < S && c < C) ? src[j * lds + c] : 0.0f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int c = c0 + r;
        const int64_t j = j0 + threadIdx.x;
        if (c < C && j < S) dst[(int64_t) c * ldd + j] = t[threadIdx.x][r];
    }
}

// per channel of x [T][C], over the rows of block b's chunk: (sum, sum of
// squares) in double into part[b][c]; threads along C (coalesced rows)
__global__ void __launch_bounds__(256) chan_partial_kernel(const float *__restrict__ x, int64_t T, int C,
                                                           int64_t rows_per, double2 *__restrict__ part) {
    const int64_t t0 = (int64_t) blockIdx.x * rows_per, t1 = min(T, t0 + rows_per);
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        double s = 0.0, q = 0.0;
#pragma unroll 4
        for (int64_t t = t0; t < t1; t++) {
            const double v = x[t * C + c];
            s += v;
            q = fma(v, v, q);
        }
        part[(int64_t) blockIdx.x * C + c] = make_double2(s, q);
    }
}

// per channel: the partials added in block order -> mean and
// 1/sqrt(var + eps), var = E[x^2] - mean^2 (double)
__global__ void chan_finalize_kernel(const double2 *__restrict__ part, int nb, int64_t T, int C, float eps,
                                     float *__restrict__ mean, float *__restrict__ inv) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    double s = 0.0, q = 0.0;
    for (int i = 0; i < nb; i++) {
        const double2 p = part[(int64_t) i * C + c];
        s += p.x;
        q += p.y;
    }
    const double m = s / (double) T;
    const double v = fmax(q / (double) T - m * m, 0.0);
    mean[c] = (float) m;
    inv[c] = (float) (1.0 / sqrt(v + (double) eps));
}

// x = gelu((x - mean[c]) * inv[c] * w[c] + b[c])  (GroupNorm, one group per channel)
// (C a multiple of 4: rows of float4, blocks over rows)
__global__ void chan_norm_gelu_kernel(float *__restrict__ x, int64_t T, int C, const float *__restrict__ mean,
                                      const float *__restrict__ inv, const float *__restrict__ w,
                                      const float *__restrict__ b) {
    const int C4 = C >> 2;
    for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
        float4 *r = (float4 *) (x + t * C);
        for (int c4 = threadIdx.x; c4 < C4; c4 += blockDim.x) {
            float4 v = r[c4];
            const int c = 4 * c4;
            v.x = gelu_erf((v.x - mean[c]) * inv[c] * __ldg(w + c) + __ldg(b + c));
            v.y = gelu_erf((v.y - mean[c + 1]) * inv[c + 1] * __ldg(w + c + 1) + __ldg(b + c + 1));
            v.z = gelu_erf((v.z - mean[c + 2]) * inv[c + 2] * __ldg(w + c + 2) + __ldg(b + c + 2));
            v.w = gelu_erf((v.w - mean[c + 3]) * inv[c + 3] * __ldg(w + c + 3) + __ldg(b + c + 3));
            r[c4] = v;
        }
    }
}


// linear interpolation with align_corners=True from T to S rows of C
__global__ void interp_kernel(const float *__restrict__ x, int64_t T, int C, int64_t S, float *__restrict__ y) {
    const int64_t n = S * C;
    for (int64_t e = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t) gridDim.x * blockDim.x) {
        const int c = (int) (e % C);
        const int64_t s = e / C;
        const double pos = S == 1 ? 0.0 : (double) s * (double) (T - 1) / (double) (S - 1);
        int64_t i0 = (int64_t) pos;
        if (i0 > T - 1) i0 = T - 1;
        const double frac = pos - (double) i0;
        float v = (float) (1.0 - frac) * x[i0 * C + c];
        if (i0 + 1 < T && frac > 0) v += (float) frac * x[(i0 + 1) * C + c];
        y[e] = v;
    }
}

// row-wise layer norm with affine over N, optionally of (x + r + rb):
//   y = LN(x + r + rb) * w + b, act: 0 none, 1 SiLU; y may alias x
__global__ void __launch_bounds__(256) layer_norm_kernel(const float *x, const float *__restrict__ r,
                                                         const float *__restrict__ rb, int N, float eps,
                                                         const float *__restrict__ w, const float *__restrict__ b,
                                                         int act, float *y) {
    __shared__ float red[8];
    extern __shared__ float row[];
    const int64_t m = blockIdx.x;
    float s = 0.0f;
    for (int i = threadIdx.x; i < N; i += blockDim.x) {
        float v = x[m * N + i];
        if (r) v += r[m * N + i] + (rb ? __ldg(rb + i) : 0.0f);
        row[i] = v;
        s += v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float mean = 0.0f;
    for (int i = 0; i < 8; i++) mean += red[i];
    mean /= (float) N;
    __syncthreads();
    float q = 0.0f;
    for (int i = threadIdx.x; i < N; i += blockDim.x) {
        const float d = row[i] - mean;
        q = fmaf(d, d, q);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = q;
    __syncthreads();
    float var = 0.0f;
    for (int i = 0; i < 8; i++) var += red[i];
    var /= (float) N;
    const float inv = 1.0f / sqrtf(var + eps);
    for (int i = threadIdx.x; i < N; i += blockDim.x) {
        float v = (row[i] - mean) * inv * __ldg(w + i) + __ldg(b + i);
        if (act == 1) v = silu(v);
        y[m * N + i] = v;
    }
}


// e[s][i] += gelu(pos[s][i] + b[i])
__global__ void pos_add_kernel(float *__restrict__ e, const float *__restrict__ pos, const float *__restrict__ b,
                               int64_t S, int H) {
    const int64_t n = S * H;
    for (int64_t q = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; q < n; q += (int64_t) gridDim.x * blockDim.x)
        e[q] += gelu_erf(pos[q] + __ldg(b + q % H));
}

// softmax over the first N entries of each ld-float row of x in place; one
// block per row
__global__ void __launch_bounds__(256) softmax_kernel(float *__restrict__ x, int N, int ld) {
    __shared__ float red[8];
    float *r = x + (int64_t) blockIdx.x * ld;
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < N; i += blockDim.x) mx = fmaxf(mx, r[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int i = 1; i < 8; i++) mx = fmaxf(mx, red[i]);
    __syncthreads();
    float s = 0.0f;
    for (int i = threadIdx.x; i < N; i += blockDim.x) {
        const float v = expf(r[i] - mx);
        r[i] = v;
        s += v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float sum = 0.0f;
    for (int i = 0; i < 8; i++) sum += red[i];
    const float inv = 1.0f / sum;
    for (int i = threadIdx.x; i < N; i += blockDim.x) r[i] *= inv;
}

// dst[s][off + i] = src[s][i] (stacking layer outputs per frame)
__global__ void copy_cols_kernel(const float *__restrict__ src, int64_t S, int H, float *__restrict__ dst, int ld,
                                 int off) {
    const int64_t n = S * H;
    for (int64_t e = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t) gridDim.x * blockDim.x)
        dst[(e / H) * ld + off + e % H] = src[e];
}

}  // namespace

cudaError_t aud_im2col(const float *x, int64_t T, int ld, int C, int K, int s, int p, int64_t OT, int groups,
                       float *out, int ldo, cudaStream_t st) {
    const dim3 grid(grid_for(OT * C * K), groups);
    im2col1d_kernel<<<grid, 256, 0, st>>>(x, T, ld, C, K, s, p, OT, out, ldo);
    return cudaGetLastError();
}
cudaError_t aud_transpose(const float *src, int64_t S, int lds, int C, float *dst, int ldd, cudaStream_t st) {
    const dim3 grid((unsigned) ((C + 31) / 32), (unsigned) ((S + 31) / 32));
    transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(src, S, lds, C, dst, ldd);
    return cudaGetLastError();
}
cudaError_t aud_group_norm_gelu(float *x, int64_t T, int C, float eps, const float *w, const float *b, float *stats,
                                cudaStream_t st) {
    // stats: mean [C], inv [C], then AUD_STAT_BLOCKS x C partials (double2)
    if (C % 4) return cudaErrorInvalidValue;
    double2 *part = (double2 *) (stats + 2 * (int64_t) ((C + 1) & ~1));
    const int64_t rows_per = (T + AUD_STAT_BLOCKS - 1) / AUD_STAT_BLOCKS;
    const int nb = (int) ((T + rows_per - 1) / rows_per);
    chan_partial_kernel<<<nb, 256, 0, st>>>(x, T, C, rows_per, part);
    chan_finalize_kernel<<<(C + 127) / 128, 128, 0, st>>>(part, nb, T, C, eps, stats, stats + C);
    chan_norm_gelu_kernel<<<(unsigned) std::min<int64_t>(T, 148 * 16), 128, 0, st>>>(x, T, C, stats, stats + C, w, b);
    return cudaGetLastError();
}
cudaError_t aud_interp(const float *x, int64_t T, int C, int64_t S, float *y, cudaStream_t st) {
    interp_kernel<<<grid_for(S * C), 256, 0, st>>>(x, T, C, S, y);
    return cudaGetLastError();
}
cudaError_t aud_layer_norm(const float *x, const float *r, const float *rb, int64_t M, int N, float eps,
                           const float *w, const float *b, bool silu_act, float *y, cudaStream_t st) {
    layer_norm_kernel<<<(unsigned) M, 256, N * sizeof(float), st>>>(x, r, rb, N, eps, w, b, silu_act ? 1 : 0, y);
    return cudaGetLastError();
}
cudaError_t aud_pos_add(float *e, const float *pos, const float *b, int64_t S, int H, cudaStream_t st) {
    pos_add_kernel<<<grid_for(S * H), 256, 0, st>>>(e, pos, b, S, H);
    return cudaGetLastError();
}
cudaError_t aud_softmax(float *x, int64_t rows, int N, int ld, cudaStream_t st) {
    softmax_kernel<<<(unsigned) rows, 256, 0, st>>>(x, N, ld);
    return cudaGetLastError();
}
cudaError_t aud_copy_cols(const float *src, int64_t S, int H, float *dst, int ld, int off, cudaStream_t st) {
    copy_cols_kernel<<<grid_for(S * H), 256, 0, st>>>(src, S, H, dst, ld, off);
    return cudaGetLastError();
}

}  // namespace tpmd
