// Kernels of the flow-matching transformer (fmt_model::forward,
// src/fmt.cpp:64-211) and its Euler/CFG sampler (src/pipeline.cpp:15-91),
// around the plain linears (the tcgen05 GEMM, tpfm_api.cu). Tokens are rows
// m = b*T + f of the three CFG branches b (uncond, full, audio-only) and T
// frames; every activation is row-major [M][width] float32 unless it feeds a
// GEMM, where it is written in the GEMM's input type TIN (float or __half).
// GEMMs other than the MLP's first (bias and GELU in its epilogue) run
// without bias; the kernel consuming their output adds it.
#include "tpmd_internal.h"

#include <algorithm>

namespace tpmd {
namespace {

template <typename T>
__device__ __forceinline__ T cvt(float v);
template <>
__device__ __forceinline__ float cvt<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half cvt<__half>(float v) { return __float2half_rn(v); }

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float s = 0.0f;
    for (int i = 0; i < nw; i++) s += red[i];
    return s;
}

// y[n] = act(W[n] . x + b[n]), one warp per row (the timestep MLP, M = 1)
__global__ void __launch_bounds__(256) gemv_kernel(const float *__restrict__ W, const float *__restrict__ x,
                                                   const float *__restrict__ b, int N, int K, int act_silu,
                                                   float *__restrict__ y) {
    const int lane = threadIdx.x & 31, n = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (n >= N) return;
    float a = 0.0f;
    for (int k = lane; k < K; k += 32) a = fmaf(__ldg(W + (int64_t) n * K + k), __ldg(x + k), a);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) {
        a += __ldg(b + n);
        y[n] = act_silu ? silu(a) : a;
    }
}

// sc[m][i] = silu(clin[m][i] + bc[i] + te[i])
template <typename TIN>
__global__ void cond_silu_kernel(const float *__restrict__ clin, const float *__restrict__ bc,
                                 const float *__restrict__ te, int M, int H, TIN *__restrict__ sc) {
    const int64_t n = (int64_t) M * H;
    for (int64_t e = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t) gridDim.x * blockDim.x) {
        const int i = (int) (e % H);
        sc[e] = cvt<TIN>(silu(clin[e] + __ldg(bc + i) + __ldg(te + i)));
    }
}

// h = LN(x) * (1 + scale) + shift per row (ggml_norm: no affine; mean and
// variance in two passes), scale/shift = mod[m][off..] + bmod[off..]. With
// x1 given, the row is first formed as x1[f] + bx + pos[f] (f = m mod T, the
// x embedding of the three branches) and stored to x.
template <typename TIN>
__global__ void __launch_bounds__(256) norm_mod_kernel(float *__restrict__ x, int H, float eps,
                                                       const float *__restrict__ mod,
                                                       const float *__restrict__ bmod, int mod_stride,
                                                       int shift_off, int scale_off, TIN *__restrict__ h,
                                                       const float *__restrict__ x1, const float *__restrict__ bx,
                                                       const float *__restrict__ pos, int T) {
    __shared__ float red[32];
    const int m = blockIdx.x;
    float *r = x + (int64_t) m * H;
    if (x1) {
        const int64_t f = m % T;
        for (int i = threadIdx.x; i < H; i += blockDim.x)
            r[i] = x1[f * H + i] + __ldg(bx + i) + __ldg(pos + f * H + i);
    }
    float s = 0.0f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) s += r[i];
    const float mean = block_sum(s, red) / (float) H;
    float q = 0.0f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const float d = r[i] - mean;
        q = fmaf(d, d, q);
    }
    const float var = block_sum(q, red) / (float) H;
    const float inv = 1.0f / sqrtf(var + eps);
    const float *md = mod + (int64_t) m * mod_stride;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const float v = (r[i] - mean) * inv;
        const float sc = md[scale_off + i] + __ldg(bmod + scale_off + i);
        const float sh = md[shift_off + i] + __ldg(bmod + shift_off + i);
        h[(int64_t) m * H + i] = cvt<TIN>(v * sc + v + sh);
    }
}

// banded self-attention per (branch, head, query row i): keys j with
// |i - j| <= window (the additive -inf mask elsewhere contributes nothing),
// scores q.k / sqrt(hd), softmax, weighted sum of v. One warp per query;
// qkv = GEMM output + bias, row m = [q | k | v] of width 3H.
template <typename TIN>
__global__ void __launch_bounds__(256) attn_kernel(const float *__restrict__ qkv, const float *__restrict__ bqkv,
                                                   int T, int H, int nh, int window, TIN *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int hd = H / nh;
    if (g >= 3 * nh * T) return;
    const int i = g % T, head = (g / T) % nh, b = g / (T * nh);
    const int j0 = max(0, i - window), j1 = min(T, i + window + 1);
    const float scale = 1.0f / sqrtf((float) hd);
    const float *qrow = qkv + ((int64_t) b * T + i) * 3 * H + head * hd;
    float sc[16];
    float mx = -INFINITY;
    for (int j = j0; j < j1; j++) {
        const float *krow = qkv + ((int64_t) b * T + j) * 3 * H + H + head * hd;
        float a = 0.0f;
        for (int d = lane; d < hd; d += 32)
            a = fmaf(qrow[d] + __ldg(bqkv + head * hd + d), krow[d] + __ldg(bqkv + H + head * hd + d), a);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        sc[j - j0] = a * scale;
        mx = fmaxf(mx, sc[j - j0]);
    }
    float sum = 0.0f;
    for (int j = j0; j < j1; j++) sum += (sc[j - j0] = expf(sc[j - j0] - mx));
    for (int d = lane; d < hd; d += 32) {
        float a = 0.0f;
        for (int j = j0; j < j1; j++)
            a = fmaf(sc[j - j0] / sum, qkv[((int64_t) b * T + j) * 3 * H + 2 * H + head * hd + d] +
                                           __ldg(bqkv + 2 * H + head * hd + d),
                     a);
        out[((int64_t) b * T + i) * H + head * hd + d] = cvt<TIN>(a);
    }
}

// the gated residual of one sub-block followed by the next layer norm, per
// row: x += (mod[gate] + bmod[gate]) * (o + bo), then h = LN(x) * (1 + scale)
// + shift with the next norm's modulation (mod2, bmod2). Each element and
// each sum is formed in the same order as a separate residual update then
// norm_mod_kernel would form them.
constexpr int RN_PER_THREAD = 16;  // H <= 16 x blockDim
template <typename TIN>
__global__ void __launch_bounds__(256) res_norm_kernel(float *__restrict__ x, const float *__restrict__ o,
                                                       const float *__restrict__ bo, const float *__restrict__ mod,
                                                       const float *__restrict__ bmod, int mod_stride, int gate_off,
                                                       int H, float eps, const float *__restrict__ mod2,
                                                       const float *__restrict__ bmod2, int shift_off, int scale_off,
                                                       TIN *__restrict__ h) {
    __shared__ float red[32];
    const int m = blockIdx.x;
    float *r = x + (int64_t) m * H;
    const float *orow = o + (int64_t) m * H;
    const float *md = mod + (int64_t) m * mod_stride;
    float xv[RN_PER_THREAD];
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < RN_PER_THREAD; k++) {
        const int i = threadIdx.x + k * blockDim.x;
        if (i < H) {
            const float g = md[gate_off + i] + __ldg(bmod + gate_off + i);
            const float v = r[i] + g * (orow[i] + __ldg(bo + i));
            r[i] = v;
            xv[k] = v;
            s += v;
        }
    }
    const float mean = block_sum(s, red) / (float) H;
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < RN_PER_THREAD; k++) {
        const int i = threadIdx.x + k * blockDim.x;
        if (i < H) {
            const float d = xv[k] - mean;
            q = fmaf(d, d, q);
        }
    }
    const float var = block_sum(q, red) / (float) H;
    const float inv = 1.0f / sqrtf(var + eps);
    const float *md2 = mod2 + (int64_t) m * mod_stride;
#pragma unroll
    for (int k = 0; k < RN_PER_THREAD; k++) {
        const int i = threadIdx.x + k * blockDim.x;
        if (i < H) {
            const float v = (xv[k] - mean) * inv;
            const float sc = md2[scale_off + i] + __ldg(bmod2 + scale_off + i);
            const float sh = md2[shift_off + i] + __ldg(bmod2 + shift_off + i);
            h[(int64_t) m * H + i] = cvt<TIN>(v * sc + v + sh);
        }
    }
}

// v = out + b; per current frame f: vc = (u + a_cfg (a - u)) + e_cfg (fu - a);
// x[f] += dt * vc; the next forward's x60 rows P.. are the new x (and their
// f16 copy, the next x_embedder GEMM's input, when x60h is given)
__global__ void cfg_euler_kernel(const float *__restrict__ vout, const float *__restrict__ bv, int T, int P,
                                 int D, float a_cfg, float e_cfg, float dt, float *__restrict__ x,
                                 float *__restrict__ x60, __half *__restrict__ x60h) {
    const int CF = T - P;
    const int64_t n = (int64_t) CF * D;
    const int64_t br = (int64_t) T * D;
    for (int64_t e = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t) gridDim.x * blockDim.x) {
        const int i = (int) (e % D);
        const int64_t q = (int64_t) P * D + e;
        const float bb = __ldg(bv + i);
        const float u = vout[q] + bb, fu = vout[br + q] + bb, a = vout[2 * br + q] + bb;
        const float vc = (u + a_cfg * (a - u)) + e_cfg * (fu - a);
        const float nx = x[e] + dt * vc;
        x[e] = nx;
        x60[q] = nx;
        if (x60h) x60h[q] = __float2half_rn(nx);
    }
}

// v_out = out + b (the plain forward's output)
__global__ void add_bias_kernel(const float *__restrict__ a, const float *__restrict__ b, int M, int N,
                                float *__restrict__ y) {
    const int64_t n = (int64_t) M * N;
    for (int64_t e = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t) gridDim.x * blockDim.x)
        y[e] = a[e] + __ldg(b + e % N);
}

__global__ void to_half_kernel(const float *__restrict__ a, int64_t n, __half *__restrict__ y) {
    for (int64_t e = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t) gridDim.x * blockDim.x)
        y[e] = __float2half_rn(a[e]);
}

inline int grid_for(int64_t n) { return (int) std::min<int64_t>((n + 255) / 256, 148 * 8); }

}  // namespace

cudaError_t fmt_gemv(const float *W, const float *x, const float *b, int N, int K, bool silu_act, float *y,
                     cudaStream_t st) {
    gemv_kernel<<<(N * 32 + 255) / 256, 256, 0, st>>>(W, x, b, N, K, silu_act ? 1 : 0, y);
    return cudaGetLastError();
}
cudaError_t fmt_cond_silu(bool f16, const float *clin, const float *bc, const float *te, int M, int H, void *sc,
                          cudaStream_t st) {
    if (f16)
        cond_silu_kernel<__half><<<grid_for((int64_t) M * H), 256, 0, st>>>(clin, bc, te, M, H, (__half *) sc);
    else
        cond_silu_kernel<float><<<grid_for((int64_t) M * H), 256, 0, st>>>(clin, bc, te, M, H, (float *) sc);
    return cudaGetLastError();
}
cudaError_t fmt_norm_mod(bool f16, float *x, int M, int H, float eps, const float *mod, const float *bmod,
                         int mod_stride, int shift_off, int scale_off, void *h, cudaStream_t st, const float *x1,
                         const float *bx, const float *pos, int T) {
    if (x1 && (!bx || !pos || T <= 0)) return cudaErrorInvalidValue;
    if (f16)
        norm_mod_kernel<__half><<<M, 256, 0, st>>>(x, H, eps, mod, bmod, mod_stride, shift_off, scale_off,
                                                   (__half *) h, x1, bx, pos, T);
    else
        norm_mod_kernel<float><<<M, 256, 0, st>>>(x, H, eps, mod, bmod, mod_stride, shift_off, scale_off,
                                                  (float *) h, x1, bx, pos, T);
    return cudaGetLastError();
}
cudaError_t fmt_attn(bool f16, const float *qkv, const float *bqkv, int T, int H, int nh, int window, void *out,
                     cudaStream_t st) {
    if (2 * window + 1 > 16 || H % nh) return cudaErrorInvalidValue;
    const int warps = 3 * nh * T;
    if (f16)
        attn_kernel<__half><<<(warps * 32 + 255) / 256, 256, 0, st>>>(qkv, bqkv, T, H, nh, window, (__half *) out);
    else
        attn_kernel<float><<<(warps * 32 + 255) / 256, 256, 0, st>>>(qkv, bqkv, T, H, nh, window, (float *) out);
    return cudaGetLastError();
}
cudaError_t fmt_res_norm(bool f16, float *x, const float *o, const float *bo, const float *mod, const float *bmod,
                         int mod_stride, int gate_off, int M, int H, float eps, const float *mod2, const float *bmod2,
                         int shift_off, int scale_off, void *h, cudaStream_t st) {
    if (H > RN_PER_THREAD * 256) return cudaErrorInvalidValue;
    if (f16)
        res_norm_kernel<__half><<<M, 256, 0, st>>>(x, o, bo, mod, bmod, mod_stride, gate_off, H, eps, mod2, bmod2,
                                                   shift_off, scale_off, (__half *) h);
    else
        res_norm_kernel<float><<<M, 256, 0, st>>>(x, o, bo, mod, bmod, mod_stride, gate_off, H, eps, mod2, bmod2,
                                                  shift_off, scale_off, (float *) h);
    return cudaGetLastError();
}
cudaError_t fmt_cfg_euler(const float *vout, const float *bv, int T, int P, int D, float a_cfg, float e_cfg,
                          float dt, float *x, float *x60, __half *x60h, cudaStream_t st) {
    cfg_euler_kernel<<<grid_for((int64_t) (T - P) * D), 256, 0, st>>>(vout, bv, T, P, D, a_cfg, e_cfg, dt, x, x60,
                                                                     x60h);
    return cudaGetLastError();
}
cudaError_t fmt_add_bias(const float *a, const float *b, int M, int N, float *y, cudaStream_t st) {
    add_bias_kernel<<<grid_for((int64_t) M * N), 256, 0, st>>>(a, b, M, N, y);
    return cudaGetLastError();
}
cudaError_t fmt_to_half(const float *a, int64_t n, __half *y, cudaStream_t st) {
    to_half_kernel<<<grid_for(n), 256, 0, st>>>(a, n, y);
    return cudaGetLastError();
}

}  // namespace tpmd
