// Kernels of the flow-matching transformer (fmt_model::forward,
// src/fmt.cpp:64-211) and its Euler/CFG sampler (src/pipeline.cpp:15-91),
// around the plain linears (the tcgen05 GEMM, tpfm_api.cu). Tokens are rows
// m = b*T + f of the three CFG branches b (uncond, full, audio-only) and T
// frames; every activation is row-major [M][width] float32 unless it feeds a
// GEMM, where it is written in the GEMM's input type TIN (float or __half).
// The block linears add their bias in the GEMM epilogue (fc1 also GELU);
// the kernel consuming the other GEMMs' output adds their bias.
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
    pdl_wait();
    pdl_trigger();
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
    pdl_wait();
    pdl_trigger();
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
    pdl_wait();
    pdl_trigger();
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
// qkv = the GEMM output (bias added in its epilogue), row m = [q | k | v] of
// width 3H. Every q, k and
// v element the warp needs is loaded up front (EPL per lane and row, MAXJ
// keys at most), so the band costs one memory round trip.
template <typename TIN, int EPL, int MAXJ>
__global__ void __launch_bounds__(128) attn_kernel(const float *__restrict__ qkv, int T, int H, int nh, int window,
                                                   TIN *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int hd = H / nh;
    if (g >= 3 * nh * T) return;
    const int i = g % T, head = (g / T) % nh, b = g / (T * nh);
    const int j0 = max(0, i - window), j1 = min(T, i + window + 1), nj = j1 - j0;
    const float scale = 1.0f / sqrtf((float) hd);
    const float *base = qkv + (int64_t) b * T * 3 * H + head * hd;
    float q[EPL], k[MAXJ][EPL], v[MAXJ][EPL];
#pragma unroll
    for (int e = 0; e < EPL; e++) {
        const int d = lane + 32 * e;
        q[e] = d < hd ? base[(int64_t) i * 3 * H + d] : 0.0f;
    }
#pragma unroll
    for (int jj = 0; jj < MAXJ; jj++)
#pragma unroll
        for (int e = 0; e < EPL; e++) {
            const int d = lane + 32 * e;
            const bool in = jj < nj && d < hd;
            const float *row = base + (int64_t) (j0 + jj) * 3 * H;
            k[jj][e] = in ? row[H + d] : 0.0f;
            v[jj][e] = in ? row[2 * H + d] : 0.0f;
        }
    float sc[MAXJ];
    float mx = -INFINITY;
#pragma unroll
    for (int jj = 0; jj < MAXJ; jj++) {
        float a = 0.0f;
#pragma unroll
        for (int e = 0; e < EPL; e++) a = fmaf(q[e], k[jj][e], a);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        sc[jj] = a * scale;
        if (jj < nj) mx = fmaxf(mx, sc[jj]);
    }
    float sum = 0.0f;
#pragma unroll
    for (int jj = 0; jj < MAXJ; jj++)
        if (jj < nj) sum += (sc[jj] = expf(sc[jj] - mx));
#pragma unroll
    for (int e = 0; e < EPL; e++) {
        const int d = lane + 32 * e;
        float a = 0.0f;
#pragma unroll
        for (int jj = 0; jj < MAXJ; jj++)
            if (jj < nj) a = fmaf(sc[jj] / sum, v[jj][e], a);
        if (d < hd) out[((int64_t) b * T + i) * H + head * hd + d] = cvt<TIN>(a);
    }
}

// the gated residual of one sub-block followed by the next layer norm, per
// row: x += (mod[gate] + bmod[gate]) * o (o: the GEMM output, its bias added
// in the GEMM epilogue), then h = LN(x) * (1 + scale)
// + shift with the next norm's modulation (mod2, bmod2). Each element and
// each sum is formed in the same order as a separate residual update then
// norm_mod_kernel would form them.
constexpr int RN_PER_THREAD = 16;  // H <= 16 x blockDim
template <typename TIN>
__global__ void __launch_bounds__(256) res_norm_kernel(float *__restrict__ x, const float *__restrict__ o,
                                                       const float *__restrict__ mod,
                                                       const float *__restrict__ bmod, int mod_stride, int gate_off,
                                                       int H, float eps, const float *__restrict__ mod2,
                                                       const float *__restrict__ bmod2, int shift_off, int scale_off,
                                                       TIN *__restrict__ h) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[32];
    const int m = blockIdx.x;
    float *r = x + (int64_t) m * H;
    const float *orow = o + (int64_t) m * H;
    const float *md = mod + (int64_t) m * mod_stride;
    const float *md2 = mod2 + (int64_t) m * mod_stride;
    float xv[RN_PER_THREAD], scv[RN_PER_THREAD], shv[RN_PER_THREAD];
    float s = 0.0f;
    // every load up front (the next norm's modulation included): one
    // memory round trip per row
#pragma unroll
    for (int k = 0; k < RN_PER_THREAD; k++) {
        const int i = threadIdx.x + k * blockDim.x;
        if (i < H) {
            scv[k] = md2[scale_off + i] + __ldg(bmod2 + scale_off + i);
            shv[k] = md2[shift_off + i] + __ldg(bmod2 + shift_off + i);
            const float g = md[gate_off + i] + __ldg(bmod + gate_off + i);
            const float v = r[i] + g * orow[i];
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
#pragma unroll
    for (int k = 0; k < RN_PER_THREAD; k++) {
        const int i = threadIdx.x + k * blockDim.x;
        if (i < H) {
            const float v = (xv[k] - mean) * inv;
            h[(int64_t) m * H + i] = cvt<TIN>(v * scv[k] + v + shv[k]);
        }
    }
}

// res_norm_kernel with one warp per row for H = 128 NV: each lane holds NV
// float4 groups (columns 4 lane + 128 j); every load of the row (x, o, both
// modulations) goes out before the first use, the sums are warp shuffles in
// a fixed order, no block barrier
template <typename TIN, int NV>
__global__ void __launch_bounds__(256) res_norm_warp_kernel(float *__restrict__ x, const float *__restrict__ o,
                                                            const float *__restrict__ mod,
                                                            const float *__restrict__ bmod, int mod_stride,
                                                            int gate_off, int M, float eps,
                                                            const float *__restrict__ mod2,
                                                            const float *__restrict__ bmod2, int shift_off,
                                                            int scale_off, TIN *__restrict__ h) {
    pdl_wait();
    pdl_trigger();
    constexpr int H = 128 * NV;
    const int lane = threadIdx.x & 31, m = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (m >= M) return;
    float4 *r4 = reinterpret_cast<float4 *>(x + (int64_t) m * H);
    const float4 *o4 = reinterpret_cast<const float4 *>(o + (int64_t) m * H);
    const float4 *g4 = reinterpret_cast<const float4 *>(mod + (int64_t) m * mod_stride + gate_off);
    const float4 *s4 = reinterpret_cast<const float4 *>(mod2 + (int64_t) m * mod_stride + scale_off);
    const float4 *t4 = reinterpret_cast<const float4 *>(mod2 + (int64_t) m * mod_stride + shift_off);
    const float4 *bg4 = reinterpret_cast<const float4 *>(bmod + gate_off);
    const float4 *bs4 = reinterpret_cast<const float4 *>(bmod2 + scale_off);
    const float4 *bt4 = reinterpret_cast<const float4 *>(bmod2 + shift_off);
    float4 xv[NV], ov[NV], gv[NV], sv[NV], tv[NV];
#pragma unroll
    for (int j = 0; j < NV; j++) {
        const int q = lane + 32 * j;
        xv[j] = r4[q];
        ov[j] = o4[q];
        gv[j] = g4[q];
        sv[j] = s4[q];
        tv[j] = t4[q];
    }
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; j++) {
        const int q = lane + 32 * j;
        const float4 bg = __ldg(bg4 + q);
        xv[j].x += (gv[j].x + bg.x) * ov[j].x;
        xv[j].y += (gv[j].y + bg.y) * ov[j].y;
        xv[j].z += (gv[j].z + bg.z) * ov[j].z;
        xv[j].w += (gv[j].w + bg.w) * ov[j].w;
        r4[q] = xv[j];
        s += xv[j].x + xv[j].y + xv[j].z + xv[j].w;
    }
#pragma unroll
    for (int w = 16; w > 0; w >>= 1) s += __shfl_xor_sync(0xffffffffu, s, w);
    const float mean = s / (float) H;
    float qs = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; j++) {
        const float a = xv[j].x - mean, b = xv[j].y - mean, c = xv[j].z - mean, d = xv[j].w - mean;
        qs = fmaf(a, a, qs);
        qs = fmaf(b, b, qs);
        qs = fmaf(c, c, qs);
        qs = fmaf(d, d, qs);
    }
#pragma unroll
    for (int w = 16; w > 0; w >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, w);
    const float inv = 1.0f / sqrtf(qs / (float) H + eps);
#pragma unroll
    for (int j = 0; j < NV; j++) {
        const int q = lane + 32 * j;
        const float4 bs = __ldg(bs4 + q), bt = __ldg(bt4 + q);
        float v[4] = {(xv[j].x - mean) * inv, (xv[j].y - mean) * inv, (xv[j].z - mean) * inv,
                      (xv[j].w - mean) * inv};
        const float sc[4] = {sv[j].x + bs.x, sv[j].y + bs.y, sv[j].z + bs.z, sv[j].w + bs.w};
        const float sh[4] = {tv[j].x + bt.x, tv[j].y + bt.y, tv[j].z + bt.z, tv[j].w + bt.w};
#pragma unroll
        for (int e = 0; e < 4; e++) v[e] = v[e] * sc[e] + v[e] + sh[e];
        TIN *hp = h + (int64_t) m * H + 4 * q;
#pragma unroll
        for (int e = 0; e < 4; e++) hp[e] = cvt<TIN>(v[e]);
    }
}

// v = out + b; per current frame f: vc = (u + a_cfg (a - u)) + e_cfg (fu - a);
// x[f] += dt * vc; the next forward's x60 rows P.. are the new x (and their
// f16 copy, the next x_embedder GEMM's input, when x60h is given)
__global__ void cfg_euler_kernel(const float *__restrict__ vout, const float *__restrict__ bv, int T, int P,
                                 int D, float a_cfg, float e_cfg, float dt, float *__restrict__ x,
                                 float *__restrict__ x60, __half *__restrict__ x60h) {
    pdl_wait();
    pdl_trigger();
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
    pdl_wait();
    pdl_trigger();
    const int64_t n = (int64_t) M * N;
    for (int64_t e = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t) gridDim.x * blockDim.x)
        y[e] = a[e] + __ldg(b + e % N);
}

__global__ void to_half_kernel(const float *__restrict__ a, int64_t n, __half *__restrict__ y) {
    pdl_wait();
    pdl_trigger();
    for (int64_t e = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t) gridDim.x * blockDim.x)
        y[e] = __float2half_rn(a[e]);
}

inline int grid_for(int64_t n) { return (int) std::min<int64_t>((n + 255) / 256, 148 * 8); }

}  // namespace

cudaError_t fmt_gemv(const float *W, const float *x, const float *b, int N, int K, bool silu_act, float *y,
                     cudaStream_t st) {
    return launch_pdl(gemv_kernel, dim3((N * 32 + 255) / 256), dim3(256), 0, st, W, x, b, N, K, silu_act ? 1 : 0, y);
}
cudaError_t fmt_cond_silu(bool f16, const float *clin, const float *bc, const float *te, int M, int H, void *sc,
                          cudaStream_t st) {
    const dim3 g(grid_for((int64_t) M * H));
    if (f16) return launch_pdl(cond_silu_kernel<__half>, g, dim3(256), 0, st, clin, bc, te, M, H, (__half *) sc);
    return launch_pdl(cond_silu_kernel<float>, g, dim3(256), 0, st, clin, bc, te, M, H, (float *) sc);
}
cudaError_t fmt_norm_mod(bool f16, float *x, int M, int H, float eps, const float *mod, const float *bmod,
                         int mod_stride, int shift_off, int scale_off, void *h, cudaStream_t st, const float *x1,
                         const float *bx, const float *pos, int T) {
    if (x1 && (!bx || !pos || T <= 0)) return cudaErrorInvalidValue;
    if (f16)
        return launch_pdl(norm_mod_kernel<__half>, dim3(M), dim3(256), 0, st, x, H, eps, mod, bmod, mod_stride,
                          shift_off, scale_off, (__half *) h, x1, bx, pos, T);
    return launch_pdl(norm_mod_kernel<float>, dim3(M), dim3(256), 0, st, x, H, eps, mod, bmod, mod_stride, shift_off,
                      scale_off, (float *) h, x1, bx, pos, T);
}
cudaError_t fmt_attn(bool f16, const float *qkv, int T, int H, int nh, int window, void *out, cudaStream_t st) {
    if (2 * window + 1 > 16 || H % nh) return cudaErrorInvalidValue;
    // 128-thread blocks: the 3 nh T warps fit the SMs in one wave
    const dim3 g((3 * nh * T * 32 + 127) / 128);
    const int hd = H / nh;
    if (hd > 128) return cudaErrorInvalidValue;
    if (hd <= 64 && window <= 2) {  // the sampler's band of five keys
        if (f16)
            return launch_pdl(attn_kernel<__half, 2, 5>, g, dim3(128), 0, st, qkv, T, H, nh, window, (__half *) out);
        return launch_pdl(attn_kernel<float, 2, 5>, g, dim3(128), 0, st, qkv, T, H, nh, window, (float *) out);
    }
    if (f16)
        return launch_pdl(attn_kernel<__half, 4, 16>, g, dim3(128), 0, st, qkv, T, H, nh, window, (__half *) out);
    return launch_pdl(attn_kernel<float, 4, 16>, g, dim3(128), 0, st, qkv, T, H, nh, window, (float *) out);
}
cudaError_t fmt_res_norm(bool f16, float *x, const float *o, const float *mod, const float *bmod,
                         int mod_stride, int gate_off, int M, int H, float eps, const float *mod2, const float *bmod2,
                         int shift_off, int scale_off, void *h, cudaStream_t st) {
    if (H > RN_PER_THREAD * 256) return cudaErrorInvalidValue;
    const bool al = !(((uintptr_t) x | (uintptr_t) o | (uintptr_t) mod | (uintptr_t) bmod |
                       (uintptr_t) mod2 | (uintptr_t) bmod2) & 15) &&
                    mod_stride % 4 == 0 && gate_off % 4 == 0 && shift_off % 4 == 0 && scale_off % 4 == 0;
    if (H == 1024 && al) {  // the sampler's width: a warp per row
        const dim3 g((M * 32 + 255) / 256);
        if (f16)
            return launch_pdl(res_norm_warp_kernel<__half, 8>, g, dim3(256), 0, st, x, o, mod, bmod, mod_stride,
                              gate_off, M, eps, mod2, bmod2, shift_off, scale_off, (__half *) h);
        return launch_pdl(res_norm_warp_kernel<float, 8>, g, dim3(256), 0, st, x, o, mod, bmod, mod_stride, gate_off,
                          M, eps, mod2, bmod2, shift_off, scale_off, (float *) h);
    }
    if (f16)
        return launch_pdl(res_norm_kernel<__half>, dim3(M), dim3(256), 0, st, x, o, mod, bmod, mod_stride,
                          gate_off, H, eps, mod2, bmod2, shift_off, scale_off, (__half *) h);
    return launch_pdl(res_norm_kernel<float>, dim3(M), dim3(256), 0, st, x, o, mod, bmod, mod_stride, gate_off, H,
                      eps, mod2, bmod2, shift_off, scale_off, (float *) h);
}
cudaError_t fmt_cfg_euler(const float *vout, const float *bv, int T, int P, int D, float a_cfg, float e_cfg,
                          float dt, float *x, float *x60, __half *x60h, cudaStream_t st) {
    return launch_pdl(cfg_euler_kernel, dim3(grid_for((int64_t) (T - P) * D)), dim3(256), 0, st, vout, bv, T, P, D,
                      a_cfg, e_cfg, dt, x, x60, x60h);
}
cudaError_t fmt_add_bias(const float *a, const float *b, int M, int N, float *y, cudaStream_t st) {
    return launch_pdl(add_bias_kernel, dim3(grid_for((int64_t) M * N)), dim3(256), 0, st, a, b, M, N, y);
}
cudaError_t fmt_to_half(const float *a, int64_t n, __half *y, cudaStream_t st) {
    return launch_pdl(to_half_kernel, dim3(grid_for(n)), dim3(256), 0, st, a, n, y);
}

}  // namespace tpmd
