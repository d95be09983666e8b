// Op-level kernels with the semantics of the reference's patched ggml ops
// ggml_bilinear_gather(_planar/_sp) and ggml_im2col_cf
// (patches/ggml-tp-ops.patch:25-60,104-111; CPU semantics patch:201-369).
//
// Both ops are HBM-bound byte movers. Design:
//  * bilinear gather: each block stages the per-point tap rows and weights in
//    shared memory (one thread per point computes them once), then the block
//    gathers channels with 16-byte vector loads (4 f32 / 8 f16 channels) so a
//    warp reads whole 128-byte lines of each tap row and writes the
//    channel-last output contiguously.
//  * im2col_cf: one thread per (output pixel, tap, 8-channel chunk): two
//    16-byte source loads, one 16-byte (f16) or two (f32) destination stores,
//    consecutive threads writing consecutive bytes of the destination row.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/tpmd.h"

namespace tpmd {
thread_local std::string g_tpk_err;
int tpk_fail(const std::string &msg) {
    g_tpk_err = msg;
    return -1;
}
}  // namespace tpmd

namespace {

int fail(const std::string &msg) { return tpmd::tpk_fail(msg); }

constexpr int GATHER_THREADS = 256;
constexpr int GATHER_PTS = 64;  // points staged per block iteration

// 16-byte vector of VEC channels converted to float
template <typename TF, int VEC>
__device__ __forceinline__ void ld_vec(const TF *p, float *v);
template <>
__device__ __forceinline__ void ld_vec<float, 4>(const float *p, float *v) {
    const float4 q = __ldg(reinterpret_cast<const float4 *>(p));
    v[0] = q.x;
    v[1] = q.y;
    v[2] = q.z;
    v[3] = q.w;
}
template <>
__device__ __forceinline__ void ld_vec<__half, 8>(const __half *p, float *v) {
    const uint4 q = __ldg(reinterpret_cast<const uint4 *>(p));
    const __half2 *h = reinterpret_cast<const __half2 *>(&q);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 f = __half22float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}
template <>
__device__ __forceinline__ void ld_vec<float, 1>(const float *p, float *v) {
    v[0] = __ldg(p);
}
template <>
__device__ __forceinline__ void ld_vec<__half, 1>(const __half *p, float *v) {
    v[0] = __half2float(__ldg(p));
}

// Tap rows and weights of one grid point, in the reference's arithmetic
// (patch:341-358): fx = (gx+1)*0.5*W - 0.5 (final multiply-add fused), taps
// k = 0..3 at (x0 + (k&1), y0 + (k>>1)), row -1 when out of bounds. A
// non-finite or absurdly large coordinate yields no taps (all zero), as the
// reference CPU op does on x86 where the int64 conversion saturates.
__device__ __forceinline__ void tap_setup(float gx, float gy, int W, int H, int *row, float *wt) {
    const float fx = fmaf((gx + 1.0f) * 0.5f, (float) W, -0.5f);
    const float fy = fmaf((gy + 1.0f) * 0.5f, (float) H, -0.5f);
    const bool sane = fabsf(fx) < 1.0e8f && fabsf(fy) < 1.0e8f;
    const float flx = floorf(fx), fly = floorf(fy);
    const int x0 = sane ? (int) flx : -4, y0 = sane ? (int) fly : -4;
    const float wx = fx - flx, wy = fy - fly;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int cx = x0 + (k & 1), cy = y0 + (k >> 1);
        const bool ok = sane && cx >= 0 && cx < W && cy >= 0 && cy < H;
        row[k] = ok ? cy * W + cx : -1;
        wt[k] = ((k & 1) ? wx : 1.0f - wx) * ((k >> 1) ? wy : 1.0f - wy);
    }
}

template <typename TF, int VEC, bool SP>
__global__ void __launch_bounds__(GATHER_THREADS)
bilinear_gather_kernel(const TF *__restrict__ feat, const float *__restrict__ grid,
                       float *__restrict__ dst, int C, int W, int H, int64_t N, int planar) {
    __shared__ int s_row[GATHER_PTS][4];
    __shared__ float s_w[GATHER_PTS][4];
    const int nchunk = C / VEC;
    for (int64_t n0 = (int64_t) blockIdx.x * GATHER_PTS; n0 < N;
         n0 += (int64_t) gridDim.x * GATHER_PTS) {
        const int npts = (N - n0 < GATHER_PTS) ? (int) (N - n0) : GATHER_PTS;
        if (threadIdx.x < npts) {
            const int64_t n = n0 + threadIdx.x;
            const float gx = planar ? grid[n] : grid[2 * n];
            const float gy = planar ? grid[N + n] : grid[2 * n + 1];
            tap_setup(gx, gy, W, H, s_row[threadIdx.x], s_w[threadIdx.x]);
        }
        __syncthreads();
        const int items = npts * nchunk;
        for (int it = threadIdx.x; it < items; it += GATHER_THREADS) {
            int pt, ch;
            if (SP) {  // point fastest: coalesced [C][N] stores
                pt = it % npts;
                ch = it / npts;
            } else {   // chunk fastest: coalesced [N][C] loads and stores
                pt = it / nchunk;
                ch = it % nchunk;
            }
            float acc[VEC];
#pragma unroll
            for (int v = 0; v < VEC; v++) acc[v] = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int row = s_row[pt][k];
                if (row < 0) continue;
                const float w = s_w[pt][k];
                float f[VEC];
                ld_vec<TF, VEC>(feat + (int64_t) row * C + (int64_t) ch * VEC, f);
#pragma unroll
                for (int v = 0; v < VEC; v++) acc[v] = fmaf(w, f[v], acc[v]);
            }
            const int64_t n = n0 + pt;
            if (SP) {
#pragma unroll
                for (int v = 0; v < VEC; v++) dst[n + N * ((int64_t) ch * VEC + v)] = acc[v];
            } else {
                float *d = dst + n * C + (int64_t) ch * VEC;
                if (VEC == 4 || VEC == 8) {
#pragma unroll
                    for (int v = 0; v < VEC; v += 4)
                        *reinterpret_cast<float4 *>(d + v) =
                            make_float4(acc[v], acc[v + 1], acc[v + 2], acc[v + 3]);
                } else {
#pragma unroll
                    for (int v = 0; v < VEC; v++) d[v] = acc[v];
                }
            }
        }
        __syncthreads();
    }
}

template <typename TF, int VEC, bool SP>
cudaError_t run_gather(const void *feat, int C, int W, int H, const float *grid, int64_t N,
                       int planar, float *dst, cudaStream_t st) {
    const int64_t tiles = (N + GATHER_PTS - 1) / GATHER_PTS;
    const int blocks = (int) std::min<int64_t>(tiles, 148 * 8);
    bilinear_gather_kernel<TF, VEC, SP><<<blocks, GATHER_THREADS, 0, st>>>(
        (const TF *) feat, grid, dst, C, W, H, N, planar);
    return cudaGetLastError();
}

// --- im2col_cf ---------------------------------------------------------------
template <typename TD>
__device__ __forceinline__ void st8(TD *d, const float *v);
template <>
__device__ __forceinline__ void st8<float>(float *d, const float *v) {
    reinterpret_cast<float4 *>(d)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4 *>(d)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
template <>
__device__ __forceinline__ void st8<__half>(__half *d, const float *v) {
    uint4 q;
    __half2 *h = reinterpret_cast<__half2 *>(&q);
#pragma unroll
    for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4 *>(d) = q;
}
__device__ __forceinline__ void st1(float *d, float v) { *d = v; }
__device__ __forceinline__ void st1(__half *d, float v) { *d = __float2half_rn(v); }

struct im2col_geom {
    int IC, IW, IH, N, KW, KH, s0, s1, p0, p1, d0, d1, OW, OH;
};

// VEC8: 8-channel chunks (IC % 8 == 0, 16-byte aligned rows), else 1 channel
template <typename TD, bool VEC8>
__global__ void __launch_bounds__(256)
im2col_cf_kernel(const float *__restrict__ src, TD *__restrict__ dst, im2col_geom g,
                 int64_t total) {
    const int per = VEC8 ? 8 : 1;
    const int nchunk = g.IC / per;
    const int ntap = g.KW * g.KH;
    const int64_t R = (int64_t) g.IC * ntap;
    for (int64_t t = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t) gridDim.x * blockDim.x) {
        const int ch = (int) (t % nchunk);
        const int64_t rest = t / nchunk;
        const int tap = (int) (rest % ntap);
        const int64_t pix = rest / ntap;
        const int ow = (int) (pix % g.OW);
        const int oh = (int) ((pix / g.OW) % g.OH);
        const int64_t n = pix / ((int64_t) g.OW * g.OH);
        const int kh = tap / g.KW, kw = tap % g.KW;
        const int iw = ow * g.s0 + kw * g.d0 - g.p0;
        const int ih = oh * g.s1 + kh * g.d1 - g.p1;
        const bool in_b = iw >= 0 && iw < g.IW && ih >= 0 && ih < g.IH;
        TD *d = dst + pix * R + (int64_t) tap * g.IC + (int64_t) ch * per;
        const float *s = src + ((n * g.IH + ih) * g.IW + iw) * (int64_t) g.IC + (int64_t) ch * per;
        if (VEC8) {
            float v[8];
            if (in_b) {
                const float4 a = __ldg(reinterpret_cast<const float4 *>(s));
                const float4 b = __ldg(reinterpret_cast<const float4 *>(s) + 1);
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
                v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) v[i] = 0.0f;
            }
            st8<TD>(d, v);
        } else {
            st1(d, in_b ? __ldg(s) : 0.0f);
        }
    }
}

// 8-channel chunks, one warp per output pixel row: chunk q of the row is
// destination element q*8 (cf rows r = ic + IC*(kw + KW*kh) make the whole
// row of one pixel contiguous, tap-major), so lane q writes the q-th 16
// (f16) or 32 (f32) bytes: every warp store is a contiguous run. The pixel's
// coordinates are divided out once per row; a chunk needs only its tap and
// channel (a shift when IC/8 is a power of two).
template <typename TD>
__global__ void __launch_bounds__(256)
im2col_cf_rows_kernel(const float *__restrict__ src, TD *__restrict__ dst, im2col_geom g, int64_t npix,
                      int lg_nchunk) {
    const int lane = threadIdx.x & 31;
    const int nchunk = g.IC / 8;
    const int rowc = nchunk * g.KW * g.KH;  // chunks per output pixel
    const int64_t R = (int64_t) g.IC * g.KW * g.KH;
    const int64_t wstride = ((int64_t) gridDim.x * blockDim.x) >> 5;
    for (int64_t pix = ((int64_t) blockIdx.x * blockDim.x + threadIdx.x) >> 5; pix < npix; pix += wstride) {
        const int ow = (int) (pix % g.OW);
        const int64_t q2 = pix / g.OW;
        const int oh = (int) (q2 % g.OH);
        const int64_t n = q2 / g.OH;
        const float *sn = src + n * g.IH * g.IW * (int64_t) g.IC;
        TD *drow = dst + pix * R;
        for (int q = lane; q < rowc; q += 32) {
            const int tap = lg_nchunk >= 0 ? q >> lg_nchunk : q / nchunk;
            const int ch = q - tap * nchunk;
            const int kh = tap / g.KW, kw = tap - kh * g.KW;
            const int iw = ow * g.s0 + kw * g.d0 - g.p0;
            const int ih = oh * g.s1 + kh * g.d1 - g.p1;
            float v[8];
            if (iw >= 0 && iw < g.IW && ih >= 0 && ih < g.IH) {
                const float4 *s4 =
                    reinterpret_cast<const float4 *>(sn + ((int64_t) ih * g.IW + iw) * g.IC + ch * 8);
                const float4 a = __ldg(s4), b = __ldg(s4 + 1);
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
                v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) v[i] = 0.0f;
            }
            st8<TD>(drow + (int64_t) q * 8, v);
        }
    }
}

template <typename TD>
cudaError_t run_im2col(const float *src, void *dst, const im2col_geom &g, cudaStream_t st) {
    const bool vec = (g.IC % 8 == 0) && ((uintptr_t) src % 16 == 0) &&
                     ((uintptr_t) dst % (sizeof(TD) * 8) == 0);
    if (vec) {
        const int64_t npix = (int64_t) g.N * g.OH * g.OW;
        const int nchunk = g.IC / 8;
        const int lg = (nchunk & (nchunk - 1)) == 0 ? __builtin_ctz((unsigned) nchunk) : -1;
        const int blocks = (int) std::min<int64_t>((npix * 32 + 255) / 256, 148 * 16);
        im2col_cf_rows_kernel<TD><<<blocks, 256, 0, st>>>(src, (TD *) dst, g, npix, lg);
        return cudaGetLastError();
    }
    const int64_t total = (int64_t) g.N * g.OH * g.OW * g.KW * g.KH * g.IC;
    const int blocks = (int) std::min<int64_t>((total + 255) / 256, 148 * 16);
    im2col_cf_kernel<TD, false><<<blocks, 256, 0, st>>>(src, (TD *) dst, g, total);
    return cudaGetLastError();
}

}  // namespace

extern "C" {

const char *tpk_last_error(void) { return tpmd::g_tpk_err.c_str(); }

int tpk_bilinear_gather(const void *feat, int feat_is_f16, int C, int W, int H,
                        const float *grid, int64_t N, int planar, int out_sp, float *dst,
                        void *stream) {
    if (C <= 0 || W <= 0 || H <= 0 || N < 0) return fail("tpk_bilinear_gather: bad shape");
    if (N == 0) return 0;  // empty grid: nothing to write (dst may be NULL)
    if (!feat || !grid || !dst) return fail("tpk_bilinear_gather: null pointer");
    cudaStream_t st = (cudaStream_t) stream;
    const int vec = feat_is_f16 ? 8 : 4;
    const bool aligned = (C % vec == 0) && ((uintptr_t) feat % 16 == 0) &&
                         (out_sp || (uintptr_t) dst % 16 == 0);
    cudaError_t e;
    if (feat_is_f16) {
        if (aligned)
            e = out_sp ? run_gather<__half, 8, true>(feat, C, W, H, grid, N, planar, dst, st)
                       : run_gather<__half, 8, false>(feat, C, W, H, grid, N, planar, dst, st);
        else
            e = out_sp ? run_gather<__half, 1, true>(feat, C, W, H, grid, N, planar, dst, st)
                       : run_gather<__half, 1, false>(feat, C, W, H, grid, N, planar, dst, st);
    } else {
        if (aligned)
            e = out_sp ? run_gather<float, 4, true>(feat, C, W, H, grid, N, planar, dst, st)
                       : run_gather<float, 4, false>(feat, C, W, H, grid, N, planar, dst, st);
        else
            e = out_sp ? run_gather<float, 1, true>(feat, C, W, H, grid, N, planar, dst, st)
                       : run_gather<float, 1, false>(feat, C, W, H, grid, N, planar, dst, st);
    }
    if (e != cudaSuccess) return fail(std::string("tpk_bilinear_gather: ") + cudaGetErrorString(e));
    return 0;
}

int tpk_im2col_cf(const float *src, int IC, int IW, int IH, int N, int KW, int KH, int s0,
                  int s1, int p0, int p1, int d0, int d1, void *dst, int dst_is_f16,
                  void *stream) {
    if (!src || !dst) return fail("tpk_im2col_cf: null pointer");
    if (IC <= 0 || IW <= 0 || IH <= 0 || N <= 0 || KW <= 0 || KH <= 0 || s0 <= 0 || s1 <= 0 ||
        d0 <= 0 || d1 <= 0 || p0 < 0 || p1 < 0)
        return fail("tpk_im2col_cf: bad shape");
    im2col_geom g{IC, IW, IH, N, KW, KH, s0, s1, p0, p1, d0, d1, 0, 0};
    g.OW = (IW + 2 * p0 - d0 * (KW - 1) - 1) / s0 + 1;
    g.OH = (IH + 2 * p1 - d1 * (KH - 1) - 1) / s1 + 1;
    if (g.OW <= 0 || g.OH <= 0) return fail("tpk_im2col_cf: source smaller than the kernel");
    if ((int64_t) IC * IW * IH >= INT32_MAX)
        return fail("tpk_im2col_cf: source image exceeds 2^31 elements");
    cudaStream_t st = (cudaStream_t) stream;
    const cudaError_t e = dst_is_f16 ? run_im2col<__half>(src, dst, g, st)
                                     : run_im2col<float>(src, dst, g, st);
    if (e != cudaSuccess) return fail(std::string("tpk_im2col_cf: ") + cudaGetErrorString(e));
    return 0;
}

}  // extern "C"
