// The per-level tail of the decoder, one pass per pixel (src/motion_dec.cpp
// :829-885 exact graph; :1077-1108 fast graph): ToFlow 1x1 modulated conv +
// bias + up-sampled flow skip, flow head (tanh + identity grid, sigmoid mask),
// bilinear warp of the level's feats (grid_sample, zeros, align_corners=false
// with the patched gather's arithmetic, patch:341-366), mask blend
// (warp = sampled*m, trunk = warp + out*(1-m)), ToRGB 1x1 + FusedLeakyReLU +
// bias + up-sampled rgb skip (upfirdn2d up=2 pad (2,1), patch:535-572).
//
// The reference runs this as ~12 separate graph nodes with transposes
// (cl_to_sp, clsp_mul/lerp, flow_grid, upfirdn2x); here it is one HBM-bound
// kernel: each pixel's channel vector is read once (conv2 output), its four
// feat taps are read with 16-byte channel-last vector loads (feats are shared
// by every frame of the batch, so they stay L2-resident), and the blended
// trunk is written once, already multiplied by the next up-conv's style.
//
// Mapping: a pixel is handled by G = OC/CPL lanes, each owning CPL
// consecutive channels; 32/G pixels per warp. Channel sums (ToFlow, ToRGB)
// reduce across the G lanes with xor shuffles. The ToFlow and ToRGB weights
// sit in shared memory lane-interleaved, [k][c][lane of the group], so the
// lanes of a warp read consecutive words (no bank conflicts).
#include "tpmd_internal.h"

#include <algorithm>

namespace tpmd {
namespace {

template <typename T, int CPL>
struct chans;
template <int CPL>
struct chans<float, CPL> {
    static __device__ __forceinline__ void load(const float *p, float *v) {
#pragma unroll
        for (int i = 0; i < CPL; i += 4) {
            const float4 q = __ldg(reinterpret_cast<const float4 *>(p + i));
            v[i] = q.x; v[i + 1] = q.y; v[i + 2] = q.z; v[i + 3] = q.w;
        }
    }
    static __device__ __forceinline__ void store(float *p, const float *v) {
#pragma unroll
        for (int i = 0; i < CPL; i += 4)
            *reinterpret_cast<float4 *>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
};
template <int CPL>
struct chans<__half, CPL> {
    static __device__ __forceinline__ void load(const __half *p, float *v) {
#pragma unroll
        for (int i = 0; i < CPL; i += 8) {
            const uint4 q = __ldg(reinterpret_cast<const uint4 *>(p + i));
            const __half2 *h = reinterpret_cast<const __half2 *>(&q);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float2 f = __half22float2(h[k]);
                v[i + 2 * k] = f.x;
                v[i + 2 * k + 1] = f.y;
            }
        }
    }
    static __device__ __forceinline__ void store(__half *p, const float *v) {
#pragma unroll
        for (int i = 0; i < CPL; i += 8) {
            uint4 q;
            __half2 *h = reinterpret_cast<__half2 *>(&q);
#pragma unroll
            for (int k = 0; k < 4; k++) h[k] = __floats2half2_rn(v[i + 2 * k], v[i + 2 * k + 1]);
            *reinterpret_cast<uint4 *>(p + i) = q;
        }
    }
};

// upfirdn2d(up=2, pad=(2,1)) of an h x h plane at output (x, y): of the
// 4x4 kernel only the taps of (x, y)'s parity meet source pixels, so four
// taps (source pixel, kernel index) serve every plane of the pixel, in the
// reference op's tap order (patch:559-569). Taps outside the plane read
// pixel 0 with weight 0.
struct up_taps {
    int off[4];  // source pixel sy * h + sx
    int k[4];    // kernel index, -1 outside the plane
};
__device__ __forceinline__ up_taps up2x_taps(int x, int y, int h) {
    up_taps t;
    const int px = x & 1, py = y & 1, nx = x >> 1, ny = y >> 1;
#pragma unroll
    for (int a = 0; a < 2; a++)
#pragma unroll
        for (int bb = 0; bb < 2; bb++) {
            const int sy = ny + py - 1 + a, sx = nx + px - 1 + bb;
            const bool in = sy >= 0 && sy < h && sx >= 0 && sx < h;
            t.off[2 * a + bb] = in ? sy * h + sx : 0;
            t.k[2 * a + bb] = in ? (px + 2 * bb) + 4 * (py + 2 * a) : -1;
        }
    return t;
}
__device__ __forceinline__ float up2x(const float *__restrict__ src, const float *__restrict__ k4,
                                      const up_taps &t) {
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++)
        acc = fmaf(__ldg(src + t.off[i]), t.k[i] >= 0 ? __ldg(k4 + t.k[i]) : 0.0f, acc);
    return acc;
}

template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <typename T, int CPL, int G>
__global__ void __launch_bounds__(256) tail_kernel(tail_params p) {
    constexpr int PW = 32 / G;  // pixels per warp
    __shared__ __align__(16) float s_fw[3 * 512];  // [k][c][g]: weight k of channel g*CPL + c
    __shared__ __align__(16) float s_rw[3 * 512];
    const int OC = p.OC, r = p.r;
    for (int i = threadIdx.x; i < 3 * OC; i += blockDim.x) {  // i = (k * CPL + c) * G + g
        const int g = i % G, c = (i / G) % CPL, k = i / (G * CPL);
        const int src = k * OC + g * CPL + c;
        s_fw[i] = __ldg(p.fW + src);
        s_rw[i] = __ldg(p.rW + src);
    }
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const int gl = lane % G, grp = lane / G;
    const int c0 = gl * CPL;
    const int64_t rr = (int64_t) r * r;
    const int64_t npix = (int64_t) p.B * rr;
    const int h = r / 2;
    const int lg = __ffs(r) - 1;  // r is a power of two
    const int64_t warp0 = ((int64_t) blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t) gridDim.x * blockDim.x) >> 5;
    const T *outp = (const T *) p.out;
    const T *featp = (const T *) p.feat;

    for (int64_t base = warp0 * PW; base < npix; base += nwarps * PW) {
        const int64_t pix = base + grp;  // npix is a multiple of PW
        const int64_t b = pix >> (2 * lg);
        const int pr = (int) (pix & (rr - 1));
        const int y = pr >> lg, x = pr & (r - 1);
        const up_taps ut = up2x_taps(x, y, h);

        float o[CPL], fs[CPL];
        chans<T, CPL>::load(outp + pix * OC + c0, o);
        chans<float, CPL>::load(p.fs + b * p.s_stride + c0, fs);
        // the up-sampled skips depend on the pixel only, so their loads are
        // issued here, in flight with the channel loads above. Groups of 8 or
        // more lanes split them: lanes 0-2 form the flow skip's three
        // channels, lanes 3-5 the rgb skip's, each with the four taps in
        // order (shuffled to the group later); narrower groups form all six
        float skv = 0.0f, skf[3] = {0.0f, 0.0f, 0.0f}, skr[3] = {0.0f, 0.0f, 0.0f};
        if constexpr (G >= 8) {
            if (gl < 6) {
                const int k = gl < 3 ? gl : gl - 3;
                const float *plane = gl < 3 ? p.skipf_prev : p.skip_prev;
                if (plane) skv = up2x(plane + (b * 3 + k) * (int64_t) h * h, gl < 3 ? p.fup : p.rup, ut);
            }
        } else {
#pragma unroll
            for (int k = 0; k < 3; k++) {
                if (p.skipf_prev) skf[k] = up2x(p.skipf_prev + (b * 3 + k) * (int64_t) h * h, p.fup, ut);
                if (p.skip_prev) skr[k] = up2x(p.skip_prev + (b * 3 + k) * (int64_t) h * h, p.rup, ut);
            }
        }
        float f0 = 0.0f, f1 = 0.0f, f2 = 0.0f;
#pragma unroll
        for (int c = 0; c < CPL; c++) {
            const float xs = o[c] * fs[c];
            f0 = fmaf(s_fw[c * G + gl], xs, f0);
            f1 = fmaf(s_fw[(CPL + c) * G + gl], xs, f1);
            f2 = fmaf(s_fw[(2 * CPL + c) * G + gl], xs, f2);
        }
        float fl[3] = {group_sum<G>(f0), group_sum<G>(f1), group_sum<G>(f2)};
        const int lead = lane - gl;  // lane 0 of this pixel's group
        if constexpr (G >= 8) {
#pragma unroll
            for (int k = 0; k < 3; k++) {
                skf[k] = __shfl_sync(0xffffffffu, skv, lead + k);
                skr[k] = __shfl_sync(0xffffffffu, skv, lead + 3 + k);
            }
        }
#pragma unroll
        for (int k = 0; k < 3; k++) {
            fl[k] += __ldg(p.fb + k);
            if (p.skipf_prev) fl[k] += skf[k];
        }
        if (p.skipf_out && gl == 0) {
#pragma unroll
            for (int k = 0; k < 3; k++) p.skipf_out[(b * 3 + k) * rr + pr] = fl[k];
        }
        const float gx = tanhf(fl[0]) + __ldg(p.lin + x);
        const float gy = tanhf(fl[1]) + __ldg(p.lin + y);
        const float m = 1.0f / (1.0f + expf(-fl[2]));

        // bilinear taps, as the patched gather computes them
        const float fx = fmaf((gx + 1.0f) * 0.5f, (float) r, -0.5f);
        const float fy = fmaf((gy + 1.0f) * 0.5f, (float) r, -0.5f);
        const bool sane = fabsf(fx) < 1.0e8f && fabsf(fy) < 1.0e8f;
        const float flx = floorf(fx), fly = floorf(fy);
        const int x0 = sane ? (int) flx : -4, y0 = sane ? (int) fly : -4;
        const float wx = fx - flx, wy = fy - fly;
        float smp[CPL];
#pragma unroll
        for (int c = 0; c < CPL; c++) smp[c] = 0.0f;
        // the four taps without branches, so their loads are in flight
        // together: a tap outside the map (zeros padding) reads pixel 0 with
        // weight 0, which adds +0 to every channel
        int trow[4];
        float twt[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int cx = x0 + (k & 1), cy = y0 + (k >> 1);
            const bool in = sane && cx >= 0 && cx < r && cy >= 0 && cy < r;
            trow[k] = in ? cy * r + cx : 0;
            twt[k] = in ? ((k & 1) ? wx : 1.0f - wx) * ((k >> 1) ? wy : 1.0f - wy) : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            float f[CPL];
            chans<T, CPL>::load(featp + (int64_t) trow[k] * OC + c0, f);
#pragma unroll
            for (int c = 0; c < CPL; c++) smp[c] = fmaf(twt[k], f[c], smp[c]);
        }

        const float om = 1.0f - m;
        float g0 = 0.0f, g1 = 0.0f, g2 = 0.0f;
#pragma unroll
        for (int c = 0; c < CPL; c++) {
            const float w = smp[c] * m;
            g0 = fmaf(s_rw[c * G + gl], w, g0);
            g1 = fmaf(s_rw[(CPL + c) * G + gl], w, g1);
            g2 = fmaf(s_rw[(2 * CPL + c) * G + gl], w, g2);
            smp[c] = w + o[c] * om;  // trunk
        }
        float rg[3] = {group_sum<G>(g0), group_sum<G>(g1), group_sum<G>(g2)};
        if (gl == 0) {
#pragma unroll
            for (int k = 0; k < 3; k++) {
                float v = rg[k] + __ldg(p.rlb + k);
                v = (v > 0.0f ? v : 0.2f * v) + __ldg(p.rb + k);
                if (p.skip_prev) v += skr[k];
                p.skip_out[(b * 3 + k) * rr + pr] = v;
            }
        }
        if (p.trunk) {
            float sn[CPL];
            chans<float, CPL>::load(p.snext + b * p.s_stride + c0, sn);
#pragma unroll
            for (int c = 0; c < CPL; c++) smp[c] *= sn[c];
            chans<T, CPL>::store((T *) p.trunk + pix * OC + c0, smp);
        }
    }
}

template <typename T, int CPL, int G>
cudaError_t run_tail(const tail_params &p, cudaStream_t st) {
    constexpr int PW = 32 / G;
    const int64_t npix = (int64_t) p.B * p.r * p.r;
    if (p.r < 2 || (p.r & (p.r - 1))) return cudaErrorInvalidValue;
    const int64_t warps = (npix + PW - 1) / PW;
    // resident blocks only (3 per SM at this kernel's registers): each block
    // stages the weights once and strides over the pixels
    const int blocks = (int) std::min<int64_t>((warps + 7) / 8, 148 * 3);
    tail_kernel<T, CPL, G><<<blocks, 256, 0, st>>>(p);
    return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch_tail(const tail_params &p, cudaStream_t st) {
    // CPL = max(channels per 16 bytes, OC/32) channels per lane, G = OC/CPL
    constexpr bool H = sizeof(T) == 2;
    switch (p.OC) {
        case 512: return run_tail<T, 16, 32>(p, st);
        case 256: return run_tail<T, 8, 32>(p, st);
        case 128:
            if constexpr (H) return run_tail<T, 8, 16>(p, st);
            else return run_tail<T, 4, 32>(p, st);
        case 64:
            if constexpr (H) return run_tail<T, 8, 8>(p, st);
            else return run_tail<T, 4, 16>(p, st);
        case 32:
            if constexpr (H) return run_tail<T, 8, 4>(p, st);
            else return run_tail<T, 4, 8>(p, st);
        default: return cudaErrorInvalidValue;
    }
}

// ToRGB's 1x1 conv (before its bias and activation) is linear, and so is
// the bilinear gather: rW . gather(feat) = gather(rW . feat). Where nothing
// else reads the gathered channels (the last level, which has no trunk), the
// tail gathers this 3-channel projection of the portrait's feats instead of
// all C channels; it is computed once per portrait.
__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

template <typename T>
__global__ void project_feats_kernel(const T *__restrict__ feat, int64_t npx, int C,
                                     const float *__restrict__ rW, float4 *__restrict__ proj) {
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < npx;
         i += (int64_t) gridDim.x * blockDim.x) {
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f;
        for (int c = 0; c < C; c++) {
            const float f = to_f(feat[i * C + c]);
            a0 = fmaf(__ldg(rW + c), f, a0);
            a1 = fmaf(__ldg(rW + C + c), f, a1);
            a2 = fmaf(__ldg(rW + 2 * C + c), f, a2);
        }
        proj[i] = make_float4(a0, a1, a2, 0.0f);
    }
}

}  // namespace

cudaError_t launch_tail(bool f16, const tail_params &p, cudaStream_t st) {
    return f16 ? dispatch_tail<__half>(p, st) : dispatch_tail<float>(p, st);
}

cudaError_t launch_project_feats(bool f16, const void *feat, int64_t npx, int C, const float *rW,
                                 float4 *proj, cudaStream_t st) {
    const int blocks = (int) std::min<int64_t>((npx + 255) / 256, 148 * 8);
    if (f16)
        project_feats_kernel<__half><<<blocks, 256, 0, st>>>((const __half *) feat, npx, C, rW, proj);
    else
        project_feats_kernel<float><<<blocks, 256, 0, st>>>((const float *) feat, npx, C, rW, proj);
    return cudaGetLastError();
}

}  // namespace tpmd
