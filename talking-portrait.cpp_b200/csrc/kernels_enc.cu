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
//  head:   five plain EqualLinears and motion = Q lambda, one block
//
// The conv is an FFMA implicit GEMM: 128 output pixels x 64 output channels
// x 16 k per step, 256 threads, 8x4 outputs per thread; per (tap, 16-channel
// slice) the block loads the strided, shifted input rows straight from
// memory (zeros outside the map), so no im2col buffer exists.
#include "tpmd_internal.h"

#include <algorithm>

namespace tpmd {
namespace {

constexpr int EBM = 128, EBN = 64, EBK = 16;

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

// blockIdx.z = split: the block sums the k-steps (tap, 16-channel chunk)
// [z * per, (z + 1) * per) of K; with several splits the raw sums go to
// p.part[z][m][n] and enc_split_reduce_kernel applies the epilogue
__global__ void __launch_bounds__(256) enc_conv_kernel(enc_conv_params p, int per) {
    __shared__ __align__(16) float As[EBK][EBM + 4];
    __shared__ __align__(16) float Bs[EBK][EBN + 4];
    const int M = p.OH * p.OW, N = p.OC, KT = p.K * p.K, Kall = KT * p.IC;
    const int m0 = blockIdx.x * EBM, n0 = blockIdx.y * EBN;
    const int tid = threadIdx.x;

    // A loads: output pixel tid%128, channels (tid/128)*8 .. +8 of the slice
    const int a_row = tid & (EBM - 1), a_c = (tid >> 7) * 8;
    const int am = m0 + a_row;
    const bool a_valid = am < M;
    const int ox = a_valid ? am % p.OW : 0, oy = a_valid ? am / p.OW : 0;
    // B loads: column tid/4, k (tid%4)*4 .. +4 of the slice
    const int b_n = tid >> 2, b_k = (tid & 3) * 4;
    const bool b_valid = n0 + b_n < N;
    const float *wrow = p.w + (int64_t) (b_valid ? n0 + b_n : 0) * Kall;
    const int tn = tid & 15, tm = tid >> 4;

    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;

    const int CK = p.IC / EBK;  // 16-channel chunks per tap
    const int ks0 = blockIdx.z * per, ks1 = min(KT * CK, ks0 + per);
    for (int tap = ks0 / CK; tap < KT && tap * CK < ks1; tap++) {
        const int iy = oy * p.stride + tap / p.K - p.pad, ix = ox * p.stride + tap % p.K - p.pad;
        const bool in_b = a_valid && iy >= 0 && iy < p.IH && ix >= 0 && ix < p.IW;
        const float *xp = p.x + ((int64_t) iy * p.IW + ix) * p.IC + a_c;
        const float *wp = wrow + (int64_t) tap * p.IC + b_k;
        const int cb = max(ks0 - tap * CK, 0) * EBK, ce = min(ks1 - tap * CK, CK) * EBK;
        for (int c0 = cb; c0 < ce; c0 += EBK) {
            float av[8], bv[4];
            if (in_b) {
                const float4 u = __ldg(reinterpret_cast<const float4 *>(xp + c0));
                const float4 v = __ldg(reinterpret_cast<const float4 *>(xp + c0) + 1);
                av[0] = u.x; av[1] = u.y; av[2] = u.z; av[3] = u.w;
                av[4] = v.x; av[5] = v.y; av[6] = v.z; av[7] = v.w;
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) av[i] = 0.0f;
            }
            if (b_valid) {
                const float4 u = __ldg(reinterpret_cast<const float4 *>(wp + c0));
                bv[0] = u.x; bv[1] = u.y; bv[2] = u.z; bv[3] = u.w;
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
            for (int kk = 0; kk < EBK; kk++) {
                const float4 a0 = *reinterpret_cast<const float4 *>(&As[kk][tm * 8]);
                const float4 a1 = *reinterpret_cast<const float4 *>(&As[kk][tm * 8 + 4]);
                const float4 bq = *reinterpret_cast<const float4 *>(&Bs[kk][tn * 4]);
                const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float bb[4] = {bq.x, bq.y, bq.z, bq.w};
#pragma unroll
                for (int i = 0; i < 8; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
            }
            __syncthreads();
        }
    }

#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int m = m0 + tm * 8 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int n = n0 + tn * 4 + j;
            if (n >= N) continue;
            float v = acc[i][j];
            if (gridDim.z > 1) {
                p.part[((int64_t) blockIdx.z * M + m) * N + n] = v;
                continue;
            }
            if (p.bias) v += __ldg(p.bias + n);
            if (p.lrelu) v = fmaxf(v, 0.2f * v);
            const int64_t dst = (int64_t) m * N + n;
            if (p.res) v += p.res[dst];
            p.y[dst] = v;
        }
    }
}

// the split-K sums in split order (deterministic), then the conv epilogue
__global__ void __launch_bounds__(256) enc_split_reduce_kernel(enc_conv_params p, int S) {
    const int64_t MN = (int64_t) p.OH * p.OW * p.OC;
    for (int64_t e = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; e < MN; e += (int64_t) gridDim.x * blockDim.x) {
        float v = p.part[e];
        for (int z = 1; z < S; z++) v += p.part[z * MN + e];
        const int n = (int) (e % p.OC);
        if (p.bias) v += __ldg(p.bias + n);
        if (p.lrelu) v = fmaxf(v, 0.2f * v);
        if (p.res) v += p.res[e];
        p.y[e] = v;
    }
}

// y[Y][X][c] = sum_{a,b} k[a][b] x[Y+a-p0][X+b-p0][c], zero outside x;
// y is (IH+p0+p1-3) x (IW+p0+p1-3); four channels per thread
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
__global__ void __launch_bounds__(512) enc_head_kernel(const float *__restrict__ app, enc_head_params h,
                                                       float *__restrict__ lam, float *__restrict__ motion) {
    __shared__ float v[2][512];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    v[0][tid] = app[tid];
    __syncthreads();
    int cur = 0;
    for (int l = 0; l < 5; l++) {
        const int out = l == 4 ? 20 : 512;
        for (int o = warp; o < out; o += 16) {
            const float *w = h.W[l] + (int64_t) o * 512;
            float a = 0.0f;
            for (int k = lane; k < 512; k += 32) a = fmaf(__ldg(w + k), v[cur][k], a);
#pragma unroll
            for (int s = 16; s > 0; s >>= 1) a += __shfl_xor_sync(0xffffffffu, a, s);
            if (lane == 0) v[cur ^ 1][o] = a + __ldg(h.b[l] + o);
        }
        __syncthreads();
        cur ^= 1;
    }
    if (tid < 20) lam[tid] = v[cur][tid];
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < 20; k++) m = fmaf(__ldg(h.Q + tid * 20 + k), v[cur][k], m);
    motion[tid] = m;
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
    if (p.IC % EBK || p.OH <= 0 || p.OW <= 0) return cudaErrorInvalidValue;
    const int64_t M = (int64_t) p.OH * p.OW;
    const int gx = (int) ((M + EBM - 1) / EBM), gy = (p.OC + EBN - 1) / EBN;
    const int ksteps = p.K * p.K * (p.IC / EBK);
    // the deep low-resolution convs launch a few blocks with long K loops:
    // split K so that about two blocks per SM work on them
    int S = 1;
    if (p.part && gx * gy < 148) {
        S = (2 * 148 + gx * gy - 1) / (gx * gy);
        S = std::min(S, 16);
        S = std::min(S, ksteps / 4);  // at least four k-steps per split
        while (S > 1 && (int64_t) S * M * p.OC > p.part_floats) S--;
        if (S < 1) S = 1;
    }
    const int per = (ksteps + S - 1) / S;
    S = (ksteps + per - 1) / per;  // no empty split
    enc_conv_kernel<<<dim3((unsigned) gx, (unsigned) gy, (unsigned) S), 256, 0, st>>>(p, per);
    if (S > 1) {
        const int64_t n = M * p.OC;
        enc_split_reduce_kernel<<<(int) std::min<int64_t>((n + 255) / 256, 148 * 8), 256, 0, st>>>(p, S);
    }
    return cudaGetLastError();
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

cudaError_t launch_enc_head(const float *app, const enc_head_params &h, float *lam, float *motion,
                            cudaStream_t st) {
    enc_head_kernel<<<1, 512, 0, st>>>(app, h, lam, motion);
    return cudaGetLastError();
}

}  // namespace tpmd
