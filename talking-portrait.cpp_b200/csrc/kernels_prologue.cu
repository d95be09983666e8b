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
// Both reductions are small f32 GEMMs (rows x frames x K <= 512). One
// register-tiled kernel serves both: a block owns 64 rows x 64 frames, K is
// staged through shared memory 64 at a time (fewer barrier round trips per
// block: the grid is about one block per SM, so each block's latency is the
// kernel's), and each thread accumulates a 4 x 4 outer product (rows
// o0 + tx + 16 i, frames b0 + 4 ty + j) in K order.
// Shared reads are conflict-free or broadcast; stores are coalesced along
// rows.
#include "tpmd_internal.h"

namespace tpmd {
namespace {

constexpr int PT = 64, PK = 64;  // tile rows and frames, K per stage

// DEN = false: s_all[b][o] = W[o] . lat[b] + bmod[o] (W [rows][512]).
// DEN = true:  per conv (a tile never spans two), inv_den[b][d_off + o] =
//              1 / sqrt(S_aug[o][:IC] . s[b]^2 + S_aug[o][IC]).
template <bool DEN>
__global__ void __launch_bounds__(256)
prologue_gemm_kernel(const float *__restrict__ w, const float *__restrict__ bmod, int rows,
                     const float *__restrict__ a, int a_stride, int B, den_table t, float *__restrict__ out,
                     int out_stride) {
    __shared__ float Ws[PT][PK + 1], As[PT][PK + 1];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int b0 = blockIdx.y * PT;
    // the tile's rows: [o0, o0 + nrow) of W (stride ldw), K columns
    int o0, nrow, K, ldw, a_off = 0, d_off = 0;
    const float *W;
    if (DEN) {
        int c = 0, tile = blockIdx.x;
        while (c < t.n) {
            const int nt = (t.row0[c + 1] - t.row0[c] + PT - 1) / PT;
            if (tile < nt) break;
            tile -= nt;
            c++;
        }
        if (c >= t.n) return;
        K = t.ic[c];
        ldw = K + 1;
        o0 = tile * PT;
        nrow = min(PT, t.row0[c + 1] - t.row0[c] - o0);
        W = w + t.saug_off[c];
        a_off = t.s_off[c];
        d_off = t.d_off[c];
    } else {
        K = 512;
        ldw = 512;
        o0 = blockIdx.x * PT;
        nrow = min(PT, rows - o0);
        W = w;
    }
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
    // loader: columns lk and lk + 32, rows lr + 8 m (columns past K load zeros,
    // which add +0 to every sum)
    const int lk = threadIdx.x & 31, lr = threadIdx.x >> 5;
    // the next K chunk is fetched into registers while this one is multiplied
    float wn[PK / 32][PT / 8], an[PK / 32][PT / 8];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int hh = 0; hh < PK / 32; hh++) {
            const int kc = k0 + lk + 32 * hh;
            const bool kin = kc < K;
#pragma unroll
            for (int m = 0; m < PT / 8; m++) {
                const int r = lr + 8 * m, b = b0 + r;
                wn[hh][m] = (kin && r < nrow) ? __ldg(W + (int64_t) (o0 + r) * ldw + kc) : 0.0f;
                an[hh][m] = (kin && b < B) ? __ldg(a + (int64_t) b * a_stride + a_off + kc) : 0.0f;
            }
        }
    };
    fetch(0);
    for (int k0 = 0; k0 < K; k0 += PK) {
#pragma unroll
        for (int hh = 0; hh < PK / 32; hh++)
#pragma unroll
            for (int m = 0; m < PT / 8; m++) {
                const int r = lr + 8 * m;
                Ws[r][lk + 32 * hh] = wn[hh][m];
                As[r][lk + 32 * hh] = DEN ? an[hh][m] * an[hh][m] : an[hh][m];
            }
        __syncthreads();
        if (k0 + PK < K) fetch(k0 + PK);
#pragma unroll 8
        for (int kk = 0; kk < PK; kk++) {
            float wv[4], av[4];
#pragma unroll
            for (int i = 0; i < 4; i++) wv[i] = Ws[tx + 16 * i][kk];
#pragma unroll
            for (int j = 0; j < 4; j++) av[j] = As[4 * ty + j][kk];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(wv[i], av[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = tx + 16 * i;
        if (r >= nrow) continue;
        const float extra = DEN ? __ldg(W + (int64_t) (o0 + r) * ldw + K) : __ldg(bmod + o0 + r);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int b = b0 + 4 * ty + j;
            if (b >= B) continue;
            if (DEN)
                out[(int64_t) b * out_stride + d_off + o0 + r] = 1.0f / sqrtf(acc[i][j] + extra);
            else
                out[(int64_t) b * out_stride + o0 + r] = acc[i][j] + extra;
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
    if (rows <= 0 || B <= 0) return cudaErrorInvalidValue;
    const dim3 grid((rows + PT - 1) / PT, (B + PT - 1) / PT);
    prologue_gemm_kernel<false><<<grid, 256, 0, st>>>(wmod, bmod, rows, lat, STYLE_DIM, B, den_table{}, s_all, rows);
    return cudaGetLastError();
}

cudaError_t launch_den(const float *saug, const den_table &t, const float *s_all, int s_stride,
                       int B, float *inv_den, int d_stride, cudaStream_t st) {
    if (t.n <= 0 || B <= 0) return cudaErrorInvalidValue;
    int tiles = 0;
    for (int c = 0; c < t.n; c++) {
        if (t.ic[c] <= 0 || t.ic[c] > 512) return cudaErrorInvalidValue;
        tiles += (t.row0[c + 1] - t.row0[c] + PT - 1) / PT;
    }
    const dim3 grid(tiles, (B + PT - 1) / PT);
    prologue_gemm_kernel<true><<<grid, 256, 0, st>>>(saug, nullptr, 0, s_all, s_stride, B, t, inv_den, d_stride);
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
