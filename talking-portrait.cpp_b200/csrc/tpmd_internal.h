// Internal interfaces between the decoder's host orchestration
// (tpmd_api.cpp) and its CUDA kernels. Not installed.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <utility>

#include <nvtx3/nvToolsExt.h>

namespace tpmd {

// A named NVTX range over a host scope (decode calls, their phases): shows
// the host side of a decode on a profiler's timeline. NVTX v3 is header-only
// and its calls do nothing unless a profiling tool is attached.
struct nvtx_range {
    explicit nvtx_range(const char *name) { nvtxRangePushA(name); }
    ~nvtx_range() { nvtxRangePop(); }
    nvtx_range(const nvtx_range &) = delete;
    nvtx_range &operator=(const nvtx_range &) = delete;
};

// Programmatic dependent launch: a kernel launched by launch_pdl may start
// while the kernel before it in the stream is still running. It calls
// pdl_wait() before touching anything that kernel writes or reads (the
// wait returns once that grid has completed and its writes are visible),
// and pdl_trigger() after its own pdl_wait(), so that when a kernel starts,
// every kernel before its predecessor has completed.
#ifdef __CUDACC__
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args &&...args) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    return cudaLaunchKernelEx(&lc, kernel, std::forward<Args>(args)...);
}
#endif

constexpr int N_LEVELS = 7;
constexpr int STYLE_DIM = 512;
constexpr int IMG = 512;
// stage channels: convs[2j] IC->OC up-conv, convs[2j+1] OC->OC
// (src/motion_dec.cpp:12-13)
constexpr int ST_IC[N_LEVELS] = {512, 512, 512, 512, 256, 128, 64};
constexpr int ST_OC[N_LEVELS] = {512, 512, 512, 256, 128, 64, 32};
constexpr int N_CONVS = 15;  // conv1 + convs.0..13 (the demodulated convs)

// One modulated 3x3 conv as an implicit GEMM over channel-last activations.
//   x  [B][H][W][IC]  this conv's input, already multiplied by its style
//   w  [N][9*IC]      N = OC (dense) or 4*OC (sub-pixel up-conv: column
//                     q = k*OC + o, parity class k = 2*by + bx); row order
//                     k = (kh*3 + kw)*IC + ic (the cf order r = ic + IC*(kw+3kh))
//   y  [B][H][W][OC] (dense) or [B][2H][2W][OC] (up)
// epilogue per output (b, o): v = acc * inv_den[b*den_stride + o] + bias[o];
// v = lrelu(v, 0.2); v *= snext[b*snext_stride + o] when snext != nullptr.
struct conv_params {
    const void *x;
    const void *w;
    void *y;
    int B, H, W, IC, OC;
    const float *inv_den;
    int den_stride;
    const float *bias;
    const float *snext;
    int snext_stride;
    int *err;  // device flag a kernel sets when a bounded wait expires
    // test hook (tcgen05 convs only): when nonzero, the kernel first waits up
    // to this many ns on an mbarrier that nothing completes, then reports the
    // expired wait through *err and skips its work
    long long stall_ns;
};

// The per-level tail after conv2 (ToFlow, flow head, bilinear warp of the
// level's feats, mask blend, ToRGB, skip up-sampling), per pixel of level r:
//   fl_k  = sum_c fW[k][c]*(out[c]*fs[c]) + fb[k] + up2x(skipf_prev)[k]
//   grid  = (tanh(fl_0) + lin[x], tanh(fl_1) + lin[y]);  m = sigmoid(fl_2)
//   warp  = gather(feat, grid) * m;  trunk = warp + out*(1 - m)
//   rgb_k = lrelu(sum_c rW[k][c]*warp[c] + rlb[k]) + rb[k] + up2x(skip_prev)[k]
struct tail_params {
    const void *out;        // [B][r][r][OC]   conv2 output
    const void *feat;       // [r*r][OC]       level feats (same dtype)
    int B, r, OC;
    const float *fW;        // [3][OC]
    const float *fs;        // ToFlow styles, fs[b*s_stride + c]
    int s_stride;
    const float *fb, *fup;  // [3], [16]
    const float *skipf_prev;  // [B][3][r/2][r/2] or nullptr (level 0)
    float *skipf_out;         // [B][3][r][r] or nullptr (last level)
    const float *rW;        // [3][OC]
    const float *rlb, *rb, *rup;
    const float *skip_prev;   // [B][3][r/2][r/2] or nullptr
    float *skip_out;          // [B][3][r][r] (the frames at r = 512)
    const float *lin;         // [r] identity grid -1 + 2i/(r-1)
    void *trunk;              // [B][r][r][OC] or nullptr (last level)
    const float *snext;       // next up-conv style, snext[b*s_stride + c]
    const float4 *proj;       // [r*r] rW . feat per feats pixel (.w = 0), or nullptr
};

// launchers; `f16` selects the f16 (else f32) instantiation
cudaError_t launch_style(const float *wmod, const float *bmod, int rows, const float *lat,
                         int B, float *s_all, cudaStream_t st);
struct den_table {
    int n;                 // convs
    int row0[N_CONVS + 1]; // first global row of each conv; row0[n] = total
    int ic[N_CONVS];
    int64_t saug_off[N_CONVS];  // float offset of the conv's S_aug in saug base
    int s_off[N_CONVS];    // its input style offset within a frame's s_all row
    int d_off[N_CONVS];    // its inv_den offset within a frame's row
};
cudaError_t launch_den(const float *saug, const den_table &t, const float *s_all, int s_stride,
                       int B, float *inv_den, int d_stride, cudaStream_t st);
cudaError_t launch_conv1_input(bool f16, const float *input, const float *s, int s_stride,
                               int B, void *x0, cudaStream_t st);
cudaError_t launch_conv_simt(bool f16, bool up, const conv_params &p, cudaStream_t st);
cudaError_t launch_tail(bool f16, const tail_params &p, cudaStream_t st);
// ---- motion encoder (f32, batch 1, channel-last) ----
struct enc_conv_params {
    const float *x;        // [IH][IW][IC]
    int IH, IW, IC;
    const float *w;        // [OC][K*K*IC], k = (kh*K + kw)*IC + ic
    int OC, K, stride, pad;
    int OH, OW;
    const float *bias;     // [OC] or nullptr
    int lrelu;             // leaky relu 0.2 after the bias
    const float *res;      // [OH][OW][OC] added last, or nullptr (may alias y)
    float *y;              // [OH][OW][OC]
    float *col;            // im2col workspace [OH*OW][K*K*IC]
    int64_t col_floats;    // its capacity
    int *err;              // the GEMM's expired-wait flag
};
struct enc_head_params {
    const float *W[5], *b[5];  // EqualLinears, [out][512]
    const float *Q;            // [512][20]
};
cudaError_t launch_enc_stem(const float *img, const float *w, const float *b, float *y, cudaStream_t st);
cudaError_t launch_enc_conv(const enc_conv_params &p, cudaStream_t st);
cudaError_t launch_enc_blur(const float *x, int IH, int IW, int C, const float *k4, int p0, int p1, float *y,
                            cudaStream_t st);
// scratch: 1024 floats (the fc chain's intermediate rows)
cudaError_t launch_enc_head(const float *app, const enc_head_params &h, float *lam, float *motion, float *scratch,
                            cudaStream_t st);
// f32 channel-last feats -> the decoder's feats storage (f16 or f32)
cudaError_t launch_convert_feats(const float *src, int64_t n, bool f16, void *dst, cudaStream_t st);

// proj[i] = (rW[0] . feat[i], rW[1] . feat[i], rW[2] . feat[i], 0) over C channels
cudaError_t launch_project_feats(bool f16, const void *feat, int64_t npx, int C, const float *rW,
                                 float4 *proj, cudaStream_t st);

// CHW f32 frames [n][3][hw] -> RGB24 bytes [n][hw][3] (tools/tp-cli.cpp:43-53)
cudaError_t launch_chw_to_rgb24(const float *chw, int64_t n, int64_t hw, uint8_t *rgb, cudaStream_t st);
// the last-error slot of the tpk_* entry points (sets it, returns -1)
int tpk_fail(const std::string &msg);

// The tcgen05 GEMM of the sampler and the audio encoder (kernels_gemm_tc.cu):
//   Y[m][n] = act((sum_k X[m][k] W[n][k] + bias[n]) * scale) (+ res[m][n]), m < M, n < N
// X and W K-major with row strides ldx, ldw (elements, 16-byte multiples);
// f32 operands by the three-pass TF32 split, else f16. Batch b (grid z)
// reads X at row b*x_row_b, column b*x_col_b (W likewise) and writes Y (or
// Yh, f16) at b*y_batch. Grids with fewer tiles than SMs split K over a
// thread-block cluster per tile.
struct gemm_desc {
    bool f32 = true;
    const void *X = nullptr;
    int64_t ldx = 0;
    const void *W = nullptr;
    int64_t ldw = 0;
    float *Y = nullptr;
    __half *Yh = nullptr;
    int64_t ldy = 0, y_batch = 0;
    int M = 0, N = 0, K = 0, batch = 1;
    int x_row_b = 0, x_col_b = 0, w_row_b = 0, w_col_b = 0;
    const float *bias = nullptr;
    float scale = 1.0f;
    int act = 0;  // 0 none, 1 GELU (erf), 2 GELU (tanh), 3 leaky ReLU (0.2)
    const float *res = nullptr;  // f32 output only: added after act, laid out as Y (may alias Y)
    int *err = nullptr;  // set when a bounded wait expires
    // launched as a programmatic dependent (launch_pdl rules); with w_const
    // W is not written by the kernels before it, so its first tiles load
    // before the wait
    bool pdl = false, w_const = false;
};
cudaError_t gemm_tc(const gemm_desc &d, cudaStream_t st);
// the GEMM kernels' shared-memory attribute on the current device (before a
// stream capture that launches them)
cudaError_t gemm_tc_prepare();

// tcgen05 path (f16)
cudaError_t launch_conv_tc(bool up, const conv_params &p, cudaStream_t st);
bool conv_tc_supported(bool up, int IC, int OC);
// conv2 with the level tail fused into its epilogue (levels with OC <= 256):
// the tail reads the conv2 output from TMEM in f32; p.y, when not null, also
// receives the conv2 output (f16) for parity taps
cudaError_t launch_conv_tail_tc(const conv_params &p, const tail_params &t, cudaStream_t st);
bool conv_tail_tc_supported(int IC, int OC, int r);

}  // namespace tpmd
