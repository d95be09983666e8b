/* CPU oracle for the talking-portrait motion decoder (motion_dec).
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker the parity tests,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg compare against.
 * Nothing in the product path (libtpmd.so, include/tpmd.h) links, loads or
 * calls it.
 *
 * It restates, in plain C++ (f32 arithmetic, OpenMP), the reference's CPU
 * semantics of:
 *   - the patched ggml ops (patches/ggml-tp-ops.patch): bilinear_gather
 *     (+_planar, +_sp), im2col_cf, bias_lrelu, subpix_lrelu, subpix_lrelu_cl,
 *     upfirdn2x, clsp_mul, clsp_lerp, flow_grid;
 *   - the load-time scale folding motion_ae_scale (src/motion_enc.cpp:14-45);
 *   - the derived decoder weights of motion_dec::prepare
 *     (src/motion_dec.cpp:31-226): S_aug, acf, tsubcf;
 *   - the decoder graph: the exact/parity graph (src/motion_dec.cpp:794-888)
 *     and a sub-pixel variant that uses the fast graph's composed up-conv
 *     kernel (src/motion_dec.cpp:397-433) in place of zero-stuff+conv+blur.
 *
 * Parity pinning: the op restatements are checked against the reference's own
 * op code (compiled from the patch by oracle/ref_build.py into oracle/_ref/)
 * and against golden vectors generated from it (tests/golden/). The decoder
 * graph as a whole has no reference-produced vectors (the reference's ggml
 * submodule is absent, so the decoder cannot be built): its composition is
 * cross-checked against an independent torch float64 formulation instead.
 */
#ifndef TP_ORACLE_H
#define TP_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- patched-op restatements ---------------------------------------- */
void orc_bilinear_gather(const void *feat, int feat_f16, int C, int W, int H,
                         const float *grid, int64_t N, int planar, int sp,
                         float *dst);
void orc_im2col_cf(const float *src, int IC, int IW, int IH, int N, int KW,
                   int KH, int s0, int s1, int p0, int p1, int d0, int d1,
                   void *dst, int dst_f16);
void orc_bias_lrelu(const float *x, const float *bias, const int64_t *ne,
                    int axis, float slope, float *y);
void orc_subpix_lrelu(const float *g0, const float *g1, const float *bias,
                      int W, int H, int OC, float slope, float *y);
void orc_subpix_lrelu_cl(const float *y4, const float *bias, int OC,
                         int64_t N, int64_t B, int W, float slope, float *y);
void orc_upfirdn2x(const float *x, const float *k4, int W, int H, int64_t CB,
                   float *y);
void orc_blur(const float *x, const float *k4, int W, int H, int64_t C, int p0, int p1,
              float *y);
void orc_clsp_mul(const float *cl, const float *m, int C, int64_t N, float *y);
void orc_clsp_lerp(const float *cl, const float *m, const float *o, int C,
                   int64_t N, float *y);
void orc_flow_grid(const float *fl, const float *xs, int64_t N, float *y);

/* motion_ae_scale: multiplier folded into tensor `name` at load; ne is the
 * ggml shape (ne[0] = torch's last dim), 4 entries. */
double orc_scale_for(const char *name, const int64_t *ne);

/* ---- derived weights (prepare) --------------------------------------- */
/* S_aug [OC][IC+1]: 0.5*sum_k W^2, last column 0.5e-8 (float32 out). */
void orc_saug(const float *W, int IC, int OC, float *saug);
/* tsubcf [4*OC][9*IC], column q = k*OC + o, row r = ic + IC*(kw + 3*kh). */
void orc_tsubcf(const float *W, const float *blur16, int IC, int OC, float *tsub);

/* ---- decoder ----------------------------------------------------------- */
typedef struct orc_dec orc_dec;
orc_dec *orc_dec_create(void);
void orc_dec_destroy(orc_dec *d);
/* folded f32 tensor in torch element order; returns 0 or -1 (unknown name
 * or size mismatch, message in orc_dec_error) */
int orc_dec_set(orc_dec *d, const char *name, const float *data, int64_t n);
/* feats[j]: [ST_OC[j], r*r] channel-last (pixel-major), r = 8<<j */
int orc_dec_set_feat(orc_dec *d, int j, const float *feat, int64_t n);
/* derive S_aug / tsubcf from the set weights */
int orc_dec_prepare(orc_dec *d);
/* mode bit 0 clear: exact graph (zero-stuff + conv + blur up-convs);
 *          set:   sub-pixel composed up-conv kernel.
 * f16 emulation bits (round to nearest even at that point, compute in f32):
 * ORC_F16_WEIGHTS conv weights, ORC_F16_FEATS feats, ORC_F16_ACTS every conv
 * input (x * style), ORC_F16_OUT the conv2 output read by the level tail.
 * WEIGHTS|FEATS|ACTS is the reference's f16 mode (f16 weights and feats,
 * f16 im2col into f32-accumulating GEMMs, src/gguf_load.cpp:149-153,
 * src/motion_dec.cpp:688,340-354); adding OUT matches storing the conv2
 * output as f16.
 * style [512] -> img [3*512*512] (CHW). keep_taps: record taps. */
#define ORC_F16_WEIGHTS 0x10
#define ORC_F16_FEATS 0x20
#define ORC_F16_ACTS 0x40
#define ORC_F16_OUT 0x80
/* ORC_F16_FOLD (mode 1): the reference's f16 fast graph as it runs
 * (src/motion_dec.cpp:283-337, 452-466 with keep_f16 weights): f16
 * modulation weights and latent in the style GEMVs, f16 constant input and
 * feats, and per conv either the style and 1/den folded into f16 weights
 * (maps larger than the weights, and every conv at r256/r512) or the styled
 * map rounded to f16 with /den after the GEMM. */
#define ORC_F16_FOLD 0x100
int orc_dec_decode(orc_dec *d, const float *style, int mode, int keep_taps,
                   float *img);
/* copy a recorded tap (names as in src/motion_dec.cpp:805-883); returns
 * its element count or -1 */
int64_t orc_dec_tap(const orc_dec *d, const char *name, float *out, int64_t cap);
const char *orc_dec_error(const orc_dec *d);
/* CHW f32 frames [n][3][hw] -> RGB24 bytes [n][hw][3] (tools/tp-cli.cpp:43-53) */
void orc_chw_to_rgb24(const float *chw, int64_t n, int64_t hw, unsigned char *rgb);
void orc_set_threads(int n);
int orc_get_threads(void);

/* ---- motion encoder (motion_enc::run, src/motion_enc.cpp:46-184) -------
 * Stem EqualConv2d(3,32,1) + FusedLeakyReLU; seven ResBlocks (3x3 conv +
 * FLReLU; Blur pad (2,2) + 3x3 stride-2 conv + FLReLU; skip: Blur pad (1,1)
 * + 1x1 stride-2 conv; sum); a 4x4 valid conv -> appearance [512]; five
 * plain EqualLinears -> lambda [20]; motion = Q lambda [512]. Tensors are
 * the scale-folded f32 host copies (motion_ae_scale folds the FLReLU sqrt2
 * and the ResBlock 1/sqrt2, src/motion_enc.cpp:9-45), torch element order.
 * image: [3][512][512] CHW (ggml [512,512,3,1]); feats[j]: [r*r][ST_OC[j]]
 * channel-last, r = 8<<j, = menc conv{6-j} (src/motion_enc.cpp:146-155);
 * any output pointer may be NULL. */
typedef struct orc_enc orc_enc;
orc_enc *orc_enc_create(void);
void orc_enc_destroy(orc_enc *e);
int orc_enc_set(orc_enc *e, const char *name, const float *data, int64_t n);
int orc_enc_run(orc_enc *e, const float *image, float *appearance, float *lambda,
                float *motion, float *const feats[7]);
const char *orc_enc_error(const orc_enc *e);

/* ---- flow-matching transformer (fmt_model, src/fmt.cpp:9-211) and its
 * chunk sampler (sample_chunk_ex, src/pipeline.cpp:15-91) ------------------
 * Dimensions as the GGUF's float.fmt.* keys give them. Tensors f32, torch
 * element order: t_embedder.mlp.{0,2}, c_embedder, x_embedder.proj,
 * pos_embed [1][T][H], blocks.i.{adaLN_modulation.1, attn.qkv, attn.proj,
 * mlp.fc1, mlp.fc2}, decoder.{adaLN_modulation.1, linear} (.weight/.bias). */
typedef struct {
    int dim_h, depth, n_heads, dim_w, dim_a, dim_e;
    int chunk_frames, prev_frames, attn_window, t_freq_dim, nfe;
    float mlp_ratio, ln_eps, a_cfg, e_cfg;
} orc_fmt_config;
typedef struct orc_fmt orc_fmt;
orc_fmt *orc_fmt_create(const orc_fmt_config *cfg);
void orc_fmt_destroy(orc_fmt *f);
int orc_fmt_set(orc_fmt *f, const char *name, const float *data, int64_t n);
/* one CFG-batched forward: x60 [T][dim_w], cond [3][T][dim_w+dim_a+dim_e],
 * t in [0,1] -> v [3][T][dim_w] (uncond, full, audio-only) */
int orc_fmt_forward(orc_fmt *f, const float *x60, const float *cond, float t, float *v);
/* one 50-frame chunk: wr [dim_w], prev_wa / prev_x [P][dim_w], cond_audio /
 * x0 [CF][dim_w], emotion (-1: none) -> motion [CF][dim_w] */
int orc_fmt_sample(orc_fmt *f, const float *wr, const float *prev_wa, const float *cond_audio,
                   const float *prev_x, const float *x0, int emotion, float *motion);
const char *orc_fmt_error(const orc_fmt *f);

/* ---- audio encoder (audio_model::encode, src/audio_enc.cpp:55-236) -----
 * Modified wav2vec2-base: 7 conv1d layers (+ GroupNorm on the first, GELU),
 * linear interpolation (align_corners) to seq_len frames, feature
 * projection, grouped positional conv, 12 post-norm transformer layers,
 * Linear(12*hidden -> dim_w) + LayerNorm + SiLU over all layer outputs. */
typedef struct {
    int n_layers, n_heads, hidden, ffn, dim_w;
    float ln_eps;
    int conv_dim[7], conv_kernel[7], conv_stride[7];
    int pos_kernel, pos_groups, sample_rate, fps;
} orc_aud_config;
typedef struct orc_aud orc_aud;
orc_aud *orc_aud_create(const orc_aud_config *cfg);
void orc_aud_destroy(orc_aud *a);
int orc_aud_set(orc_aud *a, const char *name, const float *data, int64_t n);
/* audio [n_in] -> wa [seq_len][dim_w] */
int orc_aud_encode(orc_aud *a, const float *audio, int64_t n_in, int64_t seq_len, float *wa);
const char *orc_aud_error(const orc_aud *a);

#ifdef __cplusplus
}
#endif
#endif
