/* tpfm — B200 flow-matching motion sampler (fmt_model + sample_chunk) for
 * talking-portrait.
 *
 * The transformer that turns audio features into motion coefficients, one
 * 50-frame chunk at a time (src/fmt.cpp:9-211, src/pipeline.cpp:15-91): 9
 * Euler steps of a DiT with 3-way classifier-free guidance, banded attention
 * and a 10-frame context. Conventions as in tpmd.h: opaque handle,
 * caller-owned flat float32 buffers (host), 0 / -1 status with the message
 * in tpfm_last_error, one call at a time per handle, NULL-safe destroy.
 */
#ifndef TPFM_H
#define TPFM_H

#include <stddef.h>
#include <stdint.h>

#include "tpmd.h"

#ifdef __cplusplus
extern "C" {
#endif

/* The float.fmt.* hyper-parameters (src/fmt.cpp:9-27). */
typedef struct tpfm_config {
    int dim_h, depth, n_heads, dim_w, dim_a, dim_e;
    int chunk_frames, prev_frames, attn_window, t_freq_dim, nfe;
    float mlp_ratio, ln_eps, a_cfg, e_cfg;
} tpfm_config;

/* The reference's defaults (src/fmt.h:12-18): dim_h 1024, depth 8, n_heads
 * 8, dims 512/512/7, chunk 50 + 10 context, window 2, t_freq 256, nfe 10,
 * mlp_ratio 4, ln_eps 1e-6, a_cfg 2, e_cfg 1. */
void tpfm_default_config(tpfm_config *cfg);

typedef struct tpfm_ctx tpfm_ctx;

/* dtype: TPMD_DTYPE_F32 (float32 GEMMs, no TF32) or TPMD_DTYPE_F16 (f16
 * weights and GEMM inputs, float32 accumulation and everything else).
 * NULL on failure, reason in tpfm_create_error(). */
tpfm_ctx *tpfm_create(int device, int dtype, const tpfm_config *cfg);
const char *tpfm_create_error(void);
void tpfm_destroy(tpfm_ctx *ctx);
const char *tpfm_last_error(const tpfm_ctx *ctx);

/* One float32 tensor in torch element order under its checkpoint name
 * (t_embedder.mlp.{0,2}, c_embedder, x_embedder.proj, pos_embed [1][T][H],
 * blocks.i.{adaLN_modulation.1, attn.qkv, attn.proj, mlp.fc1, mlp.fc2},
 * decoder.{adaLN_modulation.1, linear}; .weight / .bias). */
int tpfm_set_tensor(tpfm_ctx *ctx, const char *name, const float *data, int64_t n);

/* Every tensor of an fmt_{f32,f16}.gguf file (architecture "float-fmt");
 * its float.fmt.* keys must equal this handle's config. */
int tpfm_load_gguf(tpfm_ctx *ctx, const char *path);

/* Upload the weights; requires every tensor. */
int tpfm_prepare(tpfm_ctx *ctx);

/* One CFG-batched forward (fmt_model::forward): x60 [T][dim_w], cond
 * [3][T][dim_w + dim_a + dim_e], t -> v [3][T][dim_w] (uncond, full,
 * audio-only), T = chunk_frames + prev_frames. */
int tpfm_forward(tpfm_ctx *ctx, const float *x60, const float *cond, float t, float *v);

/* One chunk of the sampler (sample_chunk_ex without taps): wr [dim_w],
 * prev_wa and prev_x [prev_frames][dim_w], cond_audio and x0
 * [chunk_frames][dim_w], emotion index (-1: none) -> motion
 * [chunk_frames][dim_w]. The 9 forwards and Euler steps run as one CUDA
 * graph on the device. */
int tpfm_sample_chunk(tpfm_ctx *ctx, const float *wr, const float *prev_wa, const float *cond_audio,
                      const float *prev_x, const float *x0, int emotion, float *motion);

#ifdef __cplusplus
}
#endif
#endif
