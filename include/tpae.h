/* tpae — B200 audio encoder (audio_model) for talking-portrait.
 *
 * The modified wav2vec2-base that turns 16 kHz audio into the 25 fps
 * conditioning features of the flow-matching sampler (src/audio_enc.cpp:
 * 55-236): a 7-layer conv1d stem (GroupNorm on the first, exact-erf GELU),
 * linear interpolation to the frame rate, feature projection, grouped
 * positional conv, post-norm transformer layers, and Linear + LayerNorm +
 * SiLU over all layer outputs. float32, as the reference keeps its audio
 * encoder (src/tp.cpp:22-25). Conventions as in tpmd.h.
 */
#ifndef TPAE_H
#define TPAE_H

#include <stddef.h>
#include <stdint.h>

#include "tpmd.h"

#ifdef __cplusplus
extern "C" {
#endif

/* The float.audio.* hyper-parameters (src/audio_enc.cpp:25-45). */
typedef struct tpae_config {
    int n_layers, n_heads, hidden, ffn, dim_w;
    float ln_eps;
    int conv_dim[7], conv_kernel[7], conv_stride[7];
    int pos_kernel, pos_groups, sample_rate, fps;
} tpae_config;

/* The reference's defaults (src/audio_enc.h:10-17, src/audio_enc.cpp:25-45):
 * 12 layers, 12 heads, hidden 768, FFN 3072, dim_w 512, eps 1e-5, conv dims
 * 512, kernels 10,3,3,3,3,2,2, strides 5,2,...,2, positional conv 128 taps
 * in 16 groups, 16 kHz, 25 fps. */
void tpae_default_config(tpae_config *cfg);

typedef struct tpae_ctx tpae_ctx;

tpae_ctx *tpae_create(int device, const tpae_config *cfg);
const char *tpae_create_error(void);
void tpae_destroy(tpae_ctx *ctx);
const char *tpae_last_error(const tpae_ctx *ctx);

/* One float32 tensor in torch element order under its checkpoint name
 * (feature_extractor.conv_layers.i.conv.weight, ...conv_layers.0.layer_norm,
 * feature_projection.*, encoder.pos_conv_embed.conv.*, encoder.layer_norm,
 * encoder.layers.i.{attention.{q,k,v,out}_proj, layer_norm, feed_forward.
 * {intermediate,output}_dense, final_layer_norm}, audio_projection.{0,1}). */
int tpae_set_tensor(tpae_ctx *ctx, const char *name, const float *data, int64_t n);

/* Every tensor of an audio_{f32,f16}.gguf file (architecture
 * "float-audio"); its float.audio.* keys must equal this handle's config. */
int tpae_load_gguf(tpae_ctx *ctx, const char *path);

int tpae_prepare(tpae_ctx *ctx);

/* audio [n_in] (feature-extractor normalised, host) -> wa [seq_len][dim_w]
 * (host). Inputs that are not a multiple of seq_len*sample_rate/fps samples
 * are replicate-padded or cropped to exactly that many, as the reference
 * does. Device memory grows to the longest input seen. */
int tpae_encode(tpae_ctx *ctx, const float *audio, int64_t n_in, int64_t seq_len, float *wa);

#ifdef __cplusplus
}
#endif
#endif
