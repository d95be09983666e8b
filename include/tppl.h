/* tppl — the end-to-end talking-portrait generator on one B200: motion
 * encoder (tpme), audio encoder (tpae), flow-matching sampler (tpfm) and
 * motion decoder (tpmd) composed as the reference's generate_impl does
 * (src/pipeline.cpp:99-186, behind tp_generate / tp_generate_cb,
 * include/tp.h:37-59). Conventions as in tpmd.h.
 */
#ifndef TPPL_H
#define TPPL_H

#include <stddef.h>
#include <stdint.h>

#include "tpae.h"
#include "tpfm.h"
#include "tpmd.h"
#include "tpme.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct tppl_ctx tppl_ctx;

/* All four stages on CUDA device `device`. ftype "f32" or "f16" selects the
 * decoder's and the sampler's arithmetic (the encoders stay float32, as in
 * the reference, src/tp.cpp:22-25). fmt / audio: hyper-parameters (NULL:
 * tpfm_default_config / tpae_default_config). max_batch: frames per decoder
 * dispatch. NULL on failure, reason in tppl_create_error(). */
tppl_ctx *tppl_create(int device, const char *ftype, const tpfm_config *fmt, const tpae_config *audio,
                      int max_batch);
const char *tppl_create_error(void);
void tppl_destroy(tppl_ctx *ctx);
const char *tppl_last_error(const tppl_ctx *ctx);

/* tp_load's weight half (src/tp.cpp:13-41): audio_<ftype>.gguf,
 * fmt_<ftype>.gguf and motion_ae_<ftype>.gguf from `gguf_dir`, then every
 * stage's prepare. */
int tppl_load(tppl_ctx *ctx, const char *gguf_dir);

/* The stage handles, for loading tensors one by one; call tppl_prepare
 * afterwards. Owned by the pipeline. */
tpme_ctx *tppl_motion_encoder(tppl_ctx *ctx);
tpae_ctx *tppl_audio_encoder(tppl_ctx *ctx);
tpfm_ctx *tppl_sampler(tppl_ctx *ctx);
tpmd_ctx *tppl_decoder(tppl_ctx *ctx);
int tppl_prepare(tppl_ctx *ctx);

/* n_frames = ceil(n_samples * 25 / 16000); n_chunks = ceil(n_frames / 50)
 * (tp_n_frames / tp_n_chunks, src/tp.cpp:63-68). */
int64_t tppl_n_frames(int64_t n_samples);
int64_t tppl_n_chunks(int64_t n_frames);

/* tp_generate: image [3][512][512] CHW in [-1,1], audio [n_samples]
 * normalised 16 kHz mono, emotion index, noise [n_chunks][50][512] or NULL
 * (then drawn from `seed`, the same draw for every chunk, as the
 * reference's fixed-seed generator does) -> out_frames
 * [n_frames][3][512][512]. Returns n_frames or -1. Each sampler chunk's
 * frames are decoded on an internal worker thread (the decoder's own
 * stream) while the next chunk is sampled; the call returns when every
 * frame is in out_frames. */
int tppl_generate(tppl_ctx *ctx, const float *image, const float *audio, int64_t n_samples, int emotion,
                  const float *noise, uint64_t seed, float *out_frames);

/* tp_generate_cb: each decoded frame goes to cb (valid during the call);
 * a nonzero return stops the generation. */
typedef int (*tppl_frame_cb)(int64_t frame_idx, const float *chw, void *ud);
int tppl_generate_cb(tppl_ctx *ctx, const float *image, const float *audio, int64_t n_samples, int emotion,
                     const float *noise, uint64_t seed, tppl_frame_cb cb, void *ud);

/* The generation's intermediate products, for callers that shard the
 * decode across GPUs themselves: the decoder styles (appearance + motion,
 * [n_frames][512]) of a clip, with the decoder's feats set as a side
 * effect. Returns n_frames or -1. */
int tppl_styles(tppl_ctx *ctx, const float *image, const float *audio, int64_t n_samples, int emotion,
                const float *noise, uint64_t seed, float *styles);

/* The same styles chunk by chunk, as the sampler produces them: after each
 * 50-frame chunk, cb(frame0, n, styles, ud) with the decoder styles
 * [n][512] of frames frame0 .. frame0 + n - 1 (valid during the call; the
 * clip's padded tail frames are not passed). The decoder's feats are set
 * before the first call. A nonzero return stops the generation. Returns
 * n_frames or -1. Lets a caller decode on other GPUs while the sampler
 * runs (the reference samples every chunk before decoding,
 * src/pipeline.cpp:134-184; frames depend only on their styles). */
typedef int (*tppl_styles_fn)(int64_t frame0, int64_t n, const float *styles, void *ud);
int tppl_styles_cb(tppl_ctx *ctx, const float *image, const float *audio, int64_t n_samples, int emotion,
                   const float *noise, uint64_t seed, tppl_styles_fn cb, void *ud);

#ifdef __cplusplus
}
#endif
#endif
