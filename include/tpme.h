/* tpme — B200 motion encoder (motion_enc) for talking-portrait.
 *
 * The step in front of the decoder: once per portrait it turns the source
 * image into the appearance latent, the motion basis coefficients and the
 * feature pyramid the decoder warps (motion_enc::run,
 * src/motion_enc.cpp:46-184; called from src/pipeline.cpp through
 * tp_ctx::menc). float32 throughout, as the reference keeps its encoder
 * (src/tp.cpp:22-25). Conventions as in tpmd.h: opaque handle, caller-owned
 * flat buffers, 0 / -1 status with the message in tpme_last_error, one call
 * at a time per handle, NULL-safe destroy.
 *
 * Layouts (fastest last, as C arrays):
 *   image       [3][512][512] float32 CHW (ggml [512,512,3,1])
 *   appearance  [512]  (menc_result::appearance)
 *   lambda      [20]   (menc_result::lambda)
 *   motion      [512]  (menc_result::motion = Q lambda)
 *   feats[j]    [r*r][ST_OC[j]] channel-last, r = 8<<j (menc_result::feats,
 *               the decoder's tpmd_set_feats layout)
 */
#ifndef TPME_H
#define TPME_H

#include <stddef.h>
#include <stdint.h>

#include "tpmd.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct tpme_ctx tpme_ctx;

/* Encoder on CUDA device `device` (sm_100). NULL on failure, reason in
 * tpme_create_error(). */
tpme_ctx *tpme_create(int device);
const char *tpme_create_error(void);
void tpme_destroy(tpme_ctx *ctx);
const char *tpme_last_error(const tpme_ctx *ctx);

/* One scale-folded float32 tensor (motion_ae_scale applied, as
 * weights_t::load leaves it, src/gguf_load.cpp:160-196), torch element
 * order: every "enc.*" tensor of the motion_ae file and "dec.direction.Q"
 * ([512][20]). Unknown names or wrong sizes fail. */
int tpme_set_tensor(tpme_ctx *ctx, const char *name, const float *data, int64_t n);

/* The encoder's tensors from a motion_ae_{f32,f16}.gguf file (GGUF v3,
 * architecture "float-motion-ae", motion_ae_scale folded); decoder tensors
 * are skipped. Call tpme_prepare next. */
int tpme_load_gguf(tpme_ctx *ctx, const char *path);

/* Upload the set tensors to the device; requires every tensor. */
int tpme_prepare(tpme_ctx *ctx);

/* Encode one portrait: image (host) -> outputs (host). Any output pointer,
 * and any feats[j] (or feats itself), may be NULL. Blocks until done. */
int tpme_run(tpme_ctx *ctx, const float *image, float *appearance, float *lambda,
             float *motion, float *const feats[TPMD_N_LEVELS]);

/* Device copy of feats[j] from the last tpme_run (valid until the next run
 * or destroy): pointer and element count. Pass all seven to
 * tpmd_set_feats_device to hand the pyramid to a decoder on the same GPU
 * without a host round trip. */
int tpme_feat_device(tpme_ctx *ctx, int j, const float **dev_ptr, int64_t *count);

#ifdef __cplusplus
}
#endif
#endif
