/* tpmd — B200-native motion decoder (motion_dec) for talking-portrait.
 *
 * C ABI over hand-written sm_100a CUDA kernels. Conventions follow the
 * reference's public API (include/tp.h:1-9): no exceptions or aborts cross
 * this boundary, opaque handle, caller-owned flat buffers, fixed-width types.
 * Every int-returning entry point returns 0 on success and -1 on failure,
 * with the message in tpmd_last_error(ctx). Frees are NULL-safe.
 *
 * A handle owns one GPU (one process per GPU for multi-GPU use), one CUDA
 * stream and its device memory. It is single-threaded: one call at a time.
 *
 * Layouts (element order, fastest last, as a C array):
 *   styles  [n][512]          float32, latent = appearance + r_d[t]
 *   frames  [n][3][512][512]  float32, CHW (the reference's img output)
 *   feats[j][r*r][ST_OC[j]]   float32, channel-last (pixel-major), r = 8<<j,
 *                             ST_OC = {512,512,512,256,128,64,32}
 */
#ifndef TPMD_H
#define TPMD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TPMD_ABI_VERSION 1

/* storage/compute type of weights, feats and activations */
#define TPMD_DTYPE_F32 0 /* fp32 storage, fp32 FFMA convs (parity mode)     */
#define TPMD_DTYPE_F16 1 /* f16 storage, tcgen05 f16 convs, f32 accumulate   */

#define TPMD_N_LEVELS 7
#define TPMD_STYLE_DIM 512
#define TPMD_IMG 512

typedef struct tpmd_ctx tpmd_ctx;

int tpmd_abi_version(void);

/* Create a decoder on CUDA device `device` able to decode up to `max_batch`
 * frames per internal dispatch (the decode calls accept any n and loop).
 * Replaces the decoder half of tp_ctx::load (src/tp.cpp:13-41: backend init,
 * mdec.w binding) with ftype "f32" -> TPMD_DTYPE_F32, "f16" ->
 * TPMD_DTYPE_F16. Returns NULL on failure; the reason is in
 * tpmd_create_error() (this thread's last failed create). */
tpmd_ctx *tpmd_create(int device, int dtype, int max_batch);
const char *tpmd_create_error(void);
void tpmd_destroy(tpmd_ctx *ctx);
const char *tpmd_last_error(const tpmd_ctx *ctx);

/* motion_ae_scale (src/motion_enc.cpp:14-45): the multiplier the loader
 * folds into tensor `name` (ggml dims ne[0..3], ne[0] = torch's last dim). */
double tpmd_scale_for(const char *name, const int64_t ne[4]);

/* One scale-folded float32 tensor of the motion_ae "dec.*" set, in torch
 * element order (what weights_t holds after load, src/gguf_load.cpp:160-196;
 * 5-D modconv weights squeezed to [OC][IC][k][k]). Unknown names or wrong
 * sizes fail. */
int tpmd_set_tensor(tpmd_ctx *ctx, const char *name, const float *data, int64_t n);

/* GGUF v3 reader (weights_t::load, src/gguf_load.cpp:50-197): parses the
 * file at `path`, checks general.architecture against `expect_arch` (NULL:
 * no check) and calls `cb` once per tensor in file order with its ggml dims
 * ne[4] (fastest first, unit dims beyond the fourth dropped) and its
 * elements as float32 in torch order (f16 converted exactly), multiplied by
 * tpmd_scale_for(name, ne) when `fold_scales` is nonzero (motion_ae_scale,
 * as tp_ctx::load folds it, src/tp.cpp:32-34). `data` is valid during the
 * call only; a nonzero return from `cb` stops the read with an error. The
 * reference's acceptance rules are kept: version 3, value types
 * u32/i32/f32/bool/string, element types f32/f16, at most four non-unit
 * dims, 32-byte data alignment. Needs no GPU. On failure returns -1 and
 * writes the message (truncated to err_len, NUL-terminated) into `err`. */
typedef int (*tpmd_gguf_tensor_fn)(void *user, const char *name, const int64_t ne[4],
                                   const float *data, int64_t n);
int tpmd_gguf_read(const char *path, const char *expect_arch, int fold_scales,
                   tpmd_gguf_tensor_fn cb, void *user, char *err, size_t err_len);

/* The key/value section only (weights_t::kv_num / kv_str,
 * src/gguf_load.cpp:82-96): `cb` gets every key in file order with its
 * GGUF value type (4 u32, 5 i32, 6 f32, 7 bool: `num`; 8 string: `str`,
 * valid during the call); a nonzero return stops with an error. */
typedef int (*tpmd_gguf_kv_fn)(void *user, const char *key, int type, double num, const char *str);
int tpmd_gguf_read_kv(const char *path, const char *expect_arch, tpmd_gguf_kv_fn cb, void *user, char *err,
                      size_t err_len);

/* The decoder half of tp_ctx::load (src/tp.cpp:32-38): reads the
 * motion_ae_{f32,f16}.gguf file (architecture "float-motion-ae"), folds
 * motion_ae_scale and hands every "dec.*" tensor except dec.direction to
 * tpmd_set_tensor; encoder tensors are skipped. Call tpmd_prepare next. */
int tpmd_load_gguf(tpmd_ctx *ctx, const char *path);

/* Derive the decoder's device weights from the set tensors: S_aug, the cf
 * GEMM matrices and the sub-pixel up-conv matrices (motion_dec::prepare,
 * src/motion_dec.cpp:31-226). Requires every tensor. */
int tpmd_prepare(tpmd_ctx *ctx);

/* Per-portrait feature pyramid (motion_dec::set_feats,
 * src/motion_dec.cpp:1137-1160), host float32 as described above. */
int tpmd_set_feats(tpmd_ctx *ctx, const float *const feats[TPMD_N_LEVELS]);

/* The same pyramid from device memory on this decoder's GPU (f32,
 * channel-last, e.g. tpme_feat_device after a tpme_run), converted in place
 * on `stream` (NULL: the legacy default stream); returns after the copy.
 * The motion_enc -> motion_dec hand-off of src/pipeline.cpp:153-160 without
 * the host round trip; the reference has no counterpart. */
int tpmd_set_feats_device(tpmd_ctx *ctx, const float *const feats_dev[TPMD_N_LEVELS], void *stream);

/* Frames per internal dispatch (motion_dec::batch). */
int tpmd_batch(const tpmd_ctx *ctx);

/* styles (host) -> frames (host), n >= 1 frames; blocks until the frames
 * are in `frames`. Page-locked `frames` memory lets the device-to-host copy
 * overlap compute: on an f16 handle (n >= 4) the levels up to r128 run once
 * per group of frames and the r256 and r512 levels in parts, each part's
 * frames copied while the next part computes; the frames are the same bits
 * as tpmd_decode_device's. (motion_dec::decode_batch,
 * src/motion_dec.cpp:1194-1220, without its fixed-batch restriction.) */
int tpmd_decode(tpmd_ctx *ctx, const float *styles, int64_t n, float *frames);

/* The schedule tpmd_decode (rgb = 0) or tpmd_decode_rgb24 (rgb = 1) runs for
 * n >= 4 frames on an f16 handle created with max_batch: per group of frames
 * the levels up to r128 run once, then the r256 and r512 levels in parts,
 * each part's frames copied to the host while the next part computes. Writes
 * per group {first frame, frames, number of parts k, k part sizes} into
 * out (capacity cap entries) and returns the entries written, or -1 for bad
 * arguments, n < 4 (decoded as whole-decode sub-batches instead) or too
 * small a cap. Host-only; no counterpart in the reference (its decode_batch
 * copies each batch after computing it, src/motion_dec.cpp:1194-1220). */
int64_t tpmd_decode_schedule(int64_t n, int64_t max_batch, int rgb, int64_t *out, int64_t cap);

/* Same frames as tpmd_decode, delivered as the reference's output format:
 * interleaved RGB24 bytes rgb [n][512][512][3], each channel value v mapped
 * by clamping to [-1, 1] and (unsigned char) ((v + 1) / 2 * 255) in f32, the
 * conversion tools/tp-cli.cpp:43-53 applies before its video encoder. The
 * conversion runs on the GPU, so a quarter of the bytes cross to the host. */
int tpmd_decode_rgb24(tpmd_ctx *ctx, const float *styles, int64_t n, uint8_t *rgb);

/* Same with device pointers, enqueued on `stream` (a cudaStream_t; NULL =
 * the legacy default stream, as in CUDA's own APIs) without host
 * synchronisation. The return code covers the enqueue only: whether the
 * kernels' pipeline waits all completed is known once tpmd_device_status
 * returns 0, and the frames are valid only then. The handle's later calls
 * (on any stream, and the synchronous ones) start on the GPU after this
 * decode's work, outside a stream capture; inside one, the caller orders
 * the captured work against the handle's other calls. */
int tpmd_decode_device(tpmd_ctx *ctx, const float *styles_dev, int64_t n,
                       float *frames_dev, void *stream);

/* Device arenas: which = 0 prepared weights, 1 feats. A multi-GPU caller
 * prepares / sets feats on one rank, broadcasts each arena's bytes to the
 * other ranks (NCCL), and those ranks call tpmd_arena_adopt. */
int tpmd_arena(tpmd_ctx *ctx, int which, void **dev_ptr, size_t *bytes);
int tpmd_arena_adopt(tpmd_ctx *ctx, int which);

/* Parity taps of one frame (the reference's tap mode, src/motion_dec.cpp
 * :805-883, tools/tp-parity.cpp:235-287): decodes `style` (host [512])
 * through level `level` (0..6, r = 8<<level) and copies that level's
 * intermediates to host, CHW float32: conv1 [OC][r][r] (the up-conv output
 * as stored, i.e. multiplied by conv2's style), conv2 [OC][r][r], flowmap
 * [3][r][r] (level < 6), trunk [OC][r][r] (level < 6; multiplied by the next
 * up-conv's style), rgb [3][r][r]. Any output pointer may be NULL. */
int tpmd_decode_taps(tpmd_ctx *ctx, const float *style, int level, float *conv1,
                     float *conv2, float *flowmap, float *trunk, float *rgb);

/* Live per-kernel timing. Between begin and end, decodes launch kernels one
 * by one (no CUDA graph) with CUDA events recorded on the launch stream around
 * each; end synchronises and writes a JSON object
 * {"<kernel>": [launches, total_ms], ...} into json (cap bytes). */
int tpmd_profile_begin(tpmd_ctx *ctx);
int tpmd_profile_end(tpmd_ctx *ctx, char *json, size_t cap);

/* Kernel launches one decode of n frames issues (for accounting). */
int64_t tpmd_kernel_launches(const tpmd_ctx *ctx, int64_t n);

/* Decode without allocating anything. This entry point has no counterpart
 * in the reference. It is for callers that cannot call cudaMalloc while they
 * decode: real-time frame loops that must not risk an allocator stall or an
 * out-of-memory failure in the middle of a stream, and hosts whose own memory
 * manager owns the GPU's memory and forbids allocations behind its back.
 * Instead of the handle's workspace it uses one static device array of
 * 48 MiB inside this library, enough for one f16 frame, so it accepts n = 1
 * frame per call on a handle created with TPMD_DTYPE_F16 and rejects
 * anything larger with an error. Every GPU that loads the library holds the
 * array until process exit. The first call on each device does a one-time
 * set-up (it looks up the array's device address and zeroes its error word;
 * make that first call before any stream capture); later calls only enqueue
 * kernels on `stream` (NULL = legacy default stream), without host
 * synchronisation. All calls share the array and it keeps the last call's
 * contents, so calls whose work overlaps on the GPU (other streams, other
 * threads, other handles on the same device) race and corrupt each other's
 * frames. The frames are valid only once tpmd_device_status returns 0: an
 * expired pipeline wait stays recorded in the array until that call reads
 * and clears it. Pointers are device memory: styles_dev [n][512],
 * frames_dev [n][3][512][512]. */
int tpmd_decode_noalloc(tpmd_ctx *ctx, const float *styles_dev, int64_t n,
                        float *frames_dev, void *stream);

/* Status of the device work enqueued by tpmd_decode_device and
 * tpmd_decode_noalloc (the reference's error convention, src/tp.cpp:70-83:
 * an int status plus the last-error string). Synchronises `stream`, then
 * reads and clears the handle's device error flag and this device's
 * tpmd_decode_noalloc error word. Returns 0 when no decoder kernel reported
 * an expired pipeline wait since the last query, else -1 with the message
 * in tpmd_last_error(ctx) ("... timed out ... (results invalid)"). The
 * synchronous tpmd_decode and tpmd_decode_taps make this check themselves. */
int tpmd_device_status(tpmd_ctx *ctx, void *stream);

/* Test hook: arms the next decode of this handle so that its first tcgen05
 * conv kernel waits up to wait_ns (1 .. 2e9) on an mbarrier that nothing
 * completes, then takes its expiry path (reports through the device flag,
 * skips its work, frees its tensor memory). That decode's result is then an
 * error (tpmd_decode) or a nonzero tpmd_device_status. f16 handles only. */
int tpmd_debug_expire_wait(tpmd_ctx *ctx, long long wait_ns);

/* ---- several GPUs: frame sharding behind one handle ------------------- */

/* A group is the decoder on a clique of GPUs: one tpmd_ctx and one NCCL
 * communicator per local GPU. The reference decodes on one backend
 * (src/pipeline.cpp:153-184); frames are independent given the weights and
 * the portrait's feature pyramid, so a group shards a decode by frame with
 * no collective on the data path. Global rank 0 holds the host weights and
 * feats; tpmd_group_prepare / tpmd_group_set_feats run there and broadcast
 * the two device arenas to every other rank (ncclBroadcast over NVLink).
 * NCCL is loaded at run time (libnccl.so.2); communicators are created
 * non-blocking and every wait on them is polled under a wall-clock limit
 * (TPMD_NCCL_TIMEOUT_S, default 120 s), after which the group aborts its
 * communicators and the call fails. Group calls that communicate
 * (create, prepare, set_feats*, max) are collective: every rank makes them
 * in the same order. Conventions as above: 0 / -1 and the message in
 * tpmd_group_last_error; NULL-safe destroy; one call at a time per group. */
typedef struct tpmd_group tpmd_group;

/* All ranks in this process: devices[0..n-1] become global ranks 0..n-1
 * (n = 1 needs no NCCL). NULL on failure, reason in
 * tpmd_group_create_error(). */
tpmd_group *tpmd_group_create(const int *devices, int n, int dtype, int max_batch);
/* One process per GPU (e.g. under torchrun): global rank 0 makes an id with
 * tpmd_group_unique_id (128 bytes), the caller hands it to every rank, and
 * each rank creates its member for `device` with the same id. */
int tpmd_group_unique_id(void *id, size_t len);
tpmd_group *tpmd_group_create_rank(int device, int rank, int nranks, const void *id, size_t id_len, int dtype,
                                   int max_batch);
const char *tpmd_group_create_error(void);
void tpmd_group_destroy(tpmd_group *g);
const char *tpmd_group_last_error(const tpmd_group *g);
/* local GPUs of this group, and its place in the clique */
int tpmd_group_size(const tpmd_group *g);
int tpmd_group_ranks(const tpmd_group *g, int *rank0, int *nranks);
/* the decoder of local GPU i (for device-pointer decodes, taps, profiling) */
tpmd_ctx *tpmd_group_member(tpmd_group *g, int i);

/* Weights and feats: read on global rank 0 (other ranks' calls to
 * set_tensor / load_gguf are accepted and ignored), then broadcast. */
int tpmd_group_set_tensor(tpmd_group *g, const char *name, const float *data, int64_t n);
int tpmd_group_load_gguf(tpmd_group *g, const char *path);
int tpmd_group_prepare(tpmd_group *g);
int tpmd_group_set_feats(tpmd_group *g, const float *const feats[TPMD_N_LEVELS]);
/* feats_dev on global rank 0's device (e.g. tpme_feat_device output) */
int tpmd_group_set_feats_device(tpmd_group *g, const float *const feats_dev[TPMD_N_LEVELS], void *stream);

/* Frames of rank `rank` when n frames shard over nranks: the contiguous
 * [lo, hi) = [rank*ceil(n/nranks), ...), empty for trailing ranks. */
int tpmd_shard_range(int64_t n, int nranks, int rank, int64_t *lo, int64_t *hi);
/* Decode n frames of host styles [n][512] into host frames
 * [n][3][512][512] (the whole clip's buffers on every rank): each local GPU
 * decodes its shard on its own host thread and copies it straight into its
 * slice of `frames`; other ranks' slices are not touched. */
int tpmd_group_decode(tpmd_group *g, const float *styles, int64_t n, float *frames);
/* tpmd_group_decode with RGB24 frames (see tpmd_decode_rgb24):
 * rgb [n][512][512][3] bytes. */
int tpmd_group_decode_rgb24(tpmd_group *g, const float *styles, int64_t n, uint8_t *rgb);
/* Maximum of `value` over all ranks (NCCL all-reduce; timing as the max
 * over ranks). */
int tpmd_group_max(tpmd_group *g, double value, double *out);
/* Test hook: the communicator set-up and its failure handling against a
 * fake NCCL, without a GPU (scenario 0 initialises, 1 never finishes and the
 * limit expires, 2 reports an asynchronous error, 3 fails the init call);
 * -1 and the message in err on failure, *aborted = ncclCommAbort calls. */
int tpmd_group_selftest_nccl(int n, int scenario, double limit_s, int *aborted, char *err, size_t err_len);

/* ---- op-level kernels with the patched-op semantics ------------------ */

/* ggml_bilinear_gather / _planar / _sp (patches/ggml-tp-ops.patch:41-60,
 * 104-111; CPU semantics patch:319-369): torch grid_sample (bilinear, zeros
 * padding, align_corners=false) of a channel-last map feat [W*H][C] (f32, or
 * f16 when feat_is_f16) at N grid points. grid: [N][2] (x, y) interleaved,
 * or [2][N] planar when `planar`. dst: [N][C], or [C][N] when `out_sp`.
 * All pointers are device memory; enqueued on `stream`. */
int tpk_bilinear_gather(const void *feat, int feat_is_f16, int C, int W, int H,
                        const float *grid, int64_t N, int planar, int out_sp,
                        float *dst, void *stream);

/* ggml_im2col_cf (patch:25-39, CPU patch:201-307, CUDA patch:827-904):
 * src [N][IH][IW][IC] f32 (channels first in ggml terms: ic fastest) ->
 * dst [N][OH][OW][KH*KW*IC] with row r = ic + IC*(kw + KW*kh), zeros outside
 * the source, OW = (IW + 2*p0 - d0*(KW-1) - 1)/s0 + 1 (OH likewise).
 * dst is f16 (round to nearest even) when dst_is_f16, else f32. */
int tpk_im2col_cf(const float *src, int IC, int IW, int IH, int N, int KW, int KH,
                  int s0, int s1, int p0, int p1, int d0, int d1, void *dst,
                  int dst_is_f16, void *stream);

/* CHW f32 frames chw [n][3][H][W] -> RGB24 bytes rgb [n][H][W][3], the
 * conversion of tools/tp-cli.cpp:43-53 (clamp to [-1, 1], then
 * (unsigned char) ((v + 1) / 2 * 255) in f32, truncating), bit-exact.
 * H*W a multiple of 4, chw 16-byte and rgb 4-byte aligned; device memory,
 * enqueued on `stream`. */
int tpk_chw_to_rgb24(const float *chw, int64_t n, int H, int W, uint8_t *rgb, void *stream);

/* The library's tcgen05 GEMM, which the sampler and the audio encoder run
 * their contractions on: for b < batch,
 *   Y[b*y_batch + m*ldy + n] = act((sum_k X[m'][k'] W[n'][k'] + bias[n]) * scale)
 * with m' = b*x_row_b + m, k' = b*x_col_b + k (X rows of stride ldx), n',
 * k' of W likewise, m < M, n < N, k < K. dtype TPMD_DTYPE_F32: f32
 * operands by the three-pass TF32 split (about 2^-20 relative error per
 * product); TPMD_DTYPE_F16: f16 operands; f32 accumulation either way.
 * act 0 none, 1 GELU (erf), 2 GELU (tanh), 3 leaky ReLU (slope 0.2); bias
 * may be NULL. Strides in
 * elements, 16-byte multiples, bases 16-byte aligned; device memory.
 * Synchronous: returns once the GEMM finished on `stream`; -1 (message in
 * tpk_last_error) on a bad argument or an expired pipeline wait. */
int tpk_gemm(const void *X, int64_t ldx, const void *W, int64_t ldw, float *Y, int64_t ldy, int M, int N, int K,
             int batch, int x_row_b, int x_col_b, int w_row_b, int w_col_b, int64_t y_batch, int dtype,
             const float *bias, float scale, int act, void *stream);

/* Message of the last failed tpk_* call on this thread. */
const char *tpk_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* TPMD_H */
