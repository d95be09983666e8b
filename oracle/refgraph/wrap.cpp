// C entry points over the reference's own decoder, encoder and weight loader
// (src/motion_dec.cpp, src/motion_enc.cpp, src/gguf_load.cpp, compiled where
// they lie against the stand-in in this folder). TEST INFRASTRUCTURE ONLY:
// tests/ call these to pin the oracle at graph level. The call sequence is
// the reference's own load path (src/tp.cpp:13-41: weights_t::load with
// motion_ae_scale and the decoder's host tensors, motion_dec::prepare) and
// decode path (src/pipeline.cpp:153-175: build, set_feats, decode /
// decode_batch).
#include <cstdio>
#include <cstdlib>
#include <string>

#include "dump_standin.h"
#include "motion_dec.h"
#include "motion_enc.h"

namespace {
struct rg {
    tp::backend_t be;
    tp::weights_t w;
    tp::motion_dec dec;
    tp::motion_enc enc;
    tp::tap_writer taps;
    std::string err;
};

int fail(rg *h, const std::string &m) {
    h->err = m;
    return -1;
}

int64_t copy_out(const std::vector<float> &v, float *out, int64_t cap) {
    if (out && cap >= (int64_t) v.size()) memcpy(out, v.data(), v.size() * 4);
    return (int64_t) v.size();
}

std::vector<float> as_f32(const ggml_tensor *t) {
    std::vector<float> v((size_t) ggml_nelements(t));
    for (int64_t i = 0; i < (int64_t) v.size(); i++)
        v[(size_t) i] = t->type == GGML_TYPE_F16 ? ggml_fp16_to_fp32(((const ggml_fp16_t *) t->data)[i])
                                                 : ((const float *) t->data)[i];
    return v;
}
}  // namespace

extern "C" {

// Load a motion_ae GGUF file the way tp_ctx::load does (keep_f16 for the
// f16 fast path, encoder tensors excluded), then motion_dec::prepare.
// `gpu` selects the GPU flavour of the fast graph (two half up-convs instead
// of one wide one at the spatial stages). NULL on failure, message in err.
void *rg_create(const char *gguf_path, int keep_f16, int gpu, char *err, size_t err_len) {
    rg *h = new rg();
    h->be.gpu = gpu != 0;
    h->be.n_threads = 1;
    h->w.keep_f16 = keep_f16 != 0;
    h->w.f16_exclude_prefix = "enc.";
    h->w.want_host = tp::motion_dec_host_tensors();
    std::string e;
    bool ok = false;
    try {
        ok = h->w.load(gguf_path, h->be, "float-motion-ae", tp::motion_ae_scale, e);
        if (ok) {
            h->dec.w = &h->w;
            h->enc.w = &h->w;
            ok = h->dec.prepare(h->be, e);
        }
    } catch (const std::exception &x) {
        e = x.what();
        ok = false;
    }
    if (!ok) {
        if (err && err_len) snprintf(err, err_len, "%s", e.c_str());
        delete h;
        return nullptr;
    }
    return h;
}

void rg_destroy(void *p) { delete (rg *) p; }
const char *rg_error(void *p) { return ((rg *) p)->err.c_str(); }

// A loaded (scale-folded) weight tensor, or a tensor prepare() derived
// ("saug.<w>", "tsubcf.<w>", "acf.<w>", "wflip.<w>", "tsubsp.<w>"), as f32
// in ggml element order. Returns the element count (-1: unknown name).
int64_t rg_tensor(void *p, const char *name, float *out, int64_t cap) {
    rg *h = (rg *) p;
    const ggml_tensor *t = h->w.get(name);
    if (!t) {
        auto it = h->dec.derived.find(name);
        if (it == h->dec.derived.end()) return -1;
        t = it->second;
    }
    return copy_out(as_f32(t), out, cap);
}

// motion_dec::build: with_taps = the exact parity graph (batch 1); else the
// fast batched graph with `batch` frames per dispatch (TP_MDEC_BATCH).
// stages < 7 truncates the pyramid (TP_MDEC_STAGES): the image output is
// then that stage's rgb skip [3][r][r].
int rg_build(void *p, int with_taps, int batch, int stages) {
    rg *h = (rg *) p;
    char b[16];
    snprintf(b, sizeof b, "%d", batch);
    setenv("TP_MDEC_BATCH", b, 1);
    snprintf(b, sizeof b, "%d", stages);
    setenv("TP_MDEC_STAGES", b, 1);
    std::string e;
    bool ok;
    try {
        ok = h->dec.build(h->be, with_taps != 0, e);
    } catch (const std::exception &x) {
        ok = false;
        e = x.what();
    }
    unsetenv("TP_MDEC_BATCH");
    unsetenv("TP_MDEC_STAGES");
    return ok ? 0 : fail(h, e);
}

int rg_batch(void *p) { return ((rg *) p)->dec.batch; }

// feats[j]: [r*r][ST_OC[j]] f32, channel-last (menc_result::feats)
int rg_set_feats(void *p, const float *const feats[7]) {
    rg *h = (rg *) p;
    static const int OC[7] = {512, 512, 512, 256, 128, 64, 32};
    tp::menc_result m;
    m.feats.resize(7);
    for (int j = 0; j < 7; j++) {
        const size_t n = (size_t) (8 << j) * (8 << j) * OC[j];
        m.feats[j].assign(feats[j], feats[j] + n);
    }
    std::string e;
    return h->dec.set_feats(m, e) ? 0 : fail(h, e);
}

// motion_dec::decode of one style [512] -> img [3][512][512]; with taps,
// every registered tap is kept (rg_tap)
int rg_decode(void *p, const float *style, float *img, int want_taps) {
    rg *h = (rg *) p;
    tp::tap_sink sink;
    if (want_taps) {
        h->taps.taps.clear();
        sink.wr = &h->taps;
    }
    std::string e;
    bool ok;
    try {
        ok = h->dec.decode(h->be, style, img, sink, e);
    } catch (const std::exception &x) {
        ok = false;
        e = x.what();
    }
    return ok ? 0 : fail(h, e);
}

int rg_decode_batch(void *p, const float *styles, float *imgs) {
    rg *h = (rg *) p;
    std::string e;
    bool ok;
    try {
        ok = h->dec.decode_batch(h->be, styles, imgs, e);
    } catch (const std::exception &x) {
        ok = false;
        e = x.what();
    }
    return ok ? 0 : fail(h, e);
}

int64_t rg_tap(void *p, const char *name, float *out, int64_t cap) {
    rg *h = (rg *) p;
    auto it = h->taps.taps.find(name);
    if (it == h->taps.taps.end()) return -1;
    return copy_out(it->second, out, cap);
}

// motion_enc::run on a CHW f32 image [3][512][512]; outputs appearance [512],
// lambda [20], motion [512] and the decoder feats [r*r][ST_OC[j]] (any may
// be NULL); with taps, the encoder's taps are kept (rg_tap)
int rg_enc_run(void *p, const float *image, float *app, float *lam, float *motion, float *const feats[7],
               int want_taps) {
    rg *h = (rg *) p;
    tp::tap_sink sink;
    if (want_taps) {
        h->taps.taps.clear();
        sink.wr = &h->taps;
    }
    tp::menc_result r;
    std::string e;
    bool ok;
    try {
        ok = h->enc.run(h->be, image, r, sink, e);
    } catch (const std::exception &x) {
        ok = false;
        e = x.what();
    }
    if (!ok) return fail(h, e);
    if (app) memcpy(app, r.appearance.data(), 512 * 4);
    if (lam) memcpy(lam, r.lambda.data(), 20 * 4);
    if (motion) memcpy(motion, r.motion.data(), 512 * 4);
    for (int j = 0; j < 7 && feats; j++)
        if (feats[j]) memcpy(feats[j], r.feats[j].data(), r.feats[j].size() * 4);
    return 0;
}

}  // extern "C"
