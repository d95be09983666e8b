// End-to-end generator C ABI (include/tppl.h): the reference's
// generate_impl (src/pipeline.cpp:99-186) over the four stage handles. Host
// orchestration only; every stage runs on the GPU.
#include <algorithm>
#include <condition_variable>
#include <memory>
#include <cstdio>
#include <cstring>
#include <deque>
#include <mutex>
#include <random>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "../../include/tppl.h"

namespace {
thread_local std::string g_create_err;
constexpr int STYLE = 512, IMG_PIX = 3 * 512 * 512;
}  // namespace

struct tppl_ctx {
    std::string err, ftype;
    tpfm_config fcfg{};
    tpae_config acfg{};
    tpme_ctx *me = nullptr;
    tpae_ctx *ae = nullptr;
    tpfm_ctx *fm = nullptr;
    tpmd_ctx *md = nullptr;
    int max_batch = 50;
    ~tppl_ctx() {
        tpmd_destroy(md);
        tpfm_destroy(fm);
        tpae_destroy(ae);
        tpme_destroy(me);
    }
    int fail(const std::string &m) {
        err = m;
        return -1;
    }
};

namespace {

// stages 1-3 of generate_impl: encoder (feats to the decoder on the GPU),
// audio features, chunked sampling -> styles[t] = appearance + r_d[t];
// each chunk's styles go to `cb` (when given) as soon as they exist
int make_styles(tppl_ctx *c, const float *image, const float *audio, int64_t n_samples, int emotion,
                const float *noise, uint64_t seed, std::vector<float> &styles, tppl_styles_fn cb = nullptr,
                void *ud = nullptr) {
    const int64_t n_frames = tppl_n_frames(n_samples), n_chunks = tppl_n_chunks(n_frames);
    if (!image || !audio) return c->fail("tppl: null argument");
    if (n_frames <= 0) return c->fail("audio too short");
    const int CF = c->fcfg.chunk_frames, P = c->fcfg.prev_frames, D = c->fcfg.dim_w;
    if (CF != 50 || D != STYLE) return c->fail("tppl: the sampler must produce 50-frame chunks of 512-d motion");
    std::vector<float> app(STYLE), lam(20), motion(STYLE);
    if (tpme_run(c->me, image, app.data(), lam.data(), motion.data(), nullptr) != 0)
        return c->fail(tpme_last_error(c->me));
    const float *fd[TPMD_N_LEVELS];
    for (int j = 0; j < TPMD_N_LEVELS; j++) {
        int64_t n = 0;
        if (tpme_feat_device(c->me, j, &fd[j], &n) != 0) return c->fail(tpme_last_error(c->me));
    }
    if (tpmd_set_feats_device(c->md, fd, nullptr) != 0) return c->fail(tpmd_last_error(c->md));
    std::vector<float> wa((size_t) n_frames * c->acfg.dim_w);
    if (tpae_encode(c->ae, audio, n_samples, n_frames, wa.data()) != 0) return c->fail(tpae_last_error(c->ae));
    std::vector<float> own_noise;
    if (!noise) {
        // the same fixed-seed draw for every chunk (src/pipeline.cpp:125-132)
        own_noise.resize((size_t) CF * D);
        std::mt19937_64 g(seed);
        std::normal_distribution<float> nd(0.0f, 1.0f);
        for (float &f : own_noise) f = nd(g);
    }
    std::vector<float> r_d((size_t) n_chunks * CF * D), prev_x((size_t) P * D, 0.0f), prev_wa((size_t) P * D, 0.0f),
        wa_t((size_t) CF * D);
    styles.assign((size_t) n_frames * STYLE, 0.0f);
    for (int64_t ck = 0; ck < n_chunks; ck++) {
        const int64_t f0 = ck * CF;
        for (int64_t f = 0; f < CF; f++) {  // replicate-padded at the clip's end
            const int64_t src = std::min(f0 + f, n_frames - 1);
            memcpy(wa_t.data() + (size_t) f * D, wa.data() + (size_t) src * D, (size_t) D * 4);
        }
        float *out = r_d.data() + (size_t) ck * CF * D;
        const float *x0 = noise ? noise + (size_t) ck * CF * D : own_noise.data();
        if (tpfm_sample_chunk(c->fm, motion.data(), prev_wa.data(), wa_t.data(), prev_x.data(), x0, emotion, out) != 0)
            return c->fail(tpfm_last_error(c->fm));
        memcpy(prev_x.data(), out + (size_t) (CF - P) * D, (size_t) P * D * 4);
        memcpy(prev_wa.data(), wa_t.data() + (size_t) (CF - P) * D, (size_t) P * D * 4);
        const int64_t f1 = std::min<int64_t>(f0 + CF, n_frames);
        for (int64_t t = f0; t < f1; t++)
            for (int i = 0; i < STYLE; i++)
                styles[(size_t) t * STYLE + i] = app[(size_t) i] + r_d[(size_t) t * D + i];
        if (cb && cb(f0, f1 - f0, styles.data() + (size_t) f0 * STYLE, ud) != 0) break;
    }
    return (int) n_frames;
}

}  // namespace

extern "C" {

tppl_ctx *tppl_create(int device, const char *ftype, const tpfm_config *fmt, const tpae_config *audio,
                      int max_batch) {
    const std::string ft = ftype ? ftype : "f32";
    if ((ft != "f32" && ft != "f16") || max_batch < 1) {
        g_create_err = "tppl_create: ftype must be f32 or f16, max_batch >= 1";
        return nullptr;
    }
    tppl_ctx *c = new tppl_ctx();
    c->ftype = ft;
    c->max_batch = max_batch;
    if (fmt)
        c->fcfg = *fmt;
    else
        tpfm_default_config(&c->fcfg);
    if (audio)
        c->acfg = *audio;
    else
        tpae_default_config(&c->acfg);
    if (c->fcfg.dim_a != c->acfg.dim_w || c->fcfg.dim_w != STYLE) {
        g_create_err = "tppl_create: the sampler's dim_a must equal the audio encoder's dim_w, dim_w 512";
        delete c;
        return nullptr;
    }
    const int dt = ft == "f16" ? TPMD_DTYPE_F16 : TPMD_DTYPE_F32;
    if (!(c->me = tpme_create(device)))
        g_create_err = tpme_create_error();
    else if (!(c->ae = tpae_create(device, &c->acfg)))
        g_create_err = tpae_create_error();
    else if (!(c->fm = tpfm_create(device, dt, &c->fcfg)))
        g_create_err = tpfm_create_error();
    else if (!(c->md = tpmd_create(device, dt, max_batch)))
        g_create_err = tpmd_create_error();
    else
        return c;
    delete c;
    return nullptr;
}

const char *tppl_create_error(void) { return g_create_err.c_str(); }
void tppl_destroy(tppl_ctx *c) { delete c; }
const char *tppl_last_error(const tppl_ctx *c) { return c ? c->err.c_str() : "no context"; }
tpme_ctx *tppl_motion_encoder(tppl_ctx *c) { return c ? c->me : nullptr; }
tpae_ctx *tppl_audio_encoder(tppl_ctx *c) { return c ? c->ae : nullptr; }
tpfm_ctx *tppl_sampler(tppl_ctx *c) { return c ? c->fm : nullptr; }
tpmd_ctx *tppl_decoder(tppl_ctx *c) { return c ? c->md : nullptr; }

int tppl_prepare(tppl_ctx *c) {
    if (!c) return -1;
    if (tpme_prepare(c->me) != 0) return c->fail(tpme_last_error(c->me));
    if (tpae_prepare(c->ae) != 0) return c->fail(tpae_last_error(c->ae));
    if (tpfm_prepare(c->fm) != 0) return c->fail(tpfm_last_error(c->fm));
    if (tpmd_prepare(c->md) != 0) return c->fail(tpmd_last_error(c->md));
    return 0;
}

int tppl_load(tppl_ctx *c, const char *gguf_dir) {
    if (!c) return -1;
    const std::string dir = gguf_dir ? gguf_dir : ".";
    const std::string ma = dir + "/motion_ae_" + c->ftype + ".gguf";
    if (tpae_load_gguf(c->ae, (dir + "/audio_" + c->ftype + ".gguf").c_str()) != 0)
        return c->fail(tpae_last_error(c->ae));
    if (tpfm_load_gguf(c->fm, (dir + "/fmt_" + c->ftype + ".gguf").c_str()) != 0)
        return c->fail(tpfm_last_error(c->fm));
    if (tpme_load_gguf(c->me, ma.c_str()) != 0) return c->fail(tpme_last_error(c->me));
    if (tpmd_load_gguf(c->md, ma.c_str()) != 0) return c->fail(tpmd_last_error(c->md));
    return tppl_prepare(c);
}

int64_t tppl_n_frames(int64_t n_samples) {
    if (n_samples <= 0) return 0;
    return (n_samples * 25 + 15999) / 16000;  // ceil(n * fps / sr)
}
int64_t tppl_n_chunks(int64_t n_frames) { return (n_frames + 49) / 50; }

int tppl_styles(tppl_ctx *c, const float *image, const float *audio, int64_t n_samples, int emotion,
                const float *noise, uint64_t seed, float *styles) {
    if (!c) return -1;
    if (!styles) return c->fail("tppl_styles: null styles");
    std::vector<float> st;
    const int n = make_styles(c, image, audio, n_samples, emotion, noise, seed, st);
    if (n < 0) return -1;
    memcpy(styles, st.data(), st.size() * 4);
    return n;
}

int tppl_styles_cb(tppl_ctx *c, const float *image, const float *audio, int64_t n_samples, int emotion,
                   const float *noise, uint64_t seed, tppl_styles_fn cb, void *ud) {
    if (!c) return -1;
    if (!cb) return c->fail("tppl_styles_cb: null callback");
    std::vector<float> st;
    return make_styles(c, image, audio, n_samples, emotion, noise, seed, st, cb, ud);
}

namespace {
// Decodes chunks of frames on its own thread (the decoder's stream) while the
// calling thread samples the next chunk; the frames go straight to the
// caller's buffer. The styles vector is sized before the first chunk and
// never reallocated, so the worker reads it in place.
struct chunk_decoder {
    tpmd_ctx *md;
    const float *styles;
    float *out;
    std::mutex mu;
    std::condition_variable cv;
    std::deque<std::pair<int64_t, int64_t>> todo;  // [frame0, n)
    bool closed = false, failed = false;
    std::string err;
    std::thread th;
    chunk_decoder(tpmd_ctx *m, const float *st, float *o) : md(m), styles(st), out(o) {
        th = std::thread([this] { run(); });
    }
    void run() {
        for (;;) {
            std::pair<int64_t, int64_t> job;
            {
                std::unique_lock<std::mutex> lk(mu);
                cv.wait(lk, [this] { return closed || !todo.empty(); });
                if (todo.empty()) return;
                job = todo.front();
                todo.pop_front();
            }
            if (failed) continue;  // drain the queue after an error
            if (tpmd_decode(md, styles + (size_t) job.first * STYLE, job.second,
                            out + (size_t) job.first * IMG_PIX) != 0) {
                std::lock_guard<std::mutex> lk(mu);
                failed = true;
                err = tpmd_last_error(md);
            }
        }
    }
    void push(int64_t f0, int64_t n) {
        {
            std::lock_guard<std::mutex> lk(mu);
            todo.emplace_back(f0, n);
        }
        cv.notify_one();
    }
    bool has_failed() {
        std::lock_guard<std::mutex> lk(mu);
        return failed;
    }
    // waits for every queued chunk; false if one failed
    bool finish() {
        {
            std::lock_guard<std::mutex> lk(mu);
            closed = true;
        }
        cv.notify_one();
        if (th.joinable()) th.join();
        return !failed;
    }
    ~chunk_decoder() { finish(); }
};
}  // namespace

int tppl_generate(tppl_ctx *c, const float *image, const float *audio, int64_t n_samples, int emotion,
                  const float *noise, uint64_t seed, float *out_frames) {
    if (!c) return -1;
    if (!out_frames) return c->fail("tppl_generate: null output");
    // make_styles sizes the styles vector before its first callback; the
    // decoder thread starts on the first chunk
    std::vector<float> st;
    std::unique_ptr<chunk_decoder> dec;
    struct ctx_t {
        tppl_ctx *c;
        std::vector<float> *st;
        std::unique_ptr<chunk_decoder> *dec;
        float *out;
    } cx{c, &st, &dec, out_frames};
    auto on_chunk = [](int64_t f0, int64_t n, const float *, void *ud) -> int {
        ctx_t *x = (ctx_t *) ud;
        if (!*x->dec) x->dec->reset(new chunk_decoder(x->c->md, x->st->data(), x->out));
        if ((*x->dec)->has_failed()) return 1;
        (*x->dec)->push(f0, n);
        return 0;
    };
    const int n = make_styles(c, image, audio, n_samples, emotion, noise, seed, st, on_chunk, &cx);
    const bool ok = !dec || dec->finish();
    if (n < 0) return -1;
    if (!ok) return c->fail(dec->err);
    return n;
}

int tppl_generate_cb(tppl_ctx *c, const float *image, const float *audio, int64_t n_samples, int emotion,
                     const float *noise, uint64_t seed, tppl_frame_cb cb, void *ud) {
    if (!c) return -1;
    if (!cb) return c->fail("tppl_generate_cb: null callback");
    std::vector<float> st;
    const int n = make_styles(c, image, audio, n_samples, emotion, noise, seed, st);
    if (n < 0) return -1;
    const int bq = c->max_batch;
    std::vector<float> frames((size_t) bq * IMG_PIX);
    for (int64_t t0 = 0; t0 < n; t0 += bq) {
        const int64_t nb = std::min<int64_t>(bq, n - t0);
        if (tpmd_decode(c->md, st.data() + (size_t) t0 * STYLE, nb, frames.data()) != 0)
            return c->fail(tpmd_last_error(c->md));
        for (int64_t b = 0; b < nb; b++)
            if (cb(t0 + b, frames.data() + (size_t) b * IMG_PIX, ud) != 0) return n;
    }
    return n;
}

}  // extern "C"
