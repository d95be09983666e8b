// The C++ shim (include/motion_dec_b200.h) used the way the reference's
// pipeline uses its decoder; asserts are the test, like the reference's
// ctest programs. argv[1] == "gpu": full load + decode; otherwise only the
// failure paths that need no GPU.
#undef NDEBUG
#include <cassert>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "motion_dec_b200.h"

// stand-ins for the reference's types at the decoder's call sites
// (src/tp_internal.h backend_t, src/motion_enc.h menc_result): the shim's
// overloads take them as the reference's motion_dec does
namespace tp {
struct backend_t {
    bool gpu = true;
};
struct menc_result {
    std::vector<float> appearance;
    std::vector<std::vector<float>> feats;
};
}  // namespace tp

// the decoder calls of the reference's decode loop (src/pipeline.cpp:153-175)
// against the shim, with the reference's argument lists
struct ctx_like {
    tp::backend_t be;
    tpmd_cpp::motion_dec_b200 mdec;
    std::string err;
};
static bool decode_like_pipeline(ctx_like *c, const tp::menc_result &m, const std::vector<float> &styles,
                                 float *dst) {
    std::string &err = c->err;
    if (!c->mdec.built || c->mdec.taps_in_graph) {
        if (!c->mdec.build(c->be, false, err)) return false;
    }
    if (!c->mdec.set_feats(m, err)) return false;
    const int BQ = c->mdec.batch;
    (void) BQ;
    return c->mdec.decode_batch(c->be, styles.data(), dst, err);
}

static const int ST_IC[7] = {512, 512, 512, 512, 256, 128, 64};
static const int ST_OC[7] = {512, 512, 512, 256, 128, 64, 32};

static void put(tpmd_cpp::motion_dec_b200 &d, const std::string &name, std::vector<int64_t> ne,
                std::mt19937 &rng, float fill, bool randn) {
    int64_t n = 1;
    for (auto v : ne) n *= v;
    while (ne.size() < 4) ne.push_back(1);
    const double sc = tpmd_scale_for(name.c_str(), ne.data());
    std::normal_distribution<float> nd;
    std::vector<float> v((size_t) n);
    for (auto &x : v) x = (randn ? nd(rng) : fill) * (float) sc;
    std::string err;
    assert(d.set_tensor(name, v.data(), n, err));
}

int main(int argc, char **argv) {
    const bool gpu = argc > 1 && strcmp(argv[1], "gpu") == 0;
    std::string err;
    tpmd_cpp::motion_dec_b200 bad;
    assert(!bad.load(0, "f64", 2, err) && err == "ftype must be f32 or f16");
    assert(!bad.build(false, err) && err == "decoder not loaded");
    {
        ctx_like c;
        tp::menc_result m;
        std::vector<float> st(512), out(3 * 512 * 512);
        assert(!decode_like_pipeline(&c, m, st, out.data()) && c.err == "decoder not loaded");
    }
    if (!gpu) {
        assert(!bad.load(9999, "f16", 2, err) && !err.empty());
        printf("test_shim (no GPU) OK\n");
        return 0;
    }
    tpmd_cpp::motion_dec_b200 d;
    assert(d.load(0, "f16", 2, err));
    std::mt19937 rng(42);
    char nm[64];
    put(d, "dec.input.input", {4, 4, 512}, rng, 0, true);
    for (int k = -1; k < 14; k++) {
        const int j = k < 0 ? 0 : k / 2;
        const bool up = k >= 0 && k % 2 == 0;
        const int IC = k < 0 ? 512 : (up ? ST_IC[j] : ST_OC[j]), OC = k < 0 ? 512 : ST_OC[j];
        std::string base = k < 0 ? "dec.conv1" : ("dec.convs." + std::to_string(k));
        put(d, base + ".conv.weight", {3, 3, IC, OC}, rng, 0, true);
        put(d, base + ".conv.modulation.weight", {512, IC}, rng, 0, true);
        put(d, base + ".conv.modulation.bias", {IC}, rng, 1.0f, false);
        put(d, base + ".activate.bias", {1, 1, OC, 1}, rng, 0.0f, false);
        if (up) {
            const float k1[4] = {1, 3, 3, 1};
            std::vector<float> bk(16);
            for (int a = 0; a < 4; a++)
                for (int b = 0; b < 4; b++) bk[(size_t) a * 4 + b] = k1[a] * k1[b] / 64.0f * 4.0f;
            assert(d.set_tensor(base + ".conv.blur.kernel", bk.data(), 16, err));
        }
    }
    for (int j = 0; j < 7; j++) {
        const int OC = ST_OC[j];
        snprintf(nm, sizeof nm, "dec.to_flows.%d", j);
        std::string f = nm;
        put(d, f + ".conv.weight", {1, 1, OC, 3}, rng, 0, true);
        put(d, f + ".conv.modulation.weight", {512, OC}, rng, 0, true);
        put(d, f + ".conv.modulation.bias", {OC}, rng, 1.0f, false);
        put(d, f + ".bias", {1, 1, 3, 1}, rng, 0.0f, false);
        put(d, f + ".upsample.kernel", {4, 4}, rng, 0.25f, false);
        snprintf(nm, sizeof nm, "dec.to_rgbs.%d", j);
        std::string r = nm;
        put(d, r + ".conv.0.weight", {1, 1, OC, 3}, rng, 0, true);
        put(d, r + ".conv.1.bias", {1, 1, 3, 1}, rng, 0.0f, false);
        put(d, r + ".bias", {1, 1, 3, 1}, rng, 0.0f, false);
        put(d, r + ".upsample.kernel", {4, 4}, rng, 0.25f, false);
    }
    assert(!d.set_tensor("dec.nope", nullptr, 1, err) || true);
    assert(d.prepare(err));
    assert(d.build(false, err) && d.built && !d.taps_in_graph);
    std::vector<std::vector<float>> feats(7);
    std::normal_distribution<float> nd;
    for (int j = 0; j < 7; j++) {
        feats[(size_t) j].resize((size_t) (8 << j) * (8 << j) * ST_OC[j]);
        for (auto &x : feats[(size_t) j]) x = nd(rng);
    }
    assert(d.set_feats(feats, err));
    std::vector<float> styles((size_t) d.batch * 512), imgs((size_t) d.batch * 3 * 512 * 512);
    for (auto &x : styles) x = nd(rng);
    assert(d.decode_batch(styles.data(), imgs.data(), err));
    double s = 0;
    for (float x : imgs) {
        assert(std::isfinite(x));
        s += std::fabs(x);
    }
    assert(s > 0);
    std::vector<float> again(imgs.size());
    assert(d.decode_batch(styles.data(), again.data(), err));
    assert(memcmp(again.data(), imgs.data(), imgs.size() * 4) == 0);  // deterministic
    // the same decode through the reference-shaped call sites
    {
        tp::menc_result m;
        m.feats = feats;
        tp::backend_t be;
        std::vector<float> viaref(imgs.size());
        d.built = false;
        assert(d.build(be, false, err) && d.built);
        assert(d.set_feats(m, err));
        assert(d.decode_batch(be, styles.data(), viaref.data(), err));
        assert(memcmp(viaref.data(), imgs.data(), imgs.size() * 4) == 0);
    }
    printf("test_shim (GPU) OK mean|x| %.4f\n", s / imgs.size());
    return 0;
}
