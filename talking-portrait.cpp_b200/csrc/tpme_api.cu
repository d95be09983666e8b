// Motion encoder C ABI (include/tpme.h): the host orchestration of
// motion_enc::run (src/motion_enc.cpp:46-184) over the kernels in
// kernels_enc.cu (its convs: im2col + the library's tcgen05 GEMM, f32
// operands by the three-pass TF32 split). One stream; a fixed device
// workspace sized for the 512x512 input; the pyramid stays on the device
// after a run so the decoder can take it directly (tpmd_set_feats_device).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/tpme.h"
#include "tpmd_internal.h"

using namespace tpmd;

namespace {

const int ENC_IN[7] = {32, 64, 128, 256, 512, 512, 512};    // src/motion_enc.cpp:46
const int ENC_OUT[7] = {64, 128, 256, 512, 512, 512, 512};  // src/motion_enc.cpp:47

thread_local std::string g_create_err;

std::map<std::string, int64_t> encoder_spec() {
    std::map<std::string, int64_t> m;
    char nm[64];
    m["enc.net_app.convs.0.0.weight"] = 32 * 3;
    m["enc.net_app.convs.0.1.bias"] = 32;
    for (int i = 1; i <= 7; i++) {
        const int64_t C = ENC_IN[i - 1], Co = ENC_OUT[i - 1];
        auto put = [&](const char *suffix, int64_t n) {
            snprintf(nm, sizeof nm, "enc.net_app.convs.%d.%s", i, suffix);
            m[nm] = n;
        };
        put("conv1.0.weight", C * C * 9);
        put("conv1.1.bias", C);
        put("conv2.0.kernel", 16);
        put("conv2.1.weight", Co * C * 9);
        put("conv2.2.bias", Co);
        put("skip.0.kernel", 16);
        put("skip.1.weight", Co * C);
    }
    m["enc.net_app.convs.8.weight"] = (int64_t) 512 * 512 * 16;
    for (int i = 0; i < 5; i++) {
        const int64_t out = i == 4 ? 20 : 512;
        snprintf(nm, sizeof nm, "enc.fc.%d.weight", i);
        m[nm] = out * 512;
        snprintf(nm, sizeof nm, "enc.fc.%d.bias", i);
        m[nm] = out;
    }
    m["dec.direction.Q"] = 512 * 20;
    return m;
}

// torch [OC][IC][K][K] -> [OC][(kh*K + kw)*IC + ic] (the conv kernel's k order)
void to_tap_major(const float *w, int OC, int IC, int K, float *out) {
    for (int o = 0; o < OC; o++)
        for (int ic = 0; ic < IC; ic++)
            for (int t = 0; t < K * K; t++)
                out[((size_t) o * K * K + t) * IC + ic] = w[((size_t) o * IC + ic) * K * K + t];
}

}  // namespace

// the largest im2col: block 1's first conv, 512 x 512 pixels x 9 taps x 32 channels
constexpr size_t COL_FLOATS = (size_t) 512 * 512 * 9 * 32;

struct tpme_ctx {
    int device = 0;
    std::string err;
    std::map<std::string, int64_t> spec = encoder_spec();
    std::map<std::string, std::vector<float>> host;
    std::map<std::string, size_t> off;  // float offset of each tensor in the arena
    float *warena = nullptr;
    size_t wfloats = 0;
    bool wready = false, ran = false;
    cudaStream_t stream = nullptr;
    void *ws = nullptr;
    float *img = nullptr, *pyr[8] = {nullptr}, *x1 = nullptr, *xb = nullptr, *sb = nullptr;
    float *app = nullptr, *lam = nullptr, *mot = nullptr;
    float *col = nullptr;  // im2col rows of the current conv (COL_FLOATS)
    int *gerr = nullptr;   // the GEMMs' expired-wait flag

    bool fail(const std::string &m) {
        err = m;
        return false;
    }
    bool ck(cudaError_t e, const char *what) {
        if (e == cudaSuccess) return true;
        err = std::string(what) + ": " + cudaGetErrorString(e);
        cudaGetLastError();
        return false;
    }
    const float *W(const std::string &n) const { return warena + off.at(n); }
    ~tpme_ctx() {
        if (device >= 0) cudaSetDevice(device);
        if (ws) cudaFree(ws);
        if (gerr) cudaFree(gerr);
        if (warena) cudaFree(warena);
        if (stream) cudaStreamDestroy(stream);
    }
};

extern "C" {

tpme_ctx *tpme_create(int device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        g_create_err = "tpme_create: no such CUDA device";
        return nullptr;
    }
    cudaDeviceProp pr{};
    if (cudaGetDeviceProperties(&pr, device) != cudaSuccess || pr.major != 10) {
        cudaGetLastError();
        g_create_err = "tpme_create: needs an sm_100 (B200) GPU";
        return nullptr;
    }
    tpme_ctx *c = new tpme_ctx();
    c->device = device;
    // workspace: image, pyramid conv0..conv7, conv1 output, the two blurred maps
    size_t sizes[16], total = 0;
    int k = 0;
    sizes[k++] = (size_t) 3 * 512 * 512;
    sizes[k++] = (size_t) 512 * 512 * 32;
    for (int i = 1; i <= 7; i++) sizes[k++] = (size_t) (512 >> i) * (512 >> i) * ENC_OUT[i - 1];
    sizes[k++] = (size_t) 512 * 512 * 32;  // x1: the largest H*H*C is block 1
    sizes[k++] = (size_t) 513 * 513 * 32;  // xb: (H+1)^2*C
    sizes[k++] = (size_t) 511 * 511 * 32;  // sb: (H-1)^2*C
    sizes[k++] = 512;
    sizes[k++] = 32;
    sizes[k++] = 512;
    sizes[k++] = COL_FLOATS;  // im2col rows
    size_t offs[16];
    for (int i = 0; i < k; i++) {
        offs[i] = total;
        total += (sizes[i] + 63) & ~(size_t) 63;  // 256-byte aligned
    }
    bool ok = c->ck(cudaSetDevice(device), "cudaSetDevice") &&
              c->ck(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "stream") &&
              c->ck(cudaMalloc(&c->ws, total * 4), "cudaMalloc(encoder workspace)") &&
              c->ck(cudaMalloc(&c->gerr, sizeof(int)), "cudaMalloc(GEMM flag)") &&
              c->ck(cudaMemset(c->gerr, 0, sizeof(int)), "cudaMemset(GEMM flag)") && c->ck(gemm_tc_prepare(), "GEMM set-up");
    if (!ok) {
        g_create_err = c->err;
        delete c;
        return nullptr;
    }
    float *b = (float *) c->ws;
    int i = 0;
    c->img = b + offs[i++];
    for (int l = 0; l < 8; l++) c->pyr[l] = b + offs[i++];
    c->x1 = b + offs[i++];
    c->xb = b + offs[i++];
    c->sb = b + offs[i++];
    c->app = b + offs[i++];
    c->lam = b + offs[i++];
    c->mot = b + offs[i++];
    c->col = b + offs[i++];
    return c;
}

const char *tpme_create_error(void) { return g_create_err.c_str(); }
void tpme_destroy(tpme_ctx *c) { delete c; }
const char *tpme_last_error(const tpme_ctx *c) { return c ? c->err.c_str() : "no context"; }

int tpme_set_tensor(tpme_ctx *c, const char *name, const float *data, int64_t n) {
    if (!c) return -1;
    if (!name || !data) return c->fail("tpme_set_tensor: null argument"), -1;
    auto it = c->spec.find(name);
    if (it == c->spec.end()) return c->fail(std::string("tpme_set_tensor: unknown tensor ") + name), -1;
    if (it->second != n)
        return c->fail(std::string("tpme_set_tensor: size mismatch for ") + name + " (want " +
                       std::to_string(it->second) + ", got " + std::to_string(n) + ")"),
               -1;
    c->host[name].assign(data, data + n);
    c->wready = false;
    return 0;
}

}  // extern "C"

namespace {
int take_encoder_tensor(void *user, const char *name, const int64_t *, const float *data, int64_t n) {
    tpme_ctx *c = (tpme_ctx *) user;
    const std::string s = name;
    if (s.rfind("enc.", 0) != 0 && s != "dec.direction.Q") return 0;
    return tpme_set_tensor(c, name, data, n);
}
}  // namespace

extern "C" {

int tpme_load_gguf(tpme_ctx *c, const char *path) {
    if (!c) return -1;
    char e[1024] = {0};
    if (tpmd_gguf_read(path, "float-motion-ae", 1, take_encoder_tensor, c, e, sizeof e) != 0) {
        // a tensor tpme_set_tensor refused keeps its own message
        if (std::string(e).find("rejected by the consumer") == std::string::npos) c->fail(e);
        return -1;
    }
    return 0;
}

int tpme_prepare(tpme_ctx *c) {
    if (!c) return -1;
    for (auto &kv : c->spec)
        if (!c->host.count(kv.first)) return c->fail("tpme_prepare: missing tensor " + kv.first), -1;
    size_t total = 0;
    c->off.clear();
    for (auto &kv : c->spec) {
        c->off[kv.first] = total;
        total += ((size_t) kv.second + 63) & ~(size_t) 63;
    }
    std::vector<float> img(total, 0.0f);
    char nm[64];
    for (auto &kv : c->spec) {
        const std::vector<float> &h = c->host.at(kv.first);
        float *dst = img.data() + c->off[kv.first];
        int OC = 0, IC = 0, K = 0;
        if (kv.first == "enc.net_app.convs.8.weight") {
            OC = 512, IC = 512, K = 4;
        } else {
            for (int i = 1; i <= 7; i++) {
                snprintf(nm, sizeof nm, "enc.net_app.convs.%d.", i);
                if (kv.first.rfind(nm, 0) != 0) continue;
                const std::string rest = kv.first.substr(strlen(nm));
                if (rest == "conv1.0.weight") OC = ENC_IN[i - 1], IC = ENC_IN[i - 1], K = 3;
                if (rest == "conv2.1.weight") OC = ENC_OUT[i - 1], IC = ENC_IN[i - 1], K = 3;
            }
        }
        if (K > 1)
            to_tap_major(h.data(), OC, IC, K, dst);
        else
            memcpy(dst, h.data(), h.size() * 4);  // 1x1 convs, linears, biases, kernels, Q
    }
    if (!c->warena) {
        if (!c->ck(cudaSetDevice(c->device), "cudaSetDevice") ||
            !c->ck(cudaMalloc(&c->warena, total * 4), "cudaMalloc(encoder weights)"))
            return -1;
        c->wfloats = total;
    }
    if (!c->ck(cudaMemcpy(c->warena, img.data(), total * 4, cudaMemcpyHostToDevice), "upload encoder weights"))
        return -1;
    c->wready = true;
    return 0;
}

static int tpme_run_enqueue(tpme_ctx *c, const float *image, float *appearance, float *lambda, float *motion,
             float *const feats[TPMD_N_LEVELS]) {
    if (!c) return -1;
    if (!image) return c->fail("tpme_run: null image"), -1;
    if (!c->wready) return c->fail("tpme_run: weights not prepared (tpme_prepare)"), -1;
    cudaStream_t st = c->stream;
    auto K = [&](cudaError_t e, const char *w) { return c->ck(e, w); };
    if (!K(cudaSetDevice(c->device), "cudaSetDevice") ||
        !K(cudaMemcpyAsync(c->img, image, (size_t) 3 * 512 * 512 * 4, cudaMemcpyHostToDevice, st), "image H2D") ||
        !K(launch_enc_stem(c->img, c->W("enc.net_app.convs.0.0.weight"), c->W("enc.net_app.convs.0.1.bias"),
                           c->pyr[0], st),
           "stem"))
        return -1;
    char nm[96];
    int H = 512;
    for (int i = 1; i <= 7; i++) {
        const int C = ENC_IN[i - 1], Co = ENC_OUT[i - 1], h = H / 2;
        auto T = [&](const char *s) {
            snprintf(nm, sizeof nm, "enc.net_app.convs.%d.%s", i, s);
            return c->W(nm);
        };
        enc_conv_params p{};
        p.col = c->col, p.col_floats = COL_FLOATS, p.err = c->gerr;
        // conv1: 3x3 pad 1 + FusedLeakyReLU -> x1
        p.x = c->pyr[i - 1], p.IH = H, p.IW = H, p.IC = C;
        p.w = T("conv1.0.weight"), p.OC = C, p.K = 3, p.stride = 1, p.pad = 1, p.OH = H, p.OW = H;
        p.bias = T("conv1.1.bias"), p.lrelu = 1, p.res = nullptr, p.y = c->x1;
        if (!K(launch_enc_conv(p, st), "encoder conv1")) return -1;
        // Blur pad (2, 2) -> xb, then 3x3 stride-2 conv + FusedLeakyReLU -> pyr[i]
        if (!K(launch_enc_blur(c->x1, H, H, C, T("conv2.0.kernel"), 2, 2, c->xb, st), "encoder blur")) return -1;
        p.x = c->xb, p.IH = H + 1, p.IW = H + 1;
        p.w = T("conv2.1.weight"), p.OC = Co, p.K = 3, p.stride = 2, p.pad = 0, p.OH = h, p.OW = h;
        p.bias = T("conv2.2.bias"), p.lrelu = 1, p.res = nullptr, p.y = c->pyr[i];
        if (!K(launch_enc_conv(p, st), "encoder conv2")) return -1;
        // skip: Blur pad (1, 1) -> sb, 1x1 stride-2 conv, added to pyr[i]
        if (!K(launch_enc_blur(c->pyr[i - 1], H, H, C, T("skip.0.kernel"), 1, 1, c->sb, st), "encoder blur"))
            return -1;
        p.x = c->sb, p.IH = H - 1, p.IW = H - 1;
        p.w = T("skip.1.weight"), p.OC = Co, p.K = 1, p.stride = 2, p.pad = 0, p.OH = h, p.OW = h;
        p.bias = nullptr, p.lrelu = 0, p.res = c->pyr[i], p.y = c->pyr[i];
        if (!K(launch_enc_conv(p, st), "encoder skip")) return -1;
        H = h;
    }
    // 4x4 valid conv -> appearance; fc chain and motion
    enc_conv_params p{};
    p.col = c->col, p.col_floats = COL_FLOATS, p.err = c->gerr;
    p.x = c->pyr[7], p.IH = 4, p.IW = 4, p.IC = 512;
    p.w = c->W("enc.net_app.convs.8.weight"), p.OC = 512, p.K = 4, p.stride = 1, p.pad = 0, p.OH = 1, p.OW = 1;
    p.y = c->app;
    if (!K(launch_enc_conv(p, st), "encoder conv8")) return -1;
    enc_head_params hp{};
    for (int l = 0; l < 5; l++) {
        snprintf(nm, sizeof nm, "enc.fc.%d.weight", l);
        hp.W[l] = c->W(nm);
        snprintf(nm, sizeof nm, "enc.fc.%d.bias", l);
        hp.b[l] = c->W(nm);
    }
    hp.Q = c->W("dec.direction.Q");
    if (!K(launch_enc_head(c->app, hp, c->lam, c->mot, c->col, st), "encoder head")) return -1;
    if ((appearance && !K(cudaMemcpyAsync(appearance, c->app, 512 * 4, cudaMemcpyDeviceToHost, st), "D2H")) ||
        (lambda && !K(cudaMemcpyAsync(lambda, c->lam, 20 * 4, cudaMemcpyDeviceToHost, st), "D2H")) ||
        (motion && !K(cudaMemcpyAsync(motion, c->mot, 512 * 4, cudaMemcpyDeviceToHost, st), "D2H")))
        return -1;
    for (int j = 0; feats && j < TPMD_N_LEVELS; j++) {
        if (!feats[j]) continue;
        const int r = 8 << j;
        const size_t n = (size_t) r * r * (j < 3 ? 512 : 512 >> (j - 2));
        if (!K(cudaMemcpyAsync(feats[j], c->pyr[6 - j], n * 4, cudaMemcpyDeviceToHost, st), "feats D2H"))
            return -1;
    }
    if (!K(cudaStreamSynchronize(st), "encoder run")) return -1;
    int flag = 0;
    if (!K(cudaMemcpy(&flag, c->gerr, sizeof flag, cudaMemcpyDeviceToHost), "GEMM status")) return -1;
    if (flag) {
        cudaMemset(c->gerr, 0, sizeof(int));
        return c->fail("encoder: a GEMM pipeline wait timed out"), -1;
    }
    c->ran = true;
    return 0;
}

// On a failure after work was enqueued, the stream is drained before the
// call returns, so no copy reads or writes the caller's buffers after it.
int tpme_run(tpme_ctx *c, const float *image, float *appearance, float *lambda, float *motion,
             float *const feats[TPMD_N_LEVELS]) {
    const int rc = tpme_run_enqueue(c, image, appearance, lambda, motion, feats);
    if (rc != 0 && c && c->stream) cudaStreamSynchronize(c->stream);
    return rc;
}

int tpme_feat_device(tpme_ctx *c, int j, const float **dev_ptr, int64_t *count) {
    if (!c) return -1;
    if (j < 0 || j >= TPMD_N_LEVELS || !dev_ptr || !count) return c->fail("tpme_feat_device: bad argument"), -1;
    if (!c->ran) return c->fail("tpme_feat_device: no encoder run yet"), -1;
    const int r = 8 << j;
    *dev_ptr = c->pyr[6 - j];
    *count = (int64_t) r * r * (j < 3 ? 512 : 512 >> (j - 2));
    return 0;
}

}  // extern "C"
