// Audio encoder C ABI (include/tpae.h): audio_model::encode
// (src/audio_enc.cpp:55-236) over the library's tcgen05 GEMM with float32
// operands (three-pass TF32 split, kernels_gemm_tc.cu) and the kernels of
// kernels_audio.cu. Convolutions are im2col + GEMM (the convs' GELU and the
// linears' biases, the q scaling and the FFN GELU in the GEMM epilogue);
// q, k and v come from one GEMM over their stacked weights; attention is
// two head-batched GEMMs (heads as column blocks of the qkv rows) around a
// row softmax, the values transposed once so both operands run along j.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/tpae.h"
#include "tpmd_internal.h"

namespace tpmd {
cudaError_t aud_im2col(const float *x, int64_t T, int ld, int C, int K, int s, int p, int64_t OT, int groups,
                       float *out, int ldo, cudaStream_t st);
cudaError_t aud_transpose(const float *src, int64_t S, int lds, int C, float *dst, int ldd, cudaStream_t st);
cudaError_t aud_group_norm_gelu(float *x, int64_t T, int C, float eps, const float *w, const float *b, float *stats,
                                cudaStream_t st);
cudaError_t aud_interp(const float *x, int64_t T, int C, int64_t S, float *y, cudaStream_t st);
cudaError_t aud_layer_norm(const float *x, const float *r, const float *rb, int64_t M, int N, float eps,
                           const float *w, const float *b, bool silu_act, float *y, cudaStream_t st);
cudaError_t aud_pos_add(float *e, const float *pos, const float *b, int64_t S, int H, cudaStream_t st);
cudaError_t aud_softmax(float *x, int64_t rows, int N, int ld, cudaStream_t st);
cudaError_t aud_copy_cols(const float *src, int64_t S, int H, float *dst, int ld, int off, cudaStream_t st);
}  // namespace tpmd

using namespace tpmd;

namespace {
thread_local std::string g_create_err;
}

struct tpae_ctx {
    int device = 0;
    tpae_config c{};
    std::string err;
    std::map<std::string, int64_t> spec;
    std::map<std::string, std::vector<float>> host;
    std::map<std::string, size_t> off;
    std::map<std::string, int> kdim, ldk;  // conv weights: K, and rows padded to 4 floats
    float *w = nullptr;
    bool wready = false;
    cudaStream_t stream = nullptr;
    int *gerr = nullptr;  // the GEMMs' error flag
    float *ws = nullptr;
    size_t ws_floats = 0;

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
    const float *W(const std::string &n) const { return w + off.at(n); }
    gemm_desc desc() const {
        gemm_desc d;
        d.f32 = true;
        d.err = gerr;
        return d;
    }
    // Y[M][N] (ldy) = act((X[M][K] (ldx) W[N][K]^T (ldw) + bias) * scale)
    bool gemm(const float *X, int64_t Mr, int K, int ldx, const float *Wt, int ldw, int N, float *Y, int ldy,
              const char *what, const float *bias = nullptr, float scale = 1.0f, int act = 0) {
        gemm_desc d = desc();
        d.X = X;
        d.ldx = ldx;
        d.W = Wt;
        d.ldw = ldw;
        d.Y = Y;
        d.ldy = ldy;
        d.M = (int) Mr;
        d.N = N;
        d.K = K;
        d.bias = bias;
        d.scale = scale;
        d.act = act;
        return ck(gemm_tc(d, stream), what);
    }
    // after a synchronize: a GEMM whose pipeline wait expired
    bool gemm_status() {
        int flag = 0;
        if (!ck(cudaMemcpy(&flag, gerr, sizeof flag, cudaMemcpyDeviceToHost), "GEMM status")) return false;
        if (!flag) return true;
        cudaMemset(gerr, 0, sizeof(int));
        return fail("a GEMM pipeline wait timed out");
    }
    ~tpae_ctx() {
        if (device >= 0) cudaSetDevice(device);
        if (gerr) cudaFree(gerr);
        if (ws) cudaFree(ws);
        if (w) cudaFree(w);
        if (stream) cudaStreamDestroy(stream);
    }
};

namespace {

void build_spec(tpae_ctx *a) {
    const tpae_config &c = a->c;
    const int H = c.hidden, F = c.ffn;
    int ic = 1;
    for (int i = 0; i < 7; i++) {
        const std::string n = "feature_extractor.conv_layers." + std::to_string(i) + ".conv.weight";
        a->spec[n] = (int64_t) c.conv_dim[i] * ic * c.conv_kernel[i];
        a->kdim[n] = ic * c.conv_kernel[i];
        a->ldk[n] = (ic * c.conv_kernel[i] + 3) & ~3;
        ic = c.conv_dim[i];
    }
    a->spec["feature_extractor.conv_layers.0.layer_norm.weight"] = c.conv_dim[0];
    a->spec["feature_extractor.conv_layers.0.layer_norm.bias"] = c.conv_dim[0];
    const int C = c.conv_dim[6];
    a->spec["feature_projection.layer_norm.weight"] = C;
    a->spec["feature_projection.layer_norm.bias"] = C;
    a->spec["feature_projection.projection.weight"] = (int64_t) H * C;
    a->spec["feature_projection.projection.bias"] = H;
    a->spec["encoder.pos_conv_embed.conv.weight"] = (int64_t) H * (H / c.pos_groups) * c.pos_kernel;
    a->spec["encoder.pos_conv_embed.conv.bias"] = H;
    a->spec["encoder.layer_norm.weight"] = H;
    a->spec["encoder.layer_norm.bias"] = H;
    for (int i = 0; i < c.n_layers; i++) {
        const std::string b = "encoder.layers." + std::to_string(i) + ".";
        for (const char *pj : {"q_proj", "k_proj", "v_proj", "out_proj"}) {
            a->spec[b + "attention." + pj + ".weight"] = (int64_t) H * H;
            a->spec[b + "attention." + pj + ".bias"] = H;
        }
        a->spec[b + "layer_norm.weight"] = H;
        a->spec[b + "layer_norm.bias"] = H;
        a->spec[b + "feed_forward.intermediate_dense.weight"] = (int64_t) F * H;
        a->spec[b + "feed_forward.intermediate_dense.bias"] = F;
        a->spec[b + "feed_forward.output_dense.weight"] = (int64_t) H * F;
        a->spec[b + "feed_forward.output_dense.bias"] = H;
        a->spec[b + "final_layer_norm.weight"] = H;
        a->spec[b + "final_layer_norm.bias"] = H;
    }
    a->spec["audio_projection.0.weight"] = (int64_t) c.dim_w * H * c.n_layers;
    a->spec["audio_projection.0.bias"] = c.dim_w;
    a->spec["audio_projection.1.weight"] = c.dim_w;
    a->spec["audio_projection.1.bias"] = c.dim_w;
}

struct kv_check {
    tpae_ctx *a;
    std::string bad;
};
int check_kv(void *user, const char *key, int, double num, const char *) {
    kv_check *k = (kv_check *) user;
    const tpae_config &g = k->a->c;
    const std::string s = key;
    if (s.rfind("float.audio.", 0) != 0) return 0;
    const std::string n = s.substr(12);
    std::map<std::string, double> want = {
        {"n_layers", g.n_layers}, {"n_heads", g.n_heads}, {"hidden_size", g.hidden}, {"ffn_size", g.ffn},
        {"dim_w", g.dim_w}, {"ln_eps", g.ln_eps}, {"num_conv_pos_embeddings", g.pos_kernel},
        {"num_conv_pos_embedding_groups", g.pos_groups}, {"sample_rate", g.sample_rate}, {"fps", g.fps}};
    for (int i = 0; i < 7; i++) {
        want["conv_dim." + std::to_string(i)] = g.conv_dim[i];
        want["conv_kernel." + std::to_string(i)] = g.conv_kernel[i];
        want["conv_stride." + std::to_string(i)] = g.conv_stride[i];
    }
    auto it = want.find(n);
    if (it == want.end()) return 0;
    if (std::fabs(num - it->second) > 1e-6 * std::max(1.0, std::fabs(it->second))) {
        k->bad = s + " = " + std::to_string(num) + " differs from the handle's " + std::to_string(it->second);
        return 1;
    }
    return 0;
}
int take_tensor(void *user, const char *name, const int64_t *, const float *data, int64_t n) {
    tpae_ctx *a = (tpae_ctx *) user;
    if (!a->spec.count(name)) return 0;
    return tpae_set_tensor(a, name, data, n);
}

}  // namespace

extern "C" {

void tpae_default_config(tpae_config *cfg) {
    if (!cfg) return;
    tpae_config c{};
    c.n_layers = 12, c.n_heads = 12, c.hidden = 768, c.ffn = 3072, c.dim_w = 512, c.ln_eps = 1e-5f;
    for (int i = 0; i < 7; i++) {
        c.conv_dim[i] = 512;
        c.conv_kernel[i] = i == 0 ? 10 : (i < 5 ? 3 : 2);
        c.conv_stride[i] = i == 0 ? 5 : 2;
    }
    c.pos_kernel = 128, c.pos_groups = 16, c.sample_rate = 16000, c.fps = 25;
    *cfg = c;
}

tpae_ctx *tpae_create(int device, const tpae_config *cfg) {
    if (!cfg) {
        g_create_err = "tpae_create: null config";
        return nullptr;
    }
    bool valid = cfg->n_layers > 0 && cfg->n_heads > 0 && cfg->hidden > 0 && cfg->hidden % cfg->n_heads == 0 &&
                 cfg->ffn > 0 && cfg->dim_w > 0 && cfg->pos_groups > 0 && cfg->hidden % cfg->pos_groups == 0 &&
                 cfg->pos_kernel > 0 && cfg->sample_rate > 0 && cfg->fps > 0 && cfg->dim_w <= 4096 &&
                 cfg->hidden <= 4096 && cfg->conv_dim[6] <= 4096 &&
                 // the GEMMs' row strides (16-byte multiples) and the attention
                 // heads' whole 32-float k-blocks
                 (cfg->hidden / cfg->n_heads) % 32 == 0 && cfg->ffn % 4 == 0 && cfg->dim_w % 4 == 0 &&
                 cfg->conv_dim[0] % 4 == 0 && cfg->conv_dim[6] % 4 == 0 &&
                 ((cfg->hidden / cfg->pos_groups) * cfg->pos_kernel) % 4 == 0;
    for (int i = 0; i < 7; i++)
        valid = valid && cfg->conv_dim[i] > 0 && cfg->conv_kernel[i] > 0 && cfg->conv_stride[i] > 0;
    if (!valid) {
        g_create_err = "tpae_create: invalid config";
        return nullptr;
    }
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        g_create_err = "tpae_create: no such CUDA device";
        return nullptr;
    }
    cudaDeviceProp pr{};
    if (cudaGetDeviceProperties(&pr, device) != cudaSuccess || pr.major != 10) {
        cudaGetLastError();
        g_create_err = "tpae_create: needs an sm_100 (B200) GPU";
        return nullptr;
    }
    tpae_ctx *a = new tpae_ctx();
    a->device = device;
    a->c = *cfg;
    build_spec(a);
    bool ok = a->ck(cudaSetDevice(device), "cudaSetDevice") &&
              a->ck(cudaStreamCreateWithFlags(&a->stream, cudaStreamNonBlocking), "stream") &&
              a->ck(cudaMalloc(&a->gerr, sizeof(int)), "cudaMalloc(GEMM flag)") &&
              a->ck(cudaMemset(a->gerr, 0, sizeof(int)), "cudaMemset(GEMM flag)") &&
              a->ck(gemm_tc_prepare(), "GEMM set-up");
    if (!ok) {
        g_create_err = a->err;
        delete a;
        return nullptr;
    }
    return a;
}

const char *tpae_create_error(void) { return g_create_err.c_str(); }
void tpae_destroy(tpae_ctx *a) { delete a; }
const char *tpae_last_error(const tpae_ctx *a) { return a ? a->err.c_str() : "no context"; }

int tpae_set_tensor(tpae_ctx *a, const char *name, const float *data, int64_t n) {
    if (!a) return -1;
    if (!name || !data) return a->fail("tpae_set_tensor: null argument"), -1;
    auto it = a->spec.find(name);
    if (it == a->spec.end()) return a->fail(std::string("tpae_set_tensor: unknown tensor ") + name), -1;
    if (it->second != n)
        return a->fail(std::string("tpae_set_tensor: size mismatch for ") + name + " (want " +
                       std::to_string(it->second) + ", got " + std::to_string(n) + ")"),
               -1;
    a->host[name].assign(data, data + n);
    a->wready = false;
    return 0;
}

int tpae_load_gguf(tpae_ctx *a, const char *path) {
    if (!a) return -1;
    char e[1024] = {0};
    kv_check k{a, ""};
    if (tpmd_gguf_read_kv(path, "float-audio", check_kv, &k, e, sizeof e) != 0) {
        a->fail(k.bad.empty() ? std::string(e) : std::string(path) + ": " + k.bad);
        return -1;
    }
    if (tpmd_gguf_read(path, "float-audio", 0, take_tensor, a, e, sizeof e) != 0) {
        if (std::string(e).find("rejected by the consumer") == std::string::npos) a->fail(e);
        return -1;
    }
    return 0;
}

int tpae_prepare(tpae_ctx *a) {
    if (!a) return -1;
    for (auto &kv : a->spec)
        if (!a->host.count(kv.first)) return a->fail("tpae_prepare: missing tensor " + kv.first), -1;
    // the arena: every tensor at a 256-byte aligned offset, conv weights with
    // rows padded to ldk floats, and per layer q, k and v stacked into one
    // [3H][H] weight and one [3H] bias (one GEMM computes all three)
    const int H = a->c.hidden;
    auto is_qkv = [](const std::string &n) {
        return n.find(".attention.q_proj.") != std::string::npos || n.find(".attention.k_proj.") != std::string::npos ||
               n.find(".attention.v_proj.") != std::string::npos;
    };
    std::vector<std::pair<std::string, size_t>> items;
    for (auto &kv : a->spec) {
        if (is_qkv(kv.first)) continue;
        const auto it = a->ldk.find(kv.first);
        items.push_back({kv.first, it == a->ldk.end() ? (size_t) kv.second
                                                       : (size_t) (kv.second / a->kdim.at(kv.first)) * it->second});
    }
    for (int l = 0; l < a->c.n_layers; l++) {
        const std::string b = "encoder.layers." + std::to_string(l) + ".attention.";
        items.push_back({b + "qkv.weight", (size_t) 3 * H * H});
        items.push_back({b + "qkv.bias", (size_t) 3 * H});
    }
    size_t total = 0;
    a->off.clear();
    for (auto &it : items) {
        a->off[it.first] = total;
        total += (it.second + 63) & ~(size_t) 63;
    }
    std::vector<float> img(total, 0.0f);
    for (auto &kv : a->spec) {
        const std::string &n = kv.first;
        if (is_qkv(n)) continue;
        const auto it = a->ldk.find(n);
        if (it == a->ldk.end()) {
            memcpy(img.data() + a->off[n], a->host[n].data(), kv.second * 4);
            continue;
        }
        const int64_t K = a->kdim.at(n);
        for (int64_t r = 0; r < kv.second / K; r++)
            memcpy(img.data() + a->off[n] + r * it->second, a->host[n].data() + r * K, K * 4);
    }
    for (int l = 0; l < a->c.n_layers; l++) {
        const std::string b = "encoder.layers." + std::to_string(l) + ".attention.";
        const char *pj[3] = {"q_proj", "k_proj", "v_proj"};
        for (int j = 0; j < 3; j++) {
            memcpy(img.data() + a->off[b + "qkv.weight"] + (size_t) j * H * H, a->host[b + pj[j] + ".weight"].data(),
                   (size_t) H * H * 4);
            memcpy(img.data() + a->off[b + "qkv.bias"] + (size_t) j * H, a->host[b + pj[j] + ".bias"].data(),
                   (size_t) H * 4);
        }
    }
    if (!a->ck(cudaSetDevice(a->device), "cudaSetDevice")) return -1;
    if (a->w) cudaFree(a->w);
    a->w = nullptr;
    if (!a->ck(cudaMalloc(&a->w, total * 4), "cudaMalloc(audio weights)") ||
        !a->ck(cudaMemcpy(a->w, img.data(), total * 4, cudaMemcpyHostToDevice), "upload audio weights"))
        return -1;
    a->wready = true;
    return 0;
}

static int tpae_encode_enqueue(tpae_ctx *a, const float *audio, int64_t n_in, int64_t seq_len, float *wa) {
    if (!a) return -1;
    if (!audio || !wa || n_in < 1 || seq_len < 1) return a->fail("tpae_encode: bad argument"), -1;
    if (!a->wready) return a->fail("weights not prepared (tpae_prepare)"), -1;
    const tpae_config &c = a->c;
    // replicate-pad or crop to exactly seq_len * sample_rate / fps samples
    // unless already a multiple of it (src/audio_enc.cpp:60-70)
    const int64_t unit = (int64_t) (seq_len * c.sample_rate / c.fps);
    int64_t n = n_in;
    std::vector<float> padded;
    if (unit > 0 && n % unit != 0) {
        n = unit;
        padded.assign((size_t) n, audio[n_in - 1]);
        memcpy(padded.data(), audio, (size_t) std::min(n, n_in) * 4);
        audio = padded.data();
    }
    // shapes and workspace
    int64_t T[8];
    T[0] = n;
    size_t act = 0, col = 0;
    int ic = 1;
    for (int i = 0; i < 7; i++) {
        T[i + 1] = (T[i] - c.conv_kernel[i]) / c.conv_stride[i] + 1;
        if (T[i] < c.conv_kernel[i] || T[i + 1] < 1) return a->fail("audio too short"), -1;
        act = std::max(act, (size_t) T[i + 1] * c.conv_dim[i]);
        col = std::max(col, (size_t) T[i + 1] * ((ic * c.conv_kernel[i] + 3) & ~3));
        ic = c.conv_dim[i];
    }
    if (T[7] < 2) return a->fail("audio too short"), -1;
    const int64_t S = seq_len;
    const int H = c.hidden, F = c.ffn, L = c.n_layers, nh = c.n_heads, hd = H / nh, C6 = c.conv_dim[6];
    const int G = c.pos_groups, cg = H / G, KP = c.pos_kernel;
    // rows of the attention scores and of the transposed values: S floats
    // padded to a 16-byte multiple
    if (S > (1 << 24)) return a->fail("tpae_encode: seq_len too large"), -1;
    const int lds = (int) ((S + 3) & ~(int64_t) 3);
    col = std::max(col, (size_t) G * S * cg * KP);
    // stats: mean and 1/std per channel, then 256 x C partial (sum, sum of squares) doubles
    const size_t stat_floats = (size_t) 2 * ((c.conv_dim[0] + 1) & ~1) + (size_t) 256 * c.conv_dim[0] * 4;
    const size_t sizes[] = {(size_t) n,      act,           act,           col,          stat_floats,
                            (size_t) S * C6, (size_t) S * H, (size_t) S * 3 * H, (size_t) H * lds, (size_t) S * H,
                            (size_t) S * H,  (size_t) S * F, (size_t) nh * S * lds, (size_t) S * L * H,
                            (size_t) S * c.dim_w};
    const int ns = sizeof(sizes) / sizeof(sizes[0]);
    size_t offs[16], total = 0;
    for (int i = 0; i < ns; i++) {
        offs[i] = total;
        total += (sizes[i] + 63) & ~(size_t) 63;
    }
    if (!a->ck(cudaSetDevice(a->device), "cudaSetDevice")) return -1;
    if (total > a->ws_floats) {
        if (a->ws) cudaFree(a->ws);
        a->ws = nullptr;
        a->ws_floats = 0;
        if (!a->ck(cudaMalloc(&a->ws, total * 4), "cudaMalloc(audio workspace)")) return -1;
        a->ws_floats = total;
    }
    float *bufs[16];
    for (int i = 0; i < ns; i++) bufs[i] = a->ws + offs[i];
    float *aud = bufs[0], *x0 = bufs[1], *x1 = bufs[2], *colb = bufs[3], *stats = bufs[4], *hi = bufs[5],
          *e = bufs[6], *qkv = bufs[7], *vt = bufs[8], *att = bufs[9], *o = bufs[10], *f1 = bufs[11],
          *sc = bufs[12], *stk = bufs[13], *y = bufs[14];
    cudaStream_t st = a->stream;
    auto K = [&](cudaError_t err, const char *w) { return a->ck(err, w); };
    if (!K(cudaMemcpyAsync(aud, audio, (size_t) n * 4, cudaMemcpyHostToDevice, st), "audio H2D")) return -1;
    // conv stack: im2col + GEMM per layer; GroupNorm + GELU on the first,
    // GELU in the GEMM epilogue on the others
    const float *x = aud;
    float *dst = x0;
    ic = 1;
    for (int i = 0; i < 7; i++) {
        const int Kk = c.conv_kernel[i], s = c.conv_stride[i], O = c.conv_dim[i];
        const std::string wn = "feature_extractor.conv_layers." + std::to_string(i) + ".conv.weight";
        const int ldo = a->ldk.at(wn);
        if (!K(aud_im2col(x, T[i], ic, ic, Kk, s, 0, T[i + 1], 1, colb, ldo, st), "conv im2col") ||
            !a->gemm(colb, T[i + 1], ic * Kk, ldo, a->W(wn), ldo, O, dst, O, wn.c_str(), nullptr, 1.0f, i == 0 ? 0 : 1))
            return -1;
        if (i == 0 &&
            !K(aud_group_norm_gelu(dst, T[1], O, c.ln_eps, a->W("feature_extractor.conv_layers.0.layer_norm.weight"),
                                   a->W("feature_extractor.conv_layers.0.layer_norm.bias"), stats, st),
               "group norm"))
            return -1;
        x = dst;
        dst = dst == x0 ? x1 : x0;
        ic = O;
    }
    // interpolation to seq_len frames, feature projection (+ bias)
    if (!K(aud_interp(x, T[7], C6, S, hi, st), "interp") ||
        !K(aud_layer_norm(hi, nullptr, nullptr, S, C6, c.ln_eps, a->W("feature_projection.layer_norm.weight"),
                          a->W("feature_projection.layer_norm.bias"), false, hi, st),
           "layer norm") ||
        !a->gemm(hi, S, C6, C6, a->W("feature_projection.projection.weight"), C6, H, e, H, "feature projection",
                 a->W("feature_projection.projection.bias")))
        return -1;
    // grouped positional conv (pad K/2, first S outputs): group g's im2col
    // rows and weight rows are row blocks of one GEMM batch; GELU(+ bias) added
    {
        gemm_desc d = a->desc();
        d.X = colb;
        d.ldx = cg * KP;
        d.W = a->W("encoder.pos_conv_embed.conv.weight");
        d.ldw = cg * KP;
        d.Y = o;
        d.ldy = H;
        d.y_batch = cg;
        d.M = (int) S;
        d.N = cg;
        d.K = cg * KP;
        d.batch = G;
        d.x_row_b = (int) S;
        d.w_row_b = cg;
        if (!K(aud_im2col(e, S, H, cg, KP, 1, KP / 2, S, G, colb, cg * KP, st), "pos im2col") ||
            !K(gemm_tc(d, st), "pos conv") ||
            !K(aud_pos_add(e, o, a->W("encoder.pos_conv_embed.conv.bias"), S, H, st), "pos add") ||
            !K(aud_layer_norm(e, nullptr, nullptr, S, H, c.ln_eps, a->W("encoder.layer_norm.weight"),
                              a->W("encoder.layer_norm.bias"), false, e, st),
               "layer norm"))
            return -1;
    }
    // post-norm transformer layers
    const float scaling = 1.0f / sqrtf((float) hd);
    for (int l = 0; l < L; l++) {
        const std::string b = "encoder.layers." + std::to_string(l) + ".";
        auto Wn = [&](const char *s) { return a->W(b + s + ".weight"); };
        auto Bn = [&](const char *s) { return a->W(b + s + ".bias"); };
        // scores[h][i][j] = scaling * q_i . k_j over head h's columns; then
        // att[i][h*hd + d] = sum_j p[h][i][j] v[j][h*hd + d] against v^T
        gemm_desc ds = a->desc();
        ds.X = qkv;
        ds.ldx = 3 * H;
        ds.W = qkv + H;
        ds.ldw = 3 * H;
        ds.Y = sc;
        ds.ldy = lds;
        ds.y_batch = (int64_t) S * lds;
        ds.M = ds.N = (int) S;
        ds.K = hd;
        ds.batch = nh;
        ds.x_col_b = ds.w_col_b = hd;
        ds.scale = scaling;
        gemm_desc dv = a->desc();
        dv.X = sc;
        dv.ldx = lds;
        dv.W = vt;
        dv.ldw = lds;
        dv.Y = att;
        dv.ldy = H;
        dv.y_batch = hd;
        dv.M = (int) S;
        dv.N = hd;
        dv.K = (int) S;
        dv.batch = nh;
        dv.x_row_b = (int) S;
        dv.w_row_b = hd;
        if (!a->gemm(e, S, H, H, Wn("attention.qkv"), H, 3 * H, qkv, 3 * H, "qkv", Bn("attention.qkv")) ||
            !K(gemm_tc(ds, st), "scores") || !K(aud_softmax(sc, (int64_t) nh * S, (int) S, lds, st), "softmax") ||
            !K(aud_transpose(qkv + 2 * H, S, 3 * H, H, vt, lds, st), "values") || !K(gemm_tc(dv, st), "attention") ||
            !a->gemm(att, S, H, H, Wn("attention.out_proj"), H, H, o, H, "out proj") ||
            !K(aud_layer_norm(e, o, Bn("attention.out_proj"), S, H, c.ln_eps, Wn("layer_norm"), Bn("layer_norm"), false,
                              e, st),
               "layer norm") ||
            !a->gemm(e, S, H, H, Wn("feed_forward.intermediate_dense"), H, F, f1, F, "ffn",
                     Bn("feed_forward.intermediate_dense"), 1.0f, 1) ||
            !a->gemm(f1, S, F, F, Wn("feed_forward.output_dense"), F, H, o, H, "ffn out") ||
            !K(aud_layer_norm(e, o, Bn("feed_forward.output_dense"), S, H, c.ln_eps, Wn("final_layer_norm"),
                              Bn("final_layer_norm"), false, e, st),
               "layer norm") ||
            !K(aud_copy_cols(e, S, H, stk, L * H, l * H, st), "stack"))
            return -1;
    }
    // projection of all layer outputs: Linear (+ bias) + LayerNorm(1e-5) + SiLU
    if (!a->gemm(stk, S, L * H, L * H, a->W("audio_projection.0.weight"), L * H, c.dim_w, y, c.dim_w, "projection",
                 a->W("audio_projection.0.bias")) ||
        !K(aud_layer_norm(y, nullptr, nullptr, S, c.dim_w, 1e-5f, a->W("audio_projection.1.weight"),
                          a->W("audio_projection.1.bias"), true, y, st),
           "layer norm") ||
        !K(cudaMemcpyAsync(wa, y, (size_t) S * c.dim_w * 4, cudaMemcpyDeviceToHost, st), "wa D2H") ||
        !K(cudaStreamSynchronize(st), "audio encode") || !a->gemm_status())
        return -1;
    return 0;
}

// On a failure after work was enqueued, the stream is drained before the
// call returns, so no copy reads or writes the caller's buffers after it.
int tpae_encode(tpae_ctx *a, const float *audio, int64_t n_in, int64_t seq_len, float *wa) {
    const int rc = tpae_encode_enqueue(a, audio, n_in, seq_len, wa);
    if (rc != 0 && a && a->stream) cudaStreamSynchronize(a->stream);
    return rc;
}

}  // extern "C"
